// Block engine of the EWS hot path: A block-diagonal with 2x2 blocks (rotation-decay planes and any
// other real 2x2 blocks), state dimension N <= 8 (N even), depth 3, per-interval clock, fp32.
//
// Per interval t of sample b (h = clock[t+1] - clock[t], X = -h A, M = expm(X), dy = lift @ dx):
//     S1' = M S1 + s1
//     S2' = (M (x) M) S2 + (M S1) (x) s1 + s2
//     S3' = (M (x) M (x) M) S3 + ((M (x) M) S2) (x) s1 + (M S1) (x) s2 + s3
// the modified-Chen recursion of ews/core/chen_scan.py:124-152 with per-interval flows
// (ews/core/chen_scan.py:155-168, cached=False), and the series local terms of
// ews/core/series_leaf.py:72-127: letters b_0 = dy, b_p = (X / p) b_{p-1}, level k =
// sum_{|m|<=q} c_m b_{m1} (x) ... (x) b_{mk}, c_m = prod_j 1 / (m_j + ... + m_k + k - j + 1).
// This is the block kernel's recursion (ews/core/kernels/pallas_combine.py:1221-1289: pair-mixes of
// every tensor axis with the block flow, cross terms, local terms) written for one warp per tile.
//
// Work decomposition. One warp owns one tile (sample, chunk of Lc intervals). Lane (i, jb), i = lane / 4,
// jb = lane % 4, owns the level-3 entries S3[i][j][k] for the two components j = 2 jb, 2 jb + 1 of block
// jb and every k (16 values), S2[i][j] for those j (2), the level-2 rows S2[j][.] (16) and all of S1 (8).
// A flow mixes each axis within its 2x2 blocks: along k and j the partner is in the lane, along i it is
// in lane ^ 4 (one shuffle per value). Local terms are built per interval by the whole warp in shared
// memory from the letters: V[p][r][k] = sum_s c3_prs b_s[k], T[p][j][k] = sum_r b_r[j] V[p][r][k],
// s3[i][j][k] = sum_p b_p[i] T[p][j][k].
//
// Flows are carried as complements D = I - M (block 2x2): S <- S - D S along each axis keeps the
// rounding relative to D, as in the diagonal engine. Chunks publish their aggregates and look back over
// their predecessors (decoupled look-back with bounded waits), then re-run from the carry to emit the
// prefix rows. The backward (reverse adjoint scan) is in the second half of this file.
#include <algorithm>
#include <cstdio>

#include "ews_common.cuh"

namespace ews {
namespace blk {

constexpr int NB = 8;        // padded state dimension: 4 blocks of 2
constexpr int KQ = 9;        // coefficient slots: series order <= 8
constexpr int kWarps = 4;    // warps per CTA, each an independent tile worker
constexpr int SLOT = 16 + 8 + 64 + 512;  // chunk element: D blocks | S1 | S2 | S3
constexpr int L3ROW = 68;                 // stride of the s3 rows (index i) in a local element: bank spread
constexpr int LROW = 88 + 8 * L3ROW;       // an interval's local element D | s1 | s2 | s3, 16-byte rows
constexpr int NPAIR = KQ * (KQ + 1) / 2;  // (p, r) with p + r <= 8

struct Geom {
    int B, T, d_in, N, Lc, C, W, readout, depth;
    unsigned flags;
    int spin_limit, q, ntiles;
    int lift_n;
    int RS;  // stride of a recomputed state row (padded layout, 16-byte multiple)
    // per-warp shared memory (floats)
    int f_dys, f_dts, f_loc, f_stage, f_per_warp;  // f_loc: two staged local rows in the forward
    int b_dys, b_dts, b_dtg, b_dyg, b_loc, b_adj, b_gst, b_sst, b_gst2, b_sst2, b_per_warp;
};

struct Params {
    Geom g;
    const void* path;
    const float* clock;   // (B, T+1) knots
    const float* blocks;  // (4, 2, 2) generator blocks A_k (zero beyond N)
    const float* lift;    // (N, d_in) or null
    float* out;
    DeviceStatus* st;
    int* flags;
    float* agg;
    float* incl;
    float* carry;
    // backward
    const float* grad_out;
    float* grad_dx;
    float* grad_dtheta;
    float* partials;       // per tile: dA blocks (16) | dlift (8 x d_in)
    const float* fagg;     // the forward aggregates
    const float* fcarry;   // the forward's chunk carries (terminal backward: the recomputed chunks' starts)
    float* scratch;        // terminal backward: per warp worker, the chunk's recomputed states (Lc rows of RS)
    float* loc;            // (B, T, LROW): every interval's local element, written by local_kernel
    float c1[KQ];             // c1_p = 1 / (p + 1)
    float c2[KQ * KQ];        // c2_pr = 1 / ((p + r + 2)(r + 1))
    float c3[KQ * KQ * KQ];   // c3_prs = 1 / ((p + r + s + 3)(r + s + 2)(s + 1))
};

__host__ __device__ constexpr int align4(int n) { return (n + 3) & ~3; }

// ------------------------------------------------------------------------------ 2x2 block flows

// Complement D = I - expm(X) of a 2x2 block X, accurate when X is small: with tau = tr X / 2,
// E = X - tau I and d2 = -det E, expm(X) = e^tau (c I + s E), c = cosh sqrt(d2), s = sinh sqrt(d2) / sqrt(d2),
// so D = (-expm1(tau) - e^tau (c - 1)) I - e^tau s E.
__device__ __forceinline__ void block_complement(float x00, float x01, float x10, float x11, float D[4]) {
    const float tau = 0.5f * (x00 + x11);
    const float e00 = x00 - tau, e11 = x11 - tau;
    const float d2 = e00 * e00 + x01 * x10;
    float cm1, s;
    if (fabsf(d2) < 0.25f) {
        // c - 1 = sum_{n>=1} d2^n / (2n)!, s = sum_{n>=0} d2^n / (2n+1)!
        cm1 = d2 * (1.f / 2 + d2 * (1.f / 24 + d2 * (1.f / 720 + d2 * (1.f / 40320 + d2 * (1.f / 3628800)))));
        s = 1.f + d2 * (1.f / 6 + d2 * (1.f / 120 + d2 * (1.f / 5040 + d2 * (1.f / 362880 + d2 * (1.f / 39916800)))));
    } else if (d2 > 0.f) {
        const float d = sqrtf(d2);
        const float sh = sinhf(0.5f * d);
        cm1 = 2.f * sh * sh;
        s = sinhf(d) / d;
    } else {
        const float w = sqrtf(-d2);
        const float sn = sinf(0.5f * w);
        cm1 = -2.f * sn * sn;
        s = sinf(w) / w;
    }
    const float et = expf(tau);
    const float diag = -expm1f(tau) - et * cm1;
    const float es = et * s;
    D[0] = diag - es * e00;
    D[1] = -es * x01;
    D[2] = -es * x10;
    D[3] = diag - es * e11;
}

// v <- (I - D) v on one 2-block (v0, v1).
__device__ __forceinline__ void flow2(const float* D, float& v0, float& v1) {
    const float a = v0, b = v1;
    v0 = a - fmaf(D[0], a, D[1] * b);
    v1 = b - fmaf(D[2], a, D[3] * b);
}

// Complement of a product of commuting flows: 1 - (1 - A)(1 - B) = A + B - A B (2x2 blocks).
__device__ __forceinline__ void comp_mul2(const float* A, const float* Bm, float* out) {
    float o[4];
    o[0] = A[0] + Bm[0] - fmaf(A[0], Bm[0], A[1] * Bm[2]);
    o[1] = A[1] + Bm[1] - fmaf(A[0], Bm[1], A[1] * Bm[3]);
    o[2] = A[2] + Bm[2] - fmaf(A[2], Bm[0], A[3] * Bm[2]);
    o[3] = A[3] + Bm[3] - fmaf(A[2], Bm[1], A[3] * Bm[3]);
    out[0] = o[0];
    out[1] = o[1];
    out[2] = o[2];
    out[3] = o[3];
}

// Register-array reads at a lane-dependent index, as unrolled selects (dynamic indexing would move the
// array to local memory).
__device__ __forceinline__ float pick8(const float* v, int idx) {
    float r = v[0];
#pragma unroll
    for (int k = 1; k < 8; ++k) r = idx == k ? v[k] : r;
    return r;
}

__device__ __forceinline__ void pick_block(const float* D, int blk, float out[4]) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        float v = D[e];
#pragma unroll
        for (int b2 = 1; b2 < 4; ++b2) v = blk == b2 ? D[4 * b2 + e] : v;
        out[e] = v;
    }
}

// ------------------------------------------------------------------------------ lane elements

// A Chen group element as lane (i, jb) holds it.
struct E3 {
    float D[16];      // flow complement, block b at D[4b..4b+3] (row-major 2x2)
    float S1[8];      // all of level 1
    float S2a[2];     // S2[i][2jb + r]
    float S2b[2][8];  // S2[2jb + r][k]
    float S3[2][8];   // S3[i][2jb + r][k]
    __device__ void identity() {
#pragma unroll
        for (int e = 0; e < 16; ++e) D[e] = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            S1[k] = 0.f;
            S2b[0][k] = S2b[1][k] = 0.f;
            S3[0][k] = S3[1][k] = 0.f;
        }
        S2a[0] = S2a[1] = 0.f;
    }
};

// Right factor of a Chen product as a lane reads it: R's S1 (all), S2[i][j], S2[j][.], S3[i][j][.] and its
// flow complement. The local terms of an interval and stored chunk elements both take this form.
struct RView {
    const float* D;    // 16
    const float* S1;   // 8
    float S2a[2];
    float S2b[2][8];
    float S3[2][8];
};

// Applies the flow complement Dm (all four blocks) to every axis of L's pieces, in place.
__device__ __forceinline__ void flow_all(const float* Dm, E3& L, int i, int jb) {
    float Dj[4], Di[4];
    pick_block(Dm, jb, Dj);
    pick_block(Dm, i >> 1, Di);
    // level 1 (all components)
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) flow2(Dm + 4 * blk, L.S1[2 * blk], L.S1[2 * blk + 1]);
    // S2[j][.]: rows j = 2jb + r (block jb), columns k
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) flow2(Dm + 4 * blk, L.S2b[r][2 * blk], L.S2b[r][2 * blk + 1]);
#pragma unroll
    for (int k = 0; k < 8; ++k) flow2(Dj, L.S2b[0][k], L.S2b[1][k]);
    // S2[i][j]: along j within the lane, along i with lane ^ 4
    flow2(Dj, L.S2a[0], L.S2a[1]);
    const bool lo = (i & 1) == 0;
    {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float mine = L.S2a[r];
            const float other = __shfl_xor_sync(kFull, mine, 4);
            // row i of (I - D_i) applied to (v_{i&~1}, v_{i|1})
            L.S2a[r] = lo ? mine - fmaf(Di[0], mine, Di[1] * other) : mine - fmaf(Di[2], other, Di[3] * mine);
        }
    }
    // S3[i][j][k]: along k, along j (lane-local), along i (lane ^ 4)
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) flow2(Dm + 4 * blk, L.S3[r][2 * blk], L.S3[r][2 * blk + 1]);
#pragma unroll
    for (int k = 0; k < 8; ++k) flow2(Dj, L.S3[0][k], L.S3[1][k]);
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float mine = L.S3[r][k];
            const float other = __shfl_xor_sync(kFull, mine, 4);
            L.S3[r][k] = lo ? mine - fmaf(Di[0], mine, Di[1] * other) : mine - fmaf(Di[2], other, Di[3] * mine);
        }
}

// L <- L (x) R: L flowed by R's flow, then the truncated tensor product (ews/core/chen_scan.py:124-152).
__device__ __forceinline__ void chen_mul_r(E3& L, const float* RD, const float* R1, const float R2a[2],
                                           const float R2b[2][8], const float R3[2][8], int i, int jb) {
    flow_all(RD, L, i, jb);
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) comp_mul2(L.D + 4 * blk, RD + 4 * blk, L.D + 4 * blk);
    const float F1i = pick8(L.S1, i);
    const float F1j[2] = {pick8(L.S1, 2 * jb), pick8(L.S1, 2 * jb + 1)};
    const float R1j[2] = {pick8(R1, 2 * jb), pick8(R1, 2 * jb + 1)};
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const float f2a = L.S2a[r];
#pragma unroll
        for (int k = 0; k < 8; ++k)
            L.S3[r][k] = fmaf(f2a, R1[k], fmaf(F1i, R2b[r][k], L.S3[r][k] + R3[r][k]));
        L.S2a[r] = fmaf(F1i, R1j[r], f2a + R2a[r]);
#pragma unroll
        for (int k = 0; k < 8; ++k) L.S2b[r][k] = fmaf(F1j[r], R1[k], L.S2b[r][k] + R2b[r][k]);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) L.S1[k] += R1[k];
}

__device__ __forceinline__ void chen_mul(E3& L, const E3& R, int i, int jb) {
    chen_mul_r(L, R.D, R.S1, R.S2a, R.S2b, R.S3, i, jb);
}

// Slot layout (floats): D (16) | S1 (8) | S2 (64, row-major) | S3 (512, row-major).
__device__ __forceinline__ void store_e3(float* slot, const E3& e, int i, int jb) {
    const int lane = threadIdx.x & 31;
    if (lane == 0) {
#pragma unroll
        for (int q = 0; q < 16; ++q) slot[q] = e.D[q];
#pragma unroll
        for (int k = 0; k < 8; ++k) slot[16 + k] = e.S1[k];
    }
    if (i == 0) {  // the S2 rows of block jb
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int k = 0; k < 8; ++k) slot[24 + (2 * jb + r) * 8 + k] = e.S2b[r][k];
    }
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 8; ++k) slot[88 + i * 64 + (2 * jb + r) * 8 + k] = e.S3[r][k];
}

__device__ __forceinline__ void load_e3(const float* slot, E3& e, int i, int jb) {
#pragma unroll
    for (int q = 0; q < 16; ++q) e.D[q] = ldcg(slot + q);
#pragma unroll
    for (int k = 0; k < 8; ++k) e.S1[k] = ldcg(slot + 16 + k);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        e.S2a[r] = ldcg(slot + 24 + i * 8 + 2 * jb + r);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            e.S2b[r][k] = ldcg(slot + 24 + (2 * jb + r) * 8 + k);
            e.S3[r][k] = ldcg(slot + 88 + i * 64 + (2 * jb + r) * 8 + k);
        }
    }
}

// ------------------------------------------------------------------------------ local terms

// Per-warp shared scratch of one interval's local terms.
struct Loc {
    float* b;    // letters b[p][a], KQ x 8
    float* s1;   // 8
    float* s2;   // 64
    float* V;    // V[pair(p, r)][k], NPAIR x 8
    float* T;    // T[p][j][k], KQ x 64
    float* D;    // 16: flow complement of the interval
    static constexpr int floats = KQ * 8 + 8 + 64 + NPAIR * 8 + KQ * 64 + 16;
    __device__ Loc(float* base) {
        b = base;
        s1 = b + KQ * 8;
        s2 = s1 + 8;
        V = s2 + 64;
        T = V + NPAIR * 8;
        D = T + KQ * 64;
    }
};

// Builds the interval's local terms in lc (whole warp): dy (8, in shared memory), clock step h, blocks A.
// QT >= 0 fixes the series order at compile time (the loops unroll and the coefficients are read at fixed
// offsets); QT = -1 reads it from the parameters.
template <int QT = -1>
__device__ void build_local(const Params& p, const float* Ablk, const float* dy, float h, const Loc& lc,
                            bool level3 = true) {
    const int lane = threadIdx.x & 31;
    const int q = QT >= 0 ? QT : p.g.q;
    // flow complement of the interval, one block per lane 0..3
    if (lane < 4) {
        const float* A = Ablk + 4 * lane;
        float Dk[4];
        block_complement(-h * A[0], -h * A[1], -h * A[2], -h * A[3], Dk);
#pragma unroll
        for (int e = 0; e < 4; ++e) lc.D[4 * lane + e] = Dk[e];
    }
    // letters: lane a < 8 runs b_p[a] = (X b_{p-1})[a] / p with its block partner a ^ 1
    {
        const int a = lane & 7;
        const float* A = Ablk + 4 * (a >> 1);
        const float xs = -h;
        const float xa = (a & 1) ? A[3] : A[0];   // X[a][a] / -h
        const float xo = (a & 1) ? A[2] : A[1];   // X[a][a^1] / -h
        float v = dy[a];
        if (lane < 8) lc.b[a] = v;
        for (int pp = 1; pp <= q; ++pp) {
            const float o = __shfl_xor_sync(kFull, v, 1);
            v = (xs / (float)pp) * fmaf(xa, v, xo * o);
            if (lane < 8) lc.b[pp * 8 + a] = v;
        }
        if (lane < 8) {
            for (int pp = q + 1; pp < KQ; ++pp) lc.b[pp * 8 + a] = 0.f;
        }
    }
    __syncwarp();
    // s1 (lanes 0..7) and s2 (two entries per lane)
    if (lane < 8) {
        float acc = 0.f;
        for (int pp = q; pp >= 0; --pp) acc = fmaf(p.c1[pp], lc.b[pp * 8 + lane], acc);
        lc.s1[lane] = acc;
    }
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        const int e = lane + 32 * h2, j = e >> 3, k = e & 7;
        float acc = 0.f;
        for (int pp = 0; pp <= q; ++pp) {
            float w = 0.f;
            for (int r = q - pp; r >= 0; --r) w = fmaf(p.c2[pp * KQ + r], lc.b[r * 8 + k], w);
            acc = fmaf(lc.b[pp * 8 + j], w, acc);
        }
        lc.s2[e] = acc;
    }
    if (!level3) {
        __syncwarp();
        return;
    }
    // V[pair(p, r)][k] = sum_s c3_prs b_s[k]
    const int npair = (q + 1) * (q + 2) / 2;
    for (int e = lane; e < npair * 8; e += 32) {
        const int pr = e >> 3, k = e & 7;
        // decode pair index pr -> (pp, r) for order q
        int pp = 0, base = 0;
        while (base + (q + 1 - pp) <= pr) {
            base += q + 1 - pp;
            ++pp;
        }
        const int r = pr - base;
        float acc = 0.f;
        for (int s = q - pp - r; s >= 0; --s) acc = fmaf(p.c3[(pp * KQ + r) * KQ + s], lc.b[s * 8 + k], acc);
        lc.V[e] = acc;
    }
    __syncwarp();
    // T[p][j][k] = sum_{r <= q-p} b_r[j] V[pair(p, r)][k]
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        const int e = lane + 32 * h2, j = e >> 3, k = e & 7;
        int base = 0;
        for (int pp = 0; pp <= q; ++pp) {
            float acc = 0.f;
            for (int r = 0; r <= q - pp; ++r) acc = fmaf(lc.b[r * 8 + j], lc.V[(base + r) * 8 + k], acc);
            lc.T[pp * 64 + e] = acc;
            base += q + 1 - pp;
        }
    }
    __syncwarp();
}

// The lane's view of the local element of the interval in lc.
template <int QT = -1>
__device__ __forceinline__ void local_view(const Params& p, const Loc& lc, int i, int jb, float s2a[2],
                                           float s2b[2][8], float s3[2][8]) {
    const int q = QT >= 0 ? QT : p.g.q;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int j = 2 * jb + r;
        s2a[r] = lc.s2[i * 8 + j];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            s2b[r][k] = lc.s2[j * 8 + k];
            s3[r][k] = 0.f;
        }
    }
    for (int pp = q; pp >= 0; --pp) {
        const float bi = lc.b[pp * 8 + i];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float4* Tr = reinterpret_cast<const float4*>(lc.T + pp * 64 + (2 * jb + r) * 8);
            const float4 t0 = Tr[0], t1 = Tr[1];
            s3[r][0] = fmaf(bi, t0.x, s3[r][0]);
            s3[r][1] = fmaf(bi, t0.y, s3[r][1]);
            s3[r][2] = fmaf(bi, t0.z, s3[r][2]);
            s3[r][3] = fmaf(bi, t0.w, s3[r][3]);
            s3[r][4] = fmaf(bi, t1.x, s3[r][4]);
            s3[r][5] = fmaf(bi, t1.y, s3[r][5]);
            s3[r][6] = fmaf(bi, t1.z, s3[r][6]);
            s3[r][7] = fmaf(bi, t1.w, s3[r][7]);
        }
    }
}

// One interval: S <- S (x) local.
__device__ __forceinline__ void chen_step(const Params& p, const Loc& lc, E3& S, int i, int jb) {
    float s2a[2], s2b[2][8], s3[2][8];
    local_view(p, lc, i, jb, s2a, s2b, s3);
    chen_mul_r(S, lc.D, lc.s1, s2a, s2b, s3, i, jb);
}

// Rows staged in shared memory (the backward's state and gradient rows, the forward's prefix rows) keep
// levels 0-2 as in the row and put the level-3 rows (index i) N^2 + 4 floats apart: the lanes' accesses
// to one staged row then fall on different banks (at a stride of N^2 = 64, sixteen lanes shared a bank).
__host__ __device__ inline int row_floats_padded(int N) { return 1 + N + N * N + N * (N * N + 4); }

// Position of row element e in the padded layout; inv = ceil(2^16 / N^2) turns the division by N^2 into a
// multiply and shift, exact for the at most 512 level-3 entries.
__device__ __forceinline__ int pad_index(int e, int off3, unsigned inv) {
    return e < off3 ? e : e + 4 * (int)(((unsigned)(e - off3) * inv) >> 16);
}

// warp_load_span of one state row (real dimension N) into the padded layout (whole warp).
__device__ void warp_load_row_padded(float* __restrict__ s, const float* __restrict__ g, int N) {
    const int lane = threadIdx.x & 31;
    const int N2 = N * N, off3 = 1 + N + N2, n = off3 + N * N2;
    const unsigned inv = (65536u + N2 - 1) / N2;
    int head = (int)(((16u - ((uintptr_t)g & 15u)) & 15u) >> 2);
    if (head > n) head = n;
    if (lane < head) s[pad_index(lane, off3, inv)] = __ldcg(g + lane);
    const int nvec = (n - head) >> 2;
    const float4* gv = reinterpret_cast<const float4*>(g + head);
    for (int v = lane; v < nvec; v += 32) {
        const float4 q = __ldcg(gv + v);
        const int e = head + 4 * v;
        s[pad_index(e, off3, inv)] = q.x;
        s[pad_index(e + 1, off3, inv)] = q.y;
        s[pad_index(e + 2, off3, inv)] = q.z;
        s[pad_index(e + 3, off3, inv)] = q.w;
    }
    const int done = head + 4 * nvec;
    if (lane < n - done) s[pad_index(done + lane, off3, inv)] = __ldcg(g + done + lane);
}

// The same copy with cp.async (4-byte copies into the padded positions; the caller commits and waits).
__device__ void warp_copy_row_padded_async(float* __restrict__ s, const float* __restrict__ g, int N) {
    const int lane = threadIdx.x & 31;
    const int N2 = N * N, off3 = 1 + N + N2, n = off3 + N * N2;
    const unsigned inv = (65536u + N2 - 1) / N2;
    for (int e = lane; e < n; e += 32) cp_async4(s + pad_index(e, off3, inv), g + e);
}

// Stores a staged prefix row (padded layout) to global memory: s is placed at g's 16-byte phase (s + k is
// 16-byte aligned where g + k is), so every float4 of the row that does not straddle two level-3 rows is
// one aligned shared load; the straddling ones and the ragged ends go element by element.
__device__ void warp_store_row_padded(float* __restrict__ g, const float* __restrict__ s, int N) {
    const int lane = threadIdx.x & 31;
    const int N2 = N * N, off3 = 1 + N + N2, n = off3 + N * N2;
    const unsigned inv = (65536u + N2 - 1) / N2;
    int head = (int)(((16u - ((uintptr_t)g & 15u)) & 15u) >> 2);
    if (head > n) head = n;
    if (lane < head) g[lane] = s[pad_index(lane, off3, inv)];
    const int nvec = (n - head) >> 2;
    float4* gv = reinterpret_cast<float4*>(g + head);
    for (int v = lane; v < nvec; v += 32) {
        const int e = head + 4 * v;
        const int p0 = pad_index(e, off3, inv), p3 = pad_index(e + 3, off3, inv);
        float4 q;
        if (p3 == p0 + 3) {
            q = *reinterpret_cast<const float4*>(s + p0);
        } else {
            q.x = s[p0];
            q.y = s[pad_index(e + 1, off3, inv)];
            q.z = s[pad_index(e + 2, off3, inv)];
            q.w = s[p3];
        }
        gv[v] = q;
    }
    const int done = head + 4 * nvec;
    if (lane < n - done) g[done + lane] = s[pad_index(done + lane, off3, inv)];
}

// The shared-memory position at which a row bound for global address g is staged (16-byte phase of g).
__device__ __forceinline__ float* phase_matched(float* stage, const float* g) {
    return stage + (((uintptr_t)g & 15u) >> 2);
}

// Prefix row [1, S1, S2, S3] of a lane element into a staged row (real dimension N, padded layout).
__device__ __forceinline__ void stage_row(float* row, const E3& S, int N, int i, int jb) {
    const int lane = threadIdx.x & 31;
    const int N2 = N * N;
    if (lane == 0) {
        row[0] = 1.f;
#pragma unroll
        for (int k = 0; k < 8; ++k)
            if (k < N) row[1 + k] = S.S1[k];
    }
    if (i == 0) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int j = 2 * jb + r;
            if (j < N)
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (k < N) row[1 + N + j * N + k] = S.S2b[r][k];
        }
    }
    if (i < N) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int j = 2 * jb + r;
            if (j < N)
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (k < N) row[1 + N + N2 + i * (N2 + 4) + j * N + k] = S.S3[r][k];
        }
    }
}

// Increments (dx -> dy = lift dx, padded to 8) and clock steps of intervals [t0, t0 + n).
__device__ void load_chunk(const Params& p, const float* liftS, float* dxs, float* dys, float* dts, int b, int t0,
                           int n) {
    const Geom& g = p.g;
    const int lane = threadIdx.x & 31;
    for (int e = lane; e < n * g.d_in; e += 32) {
        const int k = e / g.d_in, cc = e - k * g.d_in;
        dxs[e] = input_increment(p.path, b, t0 + k, cc, g.T, g.d_in, g.flags);
    }
    const float* ck = p.clock + (size_t)b * (g.T + 1) + t0;
    for (int k = lane; k < n; k += 32) dts[k] = ck[k + 1] - ck[k];  // the reference's clock[1:] - clock[:-1]
    __syncwarp();
    for (int e = lane; e < n * NB; e += 32) {
        const int k = e >> 3, a = e & 7;
        float v = 0.f;
        if (a < g.N) {
            if (p.lift) {
                // lift stored channel-major (liftS[cc * NB + a]): consecutive lanes, consecutive banks
                const float* xr = dxs + k * g.d_in;
                for (int cc = 0; cc < g.d_in; ++cc) v = fmaf(liftS[cc * NB + a], xr[cc], v);
            } else {
                v = dxs[k * g.d_in + a];
            }
        }
        dys[e] = v;
    }
    __syncwarp();
}

// ------------------------------------------------------------------------------ forward kernel

// The local element of every interval, a parallel map ahead of the chains: one warp per chunk of one
// sample builds each interval's flow complement, letters and series terms (build_local, as the chain did)
// and writes [D | s1 | s2 | s3] (s3[i][j][k] at 88 + L3ROW i + 8 j + k) to p.loc.
template <int QT>
__global__ void __launch_bounds__(kWarps * 32) local_kernel(Params p) {
    extern __shared__ float smem[];
    const Geom& g = p.g;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = lane >> 2, jb = lane & 3;
    float* liftS = smem;
    float* Ablk = smem + g.lift_n;
    for (int e = threadIdx.x; e < NB * g.d_in; e += blockDim.x) {
        const int r = e / g.d_in, cc = e - r * g.d_in;
        liftS[cc * NB + r] = (p.lift && r < g.N) ? p.lift[r * g.d_in + cc] : 0.f;
    }
    for (int e = threadIdx.x; e < 16; e += blockDim.x) Ablk[e] = (e >> 2) < g.N / 2 ? p.blocks[e] : 0.f;
    __syncthreads();
    float* dxs = smem + g.lift_n + 16 + warp * g.f_per_warp;
    float* dys = dxs + g.f_dys;
    float* dts = dxs + g.f_dts;
    const Loc lc(dxs + g.f_loc);  // the forward's two staged rows hold one Loc
    const int job = blockIdx.x * kWarps + warp;
    if (job >= g.B * g.C) return;
    const int b = job / g.C, t0 = (job - b * g.C) * g.Lc;
    const int n = min(g.Lc, g.T - t0);
    load_chunk(p, liftS, dxs, dys, dts, b, t0, n);
    for (int k = 0; k < n; ++k) {
        build_local<QT>(p, Ablk, dys + k * NB, dts[k], lc);
        float s2a[2], s2b[2][8], s3[2][8];
        local_view<QT>(p, lc, i, jb, s2a, s2b, s3);
        float* row = p.loc + ((size_t)b * g.T + t0 + k) * LROW;
        if (lane < 16) row[lane] = lc.D[lane];
        if (lane < 8) row[16 + lane] = lc.s1[lane];
        row[24 + lane] = lc.s2[lane];
        row[56 + lane] = lc.s2[32 + lane];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float* d3 = row + 88 + L3ROW * i + 8 * (2 * jb + r);
            *reinterpret_cast<float4*>(d3) = make_float4(s3[r][0], s3[r][1], s3[r][2], s3[r][3]);
            *reinterpret_cast<float4*>(d3 + 4) = make_float4(s3[r][4], s3[r][5], s3[r][6], s3[r][7]);
        }
        __syncwarp();
    }
}

// Copies interval t's local element (LROW floats) into dst (one cp.async group).
__device__ __forceinline__ void fetch_local(const Params& p, int b, int t, float* dst) {
    const float* src = p.loc + ((size_t)b * p.g.T + t) * LROW;
    for (int v = threadIdx.x & 31; v < LROW / 4; v += 32) cp_async16(dst + 4 * v, src + 4 * v);
    cp_async_commit();
}

// One interval from a staged local element: S <- S (x) local.
__device__ __forceinline__ void chen_step_row(const float* row, E3& S, int i, int jb) {
    float s2a[2], s2b[2][8], s3[2][8];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int j = 2 * jb + r;
        s2a[r] = row[24 + 8 * i + j];
        const float4* b2 = reinterpret_cast<const float4*>(row + 24 + 8 * j);
        const float4* b3 = reinterpret_cast<const float4*>(row + 88 + L3ROW * i + 8 * j);
        const float4 u0 = b2[0], u1 = b2[1], w0 = b3[0], w1 = b3[1];
        s2b[r][0] = u0.x; s2b[r][1] = u0.y; s2b[r][2] = u0.z; s2b[r][3] = u0.w;
        s2b[r][4] = u1.x; s2b[r][5] = u1.y; s2b[r][6] = u1.z; s2b[r][7] = u1.w;
        s3[r][0] = w0.x; s3[r][1] = w0.y; s3[r][2] = w0.z; s3[r][3] = w0.w;
        s3[r][4] = w1.x; s3[r][5] = w1.y; s3[r][6] = w1.z; s3[r][7] = w1.w;
    }
    chen_mul_r(S, row, row + 16, s2a, s2b, s3, i, jb);
}

__global__ void __launch_bounds__(kWarps * 32) fwd_kernel(Params p) {
    extern __shared__ float smem[];
    const Geom& g = p.g;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = lane >> 2, jb = lane & 3;
    float* liftS = smem;
    float* Ablk = smem + g.lift_n;  // 16
    for (int e = threadIdx.x; e < NB * g.d_in; e += blockDim.x) {
        const int r = e / g.d_in, cc = e - r * g.d_in;
        liftS[cc * NB + r] = (p.lift && r < g.N) ? p.lift[r * g.d_in + cc] : 0.f;
    }
    for (int e = threadIdx.x; e < 16; e += blockDim.x) Ablk[e] = (e >> 2) < g.N / 2 ? p.blocks[e] : 0.f;
    __syncthreads();
    float* dxs = smem + g.lift_n + 16 + warp * g.f_per_warp;
    float* lrow = dxs + g.f_loc;  // two staged local elements
    float* stage = dxs + g.f_stage;

    for (;;) {
        const int tile = next_ticket(p.st);
        if (tile >= g.ntiles) break;
        const int c = tile / g.B, b = tile - c * g.B;
        const int t0 = c * g.Lc;
        const int len = min(g.Lc, g.T - t0);

        // pass 1: the chunk's aggregate from the identity, kept in the workspace (agg, and incl for chunk 0)
        const size_t slot = ((size_t)b * g.C + c) * SLOT;
        int* flag = p.flags + (size_t)b * g.C + c;
        {
            E3 A;
            A.identity();
            fetch_local(p, b, t0, lrow);
            for (int k = 0; k < len; ++k) {
                cp_async_wait<0>();
                __syncwarp();
                if (k + 1 < len) fetch_local(p, b, t0 + k + 1, lrow + ((k + 1) & 1) * LROW);
                chen_step_row(lrow + (k & 1) * LROW, A, i, jb);
                __syncwarp();
            }
            store_e3(p.agg + slot, A, i, jb);
            if (c == 0) store_e3(p.incl + slot, A, i, jb);
        }
        __syncwarp();
        E3 excl;
        excl.identity();
        if (c == 0) {
            if (!(g.flags & EWS_F_TEST_WITHHOLD)) publish(flag, kFlagIncl);
        } else {
            publish(flag, kFlagAgg);
            // look back: excl = incl_j (x) agg_{j+1} (x) ... (x) agg_{c-1}
            E3 acc;
            acc.identity();
            int j = c - 1;
            const int want = (g.flags & EWS_F_DETERMINISTIC) ? kFlagIncl : kFlagAgg;
            for (;;) {
                const int f = wait_slot(p.flags + (size_t)b * g.C + j, p.st, g.spin_limit, tile, want);
                if (f < 0) return;  // timeout or another tile failed: the error word is set
                E3 X;
                const size_t sj = ((size_t)b * g.C + j) * SLOT;
                load_e3((f == kFlagIncl ? p.incl : p.agg) + sj, X, i, jb);
                chen_mul(X, acc, i, jb);
                acc = X;
                if (f == kFlagIncl) break;
                --j;
            }
            excl = acc;
            E3 inc = excl;
            {
                E3 A;
                load_e3(p.agg + slot, A, i, jb);
                chen_mul(inc, A, i, jb);
            }
            __syncwarp();
            store_e3(p.incl + slot, inc, i, jb);
            publish(flag, kFlagIncl);
        }
        store_e3(p.carry + slot, excl, i, jb);

        if (g.readout == EWS_READOUT_TERMINAL) {
            if (c == g.C - 1) {
                E3 fin = excl;
                {
                    E3 A;
                    load_e3(p.agg + slot, A, i, jb);
                    chen_mul(fin, A, i, jb);
                }
                float* dst = p.out + (size_t)b * g.W;
                float* srow = phase_matched(stage, dst);
                stage_row(srow, fin, g.N, i, jb);
                __syncwarp();
                warp_store_row_padded(dst, srow, g.N);
                __syncwarp();
            }
            continue;
        }
        // pass 2: re-run the chunk from its carry and emit the prefix rows
        E3 S = excl;
        fetch_local(p, b, t0, lrow);
        for (int k = 0; k < len; ++k) {
            cp_async_wait<0>();
            __syncwarp();
            if (k + 1 < len) fetch_local(p, b, t0 + k + 1, lrow + ((k + 1) & 1) * LROW);
            chen_step_row(lrow + (k & 1) * LROW, S, i, jb);
            float* dst = p.out + ((size_t)b * g.T + t0 + k) * g.W;
            float* srow = phase_matched(stage, dst);
            stage_row(srow, S, g.N, i, jb);
            __syncwarp();
            warp_store_row_padded(dst, srow, g.N);
            __syncwarp();
        }
    }
}


// ------------------------------------------------------------------------------ backward
//
// Adjoint of one interval S' = S (x) R (R = the local element: flow M = I - D, s1, s2, s3), with
// F1 = M S1, F2 = (M (x) M) S2, F3 = (M (x) M (x) M) S3 and l' the cotangent of S':
//   dF2 = l2' + l3' . s1,   dF1 = l1' + l2' . s1 + l3' : s2
//   ds1 = l1' + F1 . l2' + F2 : l3',   ds2 = l2' + F1 . l3',   ds3 = l3'
//   l3 = (M^T)^(x)3 l3',  l2 = (M^T)^(x)2 dF2,  l1 = M^T dF1
// and dM collects, per tensor axis, the cotangent against S flowed on the other axes. The flow's
// gradient goes to X = -h A through the adjoint of the exponential's Frechet derivative (closed form on
// 2x2 blocks); the local terms' gradient goes back through the letters b_p = (X / p) b_{p-1}.

// v <- (I - D)^T v on one 2-block.
__device__ __forceinline__ void flow2T(const float* D, float& v0, float& v1) {
    const float a = v0, b = v1;
    v0 = a - fmaf(D[0], a, D[2] * b);
    v1 = b - fmaf(D[1], a, D[3] * b);
}

// Transposed flow along the i axis (partner in lane ^ 4).
__device__ __forceinline__ float flowT_i(const float* Di, float mine, bool lo) {
    const float other = __shfl_xor_sync(kFull, mine, 4);
    return lo ? mine - fmaf(Di[0], mine, Di[2] * other) : mine - fmaf(Di[1], other, Di[3] * mine);
}

// Flow along the i axis with both rows at hand (v_i, v_{i^1}).
__device__ __forceinline__ float flow_i2(const float* Di, float mine, float other, bool lo) {
    return lo ? mine - fmaf(Di[0], mine, Di[1] * other) : mine - fmaf(Di[2], other, Di[3] * mine);
}

// Adjoint lane element: cotangents of S1 (all), S2[i][j] (j in block jb) and S3[i][j][.].
struct A3 {
    float L1[8];
    float L2a[2];
    float L3[2][8];
    __device__ void zero() {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            L1[k] = 0.f;
            L3[0][k] = L3[1][k] = 0.f;
        }
        L2a[0] = L2a[1] = 0.f;
    }
    __device__ void add(const A3& o) {
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            L1[k] += o.L1[k];
            L3[0][k] += o.L3[0][k];
            L3[1][k] += o.L3[1][k];
        }
        L2a[0] += o.L2a[0];
        L2a[1] += o.L2a[1];
    }
};

// Adjoint slot layout (floats): L1 (8) | L2 (64, row-major) | L3 (512, row-major); SLOT-sized.
__device__ __forceinline__ void store_a3(float* slot, const A3& a, int i, int jb) {
    if ((threadIdx.x & 31) == 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k) slot[k] = a.L1[k];
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        slot[8 + i * 8 + 2 * jb + r] = a.L2a[r];
#pragma unroll
        for (int k = 0; k < 8; ++k) slot[72 + i * 64 + (2 * jb + r) * 8 + k] = a.L3[r][k];
    }
}

__device__ __forceinline__ void load_a3(const float* slot, A3& a, int i, int jb) {
#pragma unroll
    for (int k = 0; k < 8; ++k) a.L1[k] = ldcg(slot + k);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        a.L2a[r] = ldcg(slot + 8 + i * 8 + 2 * jb + r);
#pragma unroll
        for (int k = 0; k < 8; ++k) a.L3[r][k] = ldcg(slot + 72 + i * 64 + (2 * jb + r) * 8 + k);
    }
}

// lambda <- J(R)^T lambda for right-multiplication by R = (flow complement D, U1, U2 rows 2jb, 2jb+1).
__device__ __forceinline__ void apply_JT(A3& a, const float* D, const float* U1, const float U2b[2][8], int i,
                                         int jb) {
    float Dj[4], Di[4];
    pick_block(D, jb, Dj);
    pick_block(D, i >> 1, Di);
    const bool lo = (i & 1) == 0;
    const float U1j[2] = {pick8(U1, 2 * jb), pick8(U1, 2 * jb + 1)};
    float dF2[2];
    float part = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        float acc = a.L2a[r];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            acc = fmaf(a.L3[r][k], U1[k], acc);
            part = fmaf(a.L3[r][k], U2b[r][k], part);
        }
        dF2[r] = acc;
        part = fmaf(a.L2a[r], U1j[r], part);
    }
    part += __shfl_xor_sync(kFull, part, 1);
    part += __shfl_xor_sync(kFull, part, 2);
    const float dF1i = pick8(a.L1, i) + part;
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) flow2T(D + 4 * blk, a.L3[r][2 * blk], a.L3[r][2 * blk + 1]);
#pragma unroll
    for (int k = 0; k < 8; ++k) flow2T(Dj, a.L3[0][k], a.L3[1][k]);
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 8; ++k) a.L3[r][k] = flowT_i(Di, a.L3[r][k], lo);
    flow2T(Dj, dF2[0], dF2[1]);
#pragma unroll
    for (int r = 0; r < 2; ++r) a.L2a[r] = flowT_i(Di, dF2[r], lo);
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) a.L1[ii] = __shfl_sync(kFull, dF1i, 4 * ii);
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) flow2T(D + 4 * blk, a.L1[2 * blk], a.L1[2 * blk + 1]);
}

__device__ __forceinline__ void apply_JT_e3(A3& a, const E3& G, int i, int jb) {
    apply_JT(a, G.D, G.S1, G.S2b, i, jb);
}

// Adds gradient row t (real dimension N, padded layout) to the lane's cotangent.
__device__ __forceinline__ void add_grad_row(A3& a, const float* row, int N, int i, int jb) {
    const int N2 = N * N;
#pragma unroll
    for (int k = 0; k < 8; ++k)
        if (k < N) a.L1[k] += row[1 + k];
    if (i < N) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int j = 2 * jb + r;
            if (j < N) {
                a.L2a[r] += row[1 + N + i * N + j];
#pragma unroll
                for (int k = 0; k < 8; ++k)
                    if (k < N) a.L3[r][k] += row[1 + N + N2 + i * (N2 + 4) + j * N + k];
            }
        }
    }
}

// Entry (i, j) of level 2 / (i, j, k) of level 3 from a staged state row (padded layout), zero beyond N.
__device__ __forceinline__ float row_s1(const float* row, int N, int k) { return k < N ? row[1 + k] : 0.f; }
__device__ __forceinline__ float row_s2(const float* row, int N, int i, int j) {
    return (i < N && j < N) ? row[1 + N + i * N + j] : 0.f;
}
__device__ __forceinline__ float row_s3(const float* row, int N, int i, int j, int k) {
    return (i < N && j < N && k < N) ? row[1 + N + N * N + i * (N * N + 4) + j * N + k] : 0.f;
}

// Adjoint of expm at a 2x2 block: out = L(Y, G) with Y = X^T, the Frechet derivative of expm at Y in
// direction G. With tau = tr Y / 2, E = Y - tau I, d2 = -det E (so E^2 = d2 I) and expm(Y) = e^tau (c I + s E),
// c = cosh sqrt(d2), s = sinh sqrt(d2) / sqrt(d2): L = e^tau [g (c I + s E) + (s/2) dd I + s' dd E + s G0],
// g = tr G / 2, G0 = G - g I, dd = 2 E00 G0_00 + E01 G0_10 + E10 G0_01, s' = ds/d(d2).
__device__ __forceinline__ void expm_frechet_adjoint(const float X[4], const float G[4], float out[4]) {
    const float y00 = X[0], y01 = X[2], y10 = X[1], y11 = X[3];  // Y = X^T
    const float tau = 0.5f * (y00 + y11);
    const float e00 = y00 - tau, e11 = y11 - tau;
    const float d2 = e00 * e00 + y01 * y10;
    float c, sv, sp;
    if (fabsf(d2) < 0.25f) {
        c = 1.f + d2 * (1.f / 2 + d2 * (1.f / 24 + d2 * (1.f / 720 + d2 * (1.f / 40320 + d2 * (1.f / 3628800)))));
        sv = 1.f + d2 * (1.f / 6 + d2 * (1.f / 120 + d2 * (1.f / 5040 + d2 * (1.f / 362880 + d2 * (1.f / 39916800)))));
        // s' = sum_{n>=1} n d2^(n-1) / (2n+1)!
        sp = 1.f / 6 + d2 * (2.f / 120 + d2 * (3.f / 5040 + d2 * (4.f / 362880 + d2 * (5.f / 39916800))));
    } else if (d2 > 0.f) {
        const float d = sqrtf(d2);
        c = coshf(d);
        sv = sinhf(d) / d;
        sp = (c - sv) / (2.f * d2);
    } else {
        const float w = sqrtf(-d2);
        c = cosf(w);
        sv = sinf(w) / w;
        sp = (c - sv) / (2.f * d2);
    }
    const float g = 0.5f * (G[0] + G[3]);
    const float g00 = G[0] - g, g01 = G[1], g10 = G[2], g11 = G[3] - g;
    const float dd = 2.f * e00 * g00 + y01 * g10 + y10 * g01;
    const float et = expf(tau);
    const float di = g * c + 0.5f * sv * dd;   // coefficient of I
    const float de = g * sv + sp * dd;         // coefficient of E
    out[0] = et * (di + de * e00 + sv * g00);
    out[1] = et * (de * y01 + sv * g01);
    out[2] = et * (de * y10 + sv * g10);
    out[3] = et * (di + de * e11 + sv * g11);
}

// Per-warp shared scratch of the exact adjoint step.
struct AdjBuf {
    float* L3;    // 512: l3'
    float* L2;    // 64: l2'
    float* ds1;   // 8
    float* ds2;   // 64
    float* dT;    // KQ x 64
    float* dV;    // NPAIR x 8
    float* yz;    // 2 x KQ x 8: y_r[j] = sum_k ds2[j][k] b_r[k], z_p[k] = sum_j b_p[j] ds2[j][k]
    float* db;    // KQ x 8
    // l3' rows (index i) are L3S = 68 floats apart: the lanes' stores (rows i, columns 16 jb..) and the
    // float4 reads of a row per lane land on different banks (a 64-float stride put them all on one)
    static constexpr int L3S = 68;
    static constexpr int floats = 8 * L3S + 64 + 8 + 64 + KQ * 64 + NPAIR * 8 + 2 * KQ * 8 + KQ * 8;
    __device__ AdjBuf(float* base) {
        L3 = base;
        L2 = L3 + 8 * L3S;
        ds1 = L2 + 64;
        ds2 = ds1 + 8;
        dT = ds2 + 64;
        dV = dT + KQ * 64;
        yz = dV + NPAIR * 8;
        db = yz + 2 * KQ * 8;
    }
};

// The gradient of the interval's letters db[p][a] from ds1, ds2 (in ab) and ds3 = l3' (ab.L3), through
// the series assembly s1 = sum c1 b, s2 = sum c2 b (x) b, s3 = sum_p b_p (x) T_p (whole warp).
template <int QT = -1>
__device__ void letters_adjoint(const Params& p, const Loc& lc, const AdjBuf& ab) {
    const int lane = threadIdx.x & 31;
    const int q = QT >= 0 ? QT : p.g.q;
    const int npair = (q + 1) * (q + 2) / 2;
    // dT[p][j][k] = sum_i b_p[i] l3[i][j][k]; y, z for level 2
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
        const int e = lane + 32 * h2;
        float col[8];
#pragma unroll
        for (int ii = 0; ii < 8; ++ii) col[ii] = ab.L3[ii * AdjBuf::L3S + e];
        for (int pp = 0; pp <= q; ++pp) {
            float acc = 0.f;
#pragma unroll
            for (int ii = 0; ii < 8; ++ii) acc = fmaf(lc.b[pp * 8 + ii], col[ii], acc);
            ab.dT[pp * 64 + e] = acc;
        }
    }
    for (int e = lane; e < 2 * (q + 1) * 8; e += 32) {
        const int which = e / ((q + 1) * 8), rem = e - which * (q + 1) * 8, pp = rem >> 3, a = rem & 7;
        float acc = 0.f;
        if (which == 0) {  // y_p[a] = sum_k ds2[a][k] b_p[k]
#pragma unroll
            for (int k = 0; k < 8; ++k) acc = fmaf(ab.ds2[a * 8 + k], lc.b[pp * 8 + k], acc);
        } else {           // z_p[a] = sum_j b_p[j] ds2[j][a]
#pragma unroll
            for (int j = 0; j < 8; ++j) acc = fmaf(lc.b[pp * 8 + j], ab.ds2[j * 8 + a], acc);
        }
        ab.yz[which * KQ * 8 + pp * 8 + a] = acc;
    }
    __syncwarp();
    // dV[pair(p, r)][k] = sum_j b_r[j] dT[p][j][k]
    for (int e = lane; e < npair * 8; e += 32) {
        const int pr = e >> 3, k = e & 7;
        int pp = 0, base = 0;
        while (base + (q + 1 - pp) <= pr) {
            base += q + 1 - pp;
            ++pp;
        }
        const int r = pr - base;
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(lc.b[r * 8 + j], ab.dT[pp * 64 + j * 8 + k], acc);
        ab.dV[e] = acc;
    }
    __syncwarp();
    // db[p][a]: the three slots of level 3, both slots of level 2, level 1
    for (int o = lane; o < (q + 1) * 8; o += 32) {
        const int pp = o >> 3, a = o & 7;
        float acc = 0.f;
        // slot 1 of level 3: sum_{jk} l3[a][j][k] T[p][j][k]
        {
            const float4* Lr = reinterpret_cast<const float4*>(ab.L3 + a * AdjBuf::L3S);
            const float4* Tr = reinterpret_cast<const float4*>(lc.T + pp * 64);
#pragma unroll 4
            for (int v = 0; v < 16; ++v) {
                const float4 x = Lr[v], y = Tr[v];
                acc = fmaf(x.x, y.x, fmaf(x.y, y.y, fmaf(x.z, y.z, fmaf(x.w, y.w, acc))));
            }
        }
        // slot 2: sum_{p'} sum_k dT[p'][a][k] V[pair(p', p)][k]   (letter p in the middle)
        {
            int base = 0;
            for (int p2 = 0; p2 <= q - pp; ++p2) {
                const float* Vr = lc.V + (base + pp) * 8;
                const float* dTr = ab.dT + p2 * 64 + a * 8;
#pragma unroll
                for (int k = 0; k < 8; ++k) acc = fmaf(dTr[k], Vr[k], acc);
                base += q + 1 - p2;
            }
        }
        // slot 3: sum_{(p1, p2)} c3[p1][p2][p] dV[pair(p1, p2)][a]   (letter p last)
        {
            int base = 0;
            for (int p1 = 0; p1 <= q - pp; ++p1) {
                for (int p2 = 0; p2 <= q - pp - p1; ++p2)
                    acc = fmaf(p.c3[(p1 * KQ + p2) * KQ + pp], ab.dV[(base + p2) * 8 + a], acc);
                base += q + 1 - p1;
            }
        }
        // level 2: first slot sum_r c2[p][r] y_r[a], second slot sum_p' c2[p'][p] z_p'[a]
        for (int r = 0; r <= q - pp; ++r) acc = fmaf(p.c2[pp * KQ + r], ab.yz[r * 8 + a], acc);
        for (int p1 = 0; p1 <= q - pp; ++p1) acc = fmaf(p.c2[p1 * KQ + pp], ab.yz[KQ * 8 + p1 * 8 + a], acc);
        // level 1
        acc = fmaf(p.c1[pp], ab.ds1[a], acc);
        ab.db[o] = acc;
    }
    __syncwarp();
}

struct BwdOut {
    float dA[16];  // lane partial of dL/dA (blocks)
};

// One exact adjoint step at interval t. a holds l' (gradient row added); prow is S_{t-1} (real dims);
// lc holds the interval's local terms. Accumulates dA partials, writes dy_t (dyg, lanes 0..7) and
// dL/dh_t (lane 0 to *dtg); turns a into the cotangent of S_{t-1}.
template <int QT = -1>
__device__ void bwd_step(const Params& p, const float* Ablk, const Loc& lc, const AdjBuf& ab, const float* prow,
                         float h, A3& a, BwdOut& bo, float* dyg, float* dtg, int i, int jb) {
    const int lane = threadIdx.x & 31;
    const int N = p.g.N;
    const bool lo = (i & 1) == 0;
    const int i2 = i ^ 1;
    float Dj[4], Di[4];
    pick_block(lc.D, jb, Dj);
    pick_block(lc.D, i >> 1, Di);
    // l' to shared memory
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        ab.L2[i * 8 + 2 * jb + r] = a.L2a[r];
#pragma unroll
        for (int k = 0; k < 8; ++k) ab.L3[i * AdjBuf::L3S + (2 * jb + r) * 8 + k] = a.L3[r][k];
    }
    // F1 = M S1p (all)
    float S1p[8], F1[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) S1p[k] = F1[k] = row_s1(prow, N, k);
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) flow2(lc.D + 4 * blk, F1[2 * blk], F1[2 * blk + 1]);
    const float F1i = pick8(F1, i);
    // S2p pieces: rows i, i^1 at columns j (block jb)
    float P2[2][2];  // [row i / i^1][r]
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        P2[0][r] = row_s2(prow, N, i, 2 * jb + r);
        P2[1][r] = row_s2(prow, N, i2, 2 * jb + r);
    }
    // G1 = S2p flowed along columns (rows i, i^1); F2[i][j] = G1 flowed along rows
    float G1[2][2] = {{P2[0][0], P2[0][1]}, {P2[1][0], P2[1][1]}};
    flow2(Dj, G1[0][0], G1[0][1]);
    flow2(Dj, G1[1][0], G1[1][1]);
    float F2[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) F2[r] = flow_i2(Di, G1[0][r], G1[1][r], lo);
    // dF2, dF1
    float dF2[2];
    float part = 0.f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        float acc = a.L2a[r];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            acc = fmaf(a.L3[r][k], lc.s1[k], acc);
            part = fmaf(a.L3[r][k], lc.s2[(2 * jb + r) * 8 + k], part);
        }
        dF2[r] = acc;
        part = fmaf(a.L2a[r], lc.s1[2 * jb + r], part);
    }
    part += __shfl_xor_sync(kFull, part, 1);
    part += __shfl_xor_sync(kFull, part, 2);
    const float dF1i = pick8(a.L1, i) + part;
    float dF1[8];
#pragma unroll
    for (int ii = 0; ii < 8; ++ii) dF1[ii] = __shfl_sync(kFull, dF1i, 4 * ii);
    // ds1 = l1' + F1 . l2' + F2 : l3'  (warp reduction of lane partials)
    float P[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        P[k] = fmaf(F2[0], a.L3[0][k], F2[1] * a.L3[1][k]);
#pragma unroll
        for (int r = 0; r < 2; ++r) P[k] = (k == 2 * jb + r) ? fmaf(F1i, a.L2a[r], P[k]) : P[k];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) P[k] += __shfl_xor_sync(kFull, P[k], o);
    }
    // ds2 rows j (block jb) = l2'[j][.] + sum_i F1[i] l3'[i][j][.]
    float Q[2][8];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            float v = F1i * a.L3[r][k];
            v += __shfl_xor_sync(kFull, v, 4);
            v += __shfl_xor_sync(kFull, v, 8);
            v += __shfl_xor_sync(kFull, v, 16);
            Q[r][k] = v;
        }
    __syncwarp();
    if (lane == 0) {
#pragma unroll
        for (int k = 0; k < 8; ++k) ab.ds1[k] = a.L1[k] + P[k];
    }
    if (i == 0) {
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int k = 0; k < 8; ++k) ab.ds2[(2 * jb + r) * 8 + k] = ab.L2[(2 * jb + r) * 8 + k] + Q[r][k];
    }
    // ---- dM (block entries; lane partials): blk b entry (u, v) at dM[4b + 2u + v]
    float dM[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) dM[e] = 0.f;
    // level 1 (lane 0 alone): dM[p][q] += dF1[p] S1p[q]
    if (lane == 0) {
#pragma unroll
        for (int blk = 0; blk < 4; ++blk)
#pragma unroll
            for (int u = 0; u < 2; ++u)
#pragma unroll
                for (int v = 0; v < 2; ++v) dM[4 * blk + 2 * u + v] += dF1[2 * blk + u] * S1p[2 * blk + v];
    }
    // level 2, row axis: dM[i][q] += sum_j dF2[i][j] G1[q][j], q in {i, i^1}
    // level 2, column axis: dM[j][q] += sum_i dF2[i][j] (S2p flowed along rows)[i][q], q in block jb
    float R2[2];  // (S2p flowed along rows)[i][2jb + r']
#pragma unroll
    for (int r = 0; r < 2; ++r) R2[r] = flow_i2(Di, P2[0][r], P2[1][r], lo);
    float rowq[2];  // contributions to dM[i][i] and dM[i][i^1]
    rowq[0] = fmaf(dF2[0], G1[0][0], dF2[1] * G1[0][1]);
    rowq[1] = fmaf(dF2[0], G1[1][0], dF2[1] * G1[1][1]);
    float colq[2][2];  // dM[2jb + r][2jb + r']
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int r2 = 0; r2 < 2; ++r2) colq[r][r2] = dF2[r] * R2[r2];
    // level 3: S3p rows i, i^1 at columns j (block jb), all k
    {
        float T0[2][8], T1[2][8];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                T0[r][k] = row_s3(prow, N, i, 2 * jb + r, k);
                T1[r][k] = row_s3(prow, N, i2, 2 * jb + r, k);
            }
        // axis 3: G'' = flowed along i and j; dM[k][q] += sum_r l3'[r][k] G''[r][q]
        {
            float G[2][8], H[2][8];
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    G[r][k] = T0[r][k];
                    H[r][k] = T1[r][k];
                }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                flow2(Dj, G[0][k], G[1][k]);
                flow2(Dj, H[0][k], H[1][k]);
            }
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int k = 0; k < 8; ++k) G[r][k] = flow_i2(Di, G[r][k], H[r][k], lo);
#pragma unroll
            for (int blk = 0; blk < 4; ++blk)
#pragma unroll
                for (int u = 0; u < 2; ++u)
#pragma unroll
                    for (int v = 0; v < 2; ++v) {
                        const int k = 2 * blk + u, qq = 2 * blk + v;
                        dM[4 * blk + 2 * u + v] =
                            fmaf(a.L3[0][k], G[0][qq], fmaf(a.L3[1][k], G[1][qq], dM[4 * blk + 2 * u + v]));
                    }
        }
        // axis 2: G' = flowed along i and k; dM[j][q] += sum_k l3'[r][k] G'[r'][k], (j, q) in block jb
        {
            float G[2][8], H[2][8];
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    G[r][k] = T0[r][k];
                    H[r][k] = T1[r][k];
                }
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int blk = 0; blk < 4; ++blk) {
                    flow2(lc.D + 4 * blk, G[r][2 * blk], G[r][2 * blk + 1]);
                    flow2(lc.D + 4 * blk, H[r][2 * blk], H[r][2 * blk + 1]);
                }
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int k = 0; k < 8; ++k) G[r][k] = flow_i2(Di, G[r][k], H[r][k], lo);
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int r2 = 0; r2 < 2; ++r2) {
                    float acc = colq[r][r2];
#pragma unroll
                    for (int k = 0; k < 8; ++k) acc = fmaf(a.L3[r][k], G[r2][k], acc);
                    colq[r][r2] = acc;
                }
        }
        // axis 1: G = flowed along j and k (rows i, i^1); dM[i][q] += sum_{r,k} l3'[r][k] G_q[r][k]
        {
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int blk = 0; blk < 4; ++blk) {
                    flow2(lc.D + 4 * blk, T0[r][2 * blk], T0[r][2 * blk + 1]);
                    flow2(lc.D + 4 * blk, T1[r][2 * blk], T1[r][2 * blk + 1]);
                }
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                flow2(Dj, T0[0][k], T0[1][k]);
                flow2(Dj, T1[0][k], T1[1][k]);
            }
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                    rowq[0] = fmaf(a.L3[r][k], T0[r][k], rowq[0]);
                    rowq[1] = fmaf(a.L3[r][k], T1[r][k], rowq[1]);
                }
        }
    }
    // scatter rowq (block i>>1, row i&1, columns i and i^1) and colq (block jb) into dM
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        const bool bi = blk == (i >> 1), bj = blk == jb;
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int v = 0; v < 2; ++v) {
                float add = 0.f;
                // rowq[0] is column i itself, rowq[1] column i^1
                if (bi && u == (i & 1)) add += (v == (i & 1)) ? rowq[0] : rowq[1];
                if (bj) add += colq[u][v];
                dM[4 * blk + 2 * u + v] += add;
            }
    }
    // ---- letters: db, then the letter recursion on lanes 0..7
    __syncwarp();
    letters_adjoint<QT>(p, lc, ab);
    float dX[16];
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) {
        const float* A = Ablk + 4 * blk;
        const float X[4] = {-h * A[0], -h * A[1], -h * A[2], -h * A[3]};
        expm_frechet_adjoint(X, dM + 4 * blk, dX + 4 * blk);
    }
    {
        const int ar = lane & 7;
        const int blk = ar >> 1, u = ar & 1;
        const float* A = Ablk + 4 * blk;
        const float xd = -h * (u ? A[3] : A[0]);   // X[a][a]
        const float xt = -h * (u ? A[1] : A[2]);   // X[a^1][a]
        const int q = QT >= 0 ? QT : p.g.q;
        float cur = ab.db[q * 8 + ar];
        float dxa0 = 0.f, dxa1 = 0.f;  // dX[a][2blk], dX[a][2blk+1]
        for (int pp = q; pp >= 1; --pp) {
            const float inv = 1.f / (float)pp;
            const float curo = __shfl_xor_sync(kFull, cur, 1);
            dxa0 = fmaf(cur * inv, lc.b[(pp - 1) * 8 + 2 * blk], dxa0);
            dxa1 = fmaf(cur * inv, lc.b[(pp - 1) * 8 + 2 * blk + 1], dxa1);
            cur = ab.db[(pp - 1) * 8 + ar] + inv * fmaf(xd, cur, xt * curo);
        }
        if (lane < 8) {
            dyg[ar] = cur;
#pragma unroll
            for (int b2 = 0; b2 < 4; ++b2)
                if (b2 == blk) {
                    dX[4 * b2 + 2 * u] += dxa0;
                    dX[4 * b2 + 2 * u + 1] += dxa1;
                }
        }
    }
    // dA += -h dX, dh = -<dX, A>
    float dh = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        bo.dA[e] = fmaf(-h, dX[e], bo.dA[e]);
        dh = fmaf(-dX[e], Ablk[e], dh);
    }
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) dh += __shfl_xor_sync(kFull, dh, o);
    if (lane == 0) *dtg = dh;
    // ---- cotangent of S_{t-1}
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int blk = 0; blk < 4; ++blk) flow2T(lc.D + 4 * blk, a.L3[r][2 * blk], a.L3[r][2 * blk + 1]);
#pragma unroll
    for (int k = 0; k < 8; ++k) flow2T(Dj, a.L3[0][k], a.L3[1][k]);
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 8; ++k) a.L3[r][k] = flowT_i(Di, a.L3[r][k], lo);
    flow2T(Dj, dF2[0], dF2[1]);
#pragma unroll
    for (int r = 0; r < 2; ++r) a.L2a[r] = flowT_i(Di, dF2[r], lo);
#pragma unroll
    for (int blk = 0; blk < 4; ++blk) flow2T(lc.D + 4 * blk, dF1[2 * blk], dF1[2 * blk + 1]);
#pragma unroll
    for (int k = 0; k < 8; ++k) a.L1[k] = dF1[k];
    __syncwarp();
}

// The zero-carry local adjoint's step: lambda <- J_t^T lambda (needs only D, s1, s2 of the interval).
__device__ __forceinline__ void mu_step(const Loc& lc, A3& a, int i, int jb) {
    float U2b[2][8];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 8; ++k) U2b[r][k] = lc.s2[(2 * jb + r) * 8 + k];
    apply_JT(a, lc.D, lc.s1, U2b, i, jb);
}

// mu_step with the local element staged as a row [D | s1 | s2 | s3].
__device__ __forceinline__ void mu_step_row(const float* row, A3& a, int i, int jb) {
    float U2b[2][8];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int k = 0; k < 8; ++k) U2b[r][k] = row[24 + (2 * jb + r) * 8 + k];
    apply_JT(a, row, row + 16, U2b, i, jb);
}

template <int QT>
__global__ void __launch_bounds__(kWarps * 32) bwd_kernel(Params p) {
    extern __shared__ float smem[];
    const Geom& g = p.g;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int i = lane >> 2, jb = lane & 3;
    float* liftS = smem;
    float* Ablk = smem + g.lift_n;
    for (int e = threadIdx.x; e < NB * g.d_in; e += blockDim.x) {
        const int r = e / g.d_in, cc = e - r * g.d_in;
        liftS[cc * NB + r] = (p.lift && r < g.N) ? p.lift[r * g.d_in + cc] : 0.f;
    }
    for (int e = threadIdx.x; e < 16; e += blockDim.x) Ablk[e] = (e >> 2) < g.N / 2 ? p.blocks[e] : 0.f;
    __syncthreads();
    float* dxs = smem + g.lift_n + 16 + warp * g.b_per_warp;
    float* dys = dxs + g.b_dys;
    float* dts = dxs + g.b_dts;
    float* dtg = dxs + g.b_dtg;
    float* dyg = dxs + g.b_dyg;
    const Loc lc(dxs + g.b_loc);
    const AdjBuf ab(dxs + g.b_adj);
    float* gst = dxs + g.b_gst;  // gradient row; also the dx staging at the end of a tile
    float* sst = dxs + g.b_sst;  // S_{t-1} row
    // Terminal readout: the cotangent has one row per sample (t = T - 1), and the states S_{t-1} come from
    // re-running the chunk from the forward's carry into this warp's scratch rows (the reference's
    // block_terminal_vjp recomputes each chunk from its saved start the same way), not from a prefix stream.
    const bool term = g.readout == EWS_READOUT_TERMINAL;
    float* scr = term ? p.scratch + (size_t)(blockIdx.x * kWarps + warp) * g.Lc * g.RS : nullptr;
    // source of the cotangent row of interval t (null where it is zero)
    auto grad_row = [&](int b, int t) -> const float* {
        if (term) return t == g.T - 1 ? p.grad_out + (size_t)b * g.W : nullptr;
        return p.grad_out + ((size_t)b * g.T + t) * g.W;
    };

    for (;;) {
        const int tile = next_ticket(p.st);
        if (tile >= g.ntiles) break;
        const int cr = tile / g.B, b = tile - cr * g.B;
        const int c = g.C - 1 - cr;
        const int t0 = c * g.Lc;
        const int len = min(g.Lc, g.T - t0);
        load_chunk(p, liftS, dxs, dys, dts, b, t0, len);
        const size_t slot = ((size_t)b * g.C + c) * SLOT;
        int* flag = p.flags + (size_t)b * g.C + c;

        // ---- 1. zero-carry local adjoint over the chunk (reverse); the local elements come from the forward's
        // local_kernel, staged one interval ahead in the (idle) Loc / AdjBuf area
        A3 mu;
        mu.zero();
        float* lst = dxs + g.b_loc;
        // gradient row and local element of interval k, copied in with cp.async one interval ahead (the
        // rows into alternating buffers; fetch_local commits the group)
        float* gst2 = dxs + g.b_gst2;
        auto issue_zero_carry = [&](int k) {
            const int buf = (len - 1 - k) & 1;
            const float* gsrc = grad_row(b, t0 + k);
            if (gsrc) warp_copy_row_padded_async(buf ? gst2 : gst, gsrc, g.N);
            fetch_local(p, b, t0 + k, lst + (k & 1) * LROW);
        };
        // (terminal readout: every chunk but the last has a zero cotangent and a zero local adjoint)
        if (!term || c == g.C - 1) {
            issue_zero_carry(len - 1);
            for (int k = len - 1; k >= 0; --k) {
                if (k >= 1)
                    issue_zero_carry(k - 1);
                else
                    cp_async_commit();
                cp_async_wait<1>();
                __syncwarp();
                if (grad_row(b, t0 + k)) add_grad_row(mu, ((len - 1 - k) & 1) ? gst2 : gst, g.N, i, jb);
                mu_step_row(lst + (k & 1) * LROW, mu, i, jb);
                __syncwarp();
            }
            cp_async_wait<0>();
        }
        // ---- 2. look-back over the later chunks: the cotangent at the chunk's end
        A3 lam;
        lam.zero();
        if (c == g.C - 1) {
            store_a3(p.incl + slot, mu, i, jb);
            if (!(g.flags & EWS_F_TEST_WITHHOLD)) publish(flag, kFlagIncl);
        } else {
            store_a3(p.agg + slot, mu, i, jb);
            publish(flag, kFlagAgg);
            E3 Gacc;
            Gacc.identity();
            int j = c + 1;
            const int want = (g.flags & EWS_F_DETERMINISTIC) ? kFlagIncl : kFlagAgg;
            for (;;) {
                const int f = wait_slot(p.flags + (size_t)b * g.C + j, p.st, g.spin_limit, tile, want);
                if (f < 0) return;
                const size_t sj = ((size_t)b * g.C + j) * SLOT;
                A3 X;
                load_a3((f == kFlagIncl ? p.incl : p.agg) + sj, X, i, jb);
                apply_JT_e3(X, Gacc, i, jb);
                lam.add(X);
                if (f == kFlagIncl) break;
                E3 Gj;
                load_e3(p.fagg + sj, Gj, i, jb);
                chen_mul(Gacc, Gj, i, jb);
                ++j;
            }
            A3 out = lam;
            {
                E3 Gc;
                load_e3(p.fagg + slot, Gc, i, jb);
                apply_JT_e3(out, Gc, i, jb);
            }
            out.add(mu);
            __syncwarp();
            store_a3(p.incl + slot, out, i, jb);
            publish(flag, kFlagIncl);
        }
        // ---- terminal readout: the chunk's states S_{t0-1} .. S_{t0+len-2} recomputed from the forward's carry
        // into the scratch rows 0 .. len-1 (padded layout), the local elements staged as in pass 1
        if (term) {
            E3 S;
            load_e3(p.fcarry + slot, S, i, jb);
            stage_row(scr, S, g.N, i, jb);
            if (len > 1) fetch_local(p, b, t0, lst);
            for (int k = 0; k + 1 < len; ++k) {
                cp_async_wait<0>();
                __syncwarp();
                if (k + 2 < len) fetch_local(p, b, t0 + k + 1, lst + ((k + 1) & 1) * LROW);
                chen_step_row(lst + (k & 1) * LROW, S, i, jb);
                stage_row(scr + (size_t)(k + 1) * g.RS, S, g.N, i, jb);
                __syncwarp();
            }
            cp_async_wait<0>();
            __threadfence_block();
            __syncwarp();
        }
        // ---- 3. exact adjoint from the carry, with the gradients
        BwdOut bo;
#pragma unroll
        for (int e = 0; e < 16; ++e) bo.dA[e] = 0.f;
        A3 a = lam;
        // the rows of interval t (gradient row t, state row t-1) are copied in with cp.async one interval
        // ahead, into alternating buffers
        float* sst2 = dxs + g.b_sst2;
        auto issue_rows = [&](int k, int buf) {
            const int t = t0 + k;
            const float* gsrc = grad_row(b, t);
            if (gsrc) warp_copy_row_padded_async(buf ? gst2 : gst, gsrc, g.N);
            if (t > 0) {
                if (term)
                    warp_load_span_async(buf ? sst2 : sst, scr + (size_t)k * g.RS, g.RS);  // 16-byte aligned: lands at the buffer start
                else
                    warp_copy_row_padded_async(buf ? sst2 : sst, p.out + ((size_t)b * g.T + t - 1) * g.W, g.N);
            }
            cp_async_commit();
        };
        issue_rows(len - 1, 0);
        for (int k = len - 1; k >= 0; --k) {
            const int t = t0 + k;
            const int buf = (len - 1 - k) & 1;
            if (k >= 1)
                issue_rows(k - 1, buf ^ 1);
            else
                cp_async_commit();
            cp_async_wait<1>();
            float* grow = buf ? gst2 : gst;
            float* srow = buf ? sst2 : sst;
            if (t == 0)
                for (int e = lane; e < row_floats_padded(g.N); e += 32) srow[e] = 0.f;
            __syncwarp();
            build_local<QT>(p, Ablk, dys + k * NB, dts[k], lc, true);
            if (!term || t == g.T - 1) add_grad_row(a, grow, g.N, i, jb);
            bwd_step<QT>(p, Ablk, lc, ab, srow, dts[k], a, bo, dyg + k * NB, dtg + k, i, jb);
            __syncwarp();
        }
        cp_async_wait<0>();
        // ---- chunk outputs: dx = lift^T dy, dtheta, per-tile partials (dA, dlift)
        __syncwarp();
        for (int e = lane; e < len * g.d_in; e += 32) {
            const int k = e / g.d_in, cc = e - k * g.d_in;
            float acc = 0.f;
            if (p.lift) {
                for (int r = 0; r < g.N; ++r) acc = fmaf(liftS[cc * NB + r], dyg[k * NB + r], acc);
            } else {
                acc = dyg[k * NB + cc];
            }
            gst[e] = acc;
        }
        __syncwarp();
        warp_store_span(p.grad_dx + ((size_t)b * g.T + t0) * g.d_in, gst, len * g.d_in);
        warp_store_span(p.grad_dtheta + (size_t)b * g.T + t0, dtg, len);
        __syncwarp();
        float* part = p.partials + (size_t)tile * (16 + NB * g.d_in);
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            float v = bo.dA[e];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) v += __shfl_xor_sync(kFull, v, o);
            if (lane == 0) part[e] = v;
        }
        for (int e = lane; e < NB * g.d_in; e += 32) {
            const int r = e / g.d_in, cc = e - r * g.d_in;
            float acc = 0.f;
            if (p.lift && r < g.N)
                for (int k = 0; k < len; ++k) acc = fmaf(dyg[k * NB + r], dxs[k * g.d_in + cc], acc);
            part[16 + e] = acc;
        }
        __syncwarp();
    }
}

// Deterministic sum of the per-tile partials over all tiles (fixed order): dA blocks and the lift.
__global__ void reduce_kernel(Params p, float* grad_blocks, float* grad_lift) {
    const Geom& g = p.g;
    const int stride = 16 + NB * g.d_in;
    const int K = g.N / 2;
    const int total = 4 * K + (grad_lift ? g.N * g.d_in : 0);
    // one CTA per output entry: each thread sums a strided set of tiles in order, then a fixed tree
    __shared__ float red[256];
    for (int e = blockIdx.x; e < total; e += gridDim.x) {
        const int off = e < 4 * K ? e : 16 + (e - 4 * K);
        float acc = 0.f;
        for (int t = threadIdx.x; t < g.ntiles; t += blockDim.x) acc += ldcg(p.partials + (size_t)t * stride + off);
        red[threadIdx.x] = acc;
        __syncthreads();
        for (int h = blockDim.x / 2; h > 0; h >>= 1) {
            if (threadIdx.x < h) red[threadIdx.x] += red[threadIdx.x + h];
            __syncthreads();
        }
        if (threadIdx.x == 0) {
            if (e < 4 * K)
                grad_blocks[e] = red[0];
            else
                grad_lift[e - 4 * K] = red[0];
        }
        __syncthreads();
    }
}

}  // namespace blk
}  // namespace ews

// ------------------------------------------------------------------------------ host side

using namespace ews;
using namespace ews::blk;

namespace {

int pick_chunk(int B, int T) {
    const int want_tiles = 148 * 16;
    int C = (want_tiles + B - 1) / B;
    if (C < 1) C = 1;
    int Lc = (T + C - 1) / C;
    return std::max(8, std::min(64, Lc));
}

// The backward's zero-carry pass stages two local elements (2 LROW floats) at b_loc, across the Loc and
// AdjBuf areas that pass leaves idle; b_gst, which the same loop fills with cp.async, starts right after.
static_assert(2 * LROW <= align4(Loc::floats) + align4(AdjBuf::floats),
              "the zero-carry pass's two staged local elements must fit in the Loc + AdjBuf areas");

int make_geom(const ews_block_args* a, Geom* g) {
    if (!a || a->batch <= 0 || a->steps <= 0 || a->d_in <= 0 || a->dim <= 0) return EWS_ERR_INVALID_ARGUMENT;
    if (a->depth != 3) return EWS_ERR_UNSUPPORTED;
    if (a->dim > NB || (a->dim & 1)) return EWS_ERR_UNSUPPORTED;
    if (a->series_q < 0 || a->series_q >= KQ) return EWS_ERR_UNSUPPORTED;
    if (a->d_in > 64) return EWS_ERR_UNSUPPORTED;
    if (a->readout != EWS_READOUT_PREFIX && a->readout != EWS_READOUT_TERMINAL) return EWS_ERR_INVALID_ARGUMENT;
    if ((a->flags & EWS_F_BF16) && !(a->flags & EWS_F_INCREMENTS)) return EWS_ERR_INVALID_ARGUMENT;
    if (a->flags & (EWS_F_UNIFORM | EWS_F_BASEPOINT)) return EWS_ERR_INVALID_ARGUMENT;  // clock knots only
    g->B = a->batch;
    g->T = a->steps;
    g->d_in = a->d_in;
    g->N = a->dim;
    g->depth = a->depth;
    g->q = a->series_q;
    g->readout = a->readout;
    g->flags = a->flags;
    g->spin_limit = a->spin_limit > 0 ? a->spin_limit : kDefaultSpinLimit;
    g->W = 1 + g->N + g->N * g->N + g->N * g->N * g->N;
    g->Lc = a->chunk > 0 ? a->chunk : pick_chunk(a->batch, a->steps);
    g->C = (g->T + g->Lc - 1) / g->Lc;
    g->ntiles = g->B * g->C;
    g->lift_n = align4(NB * g->d_in);
    g->RS = align4(row_floats_padded(g->N));
    const int xs = align4(g->Lc * g->d_in), ys = g->Lc * NB, ts = align4(g->Lc);
    g->f_dys = xs;
    g->f_dts = xs + ys;
    g->f_loc = g->f_dts + ts;
    g->f_stage = g->f_loc + align4(std::max(2 * LROW, (int)Loc::floats));
    g->f_per_warp = g->f_stage + align4(row_floats_padded(g->N) + 4);  // one staged row at any phase
    g->b_dys = xs;
    g->b_dts = xs + ys;
    g->b_dtg = g->b_dts + ts;
    g->b_dyg = g->b_dtg + ts;
    g->b_loc = g->b_dyg + ys;
    g->b_adj = g->b_loc + align4(Loc::floats);
    g->b_gst = g->b_adj + align4(AdjBuf::floats);
    g->b_sst = g->b_gst + align4(std::max(row_floats_padded(g->N), g->Lc * g->d_in));
    g->b_gst2 = g->b_sst + align4(row_floats_padded(g->N));  // second buffers of the exact pass
    g->b_sst2 = g->b_gst2 + align4(row_floats_padded(g->N));
    g->b_per_warp = g->b_sst2 + align4(row_floats_padded(g->N));
    return EWS_OK;
}

size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

struct WsLayout {
    size_t status, flags, agg, incl, carry, partials, loc, scratch, total;
};

size_t bwd_smem(const Geom& g);
int num_sms();

// The backward's kernel (series order fixed at compile time), its shared memory and its persistent grid.
struct BwdPlan {
    void (*kernel)(Params);
    size_t smem;
    int grid;
};

int bwd_plan(const Geom& g, BwdPlan* bp) {
    using BK = void (*)(Params);
    static const BK kernels[KQ] = {bwd_kernel<0>, bwd_kernel<1>, bwd_kernel<2>, bwd_kernel<3>, bwd_kernel<4>,
                                   bwd_kernel<5>, bwd_kernel<6>, bwd_kernel<7>, bwd_kernel<8>};
    bp->kernel = kernels[g.q];
    bp->smem = bwd_smem(g);
    if (bp->smem > 227 * 1024) return EWS_ERR_UNSUPPORTED;
    cudaFuncSetAttribute(bp->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bp->smem);
    cudaFuncSetAttribute(bp->kernel, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    const int per_sm = resident_ctas((const void*)bp->kernel, kWarps * 32, bp->smem);
    if (per_sm < 1) return EWS_ERR_UNSUPPORTED;
    int grid = per_sm * num_sms();
    const int need = (g.ntiles + kWarps - 1) / kWarps;
    if (grid > need) grid = need;
    bp->grid = grid;
    return EWS_OK;
}

// grid: the backward's CTA count (sizes the terminal readout's per-warp scratch rows)
WsLayout bwd_layout(const Geom& g, int grid) {
    WsLayout L{};
    size_t o = 0;
    L.status = o;
    o += al256(sizeof(DeviceStatus));
    L.flags = o;
    o += al256(sizeof(int) * (size_t)g.ntiles);
    const size_t slots = al256(sizeof(float) * (size_t)g.ntiles * SLOT);
    L.agg = o;
    o += slots;
    L.incl = o;
    o += slots;
    L.partials = o;
    o += al256(sizeof(float) * (size_t)g.ntiles * (16 + NB * g.d_in));
    L.scratch = o;
    if (g.readout == EWS_READOUT_TERMINAL) o += al256(sizeof(float) * (size_t)grid * kWarps * g.Lc * g.RS);
    L.total = o;
    return L;
}

WsLayout fwd_layout(const Geom& g) {
    WsLayout L{};
    size_t o = 0;
    L.status = o;
    o += al256(sizeof(DeviceStatus));
    L.flags = o;
    o += al256(sizeof(int) * (size_t)g.ntiles);
    const size_t slots = al256(sizeof(float) * (size_t)g.ntiles * SLOT);
    L.agg = o;
    o += slots;
    L.incl = o;
    o += slots;
    L.carry = o;
    o += slots;
    L.loc = o;
    o += al256(sizeof(float) * (size_t)g.B * g.T * LROW);
    L.total = o;
    return L;
}

void series_coefficients(int q, Params* p) {
    for (int a = 0; a < KQ; ++a) {
        p->c1[a] = a <= q ? (float)(1.0 / (a + 1)) : 0.f;
        for (int b = 0; b < KQ; ++b) {
            p->c2[a * KQ + b] = a + b <= q ? (float)(1.0 / ((double)(a + b + 2) * (b + 1))) : 0.f;
            for (int c = 0; c < KQ; ++c)
                p->c3[(a * KQ + b) * KQ + c] =
                    a + b + c <= q ? (float)(1.0 / ((double)(a + b + c + 3) * (b + c + 2) * (c + 1))) : 0.f;
        }
    }
}

int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

size_t fwd_smem(const Geom& g) { return sizeof(float) * ((size_t)g.lift_n + 16 + (size_t)kWarps * g.f_per_warp); }
size_t bwd_smem(const Geom& g) { return sizeof(float) * ((size_t)g.lift_n + 16 + (size_t)kWarps * g.b_per_warp); }

}  // namespace

extern "C" int ews_block_workspace_size(const ews_block_args* a, size_t* fwd_bytes, size_t* bwd_bytes) {
    Geom g;
    const int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (fwd_bytes) *fwd_bytes = fwd_layout(g).total;
    if (bwd_bytes) {
        BwdPlan bp;
        const int pr = bwd_plan(g, &bp);
        if (pr != EWS_OK) return pr;
        *bwd_bytes = bwd_layout(g, bp.grid).total;
    }
    return EWS_OK;
}

extern "C" int ews_block_fwd(const ews_block_args* a, ews_stream_t stream) {
    Geom g;
    const int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (!a->path || !a->clock || !a->blocks || !a->out) return EWS_ERR_INVALID_ARGUMENT;
    if (!a->lift && a->d_in != a->dim) return EWS_ERR_INVALID_ARGUMENT;
    const WsLayout L = fwd_layout(g);
    if (!a->fwd_ws || a->fwd_ws_bytes < L.total) return EWS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    char* ws = (char*)a->fwd_ws;
    if (cudaMemsetAsync(ws, 0, L.agg, s) != cudaSuccess) return EWS_ERR_LAUNCH;
    Params p{};
    p.g = g;
    p.path = a->path;
    p.clock = a->clock;
    p.blocks = a->blocks;
    p.lift = a->lift;
    p.out = a->out;
    p.st = (DeviceStatus*)(ws + L.status);
    p.flags = (int*)(ws + L.flags);
    p.agg = (float*)(ws + L.agg);
    p.incl = (float*)(ws + L.incl);
    p.carry = (float*)(ws + L.carry);
    p.loc = (float*)(ws + L.loc);
    series_coefficients(g.q, &p);
    const size_t smem = fwd_smem(g);
    if (smem > 227 * 1024) return EWS_ERR_UNSUPPORTED;
    {
        // every interval's local element first: a parallel map
        using LK = void (*)(Params);
        static const LK kernels[KQ] = {local_kernel<0>, local_kernel<1>, local_kernel<2>,
                                       local_kernel<3>, local_kernel<4>, local_kernel<5>,
                                       local_kernel<6>, local_kernel<7>, local_kernel<8>};
        const LK lk = kernels[g.q];
        cudaFuncSetAttribute(lk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        lk<<<(g.B * g.C + kWarps - 1) / kWarps, kWarps * 32, smem, s>>>(p);
        if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    }
    cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    int per_sm = 0;
    per_sm = resident_ctas((const void*)fwd_kernel, kWarps * 32, smem);
    if (per_sm < 1) return EWS_ERR_UNSUPPORTED;
    int grid = per_sm * num_sms();
    const int need = (g.ntiles + kWarps - 1) / kWarps;
    if (grid > need) grid = need;
    fwd_kernel<<<grid, kWarps * 32, smem, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

extern "C" int ews_block_bwd(const ews_block_args* a, ews_stream_t stream) {
    Geom g;
    const int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (!a->path || !a->clock || !a->blocks || !a->out || !a->grad_out || !a->grad_dx || !a->grad_dtheta ||
        !a->grad_blocks)
        return EWS_ERR_INVALID_ARGUMENT;
    if (!a->lift && a->d_in != a->dim) return EWS_ERR_INVALID_ARGUMENT;
    BwdPlan bp;
    const int pr = bwd_plan(g, &bp);
    if (pr != EWS_OK) return pr;
    const WsLayout F = fwd_layout(g);
    const WsLayout L = bwd_layout(g, bp.grid);
    if (!a->fwd_ws || a->fwd_ws_bytes < F.total) return EWS_ERR_WORKSPACE;
    if (!a->bwd_ws || a->bwd_ws_bytes < L.total) return EWS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    char* ws = (char*)a->bwd_ws;
    const char* fws = (const char*)a->fwd_ws;
    if (cudaMemsetAsync(ws, 0, L.agg, s) != cudaSuccess) return EWS_ERR_LAUNCH;
    Params p{};
    p.g = g;
    p.path = a->path;
    p.clock = a->clock;
    p.blocks = a->blocks;
    p.lift = a->lift;
    p.out = a->out;
    p.grad_out = a->grad_out;
    p.grad_dx = a->grad_dx;
    p.grad_dtheta = a->grad_dtheta;
    p.st = (DeviceStatus*)(ws + L.status);
    p.flags = (int*)(ws + L.flags);
    p.agg = (float*)(ws + L.agg);
    p.incl = (float*)(ws + L.incl);
    p.partials = (float*)(ws + L.partials);
    p.fagg = (const float*)(fws + F.agg);
    p.fcarry = (const float*)(fws + F.carry);
    p.loc = (float*)(fws + F.loc);
    p.scratch = g.readout == EWS_READOUT_TERMINAL ? (float*)(ws + L.scratch) : nullptr;
    series_coefficients(g.q, &p);
    bp.kernel<<<bp.grid, kWarps * 32, bp.smem, s>>>(p);
    if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    reduce_kernel<<<2 * g.N + (a->grad_lift ? g.N * g.d_in : 0), 256, 0, s>>>(p, a->grad_blocks, a->grad_lift);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}
