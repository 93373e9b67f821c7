// Dense-A engine of the EWS hot path (any generator A, uniform clock), depth 2, N <= 32, fp32.
//
// Per interval t of sample b, with the flow M = exp(-h A) = I - D and the increment dx_t (before the lift):
//     S1' = u + s1,                      u  = M S1,   s1 = F dx
//     S2' = M S2 M^T + u s1^T + U V^T,   U = [G_a dx]_a,  V = [H_a dx]_a   (a = 0..q)
// This is the modified-Chen recursion of ews/core/chen_scan.py:124-152 (sequentially:
// ews/core/kernels/pallas_combine.py:1804-1834) with the series leaf of ews/core/series_leaf.py:72-113:
// for a uniform clock the letters are b_a = P_a dy with P_a = (-hA)^a / a!, so
// s1 = sum_p c_p P_p dy = K1 dy and s2 = sum_a (P_a dy)(K2_a dy)^T with K2_a = sum_b c_ab P_b; the lift W
// is folded into F = K1 W, G_a = P_a W, H_a = K2_a W by the caller.
//
// Work decomposition. Forward: the local terms of every interval (local_kernel), the power complements
// I - M^j (powers_kernel), every chunk's zero-carry aggregate as a parallel map (agg_kernel), the carries by
// a two-level scan over the chunks (scan_local, log-depth rounds over the groups, scan_fix), then the output
// pass on tcgen05 (fwd_tc_kernel: four chunks of a sample stacked into M = 128, two 3xTF32 products per
// step). Backward: every chunk's zero-carry adjoint as power sums (bagg_kernel), the reverse scan of the local adjoints
// (bscan_*), the exact adjoint pass with the gradient map fused in (bwd_exact_kernel), the table gradients
// (table_grad_*) and a fixed-order reduction. No kernel waits on another CTA.
//
// Flows are carried as complements D = I - M (the caller evaluates D in float64): M X = X - D X. An M
// within 1e-4 of the identity, rounded once and applied T times, drifts by ~T 2^-24; the complement keeps
// the rounding relative to D. Chunk flows compose as complements, I - (I-A)(I-B) = A + B - AB.
#include <algorithm>
#include <cstdio>

#include "ews_common.cuh"

namespace ews {
namespace dense {

constexpr int NP = 32;   // padded state dimension
constexpr int NT = 64;   // threads per tile
constexpr int MM = NP * NP;
constexpr int QMAX = 12; // series order q <= 11

struct Geom {
    int B, T, d_in, N, Lc, C, W, SW, QP, readout;
    unsigned flags;
    int spin_limit;
    int ntiles;
    int agg_pre;      // forward: the chunk aggregates come from agg_kernel (the chain runs the output pass only)
    int bwd_mode;     // backward: 2 while the exact pass runs (0 otherwise)
    int tab_n;        // floats of the F, G, H tables (N x d_in each, padded to NP rows)
    int grp0, ngrp;   // the chunk groups (TILES chunks each) that fwd_tc_kernel and bwd_exact_kernel cover
};

struct Params {
    Geom g;
    const void* path;
    const float* tab_d;  // (B, N, N) flow complement D = I - M
    const float* tab_f;  // (B, N, d_in)
    const float* tab_g;  // (B, QP, N, d_in)
    const float* tab_h;  // (B, QP, N, d_in)
    float* out;
    const float* grad_out;
    float* grad_dx;
    float* partials;  // per tile: dM (NP*NP) | dF (NP*d_in) | dG (QP*NP*d_in) | dH (QP*NP*d_in)
    DeviceStatus* st;
    int* flags;
    float* agg;
    float* incl;
    float* carry;
    const float* fagg;
    float* pw;  // per sample: flow complements C(Lc) and C(last chunk), row-major (2 MM)
    float* lcarry;     // backward: per chunk the cotangent arriving at its end [- | L1 | L2] (SW)
    float* loc;        // local terms per (sample, interval): [s1 | U_0..U_{QP-1} | V_0..V_{QP-1}], NP each
    float* coef;       // backward: per (sample, interval) the vector cotangents [ds1 | dU_a | dV_a], NP each
    float* pows;       // forward: per sample the power complements E_j = I - M^j, j = 0..Lc, row-major (Lc+1) MM
    float* gex;        // forward: per (sample, scan group) the exclusive product of the earlier groups (SW);
                       // backward: per (sample, scan group) the cotangent arriving at the group's end
    float* gsuf;       // backward: per chunk the forward aggregate of the chunks from it to its group's end
    float* srows;      // terminal backward: the window's recomputed states, per chunk Lc rows of W (row k holds
                       // S_{t0+k-1}: the carry, then the chunk's own states but its last)
};

// The cotangent row of interval t of sample b, or null where it is zero: a terminal readout has one row per
// sample (t = T - 1), a prefix readout one per interval.
__device__ __forceinline__ const float* grad_row(const Params& p, int b, int t) {
    if (p.g.readout == EWS_READOUT_TERMINAL) return t == p.g.T - 1 ? p.grad_out + (size_t)b * p.g.W : nullptr;
    return p.grad_out + ((size_t)b * p.g.T + t) * p.g.W;
}

// Terminal backward: the first of the scratch rows of chunk c_me (the tile's warp) of sample b in the window.
__device__ __forceinline__ float* window_rows(const Params& p, int grp, int warp, int b) {
    const Geom& g = p.g;
    return p.srows + ((((size_t)(grp - g.grp0) * 4 + warp) * g.B + b) * g.Lc) * g.W;
}

// Width (floats) of one interval's local terms in `loc`.
__host__ __device__ inline int loc_width(int QP) { return (1 + 2 * QP) * 32; }

__host__ __device__ inline int align4(int n) { return (n + 3) & ~3; }
__host__ __device__ inline int imax(int a, int b) { return a > b ? a : b; }

// ---------------------------------------------------------------------------------- 4x4 block GEMM

// acc (+)= A B for the thread's 4x4 block: At is A stored k-major (At[k*32+i] = A[i][k]), Bm row-major.
__device__ __forceinline__ void gemm44(const float* __restrict__ At, const float* __restrict__ Bm, float acc[4][4],
                                       int i0, int j0, bool accumulate) {
    if (!accumulate) {
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
    }
#pragma unroll 8
    for (int k = 0; k < NP; ++k) {
        const float4 a = *reinterpret_cast<const float4*>(At + k * NP + i0);
        const float4 b = *reinterpret_cast<const float4*>(Bm + k * NP + j0);
        const float av[4] = {a.x, a.y, a.z, a.w};
        const float bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(av[r], bv[c], acc[r][c]);
    }
}

__device__ __forceinline__ void store_rowmajor(float* M, const float blk[4][4], int i0, int j0) {
#pragma unroll
    for (int r = 0; r < 4; ++r)
        *reinterpret_cast<float4*>(M + (i0 + r) * NP + j0) = make_float4(blk[r][0], blk[r][1], blk[r][2], blk[r][3]);
}

__device__ __forceinline__ void store_kmajor(float* Mt, const float blk[4][4], int i0, int j0) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
        *reinterpret_cast<float4*>(Mt + (j0 + c) * NP + i0) = make_float4(blk[0][c], blk[1][c], blk[2][c], blk[3][c]);
}

__device__ __forceinline__ void load_rowmajor(const float* M, float blk[4][4], int i0, int j0) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const float4 v = *reinterpret_cast<const float4*>(M + (i0 + r) * NP + j0);
        blk[r][0] = v.x;
        blk[r][1] = v.y;
        blk[r][2] = v.z;
        blk[r][3] = v.w;
    }
}

// ---------------------------------------------------------------------------------- Chen elements
// Slot layout (floats): [P row-major (NP*NP) | S1 (NP) | S2 row-major (NP*NP)].

__device__ void store_slot(float* slot, const float* Pr, const float* S1, const float* S2r) {
    for (int e = threadIdx.x; e < MM; e += blockDim.x) {
        slot[e] = Pr[e];
        slot[MM + NP + e] = S2r[e];
    }
    if (threadIdx.x < NP) slot[MM + threadIdx.x] = S1[threadIdx.x];
}

__device__ void load_slot_smem(const float* slot, float* P, float* S1, float* S2) {
    for (int e = threadIdx.x; e < MM; e += blockDim.x) {
        P[e] = ldcg(slot + e);
        S2[e] = ldcg(slot + MM + NP + e);
    }
    if (threadIdx.x < NP) S1[threadIdx.x] = ldcg(slot + MM + threadIdx.x);
}

// One slot held in registers by a 256-thread CTA (4 + 4 floats per thread, level 1 in the first 32
// threads): the scans fetch the next element while the current product runs.
struct SlotRegs {
    float p[MM / 256], s2[MM / 256], s1;
};

__device__ __forceinline__ void slot_fetch(const float* slot, SlotRegs& r) {
#pragma unroll
    for (int k = 0; k < MM / 256; ++k) {
        r.p[k] = ldcg(slot + threadIdx.x + 256 * k);
        r.s2[k] = ldcg(slot + MM + NP + threadIdx.x + 256 * k);
    }
    r.s1 = threadIdx.x < NP ? ldcg(slot + MM + threadIdx.x) : 0.f;
}

__device__ __forceinline__ void slot_put(const SlotRegs& r, float* P, float* S1, float* S2) {
#pragma unroll
    for (int k = 0; k < MM / 256; ++k) {
        P[threadIdx.x + 256 * k] = r.p[k];
        S2[threadIdx.x + 256 * k] = r.s2[k];
    }
    if (threadIdx.x < NP) S1[threadIdx.x] = r.s1;
}

__device__ void identity_smem(float* P, float* S1, float* S2) {
    for (int e = threadIdx.x; e < MM; e += blockDim.x) {
        P[e] = 0.f;  // flow complement of the identity
        S2[e] = 0.f;
    }
    if (threadIdx.x < NP) S1[threadIdx.x] = 0.f;
}

namespace tc {

constexpr int TILES = 4;
static_assert(TILES == 4, "window_rows lays out 4 chunks per tile");
constexpr int NTH = 128;
constexpr int RQS = 33;  // padded row stride of the row/column exchange buffer

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

// x rounded to tf32 (10 explicit mantissa bits), nearest with ties away from zero, on the integer pipe: add
// half a tf32 unit to the magnitude bits, then clear the 13 low bits (a carry into the exponent is the
// correct rounding). The result is exact in tf32, so the tensor core reads it unchanged. Finite inputs only.
__device__ __forceinline__ uint32_t tf32_bits(float x) { return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u; }

// SM100 shared-memory matrix descriptor, no swizzle (start, leading / stride byte offsets, version 1).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// Instruction descriptor: kind::tf32, f32 accumulator, A and B K-major, M = 128, N = 32.
constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10) | (0u << 15) | (0u << 16) | ((32u >> 3) << 17) |
                            ((128u >> 4) << 24);

__device__ __forceinline__ void mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t"
        ".reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t"
        "}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ bool mbar_try(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float v[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,"
        "%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Offsets (floats) of the canonical no-swizzle K-major layouts, core matrices of 8 rows x 16 bytes:
// B (N = 32 rows, K = 32): [k/4][n/8][n%8][k%4]  (SBO 128 B between row groups, LBO 512 B between K chunks);
// A (M = 128 rows, K = 32): [k/4][m/8][m%8][k%4] (SBO 128 B, LBO 2048 B); one K-step of 8 spans two chunks.
__device__ __forceinline__ int bk_off(int n, int k) { return (((k >> 2) * 4 + (n >> 3)) * 32) + (n & 7) * 4 + (k & 3); }
__device__ __forceinline__ int ak_off4(int m, int kc) { return (kc * 16 + (m >> 3)) * 32 + (m & 7) * 4; }

// Writes row m of a K-major A operand as tf32 hi / lo pieces (16-byte stores).
__device__ __forceinline__ void store_a_row(float* Ahi, float* Alo, int m, const float v[32]) {
#pragma unroll
    for (int kc = 0; kc < 8; ++kc) {
        float h[4], lo[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            h[q] = __uint_as_float(tf32_bits(v[4 * kc + q]));
            lo[q] = v[4 * kc + q] - h[q];
        }
        const int off = ak_off4(m, kc);
        *reinterpret_cast<float4*>(Ahi + off) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(Alo + off) = make_float4(lo[0], lo[1], lo[2], lo[3]);
    }
}

struct TcSmem {
    float* Bhi;   // D hi, K-major (MM)
    float* Blo;   // D lo
    float* Ahi;   // A operand hi, K-major (4 MM)
    float* Alo;   // A operand lo
    float* RQ;    // TILES x 32 x RQS exchange buffer
    float* Dr;    // D row-major (or null)
    float* Dt;    // D k-major (or null)
    float* vec;   // per tile: S1 (l1) | u (v) | two staging slots of local terms
    uint64_t* bar;
    uint32_t* tmem;
    int* bcast;
};

// Per-tile vectors: S1 (or l1) | u (or v) | two staging slots for an interval's local terms.
__host__ __device__ inline int vec_per_tile(int QP) { return 2 * NP + 2 * loc_width(QP); }

// Flow table of sample b; the B operand is D (forward) or D^T (the adjoint chain, transpose = true).
__device__ void tc_load_tables(const Params& p, const TcSmem& s, int b, bool transpose = false) {
    const int N = p.g.N;
    const float* m = p.tab_d + (size_t)b * N * N;
    for (int e = threadIdx.x; e < MM; e += blockDim.x) {
        const int i = e / NP, k = e - i * NP;
        const float v = (i < N && k < N) ? m[i * N + k] : 0.f;
        if (s.Dr) s.Dr[i * NP + k] = v;
        if (s.Dt) s.Dt[k * NP + i] = v;
        const float hi = __uint_as_float(tf32_bits(v));
        const int o = transpose ? bk_off(k, i) : bk_off(i, k);
        s.Bhi[o] = hi;
        s.Blo[o] = v - hi;
    }
}

// Warp-broadcast reads of 16-byte aligned shared vectors, four entries per load (every lane reads the same
// address, one shared-memory wavefront per load).
// sum_n r[n] v[n]
__device__ __forceinline__ float dot32_bc(const float (&r)[32], const float* __restrict__ v) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
    for (int n = 0; n < 32; n += 4) {
        const float4 q = *reinterpret_cast<const float4*>(v + n);
        a0 = fmaf(r[n], q.x, a0);
        a1 = fmaf(r[n + 1], q.y, a1);
        a2 = fmaf(r[n + 2], q.z, a2);
        a3 = fmaf(r[n + 3], q.w, a3);
    }
    return (a0 + a1) + (a2 + a3);
}

// c[n] += v[n] s
__device__ __forceinline__ void axpy32_bc(float (&c)[32], const float* __restrict__ v, float s) {
#pragma unroll
    for (int n = 0; n < 32; n += 4) {
        const float4 q = *reinterpret_cast<const float4*>(v + n);
        c[n] = fmaf(q.x, s, c[n]);
        c[n + 1] = fmaf(q.y, s, c[n + 1]);
        c[n + 2] = fmaf(q.z, s, c[n + 2]);
        c[n + 3] = fmaf(q.w, s, c[n + 3]);
    }
}

// sum_k Mk[k][lane] v[k] for a row-major 32 x 32 shared matrix Mk (the lane reads its column, conflict-free)
// and a broadcast vector v.
__device__ __forceinline__ float coldot_bc(const float* __restrict__ Mk, const float* __restrict__ v, int lane) {
    float d0 = 0.f, d1 = 0.f, d2 = 0.f, d3 = 0.f;
#pragma unroll
    for (int k = 0; k < NP; k += 4) {
        const float4 q = *reinterpret_cast<const float4*>(v + k);
        d0 = fmaf(Mk[k * NP + lane], q.x, d0);
        d1 = fmaf(Mk[(k + 1) * NP + lane], q.y, d1);
        d2 = fmaf(Mk[(k + 2) * NP + lane], q.z, d2);
        d3 = fmaf(Mk[(k + 3) * NP + lane], q.w, d3);
    }
    return (d0 + d1) + (d2 + d3);
}

// u = S1 - D S1 for the lane's row (v: S1 (NP) | u (NP)).
__device__ __forceinline__ void tc_u(const TcSmem& s, float* v) {
    const int l = threadIdx.x & 31;
    v[NP + l] = v[l] - coldot_bc(s.Dt, v, l);
    __syncwarp();
}

// Starts the warp's copy of interval t's local terms (the first n floats of its `loc` row) into dst.
__device__ __forceinline__ void fetch_loc(const Params& p, int b, int t, float* dst, int n) {
    const float* src = p.loc + ((size_t)b * p.g.T + t) * loc_width(p.g.QP);
    for (int v = threadIdx.x & 31; v < n / 4; v += 32) cp_async16(dst + 4 * v, src + 4 * v);
}

}  // namespace tc

// The local terms of every interval, a parallel map over (sample, interval) run ahead of the chains:
// s1 = F dx, U_a = G_a dx, V_a = H_a dx, the lifted increment and the two factor families of the series
// leaf's level-2 term s2 = sum_a U_a V_a^T (ews/core/series_leaf.py:72-127 with the lift folded into the
// tables). One warp per interval, lane = state row; the sample's tables sit in shared memory channel-major
// (entry (m, c, i) at (m d + c) NP + i) so the lanes read consecutive words.
constexpr int LNT = 256;   // threads per CTA
constexpr int LSPAN = 64;  // intervals per CTA

__host__ __device__ inline size_t local_smem_bytes(int d_in, int QP) {
    return sizeof(float) * ((size_t)(1 + 2 * QP) * d_in * NP + (size_t)LSPAN * d_in);
}

__global__ void __launch_bounds__(LNT) local_kernel(Params p) {
    extern __shared__ float lsm[];
    const Geom& g = p.g;
    const int N = g.N, d = g.d_in, QP = g.QP, LW = loc_width(QP);
    const int nt = 1 + 2 * QP;  // tables F, G_0..G_{QP-1}, H_0..H_{QP-1}
    const int spans = (g.T + LSPAN - 1) / LSPAN;
    const int b = blockIdx.x / spans, t0 = (blockIdx.x - b * spans) * LSPAN;
    float* tab = lsm;
    float* X = tab + (size_t)nt * d * NP;  // LSPAN x d increments
    const size_t gq = (size_t)QP * N * d;
    for (int e = threadIdx.x; e < nt * NP * d; e += LNT) {
        const int m = e / (NP * d), r = e - m * NP * d, i = r / d, c = r - i * d;
        float v = 0.f;
        if (i < N) {
            if (m == 0) v = p.tab_f[((size_t)b * N + i) * d + c];
            else if (m <= QP) v = p.tab_g[(size_t)b * gq + ((size_t)(m - 1) * N + i) * d + c];
            else v = p.tab_h[(size_t)b * gq + ((size_t)(m - 1 - QP) * N + i) * d + c];
        }
        tab[(m * d + c) * NP + i] = v;
    }
    for (int e = threadIdx.x; e < LSPAN * d; e += LNT) {
        const int tt = e / d, c = e - tt * d, t = t0 + tt;
        X[e] = t < g.T ? input_increment(p.path, b, t, c, g.T, d, g.flags) : 0.f;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int tt = warp; tt < LSPAN && t0 + tt < g.T; tt += LNT / 32) {
        const float* x = X + tt * d;
        float* dst = p.loc + ((size_t)b * g.T + t0 + tt) * LW;
        for (int m = 0; m < nt; ++m) {
            const float* tm = tab + (size_t)m * d * NP + lane;
            float a0 = 0.f, a1 = 0.f;
            int c = 0;
            for (; c + 1 < d; c += 2) {
                a0 = fmaf(tm[c * NP], x[c], a0);
                a1 = fmaf(tm[(c + 1) * NP], x[c + 1], a1);
            }
            if (c < d) a0 = fmaf(tm[c * NP], x[c], a0);
            dst[m * NP + lane] = a0 + a1;  // [s1 | U_0 .. U_{QP-1} | V_0 .. V_{QP-1}]
        }
    }
}

namespace tc {

// CTA-uniform bounded wait for the MMA commit of the given parity. Returns false on timeout.
__device__ bool tc_wait(const TcSmem& s, uint32_t parity, int limit) {
    if (threadIdx.x == 0) {
        int ok = 0;
        for (int it = 0; it < limit; ++it) {
            if (mbar_try(s.bar, parity)) {
                ok = 1;
                break;
            }
        }
        s.bcast[1] = ok;
    }
    __syncthreads();
    const bool ok = s.bcast[1] != 0;
    fence_after();
    return ok;
}

}  // namespace tc

// The same local terms with the lane's rows of the tables held in registers for the whole span (d_in <= 8,
// q <= 3: ROWS = 1 + 2 QP tables): per interval two broadcast loads of the increments, ROWS x 8 FMAs and
// ROWS coalesced stores.
constexpr int LSPAN_REG = 256;

template <int ROWS>
__global__ void __launch_bounds__(LNT) local_reg_kernel(Params p) {
    __shared__ __align__(16) float X[LSPAN_REG * 8];  // the span's increments, 8 per interval (zero padded)
    const Geom& g = p.g;
    const int N = g.N, d = g.d_in, QP = g.QP, LW = loc_width(QP);
    const int spans = (g.T + LSPAN_REG - 1) / LSPAN_REG;
    const int b = blockIdx.x / spans, t0 = (blockIdx.x - b * spans) * LSPAN_REG;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float tab[ROWS][8];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const float* src = r == 0 ? p.tab_f + ((size_t)b * N + lane) * d
                           : r <= QP ? p.tab_g + (((size_t)b * QP + r - 1) * N + lane) * d
                                     : p.tab_h + (((size_t)b * QP + r - 1 - QP) * N + lane) * d;
#pragma unroll
        for (int c = 0; c < 8; ++c) tab[r][c] = (lane < N && c < d) ? __ldg(src + c) : 0.f;
    }
    for (int e = threadIdx.x; e < LSPAN_REG * 8; e += LNT) {
        const int tt = e >> 3, c = e & 7, t = t0 + tt;
        X[e] = (t < g.T && c < d) ? input_increment(p.path, b, t, c, g.T, d, g.flags) : 0.f;
    }
    __syncthreads();
    const int tend = min(LSPAN_REG, g.T - t0);
    for (int tt = warp; tt < tend; tt += LNT / 32) {
        const float4 x0 = *reinterpret_cast<const float4*>(X + tt * 8);
        const float4 x1 = *reinterpret_cast<const float4*>(X + tt * 8 + 4);
        const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        float* dst = p.loc + ((size_t)b * g.T + t0 + tt) * LW + lane;
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int c = 0; c < 8; c += 2) {
                a0 = fmaf(tab[r][c], x[c], a0);
                a1 = fmaf(tab[r][c + 1], x[c + 1], a1);
            }
            dst[r * NP] = a0 + a1;  // [s1 | U_0 .. U_{QP-1} | V_0 .. V_{QP-1}]
        }
    }
}

// Flow complements of whole chunks, per sample: C(e) = I - M^e for e = Lc and e = the last chunk's
// length, by binary powering of complements (C(a + b) = C(a) + C(b) - C(a) C(b), C(2a) = 2 C(a) - C(a)^2),
// so that no I - (a matrix near I) is ever formed. One CTA of NT threads per sample.
__global__ void __launch_bounds__(NT) power_kernel(Params p) {
    extern __shared__ float smem[];
    const Geom& g = p.g;
    const int b = blockIdx.x;
    const int N = g.N;
    const int i0 = 4 * (threadIdx.x >> 3), j0 = 4 * (threadIdx.x & 7);
    float* Dr = smem;
    float* Dt = smem + MM;
    float* W0 = smem + 2 * MM;  // C(2^j) row-major
    float* W1 = smem + 3 * MM;  // C(2^j) k-major
    float* R = smem + 4 * MM;   // accumulated complement, row-major
    const float* m = p.tab_d + (size_t)b * N * N;
    for (int e = threadIdx.x; e < MM; e += blockDim.x) {
        const int i = e / NP, k = e - i * NP;
        const float v = (i < N && k < N) ? m[i * N + k] : 0.f;
        Dr[i * NP + k] = v;
        Dt[k * NP + i] = v;
    }
    for (int which = 0; which < 2; ++which) {
        const int e_len = which == 0 ? g.Lc : g.T - (g.C - 1) * g.Lc;
        __syncthreads();
        for (int e = threadIdx.x; e < MM; e += blockDim.x) {
            R[e] = 0.f;
            W0[e] = Dr[e];
            W1[e] = Dt[e];
        }
        __syncthreads();
        int e = e_len;
        while (e > 0) {
            float blk[4][4], Rb[4][4], Bb[4][4];
            load_rowmajor(W0, Bb, i0, j0);
            if (e & 1) {
                load_rowmajor(R, Rb, i0, j0);
                gemm44(W1, R, blk, i0, j0, false);
                __syncthreads();
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int q = 0; q < 4; ++q) blk[r][q] = Rb[r][q] + Bb[r][q] - blk[r][q];
                store_rowmajor(R, blk, i0, j0);
                __syncthreads();
            }
            e >>= 1;
            if (e > 0) {
                gemm44(W1, W0, blk, i0, j0, false);
                __syncthreads();
#pragma unroll
                for (int r = 0; r < 4; ++r)
#pragma unroll
                    for (int q = 0; q < 4; ++q) blk[r][q] = 2.f * Bb[r][q] - blk[r][q];
                store_rowmajor(W0, blk, i0, j0);
                store_kmajor(W1, blk, i0, j0);
                __syncthreads();
            }
        }
        float* dst = p.pw + ((size_t)b * 2 + which) * MM;
        for (int q = threadIdx.x; q < MM; q += blockDim.x) dst[q] = R[q];
    }
}

namespace tc {
// Smem of the output pass (fwd_tc_kernel): operands, transposition buffers, D k-major and the per-tile vectors
// only (72 KB at q = 3, three CTAs per SM).
__host__ __device__ inline size_t tc_out_smem_bytes(int QP) {
    const size_t f = 2 * MM + 2 * 4 * MM + TILES * 32 * RQS + MM + TILES * vec_per_tile(QP);
    return f * sizeof(float) + 64 + 128;
}

__device__ TcSmem tc_carve_out(unsigned char* raw, const Geom& g) {
    uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 127) & ~(uintptr_t)127;
    float* p = reinterpret_cast<float*>(base);
    TcSmem s{};
    s.Bhi = p; p += MM;
    s.Blo = p; p += MM;
    s.Ahi = p; p += 4 * MM;
    s.Alo = p; p += 4 * MM;
    s.RQ = p; p += TILES * 32 * RQS;
    s.Dt = p; p += MM;
    s.vec = p; p += TILES * vec_per_tile(g.QP);
    s.bar = reinterpret_cast<uint64_t*>(p);
    s.tmem = reinterpret_cast<uint32_t*>(p + 2);
    s.bcast = reinterpret_cast<int*>(p + 4);
    return s;
}
}  // namespace tc

// The forward's output pass on tcgen05: a CTA of 4 warps stacks 4 chunks of one sample (M = 128 rows), runs
// each from its carry (computed by agg_kernel and the carry scan) and writes the prefix rows. Per step
// X = S2 - S2 D^T and M X = X - D X are 3xTF32 products in TMEM.
__global__ void __launch_bounds__(tc::NTH, 3) fwd_tc_kernel(Params p) {
    using namespace tc;
    extern __shared__ unsigned char smem_raw[];
    const Geom& g = p.g;
    TcSmem s = tc_carve_out(smem_raw, g);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int N = g.N;
    const int mbar_limit = 1 << 20;

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(s.bar)), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s.tmem)),
                     "r"(64));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *s.tmem;
    const uint32_t tP1 = tmem, tP2 = tmem + 32;
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    uint32_t phase = 0;
    bool failed = false;
    bool mma_pending = false;  // an MMA commit of `phase` may still be outstanding after a failed wait

    const uint64_t dA_hi = smem_desc(smem_u32(s.Ahi), 2048, 128), dA_lo = smem_desc(smem_u32(s.Alo), 2048, 128);
    const uint64_t dB_hi = smem_desc(smem_u32(s.Bhi), 512, 128), dB_lo = smem_desc(smem_u32(s.Blo), 512, 128);
    const int groups = (g.C + TILES - 1) / TILES;
    const int ntiles = g.B * groups;
    float* vt = s.vec + warp * vec_per_tile(g.QP);  // S1 | u | two local-term slots
    float* RQt = s.RQ + warp * 32 * RQS;
    const int LW = loc_width(g.QP);
    // terminal readout (run by the backward): the window's states go to the scratch rows, not to `out`
    const bool term = g.readout == EWS_READOUT_TERMINAL;
    (void)ntiles;

    for (;;) {
        if (tid == 0) s.bcast[0] = atomicAdd(&p.st->ticket, 1);
        __syncthreads();
        const int tile = s.bcast[0];
        __syncthreads();
        if (tile >= g.B * g.ngrp) break;
        const int grp = g.grp0 + tile / g.B, b = tile - (grp - g.grp0) * g.B;
        const int c_me = grp * TILES + warp;
        const bool valid_me = c_me < g.C;
        const int t0_me = c_me * g.Lc;
        const int len_me = valid_me ? min(g.Lc, g.T - t0_me) : 0;
        int steps = 0;
        for (int t = 0; t < TILES; ++t) {
            const int c = grp * TILES + t;
            if (c < g.C) steps = max(steps, min(g.Lc, g.T - c * g.Lc));
        }
        tc_load_tables(p, s, b);
        __syncthreads();

        // the chunk's carry; a chunk that ends early keeps feeding the MMAs (its rows are not written)
        float col[32];
        {
            const float* cs = p.carry + ((size_t)b * g.C + (valid_me ? c_me : 0)) * g.SW;
#pragma unroll
            for (int n = 0; n < 32; ++n) col[n] = valid_me ? ldcg(cs + MM + NP + n * NP + lane) : 0.f;
            vt[lane] = valid_me ? ldcg(cs + MM + lane) : 0.f;
        }
        float* wrows = term ? window_rows(p, grp, warp, b) : nullptr;
        if (term && len_me > 0 && lane < N) {
            // scratch row 0: the chunk's carry, the state its first interval starts from
            if (lane == 0) wrows[0] = 1.f;
            wrows[1 + lane] = vt[lane];
#pragma unroll
            for (int n = 0; n < 32; ++n)
                if (n < N) wrows[1 + N + n * N + lane] = col[n];
        }
        __syncwarp();
        // the intervals' local terms (computed by local_kernel), copied in one interval ahead
        if (len_me > 0) fetch_loc(p, b, t0_me, vt + 2 * NP, LW);
        cp_async_commit();
            for (int k = 0; k < steps; ++k) {
                const bool live = k < len_me;
                cp_async_wait<0>();
                __syncwarp();
                const float* stg = vt + 2 * NP + (k & 1) * LW;  // this interval's [s1 | U | V]
                if (k + 1 < len_me) fetch_loc(p, b, t0_me + k + 1, vt + 2 * NP + ((k + 1) & 1) * LW, LW);
                cp_async_commit();
                // E0: the lane's column of S2 -> its row (through the exchange buffer) -> A operand row
                float srow[32];
#pragma unroll
                for (int n = 0; n < 32; ++n) RQt[n * RQS + lane] = col[n];
                __syncwarp();
#pragma unroll
                for (int n = 0; n < 32; ++n) srow[n] = RQt[lane * RQS + n];
                __syncwarp();
                store_a_row(s.Ahi, s.Alo, 32 * warp + lane, srow);
                fence_proxy_async();
                fence_before();
                __syncthreads();
                if (tid == 0) {
                    fence_after();
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) mma_tf32(tP1, dA_hi + (ks * 4096 >> 4), dB_hi + (ks * 1024 >> 4), ks > 0);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) mma_tf32(tP1, dA_hi + (ks * 4096 >> 4), dB_lo + (ks * 1024 >> 4), 1);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) mma_tf32(tP1, dA_lo + (ks * 4096 >> 4), dB_hi + (ks * 1024 >> 4), 1);
                    mma_commit(s.bar);
                }
                // u = M S1 while the tensor core runs
                tc_u(s, vt);
                if (!tc_wait(s, phase, mbar_limit)) {
                    failed = mma_pending = true;
                    break;
                }
                phase ^= 1;
                // E1: row `lane` of X = S2 - S2 D^T -> column `lane` of X -> A operand row of X^T
                float xcol[32];
                {
                    float pr[32];
                    tmem_ld32(tP1 + lane_off, pr);
#pragma unroll
                    for (int n = 0; n < 32; ++n) RQt[lane * RQS + n] = srow[n] - pr[n];
                    __syncwarp();
#pragma unroll
                    for (int n = 0; n < 32; ++n) xcol[n] = RQt[n * RQS + lane];
                    __syncwarp();
                    store_a_row(s.Ahi, s.Alo, 32 * warp + lane, xcol);
                }
                fence_proxy_async();
                fence_before();
                __syncthreads();
                if (tid == 0) {
                    fence_after();
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) mma_tf32(tP2, dA_hi + (ks * 4096 >> 4), dB_hi + (ks * 1024 >> 4), ks > 0);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) mma_tf32(tP2, dA_hi + (ks * 4096 >> 4), dB_lo + (ks * 1024 >> 4), 1);
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) mma_tf32(tP2, dA_lo + (ks * 4096 >> 4), dB_hi + (ks * 1024 >> 4), 1);
                    mma_commit(s.bar);
                }
                if (!tc_wait(s, phase, mbar_limit)) {
                    failed = mma_pending = true;
                    break;
                }
                phase ^= 1;
                // E2: column `lane` of M X + u s1^T + U V^T
                {
                    float q2[32];
                    tmem_ld32(tP2 + lane_off, q2);
                    const float* u = vt + NP;
                    const float* s1 = stg;
                    const float s1l = s1[lane];
#pragma unroll
                    for (int n = 0; n < 32; ++n) col[n] = xcol[n] - q2[n];
                    axpy32_bc(col, u, s1l);
                    for (int a = 0; a < g.QP; ++a)
                        axpy32_bc(col, stg + NP + a * NP, stg[NP + g.QP * NP + a * NP + lane]);
                    const float s1new = u[lane] + s1l;
                    __syncwarp();
                    if (live) vt[lane] = s1new;
                    fence_before();
                    __syncwarp();
                    if (live && lane < N && (!term || k + 1 < len_me)) {
                        // the prefix row straight from registers: each level-2 row is one contiguous run
                        // (terminal: the state the next interval starts from, scratch row k + 1)
                        float* row = term ? wrows + (size_t)(k + 1) * g.W : p.out + ((size_t)b * g.T + t0_me + k) * g.W;
                        if (lane == 0) row[0] = 1.f;
                        row[1 + lane] = s1new;
#pragma unroll
                        for (int n = 0; n < 32; ++n)
                            if (n < N) row[1 + N + n * N + lane] = col[n];
                    }
                }
            }
        if (failed) break;
        __syncthreads();
    }
    // every exit drains the tensor core and frees TMEM
    if (failed && tid == 0) {
        if (atomicCAS(&p.st->error, 0, EWS_ERR_LOOKBACK_TIMEOUT) == 0) p.st->err_tile = -1;
        if (mma_pending)
            for (int it = 0; it < (1 << 20); ++it)
                if (mbar_try(s.bar, phase)) break;
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(64));
}

// ---------------------------------------------------------------------------------- chunk aggregates

// Power complements E_j = I - M^j for j = 0..Lc of each sample (one CTA per sample, four 64-thread groups),
// by doubling: with E_1..E_m known, E_{m+i} = E_m + E_i - E_m E_i for i = 1..m (all powers of M commute, so
// the complement composition needs no order). E_0 = 0, E_1 = D.
constexpr int PWT = 256;

__global__ void __launch_bounds__(PWT) powers_kernel(Params p) {
    __shared__ __align__(16) float Emt[MM];       // E_m, k-major
    __shared__ __align__(16) float Ei[4][MM];     // per group: E_i, row-major
    const Geom& g = p.g;
    const int b = blockIdx.x, N = g.N, Lc = g.Lc;
    const int grp = threadIdx.x >> 6, gt = threadIdx.x & 63;
    const int i0 = 4 * (gt >> 3), j0 = 4 * (gt & 7);
    float* E = p.pows + (size_t)b * (Lc + 1) * MM;
    const float* d = p.tab_d + (size_t)b * N * N;
    for (int e = threadIdx.x; e < MM; e += PWT) {
        const int i = e / NP, k = e - i * NP;
        E[e] = 0.f;
        E[MM + e] = (i < N && k < N) ? d[i * N + k] : 0.f;
    }
    __syncthreads();
    for (int m = 1; m < Lc; m *= 2) {
        for (int e = threadIdx.x; e < MM; e += PWT) {
            const int i = e / NP, k = e - i * NP;
            Emt[k * NP + i] = E[(size_t)m * MM + e];
        }
        __syncthreads();
        const int cnt = min(m, Lc - m);
        for (int i = 1 + grp; i <= cnt; i += 4) {
            for (int e = gt; e < MM; e += 64) Ei[grp][e] = E[(size_t)i * MM + e];
            asm volatile("bar.sync %0, 64;" ::"r"(1 + grp));
            float blk[4][4], em[4][4], ei[4][4];
            gemm44(Emt, Ei[grp], blk, i0, j0, false);
            load_rowmajor(Ei[grp], ei, i0, j0);
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) em[r][c] = Emt[(j0 + c) * NP + i0 + r];
#pragma unroll
            for (int r = 0; r < 4; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) blk[r][c] = em[r][c] + ei[r][c] - blk[r][c];
            store_rowmajor(E + (size_t)(m + i) * MM, blk, i0, j0);
            asm volatile("bar.sync %0, 64;" ::"r"(1 + grp));
        }
        __syncthreads();
    }
}

// Zero-carry aggregates of every chunk without running its chain. With the chunk's local terms
// Z_t = u_t s1_t^T + sum_a U_{t,a} V_{t,a}^T (u_t = M S1_{t-1} from the chunk's own level-1 recursion) the
// level-2 aggregate is A2 = sum_t M^{L-1-t} Z_t M^{(L-1-t)T} = sum_t sum_r (M^{L-1-t} x_{t,r}) (M^{L-1-t} y_{t,r})^T,
// a rank-(q+2) update per interval instead of a 32 x 32 x 32 conjugation, and every interval is independent
// once the powers are known (applied as complements, w = x - E x). One warp per chunk, lane = state row;
// the interval's local terms and its power complement E are copied in with cp.async one interval ahead
// (E rows padded to AGS floats so that the lanes' 16-byte reads of their rows fall in distinct banks).
constexpr int AGW = 4;   // warps per CTA
constexpr int AGS = 36;  // row stride of a staged power complement

__host__ __device__ inline int agg_warp_floats(int QP) {
    return 2 * loc_width(QP) + 2 * NP * AGS + 2 * NP + (QMAX + 1) * NP;
}

template <int QP>
__global__ void __launch_bounds__(AGW * 32, 4) agg_kernel(Params p) {
    extern __shared__ __align__(16) float agsm[];
    const Geom& g = p.g;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = blockIdx.x * AGW + warp;
    if (chunk >= g.B * g.C) return;
    const int b = chunk / g.C, c = chunk - b * g.C;
    const int N = g.N, LW = loc_width(QP), Lc = g.Lc;
    const int t0 = c * Lc, len = min(Lc, g.T - t0);
    float* locb = agsm + (size_t)warp * agg_warp_floats(QP);  // 2 x LW
    float* Eb = locb + 2 * LW;                                 // 2 x NP x AGS
    float* S1v = Eb + 2 * NP * AGS;                            // the chunk's level 1 (broadcast copy)
    float* uv = S1v + NP;                                      // u = M S1_{t-1}
    float* wy = uv + NP;                                       // (QP + 1) x NP: the flowed y vectors
    float drow[NP];
    {
        const float* d = p.tab_d + (size_t)b * N * N;
#pragma unroll
        for (int k = 0; k < NP; ++k) drow[k] = (lane < N && k < N) ? d[lane * N + k] : 0.f;
    }
    float a2[NP];
#pragma unroll
    for (int k = 0; k < NP; ++k) a2[k] = 0.f;
    float s1 = 0.f;
    S1v[lane] = 0.f;
    const float* Ebase = p.pows + (size_t)b * (Lc + 1) * MM;
    auto fetch = [&](int k) {
        float* eb = Eb + (k & 1) * NP * AGS;
        const float* src = Ebase + (size_t)(len - 1 - k) * MM;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const int e = lane + 32 * v;  // 16-byte piece e: row e / 8, column 4 (e % 8)
            cp_async16(eb + (e >> 3) * AGS + 4 * (e & 7), src + 4 * e);
        }
        tc::fetch_loc(p, b, t0 + k, locb + (k & 1) * LW, LW);
        cp_async_commit();
    };
    fetch(0);
    for (int k = 0; k < len; ++k) {
        cp_async_wait<0>();
        __syncwarp();
        const float* loc = locb + (k & 1) * LW;  // [s1 | U_0..U_{QP-1} | V_0..V_{QP-1}]
        const float* er = Eb + (k & 1) * NP * AGS + lane * AGS;
        if (k + 1 < len) fetch(k + 1);
        // u = S1 - D S1 (the level-1 state before this interval, flowed one step)
        float du0 = 0.f, du1 = 0.f;
#pragma unroll
        for (int q = 0; q < NP; q += 4) {
            const float4 v = *reinterpret_cast<const float4*>(S1v + q);
            du0 = fmaf(drow[q], v.x, du0);
            du1 = fmaf(drow[q + 1], v.y, du1);
            du0 = fmaf(drow[q + 2], v.z, du0);
            du1 = fmaf(drow[q + 3], v.w, du1);
        }
        const float u = s1 - (du0 + du1);
        uv[lane] = u;
        __syncwarp();
        // (E x_r)[lane], (E y_r)[lane] for every term at once: x = u, U_a; y = s1, V_a
        float ex[QP + 1], ey[QP + 1];
#pragma unroll
        for (int r = 0; r <= QP; ++r) ex[r] = ey[r] = 0.f;
#pragma unroll
        for (int q = 0; q < NP; q += 4) {
            const float4 e4 = *reinterpret_cast<const float4*>(er + q);
#pragma unroll
            for (int r = 0; r <= QP; ++r) {
                const float* x = r == 0 ? uv : loc + NP * r;
                const float* y = r == 0 ? loc : loc + NP * (QP + r);
                const float4 xv = *reinterpret_cast<const float4*>(x + q);
                const float4 yv = *reinterpret_cast<const float4*>(y + q);
                ex[r] = fmaf(e4.x, xv.x, fmaf(e4.y, xv.y, fmaf(e4.z, xv.z, fmaf(e4.w, xv.w, ex[r]))));
                ey[r] = fmaf(e4.x, yv.x, fmaf(e4.y, yv.y, fmaf(e4.z, yv.z, fmaf(e4.w, yv.w, ey[r]))));
            }
        }
        float wx[QP + 1];
#pragma unroll
        for (int r = 0; r <= QP; ++r) {
            const float* x = r == 0 ? uv : loc + NP * r;
            const float* y = r == 0 ? loc : loc + NP * (QP + r);
            wx[r] = x[lane] - ex[r];
            wy[r * NP + lane] = y[lane] - ey[r];
        }
        __syncwarp();
#pragma unroll
        for (int r = 0; r <= QP; ++r) {
#pragma unroll
            for (int q = 0; q < NP; q += 4) {
                const float4 yv = *reinterpret_cast<const float4*>(wy + r * NP + q);
                a2[q] = fmaf(wx[r], yv.x, a2[q]);
                a2[q + 1] = fmaf(wx[r], yv.y, a2[q + 1]);
                a2[q + 2] = fmaf(wx[r], yv.z, a2[q + 2]);
                a2[q + 3] = fmaf(wx[r], yv.w, a2[q + 3]);
            }
        }
        // S1 <- u + s1 of this interval (every lane has read S1v and uv before the barrier above)
        s1 = u + loc[lane];
        S1v[lane] = s1;
    }
    cp_async_wait<0>();
    // the slot: [flow complement C(len) | S1 | S2 row-major]
    float* as = p.agg + ((size_t)b * g.C + c) * g.SW;
    const float* C = p.pw + ((size_t)b * 2 + (c == g.C - 1 ? 1 : 0)) * MM;
    for (int e = lane; e < MM; e += 32) as[e] = C[e];
    as[MM + lane] = s1;
    float4* row = reinterpret_cast<float4*>(as + MM + NP + lane * NP);
#pragma unroll
    for (int q = 0; q < NP / 4; ++q) row[q] = make_float4(a2[4 * q], a2[4 * q + 1], a2[4 * q + 2], a2[4 * q + 3]);
}

// The same chunk aggregates with both contractions of an interval on the tensor cores (warp-level
// m16n8k8 tf32 MMAs, 3xTF32 split): the flowed vectors E [x_r | y_r] (E = E_j, 32 x 32, against the
// interval's 2 (QP + 1) vectors, two 16-wide N tiles) and the rank-(QP + 1) update W_X W_Y^T of the level-2
// aggregate. Operands are read from shared memory in fragment order (tiles padded so that every fragment
// load is conflict-free), so the warp-wide broadcast reads of the vectors are gone. Each interval's update
// is formed in a zeroed MMA accumulator and added to the running aggregate with CUDA-core (round to
// nearest) additions, so the tensor core's accumulation rounding never applies to the growing sum.
constexpr int AXS = 36;  // row stride of the vector tile (16 rows: x_0..x_7 | y_0..y_7)
constexpr int AWS = 12;  // row stride of the W_X / W_Y tiles (32 rows x 8)

__host__ __device__ inline int agg_mma_warp_floats() { return 2 * 16 * AXS + 2 * NP * AGS + NP + 2 * NP * AWS; }

__device__ __forceinline__ uint32_t tf32_hi(float v) { return tc::tf32_bits(v); }
__device__ __forceinline__ uint32_t tf32_lo(float v, uint32_t hi) { return tc::tf32_bits(v - __uint_as_float(hi)); }

__device__ __forceinline__ void mma_m16n8k8(float d[4], const uint32_t a[4], const uint32_t b[2]) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// d += A B in 3xTF32 (hi hi + hi lo + lo hi) from fp32 fragments
__device__ __forceinline__ void mma3_m16n8k8(float d[4], const float a[4], const float b[2]) {
    uint32_t ah[4], al[4], bh[2], bl[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        ah[i] = tf32_hi(a[i]);
        al[i] = tf32_lo(a[i], ah[i]);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        bh[i] = tf32_hi(b[i]);
        bl[i] = tf32_lo(b[i], bh[i]);
    }
    mma_m16n8k8(d, ah, bh);
    mma_m16n8k8(d, ah, bl);
    mma_m16n8k8(d, al, bh);
}

template <int QP>
__global__ void __launch_bounds__(AGW * 32, 3) agg_mma_kernel(Params p) {
    extern __shared__ __align__(16) float agsm[];
    const Geom& g = p.g;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = blockIdx.x * AGW + warp;
    if (chunk >= g.B * g.C) return;
    const int b = chunk / g.C, c = chunk - b * g.C;
    const int N = g.N, Lc = g.Lc;
    const int t0 = c * Lc, len = min(Lc, g.T - t0);
    const int gq = lane >> 2, cq = lane & 3;  // fragment coordinates
    float* Xb = agsm + (size_t)warp * agg_mma_warp_floats();  // 2 x 16 x AXS: rows x_0 = u, x_{1+a} = U_a, y_0 = s1, y_{1+a} = V_a
    float* Eb = Xb + 2 * 16 * AXS;                             // 2 x NP x AGS
    float* S1v = Eb + 2 * NP * AGS;                            // the chunk's level 1 (broadcast copy)
    float* WX = S1v + NP;                                      // NP x AWS: W_X[i][r]
    float* WY = WX + NP * AWS;                                 // NP x AWS: W_Y[i][r]
    // the pad rows of both vector tiles stay zero (the copies fill rows 1..QP, 8..8+QP; row 0 is u)
    for (int e = lane; e < 2 * 16 * AXS; e += 32) Xb[e] = 0.f;
    float drow[NP];
    {
        const float* d = p.tab_d + (size_t)b * N * N;
#pragma unroll
        for (int k = 0; k < NP; ++k) drow[k] = (lane < N && k < N) ? d[lane * N + k] : 0.f;
    }
    float a2[2][4][4];  // the aggregate's level 2 in accumulator-fragment order: [m tile][n tile][value]
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int v = 0; v < 4; ++v) a2[mt][nt][v] = 0.f;
    float s1 = 0.f;
    S1v[lane] = 0.f;
    __syncwarp();
    const float* Ebase = p.pows + (size_t)b * (Lc + 1) * MM;
    auto fetch = [&](int k) {
        float* eb = Eb + (k & 1) * NP * AGS;
        const float* src = Ebase + (size_t)(len - 1 - k) * MM;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const int e = lane + 32 * v;  // 16-byte piece e: row e / 8, column 4 (e % 8)
            cp_async16(eb + (e >> 3) * AGS + 4 * (e & 7), src + 4 * e);
        }
        // [s1 | U_0..U_{QP-1} | V_0..V_{QP-1}] -> rows 8, 1..QP, 9..8+QP of the vector tile
        float* xb = Xb + (k & 1) * 16 * AXS;
        const float* lsrc = p.loc + ((size_t)b * g.T + t0 + k) * loc_width(QP);
        for (int v = lane; v < (1 + 2 * QP) * 8; v += 32) {
            const int vec = v >> 3, piece = v & 7;
            const int row = vec == 0 ? 8 : vec <= QP ? vec : 8 + (vec - QP);
            cp_async16(xb + row * AXS + 4 * piece, lsrc + 4 * v);
        }
        cp_async_commit();
    };
    fetch(0);
    for (int k = 0; k < len; ++k) {
        cp_async_wait<0>();
        __syncwarp();
        float* X = Xb + (k & 1) * 16 * AXS;
        const float* E = Eb + (k & 1) * NP * AGS;
        if (k + 1 < len) fetch(k + 1);
        // u = S1 - D S1 (the level-1 state before this interval, flowed one step) -> row 0
        float du0 = 0.f, du1 = 0.f;
#pragma unroll
        for (int q = 0; q < NP; q += 4) {
            const float4 v = *reinterpret_cast<const float4*>(S1v + q);
            du0 = fmaf(drow[q], v.x, du0);
            du1 = fmaf(drow[q + 1], v.y, du1);
            du0 = fmaf(drow[q + 2], v.z, du0);
            du1 = fmaf(drow[q + 3], v.w, du1);
        }
        const float u = s1 - (du0 + du1);
        X[lane] = u;
        __syncwarp();
        // EX[i][n] = sum_k E[i][k] X[n][k]: A = E (row-major), B[k][n] = X[n][k]
        float ex[2][2][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int v = 0; v < 4; ++v) ex[mt][nt][v] = 0.f;
#pragma unroll
        for (int sk = 0; sk < 4; ++sk) {
            float af[2][4], bf[2][2];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const float* er = E + (16 * mt + gq) * AGS + 8 * sk + cq;
                af[mt][0] = er[0];
                af[mt][1] = er[8 * AGS];
                af[mt][2] = er[4];
                af[mt][3] = er[8 * AGS + 4];
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                const float* xr = X + (8 * nt + gq) * AXS + 8 * sk + cq;
                bf[nt][0] = xr[0];
                bf[nt][1] = xr[4];
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) mma3_m16n8k8(ex[mt][nt], af[mt], bf[nt]);
        }
        // W = X^T - EX at the accumulator positions -> W_X (n < 8) and W_Y (n >= 8)
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int i = 16 * mt + gq + 8 * (v >> 1), n = 2 * cq + (v & 1);
                    const float w = X[(8 * nt + n) * AXS + i] - ex[mt][nt][v];
                    (nt == 0 ? WX : WY)[i * AWS + n] = w;
                }
        __syncwarp();
        // a2 += W_X W_Y^T (K = the vectors r, zero beyond QP): A[i][r] = W_X, B[r][q] = W_Y[q][r]
        {
            float af[2][4], bf[4][2];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const float* wr = WX + (16 * mt + gq) * AWS + cq;
                af[mt][0] = wr[0];
                af[mt][1] = wr[8 * AWS];
                af[mt][2] = wr[4];
                af[mt][3] = wr[8 * AWS + 4];
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const float* wr = WY + (8 * nt + gq) * AWS + cq;
                bf[nt][0] = wr[0];
                bf[nt][1] = wr[4];
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    float dd[4] = {0.f, 0.f, 0.f, 0.f};
                    mma3_m16n8k8(dd, af[mt], bf[nt]);
#pragma unroll
                    for (int v = 0; v < 4; ++v) a2[mt][nt][v] += dd[v];
                }
        }
        // S1 <- u + s1 of this interval (every lane has read S1v, X and the W tiles before the barriers above)
        s1 = u + X[8 * AXS + lane];
        __syncwarp();
        S1v[lane] = s1;
    }
    cp_async_wait<0>();
    // the slot: [flow complement C(len) | S1 | S2 row-major]
    float* as = p.agg + ((size_t)b * g.C + c) * g.SW;
    const float* C = p.pw + ((size_t)b * 2 + (c == g.C - 1 ? 1 : 0)) * MM;
    for (int e = lane; e < MM; e += 32) as[e] = C[e];
    as[MM + lane] = s1;
    float* S2 = as + MM + NP;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = 16 * mt + gq + 8 * h, q = 8 * nt + 2 * cq;
                *reinterpret_cast<float2*>(S2 + i * NP + q) = make_float2(a2[mt][nt][2 * h], a2[mt][nt][2 * h + 1]);
            }
}

template <int QP>
static int launch_agg(const Params& p, cudaStream_t s) {
    if (QP <= 7) {  // the tensor-core form (2 (QP + 1) <= 16 vectors); the CUDA-core one beyond
        const size_t smem = sizeof(float) * (size_t)AGW * agg_mma_warp_floats();
        cudaFuncSetAttribute(agg_mma_kernel<(QP <= 7 ? QP : 7)>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        agg_mma_kernel<(QP <= 7 ? QP : 7)><<<(p.g.B * p.g.C + AGW - 1) / AGW, AGW * 32, smem, s>>>(p);
        return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
    }
    const size_t smem = sizeof(float) * (size_t)AGW * agg_warp_floats(QP);
    cudaFuncSetAttribute(agg_kernel<QP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    agg_kernel<QP><<<(p.g.B * p.g.C + AGW - 1) / AGW, AGW * 32, smem, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

static int launch_agg_q(const Params& p, cudaStream_t s) {
    switch (p.g.QP) {
        case 1: return launch_agg<1>(p, s);
        case 2: return launch_agg<2>(p, s);
        case 3: return launch_agg<3>(p, s);
        case 4: return launch_agg<4>(p, s);
        case 5: return launch_agg<5>(p, s);
        case 6: return launch_agg<6>(p, s);
        case 7: return launch_agg<7>(p, s);
        case 8: return launch_agg<8>(p, s);
        case 9: return launch_agg<9>(p, s);
        case 10: return launch_agg<10>(p, s);
        case 11: return launch_agg<11>(p, s);
        case 12: return launch_agg<12>(p, s);
    }
    return EWS_ERR_UNSUPPORTED;
}

// ---------------------------------------------------------------------------------- backward chunk aggregates

// mma.sync without `volatile`: the products have no side effects, so the compiler may interleave the three
// 3xTF32 passes of independent accumulators instead of issuing each accumulator's passes back to back.
__device__ __forceinline__ void mma_tf32_free(float d[4], const uint32_t a[4], const uint32_t b[2]) {
    asm("mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

template <int K>
__device__ __forceinline__ void tf32_split(const float (&v)[K], uint32_t (&hi)[K], uint32_t (&lo)[K]) {
#pragma unroll
    for (int i = 0; i < K; ++i) {
        hi[i] = tf32_hi(v[i]);
        lo[i] = tf32_lo(v[i], hi[i]);
    }
}

constexpr int BGW = 4;   // warps per CTA of bagg_kernel
constexpr int BES = 40;  // row stride of a staged power complement: B and transposed-A fragment reads conflict-free
constexpr int BGS = 36;  // row stride of a staged gradient tile: A fragment and float4 row reads conflict-free
constexpr int BHS = 40;  // row stride of the staged H = G M^(j+1): B fragment reads conflict-free
__host__ __device__ inline int bagg_warp_floats() { return 2 * NP * BES + 2 * NP * BGS + NP * BHS + 6 * NP; }

// The zero-carry local adjoints (mu1, mu2) of every chunk without a chain. Run from zero over a chunk, the
// reverse recursion l2 <- M^T l2 M + G_j, l1 <- M^T (l1 + l2 s1_j) + g1_j telescopes into the flow powers
// P_j = M^(j+1) = I - E_(j+1) (j the interval's index in its chunk, E the forward's power complements):
//     mu2 = sum_j P_j^T G_j P_j,      mu1 = sum_j P_j^T (g1_j + G_j s^_j),
// with s^_j = M s^_(j-1) + s1_j the chunk's level 1 from a zero start. Every term is independent: per interval
// two 32 x 32 x 32 products on the tensor core (3xTF32 mma.sync), H = G - G E and mu2 += H - E^T H (each
// through a zeroed accumulator, added on the CUDA cores), and mu1 += w - E^T w with w = g1 + G s^. One warp
// per chunk; the next interval's E, G, s1 and g1 are copied in (cp.async) while this one's products run.
__global__ void __launch_bounds__(BGW * 32, 2) bagg_kernel(Params p) {
    extern __shared__ __align__(16) float bgsm[];
    const Geom& g = p.g;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int chunk = blockIdx.x * BGW + warp;
    if (chunk >= g.B * g.C) return;
    const int b = chunk / g.C, c = chunk - b * g.C;
    const int N = g.N, Lc = g.Lc;
    const int t0 = c * Lc, len = min(Lc, g.T - t0);
    float* as = p.agg + ((size_t)b * g.C + c) * g.SW;
    if (g.readout == EWS_READOUT_TERMINAL && c != g.C - 1) {
        // terminal readout: only the sequence's last chunk has a cotangent
#pragma unroll 4
        for (int n = 0; n < NP; ++n) as[MM + NP + n * NP + lane] = 0.f;
        as[MM + lane] = 0.f;
        return;
    }
    const int gq = lane >> 2, cq = lane & 3;  // fragment coordinates
    float* Eb = bgsm + (size_t)warp * bagg_warp_floats();  // 2 x NP x BES: E_(j+1)
    float* Gb = Eb + 2 * NP * BES;                          // 2 x NP x BGS: G_j (zero beyond N)
    float* Hs = Gb + 2 * NP * BGS;                          // NP x BHS
    float* Vb = Hs + NP * BHS;                              // 2 x [s1_j | g1_j]
    float* sh = Vb + 4 * NP;                                // s^ (broadcast copy)
    float* wv = sh + NP;                                    // w (broadcast copy)
    for (int e = lane; e < 2 * NP * BGS; e += 32) Gb[e] = 0.f;
    for (int e = lane; e < 6 * NP; e += 32) Vb[e] = 0.f;
    float drow[NP];
    {
        const float* d = p.tab_d + (size_t)b * N * N;
#pragma unroll
        for (int k = 0; k < NP; ++k) drow[k] = (lane < N && k < N) ? d[lane * N + k] : 0.f;
    }
    float m2[2][4][4];  // mu2 in accumulator-fragment order: [m tile][n tile][value]
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int v = 0; v < 4; ++v) m2[mt][nt][v] = 0.f;
    float m1 = 0.f, shat = 0.f;  // mu1[lane], s^[lane]
    __syncwarp();
    const float* Ebase = p.pows + (size_t)b * (Lc + 1) * MM;
    const int LW = loc_width(g.QP);
    auto fetch = [&](int k) {
        float* eb = Eb + (k & 1) * NP * BES;
        const float* src = Ebase + (size_t)(k + 1) * MM;
#pragma unroll
        for (int v = 0; v < 8; ++v) {
            const int e = lane + 32 * v;  // 16-byte piece e: row e / 8, column 4 (e % 8)
            cp_async16(eb + (e >> 3) * BES + 4 * (e & 7), src + 4 * e);
        }
        float* vb = Vb + (k & 1) * 2 * NP;
        if (lane < 8) cp_async16(vb + 4 * lane, p.loc + ((size_t)b * g.T + t0 + k) * LW + 4 * lane);
        float* gb = Gb + (k & 1) * NP * BGS;
        const float* gr = grad_row(p, b, t0 + k);
        if (lane < N) {
            if (gr) {
                cp_async4(vb + NP + lane, gr + 1 + lane);
                for (int i = 0; i < N; ++i) cp_async4(gb + i * BGS + lane, gr + 1 + N + i * N + lane);
            } else {
                vb[NP + lane] = 0.f;
                for (int i = 0; i < N; ++i) gb[i * BGS + lane] = 0.f;
            }
        }
        cp_async_commit();
    };
    fetch(0);
    for (int k = 0; k < len; ++k) {
        cp_async_wait<0>();
        __syncwarp();
        const float* E = Eb + (k & 1) * NP * BES;
        const float* G = Gb + (k & 1) * NP * BGS;
        const float* vb = Vb + (k & 1) * 2 * NP;
        if (k + 1 < len) fetch(k + 1);
        // s^ <- s^ - D s^ + s1_j
        float du0 = 0.f, du1 = 0.f;
#pragma unroll
        for (int q = 0; q < NP; q += 4) {
            const float4 v = *reinterpret_cast<const float4*>(sh + q);
            du0 = fmaf(drow[q], v.x, du0);
            du1 = fmaf(drow[q + 1], v.y, du1);
            du0 = fmaf(drow[q + 2], v.z, du0);
            du1 = fmaf(drow[q + 3], v.w, du1);
        }
        shat = (shat - (du0 + du1)) + vb[lane];
        __syncwarp();
        sh[lane] = shat;
        __syncwarp();
        // w = g1 + G s^ (row `lane` of G)
        float w0 = vb[NP + lane], w1 = 0.f;
#pragma unroll
        for (int q = 0; q < NP; q += 4) {
            const float4 gv = *reinterpret_cast<const float4*>(G + lane * BGS + q);
            const float4 sv = *reinterpret_cast<const float4*>(sh + q);
            w0 = fmaf(gv.x, sv.x, w0);
            w1 = fmaf(gv.y, sv.y, w1);
            w0 = fmaf(gv.z, sv.z, w0);
            w1 = fmaf(gv.w, sv.w, w1);
        }
        const float w = w0 + w1;
        wv[lane] = w;
        // GE = G E (A = G row-major, B[k][n] = E[k][n]); H = G - GE at the accumulator positions
        float h[2][4][4];
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int v = 0; v < 4; ++v) h[mt][nt][v] = 0.f;
#pragma unroll
        for (int sk = 0; sk < 4; ++sk) {
            float af[2][4], bf[4][2];
            uint32_t ah[2][4], al[2][4], bh[4][2], bl[4][2];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                const float* gr = G + (16 * mt + gq) * BGS + 8 * sk + cq;
                af[mt][0] = gr[0];
                af[mt][1] = gr[8 * BGS];
                af[mt][2] = gr[4];
                af[mt][3] = gr[8 * BGS + 4];
                tf32_split(af[mt], ah[mt], al[mt]);
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const float* er = E + (8 * sk + cq) * BES + 8 * nt + gq;
                bf[nt][0] = er[0];
                bf[nt][1] = er[4 * BES];
                tf32_split(bf[nt], bh[nt], bl[nt]);
            }
            // the three passes over all eight accumulators (hi hi, hi lo, lo hi: each accumulator's order as
            // in mma3_m16n8k8)
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) mma_tf32_free(h[mt][nt], ah[mt], bh[nt]);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) mma_tf32_free(h[mt][nt], ah[mt], bl[nt]);
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) mma_tf32_free(h[mt][nt], al[mt], bh[nt]);
        }
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int i = 16 * mt + gq + 8 * (v >> 1), n = 8 * nt + 2 * cq + (v & 1);
                    h[mt][nt][v] = G[i * BGS + n] - h[mt][nt][v];
                    Hs[i * BHS + n] = h[mt][nt][v];
                }
        __syncwarp();
        // E^T H (A[i][k] = E[k][i], B[k][n] = H[k][n]); mu2 += H - E^T H
        {
            float tt[2][4][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int v = 0; v < 4; ++v) tt[mt][nt][v] = 0.f;
#pragma unroll
            for (int sk = 0; sk < 4; ++sk) {
                float af[2][4], bf[4][2];
                uint32_t ah[2][4], al[2][4], bh[4][2], bl[4][2];
#pragma unroll
                for (int mt = 0; mt < 2; ++mt) {
                    const float* ec = E + (8 * sk + cq) * BES + 16 * mt + gq;
                    af[mt][0] = ec[0];
                    af[mt][1] = ec[8];
                    af[mt][2] = ec[4 * BES];
                    af[mt][3] = ec[4 * BES + 8];
                    tf32_split(af[mt], ah[mt], al[mt]);
                }
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    const float* hr = Hs + (8 * sk + cq) * BHS + 8 * nt + gq;
                    bf[nt][0] = hr[0];
                    bf[nt][1] = hr[4 * BHS];
                    tf32_split(bf[nt], bh[nt], bl[nt]);
                }
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt) mma_tf32_free(tt[mt][nt], ah[mt], bh[nt]);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt) mma_tf32_free(tt[mt][nt], ah[mt], bl[nt]);
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int nt = 0; nt < 4; ++nt) mma_tf32_free(tt[mt][nt], al[mt], bh[nt]);
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                    for (int v = 0; v < 4; ++v) m2[mt][nt][v] += h[mt][nt][v] - tt[mt][nt][v];
        }
        // mu1 += w - E^T w
        float tw0 = 0.f, tw1 = 0.f;
#pragma unroll
        for (int q = 0; q < NP; q += 2) {
            tw0 = fmaf(E[q * BES + lane], wv[q], tw0);
            tw1 = fmaf(E[(q + 1) * BES + lane], wv[q + 1], tw1);
        }
        m1 += w - (tw0 + tw1);
        __syncwarp();  // H, w and this interval's buffers are read before the next interval writes them
    }
    cp_async_wait<0>();
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int i = 16 * mt + gq + 8 * (v >> 1), n = 8 * nt + 2 * cq + (v & 1);
                as[MM + NP + i * NP + n] = m2[mt][nt][v];
            }
    as[MM + lane] = m1;
}

// ---------------------------------------------------------------------------------- 256-thread products
// The scans' Chen products and transposed Chen maps with 256 threads (a 2 x 2 block each) instead of the
// look-back's 64: the scans are sequential chains of these products, so their latency is the scans' cost.
constexpr int CST = 256;

// acc = A B on the thread's 2 x 2 block; At is A stored k-major, Bm row-major.
__device__ __forceinline__ void gemm22(const float* __restrict__ At, const float* __restrict__ Bm, float acc[2][2],
                                       int i0, int j0) {
    acc[0][0] = acc[0][1] = acc[1][0] = acc[1][1] = 0.f;
#pragma unroll 8
    for (int k = 0; k < NP; ++k) {
        const float2 a = *reinterpret_cast<const float2*>(At + k * NP + i0);
        const float2 b = *reinterpret_cast<const float2*>(Bm + k * NP + j0);
        acc[0][0] = fmaf(a.x, b.x, acc[0][0]);
        acc[0][1] = fmaf(a.x, b.y, acc[0][1]);
        acc[1][0] = fmaf(a.y, b.x, acc[1][0]);
        acc[1][1] = fmaf(a.y, b.y, acc[1][1]);
    }
}

__device__ __forceinline__ void ld22(const float* M, float v[2][2], int i0, int j0) {
    const float2 r0 = *reinterpret_cast<const float2*>(M + i0 * NP + j0);
    const float2 r1 = *reinterpret_cast<const float2*>(M + (i0 + 1) * NP + j0);
    v[0][0] = r0.x;
    v[0][1] = r0.y;
    v[1][0] = r1.x;
    v[1][1] = r1.y;
}

__device__ __forceinline__ void st22(float* M, const float v[2][2], int i0, int j0) {
    *reinterpret_cast<float2*>(M + i0 * NP + j0) = make_float2(v[0][0], v[0][1]);
    *reinterpret_cast<float2*>(M + (i0 + 1) * NP + j0) = make_float2(v[1][0], v[1][1]);
}

// (Po, S1o, S2o) = (PL, L1, L2) (x) (PR, R1, R2), flows as complements:
//   S2 = P_R L2 P_R^T + (P_R L1) R1^T + R2,  S1 = P_R L1 + R1,  C = C_L + C_R - C_R C_L  (P_R = I - C_R).
// Outputs may alias either operand. Scratch T0, T1 (MM), vtmp (NP). Barrier-complete on return.
__device__ void chen_mul_256(const float* PL, const float* L1, const float* L2, const float* PR, const float* R1,
                             const float* R2, float* Po, float* S1o, float* S2o, float* T0, float* T1, float* vtmp) {
    const int i0 = 2 * (threadIdx.x >> 4), j0 = 2 * (threadIdx.x & 15);
    for (int e = threadIdx.x; e < MM; e += CST) {
        const int i = e / NP, k = e - i * NP;
        T0[k * NP + i] = L2[e];
        T1[k * NP + i] = PR[e];
    }
    if (threadIdx.x < NP) {
        float a0 = 0.f, a1 = 0.f;
        for (int k = 0; k < NP; k += 2) {
            a0 = fmaf(PR[threadIdx.x * NP + k], L1[k], a0);
            a1 = fmaf(PR[threadIdx.x * NP + k + 1], L1[k + 1], a1);
        }
        vtmp[threadIdx.x] = L1[threadIdx.x] - (a0 + a1);  // P_R L1
    }
    __syncthreads();
    float L2b[2][2], CLb[2][2], CRb[2][2], X[2][2], Pq[2][2], Y[2][2];
    ld22(L2, L2b, i0, j0);
    ld22(PL, CLb, i0, j0);
    ld22(PR, CRb, i0, j0);
    gemm22(T0, T1, X, i0, j0);  // L2 C_R^T
    gemm22(T1, PL, Pq, i0, j0);  // C_R C_L
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
            X[r][c] = L2b[r][c] - X[r][c];
            Pq[r][c] = CLb[r][c] + CRb[r][c] - Pq[r][c];
        }
    __syncthreads();
    st22(T0, X, i0, j0);
    __syncthreads();
    gemm22(T1, T0, Y, i0, j0);  // C_R X
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c)
            Y[r][c] = (X[r][c] - Y[r][c]) + fmaf(vtmp[i0 + r], R1[j0 + c], R2[(i0 + r) * NP + j0 + c]);
    __syncthreads();
    st22(S2o, Y, i0, j0);
    st22(Po, Pq, i0, j0);
    if (threadIdx.x < NP) S1o[threadIdx.x] = vtmp[threadIdx.x] + R1[threadIdx.x];
    __syncthreads();
}

// (L1, L2r) <- J(G)^T (L1, L2r) for G = (C row-major in Pr, level 1 U1v): L2 <- P^T L2 P,
// L1 <- P^T (L1 + L2 U1), P = I - C. Scratch T0 (MM), T1, vt (NP). Barrier-complete on return.
__device__ void apply_JT_256(const float* Pr, const float* U1v, float* L1, float* L2r, float* T0, float* T1, float* vt) {
    const int i0 = 2 * (threadIdx.x >> 4), j0 = 2 * (threadIdx.x & 15);
    if (threadIdx.x < NP) {
        float a0 = 0.f, a1 = 0.f;
        for (int k = 0; k < NP; k += 2) {
            a0 = fmaf(L2r[threadIdx.x * NP + k], U1v[k], a0);
            a1 = fmaf(L2r[threadIdx.x * NP + k + 1], U1v[k + 1], a1);
        }
        vt[threadIdx.x] = L1[threadIdx.x] + (a0 + a1);
    }
    float Z[2][2], L2b[2][2];
    gemm22(Pr, L2r, Z, i0, j0);  // C^T L2 (Pr read k-major is C^T)
    ld22(L2r, L2b, i0, j0);
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) Z[r][c] = L2b[r][c] - Z[r][c];  // P^T L2
    __syncthreads();
    // Z k-major
    T0[j0 * NP + i0] = Z[0][0];
    T0[(j0 + 1) * NP + i0] = Z[0][1];
    T0[j0 * NP + i0 + 1] = Z[1][0];
    T0[(j0 + 1) * NP + i0 + 1] = Z[1][1];
    if (threadIdx.x < NP) {
        float a0 = 0.f, a1 = 0.f;
        for (int k = 0; k < NP; k += 2) {
            a0 = fmaf(Pr[k * NP + threadIdx.x], vt[k], a0);
            a1 = fmaf(Pr[(k + 1) * NP + threadIdx.x], vt[k + 1], a1);
        }
        T1[threadIdx.x] = vt[threadIdx.x] - (a0 + a1);  // P^T (L1 + L2 U1)
    }
    __syncthreads();
    float W[2][2];
    gemm22(T0, Pr, W, i0, j0);  // Z C
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) W[r][c] = Z[r][c] - W[r][c];  // Z P
    st22(L2r, W, i0, j0);
    if (threadIdx.x < NP) L1[threadIdx.x] = T1[threadIdx.x];
    __syncthreads();
}

// Carries of every chunk from the precomputed aggregates, by a two-level scan over each sample's chunks
// instead of the chain kernel's look-back (whose first wave would walk back through every earlier aggregate):
//   scan_local_kernel:  per group of CG chunks, the inclusive products within the group (into `incl`);
//   scan_round_kernel:  the inclusive products of the group totals, in log2(groups) parallel rounds;
//   scan_fix_kernel:    per chunk, carry = (groups before) (x) incl(previous chunk of the group), and for the
//                       terminal readout the sample's total as its output row.
// Chen products are chen_mul_256, in a fixed order, so the carries are deterministic.
constexpr int CG = 8;

struct ScanSmem {
    float P0[MM], S10[NP], S20[MM];  // accumulator
    float P1[MM], S11[NP], S21[MM];  // operand
    float T0[MM], T1[MM], vtmp[NP];
};

__host__ __device__ inline int scan_groups(int C) { return (C + CG - 1) / CG; }

__global__ void __launch_bounds__(CST) scan_local_kernel(Params p) {
    __shared__ __align__(16) ScanSmem sm;
    const Geom& g = p.g;
    const int ng = scan_groups(g.C);
    const int b = blockIdx.x / ng, k = blockIdx.x - b * ng;
    const int c0 = k * CG, c1 = min(g.C, c0 + CG);
    const size_t base = (size_t)b * g.C;
    load_slot_smem(p.agg + (base + c0) * g.SW, sm.P0, sm.S10, sm.S20);
    SlotRegs nx;
    if (c0 + 1 < c1) slot_fetch(p.agg + (base + c0 + 1) * g.SW, nx);
    __syncthreads();
    store_slot(p.incl + (base + c0) * g.SW, sm.P0, sm.S10, sm.S20);
    for (int c = c0 + 1; c < c1; ++c) {
        slot_put(nx, sm.P1, sm.S11, sm.S21);
        __syncthreads();
        if (c + 1 < c1) slot_fetch(p.agg + (base + c + 1) * g.SW, nx);  // in flight during the product
        chen_mul_256(sm.P0, sm.S10, sm.S20, sm.P1, sm.S11, sm.S21, sm.P0, sm.S10, sm.S20, sm.T0, sm.T1, sm.vtmp);
        store_slot(p.incl + (base + c) * g.SW, sm.P0, sm.S10, sm.S20);
        __syncthreads();
    }
}

// One round of the group scan (Hillis-Steele, log2 of the group count rounds over B x groups CTAs):
// X_k <- X_{k-d} (x) X_k for k >= d. Round 0 (src == nullptr) reads the group totals, the inclusive value of
// each group's last chunk; after the last round X_k is the product of groups 0..k.
__global__ void __launch_bounds__(CST) scan_round_kernel(Params p, const float* src, float* dst, int d) {
    __shared__ __align__(16) ScanSmem sm;
    const Geom& g = p.g;
    const int ng = scan_groups(g.C);
    const int b = blockIdx.x / ng, k = blockIdx.x - b * ng;
    auto elem = [&](int j) -> const float* {
        return src ? src + ((size_t)b * ng + j) * g.SW
                   : p.incl + ((size_t)b * g.C + min(g.C, (j + 1) * CG) - 1) * g.SW;
    };
    load_slot_smem(elem(k), sm.P1, sm.S11, sm.S21);
    if (k >= d) {
        load_slot_smem(elem(k - d), sm.P0, sm.S10, sm.S20);
        __syncthreads();
        chen_mul_256(sm.P0, sm.S10, sm.S20, sm.P1, sm.S11, sm.S21, sm.P1, sm.S11, sm.S21, sm.T0, sm.T1, sm.vtmp);
    }
    __syncthreads();
    store_slot(dst + ((size_t)b * ng + k) * g.SW, sm.P1, sm.S11, sm.S21);
}

__global__ void __launch_bounds__(CST) scan_fix_kernel(Params p) {
    __shared__ __align__(16) ScanSmem sm;
    const Geom& g = p.g;
    const int ng = scan_groups(g.C);
    const int b = blockIdx.x / g.C, c = blockIdx.x - b * g.C;
    const int k = c / CG;
    const size_t base = (size_t)b * g.C;
    // the product of the earlier groups (the group scan's value of group k - 1; the identity for group 0)
    if (k > 0)
        load_slot_smem(p.gex + ((size_t)b * ng + k - 1) * g.SW, sm.P0, sm.S10, sm.S20);
    else
        identity_smem(sm.P0, sm.S10, sm.S20);
    __syncthreads();
    if (c > k * CG) {
        load_slot_smem(p.incl + (base + c - 1) * g.SW, sm.P1, sm.S11, sm.S21);
        __syncthreads();
        chen_mul_256(sm.P0, sm.S10, sm.S20, sm.P1, sm.S11, sm.S21, sm.P0, sm.S10, sm.S20, sm.T0, sm.T1, sm.vtmp);
    }
    store_slot(p.carry + (base + c) * g.SW, sm.P0, sm.S10, sm.S20);
    if (c == g.C - 1 && g.readout == EWS_READOUT_TERMINAL) {
        // the sample's terminal value: carry (x) the last chunk's aggregate
        load_slot_smem(p.agg + (base + c) * g.SW, sm.P1, sm.S11, sm.S21);
        __syncthreads();
        chen_mul_256(sm.P0, sm.S10, sm.S20, sm.P1, sm.S11, sm.S21, sm.P0, sm.S10, sm.S20, sm.T0, sm.T1, sm.vtmp);
        const int N = g.N;
        float* row = p.out + (size_t)b * g.W;
        if (threadIdx.x == 0) row[0] = 1.f;
        for (int e = threadIdx.x; e < N; e += blockDim.x) row[1 + e] = sm.S10[e];
        for (int e = threadIdx.x; e < N * N; e += blockDim.x) row[1 + N + e] = sm.S20[(e / N) * NP + (e % N)];
    }
}

// ---------------------------------------------------------------------------------- backward

// The backward's carries by a two-level reverse scan, the counterpart of the forward's (scan_*_kernel).
// The element of a range of chunks is (G, mu): the forward aggregate G of the range and the cotangent mu at
// the range's start from the range's own output gradients (zero carry). An earlier range a and a later b
// combine to (G_a (x) G_b, J(G_a)^T mu_b + mu_a), with J(G)^T the transposed Chen map (apply_JT_256).
//   bscan_local_kernel:  per group, the suffix elements from every chunk to the group's end (gsuf, incl);
//   bscan_round_kernel:  the suffix elements of the groups, in log2(groups) parallel rounds;
//   bscan_fix_kernel:    per chunk, the cotangent arriving at its end (lcarry), J(suffix after it)^T lam + mu.
struct BScanSmem {
    float P0[MM], S10[NP], S20[MM];  // accumulated G
    float P1[MM], S11[NP], S21[MM];  // G of a chunk
    float L2r[MM], L1[NP];           // accumulated cotangent
    float T0[MM], T1[MM], v1[NP], v2[NP], v3[NP];
};

__device__ void bscan_add_mu(BScanSmem& sm, const float* slot) {
    for (int e = threadIdx.x; e < MM; e += blockDim.x) sm.L2r[e] += ldcg(slot + MM + NP + e);
    if (threadIdx.x < NP) sm.L1[threadIdx.x] += ldcg(slot + MM + threadIdx.x);
}

__device__ void bscan_store_lam(float* slot, const BScanSmem& sm) {
    for (int e = threadIdx.x; e < MM; e += blockDim.x) slot[MM + NP + e] = sm.L2r[e];
    if (threadIdx.x < NP) slot[MM + threadIdx.x] = sm.L1[threadIdx.x];
}

// L <- J(G)^T L for G in (P1, S11) (its flow complement row-major and level 1)
__device__ void bscan_apply(BScanSmem& sm) {
    __syncthreads();
    apply_JT_256(sm.P1, sm.S11, sm.L1, sm.L2r, sm.T0, sm.v1, sm.v2);
}

__global__ void __launch_bounds__(CST) bscan_local_kernel(Params p) {
    __shared__ __align__(16) BScanSmem sm;
    const Geom& g = p.g;
    const int ng = scan_groups(g.C);
    const int b = blockIdx.x / ng, k = blockIdx.x - b * ng;
    const int c0 = k * CG, c1 = min(g.C, c0 + CG) - 1;
    const size_t base = (size_t)b * g.C;
    load_slot_smem(p.fagg + (base + c1) * g.SW, sm.P0, sm.S10, sm.S20);
    for (int e = threadIdx.x; e < MM; e += blockDim.x) sm.L2r[e] = 0.f;
    if (threadIdx.x < NP) sm.L1[threadIdx.x] = 0.f;
    __syncthreads();
    bscan_add_mu(sm, p.agg + (base + c1) * g.SW);
    __syncthreads();
    store_slot(p.gsuf + (base + c1) * g.SW, sm.P0, sm.S10, sm.S20);
    bscan_store_lam(p.incl + (base + c1) * g.SW, sm);
    // the next chunk's aggregate G_c and local cotangent mu_c, fetched one step ahead
    SlotRegs ng_, nm_;
    if (c1 - 1 >= c0) {
        slot_fetch(p.fagg + (base + c1 - 1) * g.SW, ng_);
        slot_fetch(p.agg + (base + c1 - 1) * g.SW, nm_);
    }
    for (int c = c1 - 1; c >= c0; --c) {
        slot_put(ng_, sm.P1, sm.S11, sm.S21);
        SlotRegs mu = nm_;
        if (c - 1 >= c0) {
            slot_fetch(p.fagg + (base + c - 1) * g.SW, ng_);
            slot_fetch(p.agg + (base + c - 1) * g.SW, nm_);
        }
        __syncthreads();
        bscan_apply(sm);  // mu <- J(G_c)^T mu
#pragma unroll
        for (int k = 0; k < MM / 256; ++k) sm.L2r[threadIdx.x + 256 * k] += mu.s2[k];  // + mu_c
        if (threadIdx.x < NP) sm.L1[threadIdx.x] += mu.s1;
        __syncthreads();
        chen_mul_256(sm.P1, sm.S11, sm.S21, sm.P0, sm.S10, sm.S20, sm.P0, sm.S10, sm.S20, sm.T0, sm.T1, sm.v3);
        store_slot(p.gsuf + (base + c) * g.SW, sm.P0, sm.S10, sm.S20);
        bscan_store_lam(p.incl + (base + c) * g.SW, sm);
        __syncthreads();
    }
}

// One round of the reverse group scan (Hillis-Steele over the groups): Y_k <- Y_k . Y_{k+d} for k + d < ng,
// elements (G, mu) combined as above. Round 0 (src == nullptr) reads each group's element (the suffix
// aggregate and local cotangent of its first chunk); after the last round Y_k is the element of groups
// k..ng-1. Elements are stored as two slots: G, then mu in the cotangent positions of a slot.
__global__ void __launch_bounds__(CST) bscan_round_kernel(Params p, const float* src, float* dst, int d) {
    __shared__ __align__(16) BScanSmem sm;
    const Geom& g = p.g;
    const int ng = scan_groups(g.C);
    const int b = blockIdx.x / ng, k = blockIdx.x - b * ng;
    auto gslot = [&](int j) -> const float* {
        return src ? src + ((size_t)b * ng + j) * 2 * g.SW : p.gsuf + ((size_t)b * g.C + (size_t)j * CG) * g.SW;
    };
    auto mslot = [&](int j) -> const float* {
        return src ? src + (((size_t)b * ng + j) * 2 + 1) * g.SW : p.incl + ((size_t)b * g.C + (size_t)j * CG) * g.SW;
    };
    float* out = dst + ((size_t)b * ng + k) * 2 * g.SW;
    const int kb = k + d < ng ? k + d : k;  // the later range (or the element itself, copied)
    load_slot_smem(gslot(kb), sm.P0, sm.S10, sm.S20);
    for (int e = threadIdx.x; e < MM; e += blockDim.x) sm.L2r[e] = 0.f;
    if (threadIdx.x < NP) sm.L1[threadIdx.x] = 0.f;
    __syncthreads();
    bscan_add_mu(sm, mslot(kb));
    if (kb != k) {
        load_slot_smem(gslot(k), sm.P1, sm.S11, sm.S21);
        __syncthreads();
        bscan_apply(sm);             // mu_b <- J(G_a)^T mu_b
        bscan_add_mu(sm, mslot(k));  //        + mu_a
        __syncthreads();
        chen_mul_256(sm.P1, sm.S11, sm.S21, sm.P0, sm.S10, sm.S20, sm.P0, sm.S10, sm.S20, sm.T0, sm.T1, sm.v3);
    }
    __syncthreads();
    store_slot(out, sm.P0, sm.S10, sm.S20);
    bscan_store_lam(out + g.SW, sm);
}

__global__ void __launch_bounds__(CST) bscan_fix_kernel(Params p) {
    __shared__ __align__(16) BScanSmem sm;
    const Geom& g = p.g;
    const int ng = scan_groups(g.C);
    const int b = blockIdx.x / g.C, c = blockIdx.x - b * g.C;
    const int k = c / CG, last = min(g.C, (k + 1) * CG) - 1;
    const size_t base = (size_t)b * g.C;
    if (k + 1 < ng) {
        // the cotangent arriving at the group's end: the mu of the later groups' combined element
        const float* src = p.gex + (((size_t)b * ng + k + 1) * 2 + 1) * g.SW;
        for (int e = threadIdx.x; e < MM; e += blockDim.x) sm.L2r[e] = ldcg(src + MM + NP + e);
        if (threadIdx.x < NP) sm.L1[threadIdx.x] = ldcg(src + MM + threadIdx.x);
    } else {
        for (int e = threadIdx.x; e < MM; e += blockDim.x) sm.L2r[e] = 0.f;
        if (threadIdx.x < NP) sm.L1[threadIdx.x] = 0.f;
    }
    __syncthreads();
    if (c < last) {
        load_slot_smem(p.gsuf + (base + c + 1) * g.SW, sm.P1, sm.S11, sm.S21);
        __syncthreads();
        bscan_apply(sm);
        bscan_add_mu(sm, p.incl + (base + c + 1) * g.SW);
        __syncthreads();
    }
    bscan_store_lam(p.lcarry + (base + c) * g.SW, sm);
}

// ---------------------------------------------------------------------------------- tensor-core backward
//
// The adjoint chain. With l~_t = l_t + g_t (the cotangent of S_t after adding row t of the output
// gradient) the reverse recursion of one interval is
//     l~2_{t-1} = M^T l~2_t M + g2_{t-1},      l~1_{t-1} = M^T (l~1_t + l~2_t s1_t) + g1_{t-1},
// the forward's M S M^T with D replaced by D^T. Each chunk's local adjoint mu (the recursion from zero over
// the chunk) comes from bagg_kernel's power sums, the reverse scan (bscan_*) turns those into the cotangent
// arriving at every chunk's end (`lcarry`), and the exact pass (bwd_exact_kernel) runs every chunk again from
// its carry with the gradient map fused in: two tcgen05 products per step (B operand D^T), four chunks of
// one sample stacked into M = 128; table_grad_kernel forms the table gradients and dx.
namespace tc {
// The cache lines of one output-gradient row (W floats) into L2, spread over the warp's lanes.
__device__ __forceinline__ void prefetch_row_l2(const float* row, int W) {
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(row) & ~(uintptr_t)127;
    const uintptr_t a1 = reinterpret_cast<uintptr_t>(row + W);
    for (uintptr_t a = a0 + 128 * (threadIdx.x & 31); a < a1; a += 32 * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
}
}  // namespace tc

// The exact pass of the adjoint chain with the gradient map fused in (bwd_mode 2). Per step, besides the
// chain's products P = l~2 M (row `lane` in TMEM after the first product) and M^T X, a third product gives
// Z^T = l~2^T M (A operand = the columns of l~2, same B). With S = S2_{t-1} and S1p = S1_{t-1} (prefix row
// t - 1, staged per warp) the interval contributes
//     dM += P S^T + Z^T S + du S1p^T,   du = l~1 + l~2 s1,   ds1 = l~1 + Z^T S1p  (= l~1 + l~2^T M S1p),
//     dU_a = l~2 V_a,   dV_a = l~2^T U_a,
// the same terms as the reverse of ews/core/chen_scan.py:124-152 with the series leaf's local terms. Lane l
// owns row l of dM for its chunk (registers, 32 floats); the S blocks are read as broadcast 4 x 4 tiles,
// each tile serving both the P S^T and the Z^T S terms. The vector cotangents [ds1 | dU_a | dV_a] go to
// `coef` for table_grad_kernel, dM to the chunk's partial slot; no cotangent stream is written.
//
// Shared memory: B (D, transposed orientation), the A operands of l~2 (rows) and of l~2^T (rows = columns
// of l~2), D row-major and per warp l1 | v | the interval's local terms | the staged prefix row. The row /
// column exchanges of the epilogues use the l~2^T operand's space, free at those points (101 KB, two CTAs
// per SM).
namespace tc {
constexpr int XSTG = 1064;  // staged prefix row: S1 at +4, S2 (stride NP) at +36

__host__ __device__ inline int xvec_floats(int QP) { return 2 * NP + loc_width(QP) + XSTG; }

__host__ __device__ inline size_t tc_exact_smem_bytes(int QP) {
    const size_t f = 2 * MM + 4 * 4 * MM + MM + TILES * (size_t)xvec_floats(QP);
    return f * sizeof(float) + 64 + 128;
}

struct XSmem {
    float *Bhi, *Blo, *A1hi, *A1lo, *A3hi, *A3lo, *Dr, *vec;
    uint64_t* bar;
    uint32_t* tmem;
    int* bcast;
};

__device__ XSmem tc_carve_exact(unsigned char* raw, int QP) {
    uintptr_t base = (reinterpret_cast<uintptr_t>(raw) + 127) & ~(uintptr_t)127;
    float* p = reinterpret_cast<float*>(base);
    XSmem s;
    s.Bhi = p; p += MM;
    s.Blo = p; p += MM;
    s.A1hi = p; p += 4 * MM;
    s.A1lo = p; p += 4 * MM;
    s.A3hi = p; p += 4 * MM;
    s.A3lo = p; p += 4 * MM;
    s.Dr = p; p += MM;
    s.vec = p; p += TILES * xvec_floats(QP);
    s.bar = reinterpret_cast<uint64_t*>(p);
    s.tmem = reinterpret_cast<uint32_t*>(p + 2);
    s.bcast = reinterpret_cast<int*>(p + 4);
    return s;
}

// CTA-uniform bounded wait for the MMA commit of the given parity (the exact pass's smem view).
__device__ bool tc_wait_x(const XSmem& s, uint32_t parity, int limit) {
    if (threadIdx.x == 0) {
        int ok = 0;
        for (int it = 0; it < limit; ++it) {
            if (mbar_try(s.bar, parity)) {
                ok = 1;
                break;
            }
        }
        s.bcast[1] = ok;
    }
    __syncthreads();
    const bool ok = s.bcast[1] != 0;
    fence_after();
    return ok;
}

// The three 3xTF32 K-loops of one product (hi hi, hi lo, lo hi) into the TMEM columns at `d`.
__device__ __forceinline__ void mma3x(uint32_t d, uint64_t a_hi, uint64_t a_lo, uint64_t b_hi, uint64_t b_lo) {
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) mma_tf32(d, a_hi + (ks * 4096 >> 4), b_hi + (ks * 1024 >> 4), ks > 0);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) mma_tf32(d, a_hi + (ks * 4096 >> 4), b_lo + (ks * 1024 >> 4), 1);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) mma_tf32(d, a_lo + (ks * 4096 >> 4), b_hi + (ks * 1024 >> 4), 1);
}
}  // namespace tc

template <bool FULL>
__global__ void __launch_bounds__(tc::NTH, 2) bwd_exact_kernel(Params p) {
    using namespace tc;
    extern __shared__ unsigned char smem_raw[];
    const Geom& g = p.g;
    const int QP = g.QP, LW = loc_width(QP);
    XSmem s = tc_carve_exact(smem_raw, QP);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int N = FULL ? NP : g.N;
    const int mbar_limit = 1 << 20;

    if (tid == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(s.bar)), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s.tmem)),
                     "r"(128));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    fence_before();
    __syncthreads();
    fence_after();
    const uint32_t tmem = *s.tmem;
    const uint32_t tP1 = tmem, tP2 = tmem + 32, tP3 = tmem + 64;
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    uint32_t phase = 0;
    bool failed = false;
    bool mma_pending = false;  // an MMA commit of `phase` may still be outstanding after a failed wait

    const uint64_t dA1_hi = smem_desc(smem_u32(s.A1hi), 2048, 128), dA1_lo = smem_desc(smem_u32(s.A1lo), 2048, 128);
    const uint64_t dA3_hi = smem_desc(smem_u32(s.A3hi), 2048, 128), dA3_lo = smem_desc(smem_u32(s.A3lo), 2048, 128);
    const uint64_t dB_hi = smem_desc(smem_u32(s.Bhi), 512, 128), dB_lo = smem_desc(smem_u32(s.Blo), 512, 128);
    const int groups = (g.C + TILES - 1) / TILES;
    const int ntiles = g.B * groups;
    float* vt = s.vec + warp * xvec_floats(QP);  // l1 (NP) | v (NP) | local terms (LW) | staged prefix row
    float* lb = vt + 2 * NP;                      // [s1 | U_a | V_a] of the current interval
    float* stg = lb + LW;                         // S1p at +4, S2p row-major (stride NP) at +36
    float* RQt = s.A3hi + warp * 32 * RQS;        // exchange buffer, inside the l~2^T operand's space

    // terminal readout: the states come from the window's scratch rows (fwd_tc_kernel ran the window's
    // chunks from their carries just before), not from a prefix stream
    const bool term = g.readout == EWS_READOUT_TERMINAL;
    const float* wrows = nullptr;  // the warp's chunk's scratch rows (terminal)
    int t0_w = 0;                  // the warp's chunk's first interval
    // the row holding S_{t-1}, the state interval t starts from
    auto state_row = [&](int b, int t) -> const float* {
        return term ? wrows + (size_t)(t - t0_w) * g.W : p.out + ((size_t)b * g.T + t - 1) * g.W;
    };

    // The warp's copy of prefix row t - 1 (the state the interval starts from) into the staging rows.
    auto stage_prev = [&](int b, int t) {
        const float* row = state_row(b, t);
        if (FULL) {
            for (int e = lane; e < g.W; e += 32) cp_async4(stg + 3 + e, row + e);
        } else {
            stg[4 + lane] = lane < N ? __ldg(row + 1 + lane) : 0.f;
#pragma unroll 4
            for (int i = 0; i < NP; ++i)
                stg[36 + i * NP + lane] = (i < N && lane < N) ? __ldg(row + 1 + N + i * N + lane) : 0.f;
        }
    };

    (void)ntiles;
    for (;;) {
        if (tid == 0) s.bcast[0] = atomicAdd(&p.st->ticket, 1);
        __syncthreads();
        const int tile = s.bcast[0];
        __syncthreads();
        if (tile >= g.B * g.ngrp) break;
        const int grp = g.grp0 + tile / g.B, b = tile - (grp - g.grp0) * g.B;
        const int c_me = grp * TILES + warp;
        const bool valid_me = c_me < g.C;
        const int t0_me = c_me * g.Lc;
        const int len_me = valid_me ? min(g.Lc, g.T - t0_me) : 0;
        int steps = 0;
        for (int t = 0; t < TILES; ++t) {
            const int c = grp * TILES + t;
            if (c < g.C) steps = max(steps, min(g.Lc, g.T - c * g.Lc));
        }
        if (term) {
            wrows = window_rows(p, grp, warp, b);
            t0_w = t0_me;
        }
        {
            const float* m = p.tab_d + (size_t)b * N * N;
            for (int e = tid; e < MM; e += blockDim.x) {
                const int i = e / NP, k = e - i * NP;
                const float v = (i < N && k < N) ? m[i * N + k] : 0.f;
                s.Dr[i * NP + k] = v;
                const float hi = __uint_as_float(tf32_bits(v));
                s.Bhi[bk_off(k, i)] = hi;
                s.Blo[bk_off(k, i)] = v - hi;
            }
        }
        __syncthreads();

        float dM[32];  // row `lane` of the chunk's dM
#pragma unroll
        for (int j = 0; j < 32; ++j) dM[j] = 0.f;
        float col[32];  // column `lane` of l~2
        {
            const float* cs = p.lcarry + ((size_t)b * g.C + (valid_me ? c_me : 0)) * g.SW;
#pragma unroll
            for (int n = 0; n < 32; ++n) col[n] = valid_me ? ldcg(cs + MM + NP + n * NP + lane) : 0.f;
            vt[lane] = valid_me ? ldcg(cs + MM + lane) : 0.f;
        }
        // Steps run in reverse; a chunk shorter than the tile's longest one (only the sequence's last, whose
        // carry is zero) idles on zero state until its last interval. The gradient, local terms and prefix
        // row of the interval a step starts from are fetched one step ahead (here for the first step).
        // cp.async groups per step: the local terms (waited for at the step's start), then the prefix row
        // (waited for before the dM update).
        if (len_me == steps && len_me > 0) {
            const float* gr = grad_row(p, b, t0_me + len_me - 1);
            if (lane < N && gr) {
#pragma unroll
                for (int n = 0; n < 32; ++n)
                    if (n < N) col[n] += __ldg(gr + 1 + N + n * N + lane);
                vt[lane] += __ldg(gr + 1 + lane);
            }
            fetch_loc(p, b, t0_me + len_me - 1, lb, LW);
            cp_async_commit();
            if (t0_me + len_me - 1 > 0) stage_prev(b, t0_me + len_me - 1);
            cp_async_commit();
        } else {
            cp_async_commit();
            cp_async_commit();
        }
        __syncwarp();
        for (int k = steps - 1; k >= 0; --k) {
            const bool live = k < len_me;
            const bool next = k >= 1 && k - 1 < len_me;  // the step after this one is live
            const int t = t0_me + k;
            cp_async_wait<1>();
            __syncwarp();
            if (k >= 2 && k - 2 < len_me) {
                const float* gp = grad_row(p, b, t - 2);
                if (gp) prefetch_row_l2(gp, g.W);
                if (t >= 3) prefetch_row_l2(state_row(b, t - 2), g.W);
            }
            // E0: rows of l~2 (through the exchange buffer) -> A1; columns of l~2 -> A3
            float srow[32];
#pragma unroll
            for (int n = 0; n < 32; ++n) RQt[n * RQS + lane] = col[n];
            __syncwarp();
#pragma unroll
            for (int n = 0; n < 32; ++n) srow[n] = RQt[lane * RQS + n];
            __syncthreads();  // every warp's exchange is read before A3 is written over it
            store_a_row(s.A1hi, s.A1lo, 32 * warp + lane, srow);
            store_a_row(s.A3hi, s.A3lo, 32 * warp + lane, col);
            fence_proxy_async();
            fence_before();
            __syncthreads();
            if (tid == 0) {
                fence_after();
                mma3x(tP1, dA1_hi, dA1_lo, dB_hi, dB_lo);  // l~2 D (rows)
                mma3x(tP3, dA3_hi, dA3_lo, dB_hi, dB_lo);  // l~2^T D (rows)
                mma_commit(s.bar);
            }
            // vectors while the tensor core runs: du = v = l~1 + l~2 s1; dU_a = l~2 V_a; dV_a = l~2^T U_a
            const float l1t = vt[lane];
            float du = l1t;
            if (live) {
                du += dot32_bc(srow, lb);
                float* co = p.coef + ((size_t)b * g.T + t) * LW;
                for (int a = 0; a < QP; ++a) {
                    co[(1 + a) * NP + lane] = dot32_bc(srow, lb + NP + (QP + a) * NP);  // dU_a = l~2 V_a
                    co[(1 + QP + a) * NP + lane] = dot32_bc(col, lb + NP + a * NP);   // dV_a = l~2^T U_a
                }
            }
            vt[NP + lane] = du;
            __syncwarp();
            // the next interval's local terms (this one's are consumed)
            if (next) fetch_loc(p, b, t - 1, lb, LW);
            cp_async_commit();
            if (!tc_wait_x(s, phase, mbar_limit)) {
                failed = mma_pending = true;
                break;
            }
            phase ^= 1;
            // E1: P = l~2 M (row `lane`), Z^T = l~2^T M (row `lane`); X^T rows -> A1
            float P[32], Zt[32];
            {
                float r[32], xcol[32];
                tmem_ld32(tP1 + lane_off, r);
#pragma unroll
                for (int n = 0; n < 32; ++n) P[n] = srow[n] - r[n];
                tmem_ld32(tP3 + lane_off, r);
#pragma unroll
                for (int n = 0; n < 32; ++n) Zt[n] = col[n] - r[n];
#pragma unroll
                for (int n = 0; n < 32; ++n) RQt[lane * RQS + n] = P[n];
                __syncwarp();
#pragma unroll
                for (int n = 0; n < 32; ++n) xcol[n] = RQt[n * RQS + lane];
                store_a_row(s.A1hi, s.A1lo, 32 * warp + lane, xcol);
            }
            fence_proxy_async();
            fence_before();
            __syncthreads();
            if (tid == 0) {
                fence_after();
                mma3x(tP2, dA1_hi, dA1_lo, dB_hi, dB_lo);  // X^T D (rows) = columns of D^T X
                mma_commit(s.bar);
            }
            // the next interval's gradient, loaded while the tensor core runs
            float gn[32];
            float gn1 = 0.f;
            {
                const float* gr = next ? grad_row(p, b, t - 1) : nullptr;
                const bool ld = gr && lane < N;
#pragma unroll
                for (int n = 0; n < 32; ++n) gn[n] = (ld && n < N) ? __ldg(gr + 1 + N + n * N + lane) : 0.f;
                if (ld) gn1 = __ldg(gr + 1 + lane);
            }
            // l1 <- M^T v + g1 = v - D^T v + g1
            {
                const float* v = vt + NP;
                const float nv = v[lane] - coldot_bc(s.Dr, v, lane);
                __syncwarp();
                vt[lane] = nv + gn1;
            }
            // the gradient of the interval: ds1 and dM (the prefix row t - 1 is needed from here on)
            cp_async_wait<1>();
            __syncwarp();
            if (live) {
                float* co = p.coef + ((size_t)b * g.T + t) * LW;
                if (t > 0) {
                    const float* S1p = stg + 4;
                    const float* S2p = stg + 36;
                    co[lane] = l1t + dot32_bc(Zt, S1p);
                    axpy32_bc(dM, S1p, du);
#pragma unroll
                    for (int jb = 0; jb < 8; ++jb) {
#pragma unroll
                        for (int kb = 0; kb < 8; ++kb) {
                            float sv[4][4];
#pragma unroll
                            for (int r = 0; r < 4; ++r) {
                                const float4 q = *reinterpret_cast<const float4*>(S2p + (4 * jb + r) * NP + 4 * kb);
                                sv[r][0] = q.x;
                                sv[r][1] = q.y;
                                sv[r][2] = q.z;
                                sv[r][3] = q.w;
                            }
#pragma unroll
                            for (int r = 0; r < 4; ++r)
#pragma unroll
                                for (int c = 0; c < 4; ++c) {
                                    dM[4 * jb + r] = fmaf(P[4 * kb + c], sv[r][c], dM[4 * jb + r]);  // P S^T
                                    dM[4 * kb + c] = fmaf(Zt[4 * jb + r], sv[r][c], dM[4 * kb + c]);  // Z^T S
                                }
                        }
                    }
                } else {
                    co[lane] = l1t;  // the first interval starts from the zero state
                }
            }
            __syncwarp();
            if (next && t - 1 > 0) stage_prev(b, t - 1);
            cp_async_commit();
            if (!tc_wait_x(s, phase, mbar_limit)) {
                failed = mma_pending = true;
                break;
            }
            phase ^= 1;
            // E2: column `lane` of M^T X = X - D^T X (X's column re-read from the exchange buffer), plus the
            // next interval's gradient
            {
                float q2[32];
                tmem_ld32(tP2 + lane_off, q2);
#pragma unroll
                for (int n = 0; n < 32; ++n) col[n] = (RQt[n * RQS + lane] + gn[n]) - q2[n];
                fence_before();
                __syncwarp();
            }
        }
        cp_async_wait<0>();
        if (failed) break;
        // the chunk's dM row -> its partial slot (chunk-major, the reduction's order)
        if (valid_me) {
            float* part = p.partials + (size_t)(c_me * g.B + b) * (MM + (size_t)LW * g.d_in) + lane * NP;
#pragma unroll
            for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(part + j) = make_float4(dM[j], dM[j + 1], dM[j + 2], dM[j + 3]);
        }
        __syncthreads();
    }
    // every exit drains the tensor core and frees TMEM
    if (failed && tid == 0) {
        if (atomicCAS(&p.st->error, 0, EWS_ERR_LOOKBACK_TIMEOUT) == 0) p.st->err_tile = -1;
        if (mma_pending)
            for (int it = 0; it < (1 << 20); ++it)
                if (mbar_try(s.bar, phase)) break;
    }
    fence_before();
    __syncthreads();
    fence_after();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(128));
}

namespace gm {
constexpr int TB = 8;  // intervals per block of table_grad_kernel
__host__ __device__ inline int coef_stride(int QP) { return loc_width(QP) + 4; }  // padded row of a staged coefficient block
inline size_t table_smem_bytes(const Geom& g) {
    const size_t rows = (size_t)loc_width(g.QP);
    return sizeof(float) * (2 * align4((int)(rows * g.d_in)) + TB * (size_t)coef_stride(g.QP) + align4(TB * g.d_in));
}
}  // namespace gm

// Table gradients and dx with the tables held in registers (q + 1 <= 4, d_in <= 8): lane l of each warp owns
// the table rows 32 r + l (row r of its block: F, G_a, H_a), all d_in columns, for the whole chunk; the
// warps take the chunk's intervals round robin. Per interval the lane reads its entries of c_t (coalesced),
//   dT[rows, :] += c_t[rows] dx_t^T     (registers),
//   dx_t = sum over the warp of T[rows, :]^T c_t[rows]   (a reduce-scatter of the 8 column sums, 9 shuffles),
// and the warps' dT are summed in warp order at the end.
constexpr int TG_SLAB = 8;    // intervals per staged slab of vector cotangents
constexpr int TG_STAGES = 3;  // slabs in flight

__host__ __device__ inline size_t table_reg_smem_bytes(int Lc, int QP) {
    return sizeof(float) * (8 * (size_t)Lc + (size_t)TG_STAGES * TG_SLAB * loc_width(QP));
}

// Plain (non-multicast) bulk copy of `bytes` from global to this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc::smem_u32(bar)), "r"(bytes)
                 : "memory");
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     tc::smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(tc::smem_u32(bar))
                 : "memory");
}

template <int ROWS>
__global__ void __launch_bounds__(128) table_grad_reg_kernel(Params p) {
    __shared__ __align__(16) float red[ROWS * 32 * 8];
    __shared__ __align__(8) uint64_t tbar[TG_STAGES];
    extern __shared__ __align__(16) float xs[];  // the chunk's increments (8 per interval), then the slab ring
    const Geom& g = p.g;
    const int N = g.N, d = g.d_in, QP = g.QP, LW = loc_width(QP);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x;
    const int c = tile / g.B, b = tile - c * g.B;
    const int t0 = c * g.Lc;
    const int len = min(g.Lc, g.T - t0);
    const int nslab = (len + TG_SLAB - 1) / TG_SLAB;
    float* ring = xs + 8 * g.Lc;
    // the chunk's rows of [ds1 | dU_a | dV_a] are contiguous: slabs of TG_SLAB rows by bulk copies
    const float* cbase = p.coef + ((size_t)b * g.T + t0) * LW;
    auto issue = [&](int sl) {
        const int k0 = sl * TG_SLAB, n = min(TG_SLAB, len - k0);
        bulk_load(ring + (size_t)(sl % TG_STAGES) * TG_SLAB * LW, cbase + (size_t)k0 * LW,
                  (uint32_t)(n * LW * sizeof(float)), tbar + sl % TG_STAGES);
    };
    if (tid == 0) {
        for (int k = 0; k < TG_STAGES; ++k)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tc::smem_u32(tbar + k)), "r"(1));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int sl = 0; sl < min(TG_STAGES, nslab); ++sl) issue(sl);
    }
    float tab[ROWS][8], acc[ROWS][8];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
        const bool ok = lane < N;
        const float* src = r == 0 ? p.tab_f + ((size_t)b * N + lane) * d
                           : r <= QP ? p.tab_g + (((size_t)b * QP + r - 1) * N + lane) * d
                                     : p.tab_h + (((size_t)b * QP + r - 1 - QP) * N + lane) * d;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
            tab[r][cc] = (ok && cc < d) ? src[cc] : 0.f;
            acc[r][cc] = 0.f;
        }
    }
    for (int e = tid; e < len * 8; e += blockDim.x) {
        const int k = e >> 3, cc = e & 7;
        xs[e] = cc < d ? input_increment(p.path, b, t0 + k, cc, g.T, d, g.flags) : 0.f;
    }
    __syncthreads();
    const int lim = 1 << 20;
    int sl = 0;
    for (; sl < nslab; ++sl) {
        const int slot = sl % TG_STAGES;
        const uint32_t par = (uint32_t)(sl / TG_STAGES) & 1u;
        bool ok = false;
        for (int it = 0; it < lim && !ok; ++it) ok = tc::mbar_try(tbar + slot, par);
        if (__syncthreads_or(!ok)) break;  // a copy that never landed: reported below
        const float* cs = ring + (size_t)slot * TG_SLAB * LW + lane;
        const int k0 = sl * TG_SLAB, kend = min(len, k0 + TG_SLAB);
        // the warp's two intervals of the slab (kk, kk + 4), their column sums reduce-scattered together:
        // after the exchanges lane l holds interval l / 16, column 4 bit3(l) + 2 bit2(l) + bit1(l)
        {
            const int kk = k0 + warp;
            const bool two = kk + 4 < kend;
            float sv[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) sv[i] = 0.f;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                if (j == 1 && !two) break;
                if (kk + 4 * j >= kend) break;
                const int kj = kk + 4 * j;
                const float4 x0 = *reinterpret_cast<const float4*>(xs + kj * 8);
                const float4 x1 = *reinterpret_cast<const float4*>(xs + kj * 8 + 4);
                const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int r = 0; r < ROWS; ++r) {
                    const float cur = cs[(kj - k0) * LW + 32 * r];
#pragma unroll
                    for (int cc = 0; cc < 8; ++cc) {
                        acc[r][cc] = fmaf(cur, x[cc], acc[r][cc]);
                        sv[8 * j + cc] = fmaf(tab[r][cc], cur, sv[8 * j + cc]);
                    }
                }
            }
            if (kk < kend) {
                const bool hi16 = (lane & 16) != 0, hi8 = (lane & 8) != 0, hi4 = (lane & 4) != 0;
                const bool hi2 = (lane & 2) != 0;
                float s8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float send = hi16 ? sv[i] : sv[i + 8];
                    const float keep = hi16 ? sv[i + 8] : sv[i];
                    s8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
                }
                float s4[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float send = hi8 ? s8[i] : s8[i + 4];
                    const float keep = hi8 ? s8[i + 4] : s8[i];
                    s4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
                }
                float s2[2];
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const float send = hi4 ? s4[i] : s4[i + 2];
                    const float keep = hi4 ? s4[i + 2] : s4[i];
                    s2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
                }
                float s1;
                {
                    const float send = hi2 ? s2[0] : s2[1];
                    const float keep = hi2 ? s2[1] : s2[0];
                    s1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
                }
                s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
                const int j = (lane >> 4) & 1, col = ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
                if ((lane & 1) == 0 && col < d && (j == 0 || two))
                    p.grad_dx[((size_t)b * g.T + t0 + kk + 4 * j) * d + col] = s1;
            }
        }
        __syncthreads();  // the slot is read: refill it
        if (tid == 0 && sl + TG_STAGES < nslab) issue(sl + TG_STAGES);
    }
    if (sl < nslab) {
        // a bounded wait ran out: report it, let the copies in flight land (bounded) and leave the partial
        if (tid == 0) {
            if (atomicCAS(&p.st->error, 0, EWS_ERR_LOOKBACK_TIMEOUT) == 0) p.st->err_tile = tile;
            for (int k = sl; k < min(nslab, sl + TG_STAGES); ++k) {
                bool done = false;
                for (int it = 0; it < lim && !done; ++it)
                    done = tc::mbar_try(tbar + k % TG_STAGES, (uint32_t)(k / TG_STAGES) & 1u);
            }
        }
        return;
    }
    // the warps' table gradients, summed in warp order
    for (int w = 0; w < 4; ++w) {
        if (warp == w) {
#pragma unroll
            for (int r = 0; r < ROWS; ++r)
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    float* q = red + (r * 32 + lane) * 8 + cc;
                    *q = w == 0 ? acc[r][cc] : *q + acc[r][cc];
                }
        }
        __syncthreads();
    }
    float* part = p.partials + (size_t)tile * (MM + (size_t)LW * d) + MM;
    for (int e = tid; e < LW * d; e += blockDim.x) {
        const int row = e / d, cc = e - row * d;
        part[e] = red[row * 8 + cc];
    }
}

// Table gradients and dx from the vector cotangents of a chunk: with the coefficient rows
// c_t = [ds1 | dU_a | dV_a] and the table rows T = [F | G_a | H_a] (one row per (block, state index)),
//   dT += sum_t c_t dx_t^T,   dx_t = T^T c_t,
// in blocks of TB intervals, every sum in a fixed order.
__global__ void __launch_bounds__(128) table_grad_kernel(Params p) {
    using namespace gm;
    extern __shared__ __align__(16) float smem[];
    const Geom& g = p.g;
    const int N = g.N, d = g.d_in, QP = g.QP, LW = loc_width(QP), CS = coef_stride(QP);
    const int tid = threadIdx.x;
    float* Tab = smem;                      // LW x d
    float* tacc = Tab + align4(LW * d);     // LW x d
    float* cbuf = tacc + align4(LW * d);    // TB x CS
    float* xb = cbuf + TB * CS;             // TB x d
    const int tile = blockIdx.x;
    const int c = tile / g.B, b = tile - c * g.B;
    const int t0 = c * g.Lc;
    const int len = min(g.Lc, g.T - t0);
    for (int e = tid; e < LW * d; e += blockDim.x) {
        const int row = e / d, cc = e - row * d;
        const int blk = row / NP, i = row - blk * NP;
        float v = 0.f;
        if (i < N) {
            if (blk == 0)
                v = p.tab_f[((size_t)b * N + i) * d + cc];
            else if (blk <= QP)
                v = p.tab_g[(((size_t)b * QP + blk - 1) * N + i) * d + cc];
            else
                v = p.tab_h[(((size_t)b * QP + blk - 1 - QP) * N + i) * d + cc];
        }
        Tab[e] = v;
        tacc[e] = 0.f;
    }
    for (int k0 = 0; k0 < len; k0 += TB) {
        const int n = min(TB, len - k0);
        __syncthreads();
        const float* src = p.coef + ((size_t)b * g.T + t0 + k0) * LW;
        for (int v = tid; v < n * (LW / 4); v += blockDim.x) {
            const int kk = v / (LW / 4), q = v - kk * (LW / 4);
            cp_async16(cbuf + kk * CS + 4 * q, src + (size_t)kk * LW + 4 * q);
        }
        cp_async_commit();
        for (int e = tid; e < n * d; e += blockDim.x) {
            const int kk = e / d, cc = e - kk * d;
            xb[e] = input_increment(p.path, b, t0 + k0 + kk, cc, g.T, d, g.flags);
        }
        cp_async_wait<0>();
        __syncthreads();
        for (int e = tid; e < LW; e += blockDim.x) {
            for (int cc = 0; cc < d; ++cc) {
                float acc = tacc[e * d + cc];
                for (int kk = 0; kk < n; ++kk) acc = fmaf(cbuf[kk * CS + e], xb[kk * d + cc], acc);
                tacc[e * d + cc] = acc;
            }
        }
        for (int q = tid; q < n * d; q += blockDim.x) {
            const int kk = q / d, cc = q - kk * d;
            const float* cr = cbuf + kk * CS;
            float a0 = 0.f, a1 = 0.f;
            for (int e = 0; e < LW; e += 2) {
                a0 = fmaf(Tab[e * d + cc], cr[e], a0);
                a1 = fmaf(Tab[(e + 1) * d + cc], cr[e + 1], a1);
            }
            p.grad_dx[((size_t)b * g.T + t0 + k0 + kk) * d + cc] = a0 + a1;
        }
    }
    __syncthreads();
    float* part = p.partials + (size_t)tile * (MM + (size_t)LW * d) + MM;
    for (int e = tid; e < LW * d; e += blockDim.x) part[e] = tacc[e];
}


// Deterministic per-sample reduction over chunks, compacted to the real dimensions. A CTA takes 32
// consecutive outputs; its eight warps sum interleaved eighths of the chunks (warp w: chunks w, w + 8, ...)
// and the eight partial sums are added in warp order, so the result does not depend on the schedule.
constexpr int RED_SLICES = 8;

__global__ void __launch_bounds__(32 * RED_SLICES) reduce_kernel(Params p, float* grad_d, float* grad_f, float* grad_g,
                                                                 float* grad_h) {
    __shared__ float part[RED_SLICES][32];
    const Geom& g = p.g;
    const int N = g.N, d = g.d_in;
    const int tabn = (1 + 2 * g.QP) * NP * d;
    const int stride = MM + tabn;
    const int per_sample = N * N + (1 + 2 * g.QP) * N * d;
    const size_t total = (size_t)g.B * per_sample;
    const int lane = threadIdx.x & 31, slice = threadIdx.x >> 5;
    const size_t e = (size_t)blockIdx.x * 32 + lane;
    int b = 0, r = 0, off = 0;
    float* dst = nullptr;
    if (e < total) {
        b = (int)(e / per_sample);
        r = (int)(e - (size_t)b * per_sample);
        if (r < N * N) {
            const int i = r / N, j = r - i * N;
            off = i * NP + j;
            dst = grad_d + (size_t)b * N * N + r;
        } else {
            const int q = r - N * N, blk = q / (N * d), rem = q - blk * N * d, i = rem / d, cc = rem - i * d;
            off = MM + blk * NP * d + i * d + cc;
            if (blk == 0) dst = grad_f + (size_t)b * N * d + rem;
            else if (blk <= g.QP) dst = grad_g + ((size_t)b * g.QP + (blk - 1)) * N * d + rem;
            else dst = grad_h + ((size_t)b * g.QP + (blk - 1 - g.QP)) * N * d + rem;
        }
    }
    float acc = 0.f;
    if (dst)
#pragma unroll 4
        for (int cr = slice; cr < g.C; cr += RED_SLICES) acc += p.partials[((size_t)cr * g.B + b) * stride + off];
    part[slice][lane] = acc;
    __syncthreads();
    if (slice == 0 && dst) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < RED_SLICES; ++k) s += part[k][lane];
        *dst = r < N * N ? -s : s;  // the flow block accumulates dL/dM; dL/dD = -dL/dM
    }
}

// ---------------------------------------------------------------------------------- host side

// A second stream per (host thread, device) for the forward's independent prologue kernels, forked from
// and joined back into the caller's stream with events (both capture into a CUDA graph as a fork / join).
// Created on the first call outside a capture; while none exists a capturing call stays on one stream.
struct SideStream {
    cudaStream_t s2 = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};

static SideStream* side_stream(cudaStream_t s) {
    constexpr int kMaxDev = 64;
    thread_local SideStream per_dev[kMaxDev];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return nullptr;
    SideStream& ss = per_dev[dev];
    if (!ss.s2) {
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return nullptr;
        if (cudaStreamCreateWithFlags(&ss.s2, cudaStreamNonBlocking) != cudaSuccess) {
            ss.s2 = nullptr;
            return nullptr;
        }
        if (cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
            cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
            cudaStreamDestroy(ss.s2);
            ss.s2 = nullptr;
            return nullptr;
        }
    }
    return &ss;
}

static int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

static int make_geom(const ews_dense_args* a, Geom* g) {
    if (!a || a->batch <= 0 || a->steps <= 0 || a->d_in <= 0 || a->dim <= 0) return EWS_ERR_INVALID_ARGUMENT;
    if (a->depth != 2 || a->dim > NP || a->d_in > 32) return EWS_ERR_UNSUPPORTED;
    if (a->series_q < 0 || a->series_q + 1 > QMAX) return EWS_ERR_UNSUPPORTED;
    if (!(a->flags & EWS_F_UNIFORM)) return EWS_ERR_UNSUPPORTED;
    if (a->readout != EWS_READOUT_PREFIX && a->readout != EWS_READOUT_TERMINAL) return EWS_ERR_INVALID_ARGUMENT;
    if ((a->flags & EWS_F_BF16) && !(a->flags & EWS_F_INCREMENTS)) return EWS_ERR_INVALID_ARGUMENT;
    g->B = a->batch;
    g->T = a->steps;
    g->d_in = a->d_in;
    g->N = a->dim;
    g->QP = a->series_q + 1;
    g->W = 1 + g->N + g->N * g->N;
    g->SW = MM + NP + MM;
    g->readout = a->readout;
    g->flags = a->flags;
    g->spin_limit = a->spin_limit > 0 ? a->spin_limit : kDefaultSpinLimit;
    if (a->chunk > 0) {
        g->Lc = a->chunk;
    } else {
        // The chains stack 4 chunks of a sample per CTA: the forward's output pass runs 3 CTAs per SM, the
        // backward's exact pass 2 (the zero-carry adjoints are power sums, whose cost does not depend on the
        // chunk length). Pick the chunk length that minimises the passes' waves x (steps + a per-tile
        // overhead of ~10 steps), weighted by their measured costs per wave-step (~5.8 us for the output
        // pass, ~11.7 us for the exact pass at N = 32), plus the scans and per-chunk kernels, which grow
        // with the number of chunks (~0.13 us each).
        const int sms = num_sms();
        double best = 1e30;
        int bestL = 256;
        for (int L = 16; L <= 512; ++L) {
            const int C = (g->T + L - 1) / L;
            const long G = (long)g->B * ((C + 3) / 4);
            const long w3 = (G + 3L * sms - 1) / (3L * sms);
            const long w2 = (G + 2L * sms - 1) / (2L * sms);
            const double cost = (L + 10.0) * (5.8 * (double)w3 + 11.7 * (double)w2) + 0.13 * (double)g->B * C;
            if (cost < best) {
                best = cost;
                bestL = L;
            }
        }
        g->Lc = bestL;
    }
    g->C = (g->T + g->Lc - 1) / g->Lc;
    g->ntiles = g->B * g->C;
    g->grp0 = 0;
    g->ngrp = (g->C + tc::TILES - 1) / tc::TILES;
    return EWS_OK;
}

// The output pass's launch (fwd_tc_kernel: shared memory, persistent grid) and, for the terminal backward,
// the chunk groups per window: enough tiles to fill that grid once, so the scratch rows are bounded by the
// grid, not by the sequence.
struct OutPlan {
    size_t smem;
    int grid, wgrp;
};

static int out_plan(const Geom& g, OutPlan* op) {
    op->smem = tc::tc_out_smem_bytes(g.QP);
    if (op->smem > 227 * 1024) return EWS_ERR_UNSUPPORTED;
    cudaFuncSetAttribute(fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)op->smem);
    cudaFuncSetAttribute(fwd_tc_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
    const int per_sm = resident_ctas((const void*)fwd_tc_kernel, tc::NTH, op->smem);
    if (per_sm < 1) return EWS_ERR_UNSUPPORTED;
    op->grid = per_sm * num_sms();
    const int groups = (g.C + tc::TILES - 1) / tc::TILES;
    op->wgrp = std::min(groups, (op->grid + g.B - 1) / g.B);
    return EWS_OK;
}

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

struct WsLayout {
    size_t status, flags, agg, incl, carry, partials, pw, loc, pows, gex, srows, total;
};

static WsLayout fwd_layout(const Geom& g) {
    WsLayout L{};
    size_t o = 0;
    L.status = o;
    o += al256(sizeof(DeviceStatus));
    L.flags = o;
    o += al256(sizeof(int) * (size_t)g.ntiles);
    const size_t slots = al256(sizeof(float) * (size_t)g.ntiles * g.SW);
    L.agg = o;
    o += slots;
    L.incl = o;
    o += slots;
    L.carry = o;
    o += slots;
    L.pw = o;
    o += al256(sizeof(float) * (size_t)g.B * 2 * MM);
    L.loc = o;  // the intervals' local terms, written by local_kernel and read by agg_kernel and both chains
    o += al256(sizeof(float) * (size_t)g.B * g.T * loc_width(g.QP));
    L.pows = o;  // power complements for agg_kernel
    o += al256(sizeof(float) * (size_t)g.B * (g.Lc + 1) * MM);
    L.gex = o;   // the group scan's two round buffers
    o += 2 * al256(sizeof(float) * (size_t)g.B * scan_groups(g.C) * g.SW);
    L.total = o;
    return L;
}

// wgrp: the terminal backward's chunk groups per window (out_plan); unused for the prefix readout
static WsLayout bwd_layout(const Geom& g, int wgrp) {
    WsLayout L{};
    size_t o = 0;
    L.status = o;
    o += al256(sizeof(DeviceStatus));
    L.flags = o;
    o += al256(sizeof(int) * (size_t)g.ntiles);
    const size_t slots = al256(sizeof(float) * (size_t)g.ntiles * g.SW);
    L.agg = o;
    o += slots;
    L.incl = o;
    o += slots;
    L.partials = o;
    o += al256(sizeof(float) * (size_t)g.ntiles * (MM + (1 + 2 * g.QP) * NP * g.d_in));
    L.carry = o;  // per chunk: the cotangent arriving at its end
    o += slots;
    L.loc = o;    // the vector cotangents [ds1 | dU_a | dV_a] per interval
    o += al256(sizeof(float) * (size_t)g.B * g.T * loc_width(g.QP));
    L.pows = o;   // the reverse scan's suffix aggregates (gsuf)
    o += slots;
    L.gex = o;    // the reverse group scan's two round buffers of (G, mu) elements
    o += 2 * al256(sizeof(float) * (size_t)g.B * scan_groups(g.C) * 2 * g.SW);
    L.srows = o;  // terminal: the window's recomputed states
    if (g.readout == EWS_READOUT_TERMINAL)
        o += al256(sizeof(float) * (size_t)wgrp * tc::TILES * g.B * g.Lc * g.W);
    L.total = o;
    return L;
}


}  // namespace dense
}  // namespace ews

using namespace ews;
using namespace ews::dense;

extern "C" int ews_dense_workspace_size(const ews_dense_args* a, size_t* fwd_bytes, size_t* bwd_bytes) {
    Geom g;
    const int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (fwd_bytes) *fwd_bytes = fwd_layout(g).total;
    if (bwd_bytes) {
        int wgrp = 0;
        if (g.readout == EWS_READOUT_TERMINAL) {
            OutPlan op;
            const int pr = out_plan(g, &op);
            if (pr != EWS_OK) return pr;
            wgrp = op.wgrp;
        }
        *bwd_bytes = bwd_layout(g, wgrp).total;
    }
    return EWS_OK;
}

extern "C" int ews_dense_launches(const ews_dense_args* a, int* fwd_launches, int* bwd_launches) {
    Geom g;
    const int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    int rounds = 1;  // the group scans' rounds
    while ((1 << rounds) < scan_groups(g.C)) ++rounds;
    // forward: power, local, powers, agg, scan_local, rounds, scan_fix [, fwd_tc for the prefix readout];
    // backward: bagg, bscan_local, rounds, bscan_fix, bwd_exact, table_grad, reduce (terminal readout:
    // fwd_tc and bwd_exact once per window of chunk groups)
    if (fwd_launches) *fwd_launches = 6 + rounds + (g.readout == EWS_READOUT_PREFIX ? 1 : 0);
    if (bwd_launches) {
        int windows = 1;
        if (g.readout == EWS_READOUT_TERMINAL) {
            OutPlan op;
            const int pr = out_plan(g, &op);
            if (pr != EWS_OK) return pr;
            windows = (g.ngrp + op.wgrp - 1) / op.wgrp;
        }
        *bwd_launches = 5 + rounds + 2 * windows - (g.readout == EWS_READOUT_TERMINAL ? 0 : 1);
    }
    return EWS_OK;
}

extern "C" int ews_dense_fwd(const ews_dense_args* a, ews_stream_t stream) {
    Geom g;
    const int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (!a->path || !a->out || !a->tab_d || !a->tab_f || !a->tab_g || !a->tab_h) return EWS_ERR_INVALID_ARGUMENT;
    const WsLayout L = fwd_layout(g);
    if (!a->fwd_ws || a->fwd_ws_bytes < L.total) return EWS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    char* ws = (char*)a->fwd_ws;
    if (cudaMemsetAsync(ws, 0, L.agg, s) != cudaSuccess) return EWS_ERR_LAUNCH;
    Params p{};
    p.g = g;
    p.path = a->path;
    p.tab_d = a->tab_d;
    p.tab_f = a->tab_f;
    p.tab_g = a->tab_g;
    p.tab_h = a->tab_h;
    p.out = a->out;
    p.st = (DeviceStatus*)(ws + L.status);
    p.flags = (int*)(ws + L.flags);
    p.agg = (float*)(ws + L.agg);
    p.incl = (float*)(ws + L.incl);
    p.carry = (float*)(ws + L.carry);
    p.pw = (float*)(ws + L.pw);
    p.loc = (float*)(ws + L.loc);
    const size_t lsmem = local_smem_bytes(g.d_in, g.QP);
    if (lsmem > 227 * 1024) return EWS_ERR_UNSUPPORTED;
    cudaFuncSetAttribute(local_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsmem);
    p.pows = (float*)(ws + L.pows);
    p.g.agg_pre = 1;
    // the flow powers (B CTAs each) beside the local terms (B x spans CTAs): independent until agg_kernel
    SideStream* ss = side_stream(s);
    cudaStream_t sp = s;
    if (ss && cudaEventRecord(ss->fork, s) == cudaSuccess && cudaStreamWaitEvent(ss->s2, ss->fork, 0) == cudaSuccess)
        sp = ss->s2;
    power_kernel<<<g.B, NT, 5 * MM * sizeof(float), sp>>>(p);
    powers_kernel<<<g.B, PWT, 0, sp>>>(p);
    if (g.QP <= 4 && g.d_in <= 8) {
        const int rspans = (g.T + LSPAN_REG - 1) / LSPAN_REG;
        const int rows = 1 + 2 * g.QP;
        if (rows == 3) local_reg_kernel<3><<<g.B * rspans, LNT, 0, s>>>(p);
        else if (rows == 5) local_reg_kernel<5><<<g.B * rspans, LNT, 0, s>>>(p);
        else if (rows == 7) local_reg_kernel<7><<<g.B * rspans, LNT, 0, s>>>(p);
        else local_reg_kernel<9><<<g.B * rspans, LNT, 0, s>>>(p);
    } else {
        const int spans = (g.T + LSPAN - 1) / LSPAN;
        local_kernel<<<g.B * spans, LNT, lsmem, s>>>(p);
    }
    if (sp != s && (cudaEventRecord(ss->join, sp) != cudaSuccess || cudaStreamWaitEvent(s, ss->join, 0) != cudaSuccess))
        return EWS_ERR_LAUNCH;
    if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    {
        const int arc = launch_agg_q(p, s);
        if (arc != EWS_OK) return arc;
    }
    p.gex = (float*)(ws + L.gex);
    scan_local_kernel<<<g.B * scan_groups(g.C), CST, 0, s>>>(p);
    if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    {
        const int ng = scan_groups(g.C);
        float* h0 = (float*)(ws + L.gex);
        float* h1 = h0 + al256(sizeof(float) * (size_t)g.B * ng * g.SW) / sizeof(float);
        int rounds = 1;
        while ((1 << rounds) < ng) ++rounds;
        for (int r = 0; r < rounds; ++r) {
            scan_round_kernel<<<g.B * ng, CST, 0, s>>>(p, r == 0 ? nullptr : ((r & 1) ? h0 : h1), (r & 1) ? h1 : h0, 1 << r);
            if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
        }
        p.gex = ((rounds - 1) & 1) ? h1 : h0;  // the inclusive group products
    }
    scan_fix_kernel<<<g.B * g.C, CST, 0, s>>>(p);
    if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    if (g.readout == EWS_READOUT_TERMINAL) return EWS_OK;  // the scan wrote the terminal rows
    OutPlan op;
    const int pr = out_plan(g, &op);
    if (pr != EWS_OK) return pr;
    const int grid = std::min(op.grid, g.B * g.ngrp);
    fwd_tc_kernel<<<grid, tc::NTH, op.smem, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

extern "C" int ews_dense_bwd(const ews_dense_args* a, ews_stream_t stream) {
    Geom g;
    int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (!a->path || !a->out || !a->grad_out || !a->grad_dx || !a->grad_d || !a->grad_f || !a->grad_g || !a->grad_h)
        return EWS_ERR_INVALID_ARGUMENT;
    const bool term = g.readout == EWS_READOUT_TERMINAL;
    OutPlan op{};
    if (term) {
        rc = out_plan(g, &op);
        if (rc != EWS_OK) return rc;
    }
    const WsLayout F = fwd_layout(g);
    const WsLayout L = bwd_layout(g, op.wgrp);
    if (!a->fwd_ws || a->fwd_ws_bytes < F.total) return EWS_ERR_WORKSPACE;
    if (!a->bwd_ws || a->bwd_ws_bytes < L.total) return EWS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    char* ws = (char*)a->bwd_ws;
    const char* fws = (const char*)a->fwd_ws;
    if (cudaMemsetAsync(ws, 0, L.agg, s) != cudaSuccess) return EWS_ERR_LAUNCH;
    Params p{};
    p.g = g;
    p.path = a->path;
    p.tab_d = a->tab_d;
    p.tab_f = a->tab_f;
    p.tab_g = a->tab_g;
    p.tab_h = a->tab_h;
    p.out = a->out;
    p.grad_out = a->grad_out;
    p.grad_dx = a->grad_dx;
    p.partials = (float*)(ws + L.partials);
    p.st = (DeviceStatus*)(ws + L.status);
    p.flags = (int*)(ws + L.flags);
    p.agg = (float*)(ws + L.agg);
    p.incl = (float*)(ws + L.incl);
    p.fagg = (const float*)(fws + F.agg);
    p.carry = (float*)(fws + F.carry);  // the forward's chunk carries (the terminal backward re-runs the chunks)
    p.loc = (float*)(fws + F.loc);
    p.lcarry = (float*)(ws + L.carry);
    {
        const int groups = (g.C + tc::TILES - 1) / tc::TILES;
        // zero-carry local adjoints (power sums, parallel over the chunks) -> reverse scan over the chunks ->
        // exact pass from the carries
        p.pows = (float*)(fws + F.pows);
        {
            const size_t bsm = sizeof(float) * (size_t)BGW * bagg_warp_floats();
            cudaFuncSetAttribute(bagg_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsm);
            bagg_kernel<<<(g.B * g.C + BGW - 1) / BGW, BGW * 32, bsm, s>>>(p);
        }
        if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
        p.gsuf = (float*)(ws + L.pows);
        p.gex = (float*)(ws + L.gex);
        const int ng = scan_groups(g.C);
        bscan_local_kernel<<<g.B * ng, CST, 0, s>>>(p);
        if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
        {
            float* h0 = (float*)(ws + L.gex);
            float* h1 = h0 + al256(sizeof(float) * (size_t)g.B * ng * 2 * g.SW) / sizeof(float);
            int rounds = 1;
            while ((1 << rounds) < ng) ++rounds;
            for (int r = 0; r < rounds; ++r) {
                bscan_round_kernel<<<g.B * ng, CST, 0, s>>>(p, r == 0 ? nullptr : ((r & 1) ? h0 : h1), (r & 1) ? h1 : h0,
                                                           1 << r);
                if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
            }
            p.gex = ((rounds - 1) & 1) ? h1 : h0;  // the suffix elements of the groups
        }
        bscan_fix_kernel<<<g.B * g.C, CST, 0, s>>>(p);
        if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
        // the exact pass with the gradient map: vector cotangents to `coef`, dM to the chunk partials
        p.coef = (float*)(ws + L.loc);
        const size_t xsmem = tc::tc_exact_smem_bytes(g.QP);
        if (xsmem > 227 * 1024) return EWS_ERR_UNSUPPORTED;
        auto* xk = g.N == NP ? bwd_exact_kernel<true> : bwd_exact_kernel<false>;
        cudaFuncSetAttribute(xk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)xsmem);
        cudaFuncSetAttribute(xk, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
        const int xper = resident_ctas((const void*)xk, tc::NTH, xsmem);
        if (xper < 1) return EWS_ERR_UNSUPPORTED;
        // prefix readout: one window of every chunk group, the states read from `out`; terminal readout: per
        // window of op.wgrp groups, the output pass re-runs the window's chunks from the forward's carries into
        // the scratch rows, then the exact pass reads them
        const int wgrp = term ? op.wgrp : groups;
        if (term) p.srows = (float*)(ws + L.srows);
        for (int g0 = 0; g0 < groups; g0 += wgrp) {
            p.g.grp0 = g0;
            p.g.ngrp = std::min(wgrp, groups - g0);
            if (term) {
                if (cudaMemsetAsync(ws + L.status, 0, sizeof(int), s) != cudaSuccess) return EWS_ERR_LAUNCH;
                p.g.bwd_mode = 0;
                fwd_tc_kernel<<<std::min(op.grid, g.B * p.g.ngrp), tc::NTH, op.smem, s>>>(p);
                if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
            }
            if (cudaMemsetAsync(ws + L.status, 0, sizeof(int), s) != cudaSuccess) return EWS_ERR_LAUNCH;  // the ticket
            p.g.bwd_mode = 2;
            xk<<<std::min(xper * num_sms(), g.B * p.g.ngrp), tc::NTH, xsmem, s>>>(p);
            if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
        }
        p.g.bwd_mode = 0;
        p.g.grp0 = 0;
        p.g.ngrp = groups;
    }
    {
        const size_t tsmem = gm::table_smem_bytes(g);
        if (tsmem > 227 * 1024) return EWS_ERR_UNSUPPORTED;
        if (g.QP <= 4 && g.d_in <= 8) {
            const int rows = 1 + 2 * g.QP;
            const size_t xsm = table_reg_smem_bytes(g.Lc, g.QP);  // the chunk's increments and the slab ring
            const void* tk = rows == 3 ? (const void*)table_grad_reg_kernel<3>
                             : rows == 5 ? (const void*)table_grad_reg_kernel<5>
                             : rows == 7 ? (const void*)table_grad_reg_kernel<7>
                                         : (const void*)table_grad_reg_kernel<9>;
            cudaFuncSetAttribute(tk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)xsm);
            if (rows == 3) table_grad_reg_kernel<3><<<g.C * g.B, 128, xsm, s>>>(p);
            else if (rows == 5) table_grad_reg_kernel<5><<<g.C * g.B, 128, xsm, s>>>(p);
            else if (rows == 7) table_grad_reg_kernel<7><<<g.C * g.B, 128, xsm, s>>>(p);
            else table_grad_reg_kernel<9><<<g.C * g.B, 128, xsm, s>>>(p);
        } else {
            cudaFuncSetAttribute(table_grad_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsmem);
            table_grad_kernel<<<g.C * g.B, 128, tsmem, s>>>(p);
        }
        if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    }
    const size_t total = (size_t)g.B * (g.N * g.N + (1 + 2 * g.QP) * g.N * g.d_in);
    reduce_kernel<<<(unsigned)((total + 31) / 32), 32 * RED_SLICES, 0, s>>>(p, a->grad_d, a->grad_f, a->grad_g,
                                                                           a->grad_h);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}
