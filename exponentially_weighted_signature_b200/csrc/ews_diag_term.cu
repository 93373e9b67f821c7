// Diagonal engine, uniform clock, terminal readout: the terminal value in closed form.
//
// With the per-step flow rho = exp(x) (x = -h lambda per sample), the series tables Q1, Q2 and the lifted
// increments dy_t, the depth-2 recursion of the uniform diagonal engine
//     S1_t = rho S1_{t-1} + Q1 dy_t,
//     S2_t = (rho rho^T) S2_{t-1} + (rho S1_{t-1}) (Q1 dy_t)^T + Q2 (dy_t dy_t^T)      (elementwise products)
// unrolls, with the interval weights w_t = rho^(T-1-t) and r_t = w_t dy_t, into
//     S1_T = Q1 sum_t r_t,     S2_T = diag(Q1) M diag(Q1) + Q2 G,
//     M = sum_t (sum_{tau < t} r_tau) r_t^T,    G = sum_t r_t r_t^T:
// the decay of every earlier interval cancels against the weights (rho^(t-1-tau) w_t rho = w_tau), so the
// terminal value is a reweighted depth-2 signature, two Gram-type products over the path and a running sum,
// with no sequential dependence but the running sum. It is the same value as the reference's terminal
// reduction of the Chen products (ews/core/chen_scan.py:218-298 with the series leaf
// ews/core/series_leaf.py:72-127 and cached uniform flows, chen_scan.py:155-168), evaluated in another order.
//
// The backward, with G1 = dL/dS1_T and G2 = dL/dS2_T: dM = diag(Q1) G2 diag(Q1), dG = Q2 G2,
//     dr_t = dM^T P_t + dM Z_t + (dG + dG^T) r_t + Q1 G1,    P_t = sum_{tau < t} r_tau,  Z_t = sum_{tau > t} r_tau,
// and since P_t + r_t + Z_t = s,  dr_t = (dM^T - dM) P_t + (dG + dG^T - dM) r_t + dM s + Q1 G1: two
// matrix-vector products per interval,
//     d(dy_t) = w_t dr_t,   dL/dx += sum_t (T-1-t) dr_t r_t,   dL/dQ2 = G2 G,
//     dL/dQ1_i = sum_j G2_ij M_ij Q1_j + G2_ji Q1_j M_ji + G1_i s_i   (s = sum_t r_t).
//
// Work: one CTA per (sample, segment of the path); a segment runs in chunks of TL intervals through shared
// memory, its own running sum starting at zero; a finishing kernel combines the segments in order
// (M = sum_seg (P_seg s_seg^T + M_seg), P_seg the sum of the earlier segments). Float32 throughout; the
// weights are exp(x k) with the product x k split exactly (x k = hi + lo) so their error stays at a few
// ulps for every k.

#include <cuda_runtime.h>

#include "../../include/ews_b200.h"
#include "ews_common.cuh"

namespace ews {
namespace diagterm {

constexpr int NP = 32;   // padded state dimension
constexpr int MM = NP * NP;
constexpr int TL = 128;  // intervals per chunk
constexpr int TNT = 256; // threads per CTA
constexpr int PW = 2 * MM + NP;  // per-segment partial: M | G | s
constexpr int LTS = NP + 4;      // row stride of lift^T in shared memory (float4 rows, 2-way banks at most)
constexpr int XTS = TL + 4;      // row stride of the channel-major increments

struct TP {
    int B, T, d_in, N, S, seg;  // S segments of `seg` intervals per sample
    unsigned flags;
    const void* path;
    const float* lift;
    const float* tab_x;
    const float* tab_q1;
    const float* tab_q2;
    float* out;
    float* part;   // (B, S, PW): per segment M | G | s from a zero running sum
    float* save;   // (B, PW): M | G | s of the whole path
    float* spre;   // (B, S, NP): sum of r over the earlier segments
    const float* grad_out;
    float* grad_dx;
    float* grad_lift;
    float* grad_x;
    float* grad_q1;
    float* grad_q2;
    float* dmat;   // (B, 2 MM + NP): A1 = dM^T - dM | A2 = dG + dG^T - dM | c = dM s + Q1 G1 (rows j)
    float* bpart;  // (B, S, NP + NP d_in): dL/dx partial | lift-gradient partial
};

// Shared-memory layout shared by both directions (floats).
struct TS {
    float *liftT, *xs, *dxs, *R, *P, *tot, *carry;
};

__device__ __forceinline__ TS carve(float* sm, int d_in) {
    TS s;
    float* q = sm;
    s.R = q; q += TL * NP;
    s.P = q; q += TL * NP;
    s.liftT = q; q += 32 * LTS;  // lift^T: liftT[c LTS + i]
    s.dxs = q; q += 32 * XTS;    // increments, channel-major: dxs[c XTS + t]
    s.xs = q; q += NP;
    s.tot = q; q += 8 * NP;
    s.carry = q; q += NP;
    return s;
}

__host__ __device__ inline size_t smem_bytes() { return sizeof(float) * (2 * TL * NP + 32 * LTS + 32 * XTS + 10 * NP); }

// The compressed depth-2 log-signature: N letters, then the Lyndon words (i, j), i < j, in lexicographic
// order (signax 0.2.1's coordinates); (i, j) sits at i (2N - i - 1) / 2 + (j - i - 1) after the letters.
__host__ __device__ inline int logsig_width(int N) { return N + N * (N - 1) / 2; }
__host__ __device__ inline int lyndon2_index(int i, int j, int N) { return i * (2 * N - i - 1) / 2 + (j - i - 1); }

// w = exp(x k) for an integer k >= 0: x k = hi + lo exactly, exp(hi) (1 + lo).
__device__ __forceinline__ float weight(float x, int k) {
    const float kf = (float)k;
    const float hi = x * kf;
    const float lo = fmaf(x, kf, -hi);
    return expf(hi) * (1.f + lo);
}

// The chunk's increments into dxs[c XTS + t] (channel-major), then r_t = w_t (lift dx_t) into R (rows
// t < len; zeros beyond, and in the padded columns). Thread (g, i) forms rows 4 g + 32 m .. + 3 of column
// i: one lift entry and one float4 of increments per 4 FMAs.
__device__ void chunk_r(const TP& p, const TS& s, int b, int t0, int len) {
    const int d = p.d_in, N = p.N;
    for (int e = threadIdx.x; e < TL * d; e += TNT) {
        const int c = e / TL, t = e - c * TL;
        s.dxs[c * XTS + t] = t < len ? input_increment(p.path, b, t0 + t, c, p.T, d, p.flags) : 0.f;
    }
    __syncthreads();
    const int g = threadIdx.x >> 5, i = threadIdx.x & 31;
    const float xi = s.xs[i];
#pragma unroll
    for (int m = 0; m < TL / 32; ++m) {
        const int tb = 4 * g + 32 * m;
        float dy[4] = {0.f, 0.f, 0.f, 0.f};
        if (p.lift) {
            for (int c = 0; c < d; ++c) {
                const float l = s.liftT[c * LTS + i];
                const float4 x = *reinterpret_cast<const float4*>(s.dxs + c * XTS + tb);
                dy[0] = fmaf(l, x.x, dy[0]);
                dy[1] = fmaf(l, x.y, dy[1]);
                dy[2] = fmaf(l, x.z, dy[2]);
                dy[3] = fmaf(l, x.w, dy[3]);
            }
        } else if (i < d) {
            const float4 x = *reinterpret_cast<const float4*>(s.dxs + i * XTS + tb);
            dy[0] = x.x;
            dy[1] = x.y;
            dy[2] = x.z;
            dy[3] = x.w;
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int t = tb + u;
            s.R[t * NP + i] = (t < len && i < N) ? weight(xi, p.T - 1 - (t0 + t)) * dy[u] : 0.f;
        }
    }
    __syncthreads();
}

// P[t] = carry + sum_{tau < t} R[tau] (exclusive, within the chunk), then carry += sum_t R[t]. Thread
// (g, i) sums rows 16 g .. 16 g + 15 of column i; the 8 group totals are combined in order.
__device__ void chunk_prefix(const TS& s) {
    const int g = threadIdx.x >> 5, i = threadIdx.x & 31;
    float run = 0.f;
    for (int t = 16 * g; t < 16 * g + 16; ++t) {
        s.P[t * NP + i] = run;
        run += s.R[t * NP + i];
    }
    s.tot[g * NP + i] = run;
    __syncthreads();
    float base = s.carry[i];
    for (int h = 0; h < g; ++h) base += s.tot[h * NP + i];
    for (int t = 16 * g; t < 16 * g + 16; ++t) s.P[t * NP + i] += base;
    __syncthreads();
    if (g == 0) {
        float c = s.carry[i];
        for (int h = 0; h < 8; ++h) c += s.tot[h * NP + i];
        s.carry[i] = c;
    }
    __syncthreads();
}

__device__ void load_common(const TP& p, const TS& s, int b) {
    const int d = p.d_in, N = p.N;
    for (int e = threadIdx.x; e < 32 * NP; e += TNT) {
        const int c = e >> 5, i = e & 31;
        s.liftT[c * LTS + i] = (p.lift && c < d && i < N) ? p.lift[i * d + c] : 0.f;
    }
    if (threadIdx.x < NP) s.xs[threadIdx.x] = threadIdx.x < N ? p.tab_x[(size_t)b * N + threadIdx.x] : 0.f;
}

// ---------------------------------------------------------------------------------- forward

__global__ void __launch_bounds__(TNT) fwd_kernel(TP p) {
    extern __shared__ __align__(16) float sm[];
    const TS s = carve(sm, p.d_in);
    const int b = blockIdx.x / p.S, sg = blockIdx.x - b * p.S;
    const int tb = sg * p.seg, te = min(p.T, tb + p.seg);
    load_common(p, s, b);
    if (threadIdx.x < NP) s.carry[threadIdx.x] = 0.f;
    // [M; G] (64 x 32) in 4 x 4 blocks: thread (h, rb, cb) owns rows 4 rb (M for rb < 8, G beyond) and
    // columns 4 cb over the chunk rows k of half h; the halves are added at the end
    const int h = threadIdx.x >> 7, u = threadIdx.x & 127;
    const int a0 = 4 * (u >> 3), j0 = 4 * (u & 7);
    const float* Abase = a0 < 32 ? s.P + a0 : s.R + (a0 - 32);
    float acc[4][4];
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = 0.f;
    for (int t0 = tb; t0 < te; t0 += TL) {
        const int len = min(TL, te - t0);
        __syncthreads();
        chunk_r(p, s, b, t0, len);
        chunk_prefix(s);
        const int k1 = min(len, (h + 1) * (TL / 2));
#pragma unroll 4
        for (int k = h * (TL / 2); k < k1; ++k) {
            const float4 av = *reinterpret_cast<const float4*>(Abase + k * NP);
            const float4 bv = *reinterpret_cast<const float4*>(s.R + k * NP + j0);
            const float ar[4] = {av.x, av.y, av.z, av.w};
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                acc[r][0] = fmaf(ar[r], bv.x, acc[r][0]);
                acc[r][1] = fmaf(ar[r], bv.y, acc[r][1]);
                acc[r][2] = fmaf(ar[r], bv.z, acc[r][2]);
                acc[r][3] = fmaf(ar[r], bv.w, acc[r][3]);
            }
        }
    }
    __syncthreads();
    float* red = s.P;  // the second half's blocks, then added by the first half
    if (h == 1)
#pragma unroll
        for (int r = 0; r < 4; ++r)
            *reinterpret_cast<float4*>(red + (a0 + r) * NP + j0) = make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
    __syncthreads();
    float* pp = p.part + ((size_t)b * p.S + sg) * PW;
    if (h == 0) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float4 o = *reinterpret_cast<const float4*>(red + (a0 + r) * NP + j0);
            const int a = a0 + r;
            float* dst = pp + (a < 32 ? a * NP : MM + (a - 32) * NP) + j0;
            *reinterpret_cast<float4*>(dst) = make_float4(acc[r][0] + o.x, acc[r][1] + o.y, acc[r][2] + o.z, acc[r][3] + o.w);
        }
    }
    if (threadIdx.x < NP) pp[2 * MM + threadIdx.x] = s.carry[threadIdx.x];
}

// Combines the segments of sample b in order and writes its terminal row [1, Q1 s, Q1 M Q1 + Q2 G].
__global__ void __launch_bounds__(TNT) fin_kernel(TP p) {
    __shared__ float Sc[NP], ss[NP];
    const int b = blockIdx.x, N = p.N;
    float M[4], G[4];
#pragma unroll
    for (int m = 0; m < 4; ++m) M[m] = G[m] = 0.f;
    if (threadIdx.x < NP) Sc[threadIdx.x] = 0.f;
    __syncthreads();
    for (int sg = 0; sg < p.S; ++sg) {
        const float* pp = p.part + ((size_t)b * p.S + sg) * PW;
        if (threadIdx.x < NP) {
            ss[threadIdx.x] = pp[2 * MM + threadIdx.x];
            p.spre[((size_t)b * p.S + sg) * NP + threadIdx.x] = Sc[threadIdx.x];
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int e = threadIdx.x + TNT * m, i = e >> 5, j = e & 31;
            M[m] += fmaf(Sc[i], ss[j], pp[e]);
            G[m] += pp[MM + e];
        }
        __syncthreads();
        if (threadIdx.x < NP) Sc[threadIdx.x] += ss[threadIdx.x];
        __syncthreads();
    }
    float* sv = p.save + (size_t)b * PW;
    const float* q1 = p.tab_q1 + (size_t)b * N;
    const float* q2 = p.tab_q2 + (size_t)b * N * N;
    if (p.flags & EWS_F_LOGSIG) {
        // the log-signature epilogue (ews/layer.py:488-498): log(1 + X) = (X1, X2 - X1 X1^T / 2) at depth 2,
        // compressed to the Lyndon words (level 1: every letter; level 2: i < j, lexicographic)
        float* x1 = ss;  // the segment sums are no longer needed
        if (threadIdx.x < NP) x1[threadIdx.x] = threadIdx.x < N ? q1[threadIdx.x] * Sc[threadIdx.x] : 0.f;
        __syncthreads();
        float* row = p.out + (size_t)b * logsig_width(N);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const int e = threadIdx.x + TNT * m, i = e >> 5, j = e & 31;
            sv[e] = M[m];
            sv[MM + e] = G[m];
            if (i < j && j < N)
                row[N + lyndon2_index(i, j, N)] =
                    fmaf(q1[i] * M[m], q1[j], q2[i * N + j] * G[m]) - 0.5f * x1[i] * x1[j];
        }
        if (threadIdx.x < NP) {
            sv[2 * MM + threadIdx.x] = Sc[threadIdx.x];
            if (threadIdx.x < N) row[threadIdx.x] = x1[threadIdx.x];
        }
        return;
    }
    float* row = p.out + (size_t)b * (1 + N + N * N);
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const int e = threadIdx.x + TNT * m, i = e >> 5, j = e & 31;
        sv[e] = M[m];
        sv[MM + e] = G[m];
        if (i < N && j < N) row[1 + N + i * N + j] = fmaf(q1[i] * M[m], q1[j], q2[i * N + j] * G[m]);
    }
    if (threadIdx.x < NP) {
        sv[2 * MM + threadIdx.x] = Sc[threadIdx.x];
        if (threadIdx.x < N) row[1 + threadIdx.x] = q1[threadIdx.x] * Sc[threadIdx.x];
    }
    if (threadIdx.x == 0) row[0] = 1.f;
}

// ---------------------------------------------------------------------------------- backward

// Per sample: the coefficients of dr_t (A1, A2, c) and the table gradients dL/dQ1, dL/dQ2.
__global__ void __launch_bounds__(TNT) prep_kernel(TP p) {
    __shared__ float G2[MM], Ms[MM], dMs[MM], q1s[NP], g1s[NP];
    const int b = blockIdx.x, N = p.N, W = 1 + N + N * N;
    const bool logsig = (p.flags & EWS_F_LOGSIG) != 0;
    const float* go = p.grad_out + (size_t)b * (logsig ? logsig_width(N) : W);
    const float* sv = p.save + (size_t)b * PW;
    const float* q2 = p.tab_q2 + (size_t)b * N * N;
    float* dm = p.dmat + (size_t)b * (2 * MM + NP);
    if (threadIdx.x < NP) q1s[threadIdx.x] = threadIdx.x < N ? p.tab_q1[(size_t)b * N + threadIdx.x] : 0.f;
    for (int e = threadIdx.x; e < MM; e += TNT) {
        const int i = e >> 5, j = e & 31;
        if (logsig)  // the log epilogue's adjoint at level 2: only the Lyndon entries i < j carry a cotangent
            G2[e] = (i < j && j < N) ? go[N + lyndon2_index(i, j, N)] : 0.f;
        else
            G2[e] = (i < N && j < N) ? go[1 + N + i * N + j] : 0.f;
        Ms[e] = sv[e];
    }
    __syncthreads();
    if (threadIdx.x < NP) {
        // level 1: g1 = dlog1 - (G2 + G2^T) X1 / 2 with X1 = Q1 s under the log epilogue, else the row's own
        const int i = threadIdx.x;
        float g1 = 0.f;
        if (i < N) {
            if (logsig) {
                float acc = 0.f;
                for (int j = 0; j < N; ++j) acc = fmaf(G2[i * NP + j] + G2[j * NP + i], q1s[j] * sv[2 * MM + j], acc);
                g1 = go[i] - 0.5f * acc;
            } else {
                g1 = go[1 + i];
            }
        }
        g1s[i] = g1;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < MM; e += TNT) {
        const int i = e >> 5, j = e & 31;
        dMs[e] = q1s[i] * G2[e] * q1s[j];
    }
    __syncthreads();
    // entry e = (j, i) of the rows-j layout
    for (int e = threadIdx.x; e < MM; e += TNT) {
        const int j = e >> 5, i = e & 31;
        const bool ok = i < N && j < N;
        const float hji = ok ? q2[j * N + i] * G2[j * NP + i] : 0.f;
        const float hij = ok ? q2[i * N + j] * G2[i * NP + j] : 0.f;
        dm[e] = dMs[i * NP + j] - dMs[j * NP + i];
        dm[MM + e] = hji + hij - dMs[j * NP + i];
        if (ok) p.grad_q2[((size_t)b * N + j) * N + i] = G2[j * NP + i] * sv[MM + j * NP + i];
    }
    if (threadIdx.x < NP) {
        const int i = threadIdx.x;
        const float g1 = g1s[i];
        float cs = q1s[i] * g1;
        for (int k = 0; k < NP; ++k) cs = fmaf(dMs[i * NP + k], sv[2 * MM + k], cs);
        dm[2 * MM + i] = cs;
        if (i < N) {
            float acc = g1 * sv[2 * MM + i];
            for (int j = 0; j < N; ++j)
                acc += G2[i * NP + j] * Ms[i * NP + j] * q1s[j] + G2[j * NP + i] * q1s[j] * Ms[j * NP + i];
            p.grad_q1[(size_t)b * N + i] = acc;
        }
    }
}

__global__ void __launch_bounds__(TNT, 2) bwd_kernel(TP p) {
    extern __shared__ __align__(16) float sm[];
    const TS s = carve(sm, p.d_in);
    const int b = blockIdx.x / p.S, sg = blockIdx.x - b * p.S;
    const int tb = sg * p.seg, te = min(p.T, tb + p.seg);
    const int N = p.N, d = p.d_in;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    load_common(p, s, b);
    const float* dm = p.dmat + (size_t)b * (2 * MM + NP);
    if (threadIdx.x < NP) s.carry[threadIdx.x] = p.spre[((size_t)b * p.S + sg) * NP + threadIdx.x];
    // lane j: row j of A1 and of A2, and c_j
    float A1[32], A2[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        A1[i] = dm[lane * NP + i];
        A2[i] = dm[MM + lane * NP + i];
    }
    const float cj = dm[2 * MM + lane];
    const float xj = lane < N ? p.tab_x[(size_t)b * N + lane] : 0.f;
    float xlog = 0.f;  // lane j: sum_t (T-1-t) dr_t[j] r_t[j]
    // lift gradient: thread tid = (lh, liq, lc) of 2 x 8 x 16 owns entries (4 liq + u, lc) for chunk rows in
    // half lh (d_in <= 16 here; larger d_in loops over channel groups below)
    const int nl = p.lift ? N * d : 0;
    const int lh = threadIdx.x >> 7, liq = (threadIdx.x >> 4) & 7, lc0 = threadIdx.x & 15;
    float dlg[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int t0 = tb; t0 < te; t0 += TL) {
        const int len = min(TL, te - t0);
        __syncthreads();
        chunk_r(p, s, b, t0, len);
        chunk_prefix(s);
        // dr_t[j] for the warp's rows t = warp, warp + 8, ..., two rows at a time; d(dy_t) = w_t dr_t replaces
        // R[t] after use
        for (int t = warp; t < len; t += 2 * (TNT / 32)) {
            const int t2 = t + TNT / 32;
            const bool two = t2 < len;
            const int u2 = two ? t2 : t;
            float x0 = cj, x1 = 0.f, x2 = 0.f, x3 = 0.f, y0 = cj, y1 = 0.f, y2 = 0.f, y3 = 0.f;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 pv = *reinterpret_cast<const float4*>(s.P + t * NP + 4 * q);
                const float4 rv = *reinterpret_cast<const float4*>(s.R + t * NP + 4 * q);
                const float4 pw = *reinterpret_cast<const float4*>(s.P + u2 * NP + 4 * q);
                const float4 rw = *reinterpret_cast<const float4*>(s.R + u2 * NP + 4 * q);
                x0 = fmaf(A1[4 * q], pv.x, x0);
                x1 = fmaf(A2[4 * q], rv.x, x1);
                y0 = fmaf(A1[4 * q], pw.x, y0);
                y1 = fmaf(A2[4 * q], rw.x, y1);
                x2 = fmaf(A1[4 * q + 1], pv.y, x2);
                x3 = fmaf(A2[4 * q + 1], rv.y, x3);
                y2 = fmaf(A1[4 * q + 1], pw.y, y2);
                y3 = fmaf(A2[4 * q + 1], rw.y, y3);
                x0 = fmaf(A1[4 * q + 2], pv.z, x0);
                x1 = fmaf(A2[4 * q + 2], rv.z, x1);
                y0 = fmaf(A1[4 * q + 2], pw.z, y0);
                y1 = fmaf(A2[4 * q + 2], rw.z, y1);
                x2 = fmaf(A1[4 * q + 3], pv.w, x2);
                x3 = fmaf(A2[4 * q + 3], rv.w, x3);
                y2 = fmaf(A1[4 * q + 3], pw.w, y2);
                y3 = fmaf(A2[4 * q + 3], rw.w, y3);
            }
            const float dr = (x0 + x1) + (x2 + x3);
            const float dr2 = (y0 + y1) + (y2 + y3);
            const int k = p.T - 1 - (t0 + t);
            const int k2 = p.T - 1 - (t0 + u2);
            const float rj = s.R[t * NP + lane];
            const float rj2 = s.R[u2 * NP + lane];
            xlog = fmaf(dr * rj, (float)k, xlog);
            if (two) xlog = fmaf(dr2 * rj2, (float)k2, xlog);
            __syncwarp();
            s.R[t * NP + lane] = lane < N ? weight(xj, k) * dr : 0.f;  // d(dy_t)
            if (two) s.R[t2 * NP + lane] = lane < N ? weight(xj, k2) * dr2 : 0.f;
        }
        __syncthreads();
        // dL/d(increment) = lift^T d(dy_t): thread per (t, c), rows of d(dy_t) and of lift^T as float4
        for (int e = threadIdx.x; e < len * d; e += TNT) {
            const int t = e / d, c = e - t * d;
            float v;
            if (p.lift) {
                const float* gr = s.R + t * NP;
                const float* lr = s.liftT + c * LTS;
                float a0 = 0.f, a1 = 0.f;
#pragma unroll
                for (int i = 0; i < NP; i += 4) {
                    const float4 gv = *reinterpret_cast<const float4*>(gr + i);
                    const float4 lv = *reinterpret_cast<const float4*>(lr + i);
                    a0 = fmaf(lv.x, gv.x, a0);
                    a1 = fmaf(lv.y, gv.y, a1);
                    a0 = fmaf(lv.z, gv.z, a0);
                    a1 = fmaf(lv.w, gv.w, a1);
                }
                v = a0 + a1;
            } else {
                v = s.R[t * NP + c];
            }
            p.grad_dx[((size_t)b * p.T + t0 + t) * d + c] = v;
        }
        // lift gradient: thread (h, iq, c) accumulates entries (4 iq .. 4 iq + 3, c) over the chunk rows of
        // half h: one float4 of d(dy_t) and one increment per 4 FMAs
        if (nl) {
            const int t1 = min(len, (lh + 1) * (TL / 2));
#pragma unroll
            for (int cg = 0; cg < 2; ++cg) {
                const int c = lc0 + 16 * cg;
                if (c < d)
                    for (int t = lh * (TL / 2); t < t1; ++t) {
                        const float4 gv = *reinterpret_cast<const float4*>(s.R + t * NP + 4 * liq);
                        const float xv = s.dxs[c * XTS + t];
                        dlg[cg][0] = fmaf(gv.x, xv, dlg[cg][0]);
                        dlg[cg][1] = fmaf(gv.y, xv, dlg[cg][1]);
                        dlg[cg][2] = fmaf(gv.z, xv, dlg[cg][2]);
                        dlg[cg][3] = fmaf(gv.w, xv, dlg[cg][3]);
                    }
            }
        }
    }
    // partials: dL/dx (lanes summed over the warps) and the lift gradient
    __syncthreads();
    s.tot[warp * NP + lane] = xlog;
    __syncthreads();
    float* bp = p.bpart + ((size_t)b * p.S + sg) * (NP + NP * d);
    if (threadIdx.x < NP) {
        float v = 0.f;
        for (int w = 0; w < TNT / 32; ++w) v += s.tot[w * NP + threadIdx.x];
        bp[threadIdx.x] = v;
    }
    if (nl) {
        // the two halves' lift-gradient blocks, added in order
        float* red = s.P;
        __syncthreads();
        if (lh == 1)
#pragma unroll
            for (int cg = 0; cg < 2; ++cg)
#pragma unroll
                for (int u = 0; u < 4; ++u) red[(4 * liq + u) * NP + lc0 + 16 * cg] = dlg[cg][u];
        __syncthreads();
        if (lh == 0)
#pragma unroll
            for (int cg = 0; cg < 2; ++cg)
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const int i = 4 * liq + u, c = lc0 + 16 * cg;
                    if (i < N && c < d) bp[NP + i * d + c] = dlg[cg][u] + red[i * NP + c];
                }
    }
}

// dL/dx per sample (its segments in order): one thread per entry.
__global__ void reduce_x_kernel(TP p) {
    const int N = p.N, pw = NP + NP * p.d_in;
    const int e = blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= p.B * N) return;
    const int b = e / N, i = e - b * N;
    float v = 0.f;
    for (int sg = 0; sg < p.S; ++sg) v += p.bpart[((size_t)b * p.S + sg) * pw + i];
    p.grad_x[e] = v;
}

// The lift gradient: one CTA per entry, a fixed-order tree over all (sample, segment) partials.
__global__ void __launch_bounds__(TNT) reduce_lift_kernel(TP p) {
    __shared__ float red[TNT];
    const int pw = NP + NP * p.d_in, o = blockIdx.x;
    const size_t n = (size_t)p.B * p.S;
    float v = 0.f;
    for (size_t u = threadIdx.x; u < n; u += TNT) v += p.bpart[u * pw + NP + o];
    red[threadIdx.x] = v;
    __syncthreads();
    for (int w = TNT / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) red[threadIdx.x] += red[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) p.grad_lift[o] = red[0];
}

// ---------------------------------------------------------------------------------- host side

static int segments(int B, int T) {
    int sms = 148;
    {
        int dev = 0;
        cudaGetDevice(&dev);
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0) sms = n;
    }
    const int want = 4 * 3 * sms;  // about four waves of three CTAs per SM
    const int maxS = (T + TL - 1) / TL;
    int S = (want + B - 1) / B;
    return S < 1 ? 1 : (S > maxS ? maxS : S);
}

static TP make_tp(const ews_diag_args* a) {
    TP p{};
    p.B = a->batch;
    p.T = a->steps;
    p.d_in = a->d_in;
    p.N = a->dim;
    p.flags = a->flags;
    p.S = segments(p.B, p.T);
    const int chunks = (p.T + TL - 1) / TL;
    p.seg = ((chunks + p.S - 1) / p.S) * TL;
    p.S = (p.T + p.seg - 1) / p.seg;
    return p;
}

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

struct TLay {
    size_t part, save, spre, total;       // forward workspace
    size_t dmat, bpart, btotal;           // backward workspace
};

// Both workspaces begin with a DeviceStatus block, as every workspace of the library does, so a caller
// can fold any workspace's error word the same way (ews_status_fold). This path has no waits: the call
// clears the block and nothing sets it.
static TLay layout(const TP& p) {
    TLay L{};
    size_t o = al256(sizeof(DeviceStatus));
    L.part = o;
    o += al256(sizeof(float) * (size_t)p.B * p.S * PW);
    L.save = o;
    o += al256(sizeof(float) * (size_t)p.B * PW);
    L.spre = o;
    o += al256(sizeof(float) * (size_t)p.B * p.S * NP);
    L.total = o;
    o = al256(sizeof(DeviceStatus));
    L.dmat = o;
    o += al256(sizeof(float) * (size_t)p.B * (2 * MM + NP));
    L.bpart = o;
    o += al256(sizeof(float) * (size_t)p.B * p.S * (NP + NP * p.d_in));
    L.btotal = o;
    return L;
}

}  // namespace diagterm

// The closed-form terminal path applies to the uniform clock, depth 2, terminal readout, d_in <= 32 and
// (with a lift) dim * d_in <= 1024, without a basepoint, unless EWS_F_TERMINAL_SCAN asks for the scan.
bool diag_term_applies(const ews_diag_args* a) {
    if (!a || a->depth != 2 || a->readout != EWS_READOUT_TERMINAL) return false;
    if (!(a->flags & EWS_F_UNIFORM)) return false;
    if (a->flags & (EWS_F_BASEPOINT | EWS_F_TERMINAL_SCAN | EWS_F_TEST_WITHHOLD)) return false;
    if (a->dim > 32 || a->d_in > 32 || a->dim * a->d_in > 4 * diagterm::TNT) return false;
    return true;
}

void diag_term_workspace(const ews_diag_args* a, size_t* fwd_bytes, size_t* bwd_bytes) {
    const diagterm::TP p = diagterm::make_tp(a);
    const diagterm::TLay L = diagterm::layout(p);
    if (fwd_bytes) *fwd_bytes = L.total;
    if (bwd_bytes) *bwd_bytes = L.btotal;
}

int diag_term_fwd(const ews_diag_args* a, cudaStream_t s) {
    using namespace diagterm;
    TP p = make_tp(a);
    const TLay L = layout(p);
    if (!a->fwd_ws || a->fwd_ws_bytes < L.total) return EWS_ERR_WORKSPACE;
    char* ws = (char*)a->fwd_ws;
    if (cudaMemsetAsync(ws, 0, sizeof(DeviceStatus), s) != cudaSuccess) return EWS_ERR_LAUNCH;
    p.path = a->path;
    p.lift = a->lift;
    p.tab_x = a->tab_x;
    p.tab_q1 = a->tab_q1;
    p.tab_q2 = a->tab_q2;
    p.out = a->out;
    p.part = (float*)(ws + L.part);
    p.save = (float*)(ws + L.save);
    p.spre = (float*)(ws + L.spre);
    const size_t smem = smem_bytes();
    cudaFuncSetAttribute(fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    fwd_kernel<<<p.B * p.S, TNT, smem, s>>>(p);
    if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    fin_kernel<<<p.B, TNT, 0, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

int diag_term_bwd(const ews_diag_args* a, cudaStream_t s) {
    using namespace diagterm;
    TP p = make_tp(a);
    const TLay L = layout(p);
    if (!a->fwd_ws || a->fwd_ws_bytes < L.total) return EWS_ERR_WORKSPACE;
    if (!a->bwd_ws || a->bwd_ws_bytes < L.btotal) return EWS_ERR_WORKSPACE;
    if (a->lift && !a->grad_lift) return EWS_ERR_INVALID_ARGUMENT;
    char* fws = (char*)a->fwd_ws;
    char* ws = (char*)a->bwd_ws;
    if (cudaMemsetAsync(ws, 0, sizeof(DeviceStatus), s) != cudaSuccess) return EWS_ERR_LAUNCH;
    p.path = a->path;
    p.lift = a->lift;
    p.tab_x = a->tab_x;
    p.tab_q1 = a->tab_q1;
    p.tab_q2 = a->tab_q2;
    p.part = (float*)(fws + L.part);
    p.save = (float*)(fws + L.save);
    p.spre = (float*)(fws + L.spre);
    p.grad_out = a->grad_out;
    p.grad_dx = a->grad_dx;
    p.grad_lift = a->grad_lift;
    p.grad_x = a->grad_x;
    p.grad_q1 = a->grad_q1;
    p.grad_q2 = a->grad_q2;
    p.dmat = (float*)(ws + L.dmat);
    p.bpart = (float*)(ws + L.bpart);
    prep_kernel<<<p.B, TNT, 0, s>>>(p);
    if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    const size_t smem = smem_bytes();
    cudaFuncSetAttribute(bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    bwd_kernel<<<p.B * p.S, TNT, smem, s>>>(p);
    if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    reduce_x_kernel<<<(p.B * p.N + 255) / 256, 256, 0, s>>>(p);
    if (cudaGetLastError() != cudaSuccess) return EWS_ERR_LAUNCH;
    if (p.lift) reduce_lift_kernel<<<p.N * p.d_in, TNT, 0, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

}  // namespace ews
