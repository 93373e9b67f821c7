// Diagonal engine of the EWS hot path (A = diag(lambda)), depth 2, state dimension N <= 32, fp32.
//
// Per interval t of sample b (x = -h lambda, rho = exp(x), dy = lift @ dx):
//     S1' = rho o S1 + s1,                 s1_i  = Q1_i dy_i
//     S2' = (rho rho^T) o S2 + (rho o S1) s1^T + s2,   s2_ij = Q2_ij dy_i dy_j
// which is the modified-Chen recursion of ews/core/chen_scan.py:124-152 for a diagonal flow
// (ews/core/kernels/pallas_combine.py:1804-1834 is the same recursion sequentially), with the series
// local terms of ews/core/series_leaf.py:72-113 folded into the tables Q1, Q2.
//
// Work decomposition. One warp owns one tile = (sample, chunk of Lc intervals). Lane (ti, tj), ti in
// [0,4), tj in [0,8), owns the RI x RJ block (RI = NP/4, RJ = NP/8) of the level-2 state with rows
// ti*RI.. and columns tj*RJ.., plus the level-1 entries of its rows (kept redundantly by the 8 lanes of
// a row group). Row sums are xor-shuffles over lane bits 0-2, column sums over bits 3-4. Tiles are
// taken in order from an atomic ticket, so every tile a chunk waits for is already running: chunks
// publish their aggregate, look back over their predecessors (decoupled look-back) and re-run the
// recursion from the carry to emit the prefix rows. Every wait is bounded.
//
// Flows are carried as complements delta = 1 - rho = -expm1(x): S rho = S - delta S and
// rho_i rho_j = 1 - (delta_i + delta_j - delta_i delta_j). A rho within 1e-4 of one, rounded once and applied
// T times, drifts by ~T 2^-24 (the reference's float32 path loses 5e-5 relative at T = 4096 that way); the
// complement keeps the flow's rounding relative to delta instead.
//
// Per-interval clock (the reference's "displacement" mode): x_t = dtheta_t r with the clock step of each
// interval, and Q1(x_t), Q2(x_t) evaluated in the kernel from the series coefficients (Horner); the
// backward also returns dL/d(dtheta_t) and dL/dr.
//
// Backward: the adjoint of step t is lambda2 <- rho rho^T o lambda2, lambda1 <- rho o (lambda1 +
// lambda2 s1). Chunks compute a zero-carry local adjoint, look back over the later chunks (whose
// transposed chunk maps come from the forward aggregates) and then run the exact adjoint from the
// carry, accumulating the gradients. Prefix readouts read S_{t-1} back from the forward output;
// terminal readouts use the closed form lambda2_t = e^{(T-1-t)(x_i+x_j)} g2 and recompute S forward.
#include <algorithm>
#include <cstdio>
#include <mutex>

#include "ews_common.cuh"

namespace ews {
namespace diag {

constexpr int kWarps = 4;  // warps per CTA; each warp is an independent tile worker
constexpr int kQNU = 9;    // coefficient slots of the in-kernel series tables (series order <= 8)

struct Geom {
    int B, T, d_in, N, NP, Lc, C, W, SW, readout;
    unsigned flags;
    int spin_limit;
    int SR;      // prefix rows staged per span store
    int ntiles;  // B * C
    int nu;      // per-interval clock (tables evaluated per step)
    // per-warp shared-memory carve-up (floats), after the CTA's lift matrix (lift_n floats)
    int lift_n;
    int f_dys, f_dts, f_stage, f_per_warp;                     // forward: dxs at 0
    int b_dys, b_dts, b_dtg, b_dyg, b_lam1, b_gst, b_gst2, b_sst, b_sst2, b_per_warp;  // backward: dxs at 0
};

struct Params {
    Geom g;
    const void* path;
    const float* lift;
    const float* tab_x;
    const float* tab_q1;
    const float* tab_q2;
    float* out;
    // backward
    const float* grad_out;
    float* grad_dx;
    float* partials;  // per tile: gx (NP), dq1 (NP), dq2 (NP*NP), dlift (NP*d_in)
    // look-back state
    DeviceStatus* st;
    int* flags;
    float* agg;     // forward: chunk aggregates; backward: local adjoints
    float* incl;    // inclusive values
    float* carry;   // forward: exclusive prefix per chunk (kept for the backward)
    const float* fagg;    // backward: the forward aggregates
    const float* fcarry;  // backward: the forward carries
    // per-interval clock
    const float* clock;   // (B, T+1) knots
    float* grad_dtheta;   // (B, T)
    float c1[kQNU];       // Q1 coefficients c1_p / p!
    float c2[kQNU * kQNU];  // Q2 coefficients c2_ab / (a! b!), row a
};

__host__ __device__ inline int align4(int n) { return (n + 3) & ~3; }

// --------------------------------------------------------------------------------- lane elements

template <int RI, int RJ>
struct Elem {  // a Chen group element restricted to a lane's block: flow complements, level 1, level 2
    float Dr[RI], Dc[RJ], S1r[RI], S1c[RJ], S2[RI][RJ];
    __device__ void identity() {
#pragma unroll
        for (int r = 0; r < RI; ++r) {
            Dr[r] = 0.f;
            S1r[r] = 0.f;
#pragma unroll
            for (int c = 0; c < RJ; ++c) S2[r][c] = 0.f;
        }
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            Dc[c] = 0.f;
            S1c[c] = 0.f;
        }
    }
};

// Complement of a product of flows: 1 - (1-a)(1-b) = a + b - ab.
__device__ __forceinline__ float comp_mul(float a, float b) { return fmaf(-a, b, a + b); }

// res = L (x) R: L flowed by R's flow, then the truncated tensor product (ews/core/chen_scan.py:124-152).
template <int RI, int RJ>
__device__ __forceinline__ void chen_mul(const Elem<RI, RJ>& L, const Elem<RI, RJ>& R, Elem<RI, RJ>& out) {
    Elem<RI, RJ> o;
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const float u = fmaf(-R.Dr[r], L.S1r[r], L.S1r[r]);
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            const float dd = comp_mul(R.Dr[r], R.Dc[c]);
            o.S2[r][c] = fmaf(-dd, L.S2[r][c], L.S2[r][c] + fmaf(u, R.S1c[c], R.S2[r][c]));
        }
        o.S1r[r] = u + R.S1r[r];
        o.Dr[r] = comp_mul(L.Dr[r], R.Dr[r]);
    }
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        o.S1c[c] = fmaf(-R.Dc[c], L.S1c[c], L.S1c[c] + R.S1c[c]);
        o.Dc[c] = comp_mul(L.Dc[c], R.Dc[c]);
    }
    out = o;
}

// Slot layout (floats): [flow complement (NP) | S1 (NP) | S2 (NP x NP)].
template <int RI, int RJ>
__device__ __forceinline__ void store_elem(float* slot, const Elem<RI, RJ>& e, int NP, int i0, int j0, int tj) {
    if (tj == 0) {
#pragma unroll
        for (int r = 0; r < RI; ++r) {
            slot[i0 + r] = e.Dr[r];
            slot[NP + i0 + r] = e.S1r[r];
        }
    }
#pragma unroll
    for (int r = 0; r < RI; ++r)
#pragma unroll
        for (int c = 0; c < RJ; ++c) slot[2 * NP + (i0 + r) * NP + j0 + c] = e.S2[r][c];
}

template <int RI, int RJ>
__device__ __forceinline__ void load_elem(const float* slot, Elem<RI, RJ>& e, int NP, int i0, int j0) {
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        e.Dr[r] = ldcg(slot + i0 + r);
        e.S1r[r] = ldcg(slot + NP + i0 + r);
#pragma unroll
        for (int c = 0; c < RJ; ++c) e.S2[r][c] = ldcg(slot + 2 * NP + (i0 + r) * NP + j0 + c);
    }
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        e.Dc[c] = ldcg(slot + j0 + c);
        e.S1c[c] = ldcg(slot + NP + j0 + c);
    }
}

// --------------------------------------------------------------------------------- tables, inputs

// Horner evaluation of sum_a coef[a] x^a over the kQNU slots (zero above the series order) and of its
// derivative.
__device__ __forceinline__ float poly(const float* coef, float x) {
    float acc = 0.f;
#pragma unroll
    for (int a = kQNU - 1; a >= 0; --a) acc = fmaf(acc, x, coef[a]);
    return acc;
}

__device__ __forceinline__ float dpoly(const float* coef, float x) {
    float acc = 0.f;
#pragma unroll
    for (int a = kQNU - 1; a >= 1; --a) acc = fmaf(acc, x, (float)a * coef[a]);
    return acc;
}

template <int RI, int RJ>
struct Tables {
    float xr[RI], xc[RJ], dr[RI], dc[RJ], q1r[RI], q1c[RJ], q2[RI][RJ];  // d = 1 - rho = -expm1(x)
    float rr[RI], rc[RJ];  // per-interval clock: rates r, x = dtheta r
    __device__ void load_rates(const Params& p, int b, int i0, int j0) {
        const int N = p.g.N;
        const float* tr = p.tab_x + (size_t)b * N;
#pragma unroll
        for (int r = 0; r < RI; ++r) rr[r] = i0 + r < N ? tr[i0 + r] : 0.f;
#pragma unroll
        for (int c = 0; c < RJ; ++c) rc[c] = j0 + c < N ? tr[j0 + c] : 0.f;
    }
    // The tables of one interval of clock step dth: Q1(x) = sum_p c1_p x^p, Q2(x, y) = sum_a x^a w_a(y)
    // with w_a(y) = sum_b c2_ab y^b (the series leaf's coefficients, ews/core/series_leaf.py:72-113).
    __device__ void at(const Params& p, float dth) {
#pragma unroll
        for (int r = 0; r < RI; ++r) {
            xr[r] = dth * rr[r];
            dr[r] = -expm1f(xr[r]);
            q1r[r] = poly(p.c1, xr[r]);
        }
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            xc[c] = dth * rc[c];
            dc[c] = -expm1f(xc[c]);
            q1c[c] = poly(p.c1, xc[c]);
            float w[kQNU];
#pragma unroll
            for (int a = 0; a < kQNU; ++a) w[a] = poly(p.c2 + a * kQNU, xc[c]);
#pragma unroll
            for (int r = 0; r < RI; ++r) {
                float acc = 0.f;
#pragma unroll
                for (int a = kQNU - 1; a >= 0; --a) acc = fmaf(acc, xr[r], w[a]);
                q2[r][c] = acc;
            }
        }
    }
    __device__ void load(const Params& p, int b, int i0, int j0) {
        const int N = p.g.N;
        const float* tx = p.tab_x + (size_t)b * N;
        const float* t1 = p.tab_q1 + (size_t)b * N;
        const float* t2 = p.tab_q2 + (size_t)b * N * N;
#pragma unroll
        for (int r = 0; r < RI; ++r) {
            const int i = i0 + r;
            xr[r] = i < N ? tx[i] : 0.f;
            dr[r] = -expm1f(xr[r]);
            q1r[r] = i < N ? t1[i] : 0.f;
#pragma unroll
            for (int c = 0; c < RJ; ++c) {
                const int j = j0 + c;
                q2[r][c] = (i < N && j < N) ? t2[i * N + j] : 0.f;
            }
        }
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            const int j = j0 + c;
            xc[c] = j < N ? tx[j] : 0.f;
            dc[c] = -expm1f(xc[c]);
            q1c[c] = j < N ? t1[j] : 0.f;
        }
    }
};

// Lifted increments of steps [t0, t0 + n) into dys[k * NP + i] (zero for padded i >= N). The increments
// themselves go to dxs[k * d_in + c] first.
__device__ void load_increments(const Params& p, const float* liftS, float* dxs, float* dys, float* dts, int b,
                                int t0, int n) {
    const Geom& g = p.g;
    const int lane = threadIdx.x & 31;
    if (g.nu) {
        const float* ck = p.clock + (size_t)b * (g.T + 1) + t0;
        for (int k = lane; k < n; k += 32) dts[k] = ck[k + 1] - ck[k];  // the reference's clock[1:] - clock[:-1]
    }
    for (int e = lane; e < n * g.d_in; e += 32) {
        const int k = e / g.d_in, cc = e - k * g.d_in;
        dxs[e] = input_increment(p.path, b, t0 + k, cc, g.T, g.d_in, g.flags);
    }
    __syncwarp();
    for (int e = lane; e < n * g.NP; e += 32) {
        const int k = e / g.NP, i = e - k * g.NP;
        float v = 0.f;
        if (i < g.N) {
            if (p.lift) {
                // lift stored channel-major (liftS[cc * NP + i]): consecutive lanes, consecutive banks
                const float* xr = dxs + k * g.d_in;
                for (int cc = 0; cc < g.d_in; ++cc) v = fmaf(liftS[cc * g.NP + i], xr[cc], v);
            } else {
                v = dxs[k * g.d_in + i];
            }
        }
        dys[e] = v;
    }
    __syncwarp();
}

// --------------------------------------------------------------------------------- the step

// The flow complement of a step: delta, except the identity (delta = 0) for the basepoint interval
// (ews/core/chen_scan.py:160-166).
template <int RI, int RJ>
__device__ __forceinline__ void step_flow(const Tables<RI, RJ>& tb, bool identity, float fr[RI], float fc[RJ]) {
#pragma unroll
    for (int r = 0; r < RI; ++r) fr[r] = identity ? 0.f : tb.dr[r];
#pragma unroll
    for (int c = 0; c < RJ; ++c) fc[c] = identity ? 0.f : tb.dc[c];
}

// One modified-Chen step S <- flow(S) (x) (s1, s2) on a lane's block, also accumulating the flow product.
// bp: the basepoint interval (dtheta = 0), whose series local terms are those of x = 0: Q1 = 1, Q2 = 1/2.
template <int RI, int RJ>
__device__ __forceinline__ void chen_step(const Tables<RI, RJ>& tb, const float* dyk, int i0, int j0,
                                          Elem<RI, RJ>& S, const float fr[RI], const float fc[RJ], bool bp = false) {
    float dyr[RI], dyc[RJ], s1c[RJ];
#pragma unroll
    for (int r = 0; r < RI; ++r) dyr[r] = dyk[i0 + r];
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        dyc[c] = dyk[j0 + c];
        s1c[c] = (bp ? 1.f : tb.q1c[c]) * dyc[c];
    }
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const float u = fmaf(-fr[r], S.S1r[r], S.S1r[r]);
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            const float loc = (bp ? 0.5f : tb.q2[r][c]) * (dyr[r] * dyc[c]);
            const float dd = comp_mul(fr[r], fc[c]);
            S.S2[r][c] = fmaf(-dd, S.S2[r][c], S.S2[r][c] + fmaf(u, s1c[c], loc));
        }
        S.S1r[r] = fmaf(bp ? 1.f : tb.q1r[r], dyr[r], u);
        S.Dr[r] = comp_mul(S.Dr[r], fr[r]);
    }
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        S.S1c[c] = fmaf(-fc[c], S.S1c[c], S.S1c[c] + s1c[c]);
        S.Dc[c] = comp_mul(S.Dc[c], fc[c]);
    }
}

// The emitting pass's step: as chen_step without the flow-product bookkeeping (the carry already holds
// the chunk's start), with the pair complements dd = 1 - rho_i rho_j given (constant under a uniform clock).
template <int RI, int RJ>
__device__ __forceinline__ void chen_step_emit(const Tables<RI, RJ>& tb, const float* dyk, int i0, int j0,
                                               Elem<RI, RJ>& S, const float fr[RI], const float fc[RJ],
                                               const float dd[RI][RJ], bool bp) {
    float dyr[RI], s1c[RJ], dq[RJ];
#pragma unroll
    for (int r = 0; r < RI; ++r) dyr[r] = dyk[i0 + r];
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        const float dyc = dyk[j0 + c];
        s1c[c] = (bp ? 1.f : tb.q1c[c]) * dyc;
        dq[c] = dyc;
    }
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const float u = fmaf(-fr[r], S.S1r[r], S.S1r[r]);
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            const float loc = (bp ? 0.5f : tb.q2[r][c]) * (dyr[r] * dq[c]);
            S.S2[r][c] = fmaf(-dd[r][c], S.S2[r][c], S.S2[r][c] + fmaf(u, s1c[c], loc));
        }
        S.S1r[r] = fmaf(bp ? 1.f : tb.q1r[r], dyr[r], u);
    }
}

// Uniform clock, not the basepoint interval: S2' = S2 - dd o S2 + dy_j (u_i q1_j + q2_ij dy_i) with
// u = rho o S1, the pair complements dd constant (four floating-point operations per entry).
template <int RI, int RJ>
__device__ __forceinline__ void chen_step_u(const Tables<RI, RJ>& tb, const float* dyk, int i0, int j0,
                                            Elem<RI, RJ>& S, const float dd[RI][RJ]) {
    float dyr[RI], dyc[RJ];
#pragma unroll
    for (int r = 0; r < RI; ++r) dyr[r] = dyk[i0 + r];
#pragma unroll
    for (int c = 0; c < RJ; ++c) dyc[c] = dyk[j0 + c];
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const float u = fmaf(-tb.dr[r], S.S1r[r], S.S1r[r]);
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            const float t = fmaf(u, tb.q1c[c], tb.q2[r][c] * dyr[r]);
            const float s2 = fmaf(t, dyc[c], S.S2[r][c]);
            S.S2[r][c] = fmaf(-dd[r][c], S.S2[r][c], s2);
        }
        S.S1r[r] = fmaf(tb.q1r[r], dyr[r], u);
    }
}

// Prefix row [1, S1, S2] of a lane element to global memory (real dimension N). Every lane of a row group
// writes its rows' level-1 entries (same value, same address), so no store is predicated on the lane.
template <int RI, int RJ>
__device__ __forceinline__ void emit_row_all(float* row, const Elem<RI, RJ>& S, int N, int i0, int j0) {
    row[0] = 1.f;
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const int i = i0 + r;
        if (i < N) {
            row[1 + i] = S.S1r[r];
#pragma unroll
            for (int c = 0; c < RJ; ++c) {
                const int j = j0 + c;
                if (j < N) row[1 + N + i * N + j] = S.S2[r][c];
            }
        }
    }
}

// Writes prefix row [1, S1, S2] of a lane element straight to global memory (real dimension N).
template <int RI, int RJ>
__device__ __forceinline__ void emit_row(float* row, const Elem<RI, RJ>& S, int N, int i0, int j0, int tj,
                                         int lane) {
    if (lane == 0) row[0] = 1.f;
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const int i = i0 + r;
        if (i < N) {
            if (tj == 0) row[1 + i] = S.S1r[r];
#pragma unroll
            for (int c = 0; c < RJ; ++c) {
                const int j = j0 + c;
                if (j < N) row[1 + N + i * N + j] = S.S2[r][c];
            }
        }
    }
}

// Writes row [1, S1, S2] of a lane element into a staged row (real dimension N, row width W).
template <int RI, int RJ>
__device__ __forceinline__ void stage_row(float* row, const Elem<RI, RJ>& S, int N, int i0, int j0, int tj,
                                          int lane) {
    if (lane == 0) row[0] = 1.f;
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const int i = i0 + r;
        if (i < N) {
            if (tj == 0) row[1 + i] = S.S1r[r];
#pragma unroll
            for (int c = 0; c < RJ; ++c) {
                const int j = j0 + c;
                if (j < N) row[1 + N + i * N + j] = S.S2[r][c];
            }
        }
    }
}

// --------------------------------------------------------------------------------- forward kernel

template <int NP, bool NU, bool FULL>
__global__ void __launch_bounds__(kWarps * 32) fwd_kernel(Params p) {
    // FULL: N == NP, so row indices and bounds are compile-time constants
    constexpr int RI = NP / 4, RJ = NP / 8;
    extern __shared__ float smem[];
    const Geom& g = p.g;
    const int Nr = FULL ? NP : g.N;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* liftS = smem;
    for (int e = threadIdx.x; e < NP * g.d_in; e += blockDim.x) {
        const int r = e / g.d_in, cc = e - r * g.d_in;
        const float w = (p.lift && r < g.N) ? p.lift[r * g.d_in + cc] : 0.f;
        liftS[cc * NP + r] = w;                    // channel-major: the lift of the increments
        liftS[g.lift_n / 2 + r * g.d_in + cc] = w;  // row-major: the gradient's map back to dx
    }
    __syncthreads();
    float* dxs = smem + g.lift_n + warp * g.f_per_warp;
    float* dys = dxs + g.f_dys;
    float* dts = dxs + g.f_dts;
    float* stage = dxs + g.f_stage;

    const int ti = lane >> 3, tj = lane & 7;
    const int i0 = ti * RI, j0 = tj * RJ;
    const bool basepoint = (g.flags & EWS_F_BASEPOINT) != 0;

    for (;;) {
        const int tile = next_ticket(p.st);
        if (tile >= g.ntiles) break;
        const int c = tile / g.B, b = tile - c * g.B;
        const int t0 = c * g.Lc;
        const int len = min(g.Lc, g.T - t0);
        Tables<RI, RJ> tb;
        if (NU)
            tb.load_rates(p, b, i0, j0);
        else
            tb.load(p, b, i0, j0);
        load_increments(p, liftS, dxs, dys, dts, b, t0, len);

        // pass 1: the chunk's aggregate from the identity. Under a uniform clock the aggregate's flow
        // complement is 1 - rho^n = -expm1(n x) for the n non-basepoint intervals, so the steps skip the
        // flow bookkeeping and use the constant pair complements.
        Elem<RI, RJ> A;
        A.identity();
        if (NU) {
            for (int k = 0; k < len; ++k) {
                float fr[RI], fc[RJ];
                tb.at(p, dts[k]);
                step_flow(tb, false, fr, fc);
                chen_step(tb, dys + k * NP, i0, j0, A, fr, fc, false);
            }
        } else {
            float dd[RI][RJ];
#pragma unroll
            for (int r = 0; r < RI; ++r)
#pragma unroll
                for (int cc = 0; cc < RJ; ++cc) dd[r][cc] = comp_mul(tb.dr[r], tb.dc[cc]);
            // the basepoint interval (k = 0 of chunk 0) runs apart from the loop
            const int kf = (basepoint && t0 == 0) ? 1 : 0;
            if (kf) {
                float fr[RI], fc[RJ], d0[RI][RJ];
                step_flow(tb, true, fr, fc);
#pragma unroll
                for (int r = 0; r < RI; ++r)
#pragma unroll
                    for (int cc = 0; cc < RJ; ++cc) d0[r][cc] = 0.f;
                chen_step_emit(tb, dys, i0, j0, A, fr, fc, d0, true);
            }
            for (int k = kf; k < len; ++k) chen_step_u(tb, dys + k * NP, i0, j0, A, dd);
            const float fn = (float)(len - kf);
#pragma unroll
            for (int r = 0; r < RI; ++r) A.Dr[r] = -expm1f(fn * tb.xr[r]);
#pragma unroll
            for (int cc = 0; cc < RJ; ++cc) A.Dc[cc] = -expm1f(fn * tb.xc[cc]);
            // level 1 by columns, from the lanes holding those rows (column j0 + c is row (tj&1)*RJ + c of
            // row group tj/2, on the lane of that group with the same tj)
            const int src = (tj >> 1) * 8 + tj;
#pragma unroll
            for (int cc = 0; cc < RJ; ++cc) {
                const float send = (tj & 1) ? A.S1r[RJ + cc] : A.S1r[cc];
                A.S1c[cc] = __shfl_sync(kFull, send, src);
            }
        }
        const size_t slot = ((size_t)b * g.C + c) * g.SW;
        int* flag = p.flags + (size_t)b * g.C + c;
        Elem<RI, RJ> excl;
        excl.identity();
        if (c == 0) {
            store_elem(p.incl + slot, A, NP, i0, j0, tj);
            if (!(g.flags & EWS_F_TEST_WITHHOLD)) publish(flag, kFlagIncl);
        } else {
            store_elem(p.agg + slot, A, NP, i0, j0, tj);
            publish(flag, kFlagAgg);
            // look back over the predecessors: excl = incl_j (x) agg_{j+1} (x) ... (x) agg_{c-1}
            Elem<RI, RJ> acc;
            acc.identity();
            int j = c - 1;
            const int want = (g.flags & EWS_F_DETERMINISTIC) ? kFlagIncl : kFlagAgg;
            for (;;) {
                const int f = wait_slot(p.flags + (size_t)b * g.C + j, p.st, g.spin_limit, tile, want);
                if (f < 0) return;  // timeout or another tile failed: the error word is set
                Elem<RI, RJ> X;
                const size_t sj = ((size_t)b * g.C + j) * g.SW;
                if (f == kFlagIncl) {
                    load_elem(p.incl + sj, X, NP, i0, j0);
                    chen_mul(X, acc, excl);
                    break;
                }
                load_elem(p.agg + sj, X, NP, i0, j0);
                chen_mul(X, acc, acc);
                --j;
            }
            Elem<RI, RJ> inc;
            chen_mul(excl, A, inc);
            store_elem(p.incl + slot, inc, NP, i0, j0, tj);
            publish(flag, kFlagIncl);
        }
        store_elem(p.carry + slot, excl, NP, i0, j0, tj);
        // the forward aggregates are kept for the backward: chunk 0 stored it as incl
        if (c == 0) store_elem(p.agg + slot, A, NP, i0, j0, tj);

        if (g.readout == EWS_READOUT_TERMINAL) {
            if (c == g.C - 1) {
                Elem<RI, RJ> fin;
                chen_mul(excl, A, fin);
                stage_row(stage, fin, Nr, i0, j0, tj, lane);
                __syncwarp();
                warp_store_span(p.out + (size_t)b * g.W, stage, g.W);
                __syncwarp();
            }
            continue;
        }
        // pass 2: re-run the chunk from its carry and write the prefix rows from registers
        Elem<RI, RJ> S = excl;
        float dd[RI][RJ];
        if (!NU) {
#pragma unroll
            for (int r = 0; r < RI; ++r)
#pragma unroll
                for (int c = 0; c < RJ; ++c) dd[r][c] = comp_mul(tb.dr[r], tb.dc[c]);
        }
        float* orow = p.out + ((size_t)b * g.T + t0) * g.W;
        if (!NU) {
            const int kf = (basepoint && t0 == 0) ? 1 : 0;
            if (kf) {
                float fr[RI], fc[RJ], d0[RI][RJ];
                step_flow(tb, true, fr, fc);
#pragma unroll
                for (int r = 0; r < RI; ++r)
#pragma unroll
                    for (int c = 0; c < RJ; ++c) d0[r][c] = 0.f;
                chen_step_emit(tb, dys, i0, j0, S, fr, fc, d0, true);
                emit_row_all(orow, S, Nr, i0, j0);
                orow += g.W;
            }
            for (int k = kf; k < len; ++k, orow += g.W) {
                chen_step_u(tb, dys + k * NP, i0, j0, S, dd);
                emit_row_all(orow, S, Nr, i0, j0);
            }
        } else {
            // per-interval clock (no basepoint interval): the tables and pair complements of every step
            for (int k = 0; k < len; ++k, orow += g.W) {
                float fr[RI], fc[RJ];
                tb.at(p, dts[k]);
                step_flow(tb, false, fr, fc);
#pragma unroll
                for (int r = 0; r < RI; ++r)
#pragma unroll
                    for (int c = 0; c < RJ; ++c) dd[r][c] = comp_mul(fr[r], fc[c]);
                chen_step_emit(tb, dys + k * NP, i0, j0, S, fr, fc, dd, false);
                emit_row(orow, S, Nr, i0, j0, tj, lane);
            }
        }
    }
}

// --------------------------------------------------------------------------------- backward

// Adjoint lane element: cotangents of S1 (rows) and S2 (block).
template <int RI, int RJ>
struct Adj {
    float L1r[RI], L2[RI][RJ];
    __device__ void zero() {
#pragma unroll
        for (int r = 0; r < RI; ++r) {
            L1r[r] = 0.f;
#pragma unroll
            for (int c = 0; c < RJ; ++c) L2[r][c] = 0.f;
        }
    }
};

__device__ __forceinline__ float row_sum(float v) {  // over the 8 lanes of a row group
    v += __shfl_xor_sync(kFull, v, 1);
    v += __shfl_xor_sync(kFull, v, 2);
    v += __shfl_xor_sync(kFull, v, 4);
    return v;
}

__device__ __forceinline__ float col_sum(float v) {  // over the 4 lanes of a column group
    v += __shfl_xor_sync(kFull, v, 8);
    v += __shfl_xor_sync(kFull, v, 16);
    return v;
}

// Values a lane holds for its rows, delivered to the lanes whose columns they are: column j0 + c lives in
// row group tj/2 at offset (tj&1)*RJ + c; the source lane with the same tj sends it.
template <int RI, int RJ>
__device__ __forceinline__ void rows_to_cols(const float vr[RI], float vc[RJ], int tj) {
    const int src = (tj >> 1) * 8 + tj;
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        const float send = (tj & 1) ? vr[RJ + c] : vr[c];
        vc[c] = __shfl_sync(kFull, send, src);
    }
}

// Transposed Jacobian of right-multiplication by G = (P, U1, U2): mu2 = P P^T o l2,
// mu1 = P o (l1 + l2 U1), with P = 1 - D. Applied in place.
template <int RI, int RJ>
__device__ __forceinline__ void apply_JT(const Elem<RI, RJ>& G, Adj<RI, RJ>& a) {
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        float w = 0.f;
#pragma unroll
        for (int c = 0; c < RJ; ++c) w = fmaf(a.L2[r][c], G.S1c[c], w);
        w = row_sum(w) + a.L1r[r];
        a.L1r[r] = fmaf(-G.Dr[r], w, w);
#pragma unroll
        for (int c = 0; c < RJ; ++c) a.L2[r][c] = fmaf(-comp_mul(G.Dr[r], G.Dc[c]), a.L2[r][c], a.L2[r][c]);
    }
}

// Adjoint slot layout (floats): [L1 (NP) | pad (NP) | L2 (NP x NP)] (same size as a forward slot).
template <int RI, int RJ>
__device__ __forceinline__ void store_adj(float* slot, const Adj<RI, RJ>& a, int NP, int i0, int j0, int tj) {
    if (tj == 0) {
#pragma unroll
        for (int r = 0; r < RI; ++r) slot[i0 + r] = a.L1r[r];
    }
#pragma unroll
    for (int r = 0; r < RI; ++r)
#pragma unroll
        for (int c = 0; c < RJ; ++c) slot[2 * NP + (i0 + r) * NP + j0 + c] = a.L2[r][c];
}

template <int RI, int RJ>
__device__ __forceinline__ void load_adj(const float* slot, Adj<RI, RJ>& a, int NP, int i0, int j0) {
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        a.L1r[r] = ldcg(slot + i0 + r);
#pragma unroll
        for (int c = 0; c < RJ; ++c) a.L2[r][c] = ldcg(slot + 2 * NP + (i0 + r) * NP + j0 + c);
    }
}

template <int RI, int RJ>
__device__ __forceinline__ void adj_add(Adj<RI, RJ>& a, const Adj<RI, RJ>& b) {
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        a.L1r[r] += b.L1r[r];
#pragma unroll
        for (int c = 0; c < RJ; ++c) a.L2[r][c] += b.L2[r][c];
    }
}

// Reads row t of a (B, T, W) stream into a lane's (level-1 rows, level-2 block) pieces; real dims N.
template <int RI, int RJ>
__device__ __forceinline__ void read_row(const float* row, float v1[RI], float v2[RI][RJ], int N, int i0, int j0) {
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const int i = i0 + r;
        v1[r] = i < N ? row[1 + i] : 0.f;
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            const int j = j0 + c;
            v2[r][c] = (i < N && j < N) ? row[1 + N + i * N + j] : 0.f;
        }
    }
}

// Gradient accumulators of a lane.
template <int RI, int RJ>
struct Grads {
    float gxr[RI], gxc[RJ], dq1c[RJ], dq2[RI][RJ];
    float F[RI][RJ];  // uniform clock: sum_t lambda2_t o S2_{t-1}, scaled by rho_i rho_j once per chunk
    __device__ void zero() {
#pragma unroll
        for (int r = 0; r < RI; ++r) {
            gxr[r] = 0.f;
#pragma unroll
            for (int c = 0; c < RJ; ++c) {
                dq2[r][c] = 0.f;
                F[r][c] = 0.f;
            }
        }
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            gxc[c] = 0.f;
            dq1c[c] = 0.f;
        }
    }
};

// One exact adjoint step at interval t: a holds the cotangent of S_t (g_t already added); S1p/S2p are
// S_{t-1}. Accumulates the gradients, writes dy_t to dyg[0..NP) and turns a into the cotangent of S_{t-1}.
// Per-interval clock (NU): the x-gradient of the step (flow and tables) goes to dL/d(dtheta_t) = r . gx
// (written by lane 0 to *dtg) and to dL/dr += dtheta_t gx (row / column partials in gr.gxr / gr.gxc).
template <int RI, int RJ, bool NU>
__device__ __forceinline__ void bwd_step(const Params& p, const Tables<RI, RJ>& tb, const float fr[RI],
                                         const float fc[RJ], const float* dyk, const float S1p[RI],
                                         const float S2p[RI][RJ], Adj<RI, RJ>& a, Grads<RI, RJ>& gr, float* dyg,
                                         float dth, float* dtg, int i0, int j0, int ti, int tj, bool bp = false) {
    float dyr[RI], dyc[RJ], s1c[RJ], u[RI];
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        dyr[r] = dyk[i0 + r];
        u[r] = fmaf(-fr[r], S1p[r], S1p[r]);
    }
    float q1c[RJ];
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        dyc[c] = dyk[j0 + c];
        q1c[c] = bp ? 1.f : tb.q1c[c];
        s1c[c] = q1c[c] * dyc[c];
    }
    const float table_w = bp ? 0.f : 1.f;  // the basepoint interval does not read the tables
    // row sums: w (adjoint recursion), z (dy from s2, row side)
    float w[RI], z[RI];
    // column partials: y (ds1), v (dy from s2, column side)
    float y[RJ], v[RJ];
    float rowx[RI], colx[RJ];  // NU: this step's x-gradient partials
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        y[c] = 0.f;
        v[c] = 0.f;
        colx[c] = 0.f;
    }
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        float wr = 0.f, zr = 0.f, fx = 0.f;
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            const float l2 = a.L2[r][c];
            const float l2q = l2 * (bp ? 0.5f : tb.q2[r][c]);
            wr = fmaf(l2, s1c[c], wr);
            zr = fmaf(l2q, dyc[c], zr);
            y[c] = fmaf(l2, u[r], y[c]);
            v[c] = fmaf(l2q, dyr[r], v[c]);
            // flow gradient (w.r.t. x = log rho) of rho_i rho_j S2_ij, credited to i and to j
            const float fl = l2 * (1.f - comp_mul(fr[r], fc[c])) * S2p[r][c];
            fx = fmaf(l2, u[r] * s1c[c], fx + fl);
            if (NU) {
                colx[c] += fl;
            } else {
                gr.gxc[c] += fl;
                gr.dq2[r][c] = fmaf(table_w * l2, dyr[r] * dyc[c], gr.dq2[r][c]);
            }
        }
        w[r] = row_sum(wr);
        z[r] = row_sum(zr);
        const float rx = fx + (tj == 0 ? a.L1r[r] * u[r] : 0.f);
        if (NU)
            rowx[r] = rx;
        else
            gr.gxr[r] += rx;
    }
    if (NU) {
        // table derivatives: dQ2/dx_i = sum_a a x_i^(a-1) w_a(x_j), dQ2/dx_j = sum_a x_i^a w'_a(x_j)
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            float wv[kQNU], wd[kQNU];
#pragma unroll
            for (int q = 0; q < kQNU; ++q) {
                wv[q] = poly(p.c2 + q * kQNU, tb.xc[c]);
                wd[q] = dpoly(p.c2 + q * kQNU, tb.xc[c]);
            }
#pragma unroll
            for (int r = 0; r < RI; ++r) {
                const float L = a.L2[r][c] * (dyr[r] * dyc[c]);
                const float x = tb.xr[r];
                float gxv = 0.f, gyv = 0.f;
#pragma unroll
                for (int q = kQNU - 1; q >= 1; --q) gxv = fmaf(gxv, x, (float)q * wv[q]);
#pragma unroll
                for (int q = kQNU - 1; q >= 0; --q) gyv = fmaf(gyv, x, wd[q]);
                rowx[r] = fmaf(L, gxv, rowx[r]);
                colx[c] = fmaf(L, gyv, colx[c]);
            }
        }
    }
    float l1c[RJ], zc[RJ];
    rows_to_cols<RI, RJ>(a.L1r, l1c, tj);
    rows_to_cols<RI, RJ>(z, zc, tj);
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        const float ds1 = l1c[c] + col_sum(y[c]);
        const float vv = col_sum(v[c]);
        if (NU) {
            if (ti == 0) colx[c] = fmaf(ds1 * dyc[c], dpoly(p.c1, tb.xc[c]), colx[c]);
        } else {
            gr.dq1c[c] = fmaf(table_w * ds1, dyc[c], gr.dq1c[c]);
        }
        if (ti == 0) dyg[j0 + c] = fmaf(ds1, q1c[c], vv + zc[c]);
    }
    if (NU) {
        float contrib = 0.f;
#pragma unroll
        for (int r = 0; r < RI; ++r) {
            contrib = fmaf(tb.rr[r], rowx[r], contrib);
            gr.gxr[r] = fmaf(dth, rowx[r], gr.gxr[r]);
        }
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            contrib = fmaf(tb.rc[c], colx[c], contrib);
            gr.gxc[c] = fmaf(dth, colx[c], gr.gxc[c]);
        }
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) contrib += __shfl_xor_sync(kFull, contrib, o);
        if ((threadIdx.x & 31) == 0) *dtg = contrib;
    }
    // cotangent of S_{t-1}
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const float lw = a.L1r[r] + w[r];
        a.L1r[r] = fmaf(-fr[r], lw, lw);
#pragma unroll
        for (int c = 0; c < RJ; ++c) a.L2[r][c] = fmaf(-comp_mul(fr[r], fc[c]), a.L2[r][c], a.L2[r][c]);
    }
}

// The transposed step alone (no gradients): used for the zero-carry local adjoint.
template <int RI, int RJ>
__device__ __forceinline__ void adj_step(const Tables<RI, RJ>& tb, const float fr[RI], const float fc[RJ],
                                         const float* dyk, Adj<RI, RJ>& a, int j0, bool bp = false) {
    float s1c[RJ];
#pragma unroll
    for (int c = 0; c < RJ; ++c) s1c[c] = (bp ? 1.f : tb.q1c[c]) * dyk[j0 + c];
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        float wr = 0.f;
#pragma unroll
        for (int c = 0; c < RJ; ++c) wr = fmaf(a.L2[r][c], s1c[c], wr);
        wr = row_sum(wr) + a.L1r[r];
        a.L1r[r] = fmaf(-fr[r], wr, wr);
#pragma unroll
        for (int c = 0; c < RJ; ++c) a.L2[r][c] = fmaf(-comp_mul(fr[r], fc[c]), a.L2[r][c], a.L2[r][c]);
    }
}

// Uniform clock, not the basepoint interval: the transposed step with the pair complements dd = 1 - rho_i rho_j
// given (they are constant over the path).
template <int RI, int RJ>
__device__ __forceinline__ void adj_step_u(const Tables<RI, RJ>& tb, const float dd[RI][RJ], const float* dyk,
                                           Adj<RI, RJ>& a, int j0) {
    float s1c[RJ];
#pragma unroll
    for (int c = 0; c < RJ; ++c) s1c[c] = tb.q1c[c] * dyk[j0 + c];
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        float wr = 0.f;
#pragma unroll
        for (int c = 0; c < RJ; ++c) wr = fmaf(a.L2[r][c], s1c[c], wr);
        wr = row_sum(wr) + a.L1r[r];
        a.L1r[r] = fmaf(-tb.dr[r], wr, wr);
#pragma unroll
        for (int c = 0; c < RJ; ++c) a.L2[r][c] = fmaf(-dd[r][c], a.L2[r][c], a.L2[r][c]);
    }
}

// Uniform clock, not the basepoint interval: bwd_step with the pair complements given. The flow gradient's
// level-2 part rho_i rho_j lambda2 S2_{t-1} is accumulated as sum_t lambda2 o S2_{t-1} (gr.F) and scaled by
// the constant rho_i rho_j once per chunk (lane blocks up to 18 entries; larger ones credit it every step,
// which needs no accumulator registers); its level-1 part sum_j lambda2_ij u_i s1_j = u_i (lambda2 s1)_i
// reuses the adjoint recursion's row partials. l1w = 1 on the lane that credits lambda1 u (tj == 0).
template <int RI, int RJ>
__host__ __device__ constexpr bool accumulate_flow_terms() { return RI * RJ <= 18; }

template <int RI, int RJ>
__device__ __forceinline__ void bwd_step_u(const Tables<RI, RJ>& tb, const float dd[RI][RJ], const float* dyk,
                                           const float S1p[RI], const float S2p[RI][RJ], Adj<RI, RJ>& a,
                                           Grads<RI, RJ>& gr, float* dyg, int i0, int j0, int ti, int tj, float l1w) {
    float dyr[RI], dyc[RJ], s1c[RJ], u[RI];
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        dyr[r] = dyk[i0 + r];
        u[r] = fmaf(-tb.dr[r], S1p[r], S1p[r]);
    }
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        dyc[c] = dyk[j0 + c];
        s1c[c] = tb.q1c[c] * dyc[c];
    }
    float w[RI], z[RI], y[RJ], v[RJ];
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        y[c] = 0.f;
        v[c] = 0.f;
    }
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        float wr = 0.f, zr = 0.f, fx = 0.f;
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            const float l2 = a.L2[r][c];
            const float l2q = l2 * tb.q2[r][c];
            wr = fmaf(l2, s1c[c], wr);
            zr = fmaf(l2q, dyc[c], zr);
            y[c] = fmaf(l2, u[r], y[c]);
            v[c] = fmaf(l2q, dyr[r], v[c]);
            if (accumulate_flow_terms<RI, RJ>()) {
                gr.F[r][c] = fmaf(l2, S2p[r][c], gr.F[r][c]);
            } else {
                float fl = l2 * S2p[r][c];
                fl = fmaf(-dd[r][c], fl, fl);
                fx += fl;
                gr.gxc[c] += fl;
            }
            gr.dq2[r][c] = fmaf(l2, dyr[r] * dyc[c], gr.dq2[r][c]);
        }
        gr.gxr[r] = fmaf(u[r], fmaf(l1w, a.L1r[r], wr), gr.gxr[r] + fx);
        w[r] = row_sum(wr);
        z[r] = row_sum(zr);
    }
    float l1c[RJ], zc[RJ];
    rows_to_cols<RI, RJ>(a.L1r, l1c, tj);
    rows_to_cols<RI, RJ>(z, zc, tj);
#pragma unroll
    for (int c = 0; c < RJ; ++c) {
        const float ds1 = l1c[c] + col_sum(y[c]);
        const float vv = col_sum(v[c]);
        gr.dq1c[c] = fmaf(ds1, dyc[c], gr.dq1c[c]);
        if (ti == 0) dyg[j0 + c] = fmaf(ds1, tb.q1c[c], vv + zc[c]);
    }
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const float lw = a.L1r[r] + w[r];
        a.L1r[r] = fmaf(-tb.dr[r], lw, lw);
#pragma unroll
        for (int c = 0; c < RJ; ++c) a.L2[r][c] = fmaf(-dd[r][c], a.L2[r][c], a.L2[r][c]);
    }
}

// Stages n floats from global memory at the shared-memory offset off (floats from base) with cp.async and
// returns the offset of the first element (the copy keeps the source's 16-byte phase). Offsets rather than
// pointers keep the later reads in the shared address space.
__device__ __forceinline__ int stage_span(float* base, int off, const float* src, int n) {
    const int shift = (int)(((uintptr_t)src & 15u) >> 2);
    warp_load_span_async(base + off, src, n);
    return off + shift;
}

// Under a uniform clock, lane blocks of up to 8 level-2 entries (N <= 16) read the backward's rows straight
// into registers, one row ahead; larger blocks and the per-interval clock (whose tables take the registers)
// stage blocks of rows in shared memory with cp.async.
template <int RI, int RJ, bool NU>
__host__ __device__ constexpr bool rows_in_registers() { return !NU && RI * RJ <= 8; }

// Rows the register path asks L2 for ahead of its loads (the loads themselves run one row ahead).
constexpr int kPrefetchRows = 6;

template <int RI, int RJ>
__device__ __forceinline__ void add_grad_vals(Adj<RI, RJ>& a, const float g1[RI], const float g2[RI][RJ]) {
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        a.L1r[r] += g1[r];
#pragma unroll
        for (int c = 0; c < RJ; ++c) a.L2[r][c] += g2[r][c];
    }
}

template <int RI, int RJ>
__device__ __forceinline__ void copy_vals(float d1[RI], float d2[RI][RJ], const float s1[RI], const float s2[RI][RJ]) {
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        d1[r] = s1[r];
#pragma unroll
        for (int c = 0; c < RJ; ++c) d2[r][c] = s2[r][c];
    }
}

template <int RI, int RJ>
__device__ __forceinline__ void add_grad_row(Adj<RI, RJ>& a, const float* row, int N, int i0, int j0) {
    float g1[RI], g2[RI][RJ];
    read_row<RI, RJ>(row, g1, g2, N, i0, j0);
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        a.L1r[r] += g1[r];
#pragma unroll
        for (int c = 0; c < RJ; ++c) a.L2[r][c] += g2[r][c];
    }
}

// Writes dx (the gradient of the input increments) of the chunk and accumulates the lift gradient.
template <int RI, int RJ>
__device__ void finish_chunk(const Params& p, const float* liftS, const float* dxs, const float* dyg, const float* dtg,
                             float* stage, int b, int t0, int len, int tile, const Grads<RI, RJ>& gr, int i0, int j0,
                             int ti, int tj) {
    const Geom& g = p.g;
    const int lane = threadIdx.x & 31;
    const int NP = g.NP;
    __syncwarp();
    if (g.nu) warp_store_span(p.grad_dtheta + (size_t)b * g.T + t0, dtg, len);
    // dx_t = lift^T dy_t, staged contiguously, then one span store
    for (int e = lane; e < len * g.d_in; e += 32) {
        const int k = e / g.d_in, cc = e - k * g.d_in;
        float acc = 0.f;
        if (p.lift) {
            const float* liftR = liftS + g.lift_n / 2;
            for (int i = 0; i < g.N; ++i) acc = fmaf(liftR[i * g.d_in + cc], dyg[k * NP + i], acc);
        } else {
            acc = dyg[k * NP + cc];
        }
        stage[e] = acc;
    }
    __syncwarp();
    warp_store_span(p.grad_dx + ((size_t)b * g.T + t0) * g.d_in, stage, len * g.d_in);
    __syncwarp();
    float* part = p.partials + (size_t)tile * (2 * NP + NP * NP + NP * g.d_in);
    // lift gradient: sum_t dy_t dx_t^T (dx recomputed from the input)
    if (p.lift) {
        for (int e = lane; e < NP * g.d_in; e += 32) {
            const int i = e / g.d_in, cc = e - i * g.d_in;
            float acc = 0.f;
            if (i < g.N)
                for (int k = 0; k < len; ++k)
                    acc = fmaf(dyg[k * NP + i], dxs[k * g.d_in + cc], acc);
            part[2 * NP + NP * NP + e] = acc;
        }
    }
    // flow gradient = row part (summed over the row group's lanes) + column part (over the column group's);
    // the row owner (tj == 0) writes first, the column owner (ti == 0) adds after a warp barrier
#pragma unroll
    for (int r = 0; r < RI; ++r) {
        const float s = row_sum(gr.gxr[r]);
        if (tj == 0) part[i0 + r] = s;
    }
    float colpart[RJ];
#pragma unroll
    for (int c = 0; c < RJ; ++c) colpart[c] = col_sum(gr.gxc[c]);
    __syncwarp();
    if (ti == 0) {
#pragma unroll
        for (int c = 0; c < RJ; ++c) {
            part[j0 + c] += colpart[c];
            part[NP + j0 + c] = gr.dq1c[c];  // identical on the 4 lanes of a column group
        }
    }
#pragma unroll
    for (int r = 0; r < RI; ++r)
#pragma unroll
        for (int c = 0; c < RJ; ++c) part[2 * NP + (i0 + r) * NP + j0 + c] = gr.dq2[r][c];
}

template <int NP, bool NU, bool FULL>
__global__ void __launch_bounds__(kWarps * 32) bwd_kernel(Params p) {
    // FULL: N == NP, so row indices and bounds are compile-time constants
    constexpr int RI = NP / 4, RJ = NP / 8;
    extern __shared__ float smem[];
    const Geom& g = p.g;
    const int Nr = FULL ? NP : g.N;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float* liftS = smem;
    for (int e = threadIdx.x; e < NP * g.d_in; e += blockDim.x) {
        const int r = e / g.d_in, cc = e - r * g.d_in;
        const float w = (p.lift && r < g.N) ? p.lift[r * g.d_in + cc] : 0.f;
        liftS[cc * NP + r] = w;                    // channel-major: the lift of the increments
        liftS[g.lift_n / 2 + r * g.d_in + cc] = w;  // row-major: the gradient's map back to dx
    }
    __syncthreads();
    // per warp: dxs, dys, dyg (Lc x NP), lam1 (Lc x NP, terminal only), gst (gradient rows, and the dx
    // staging), sst (forward rows, prefix only)
    float* dxs = smem + g.lift_n + warp * g.b_per_warp;
    float* dys = dxs + g.b_dys;
    float* dts = dxs + g.b_dts;  // per-interval clock steps
    float* dtg = dxs + g.b_dtg;  // dL/d(dtheta) of the chunk's intervals
    float* dyg = dxs + g.b_dyg;
    float* lam1 = dxs + g.b_lam1;
    float* gst = dxs + g.b_gst;

    const int ti = lane >> 3, tj = lane & 7;
    const int i0 = ti * RI, j0 = tj * RJ;
    const bool basepoint = (g.flags & EWS_F_BASEPOINT) != 0;
    const bool terminal = g.readout == EWS_READOUT_TERMINAL;

    for (;;) {
        const int tile = next_ticket(p.st);
        if (tile >= g.ntiles) break;
        const int cr = tile / g.B, b = tile - cr * g.B;
        const int c = g.C - 1 - cr;
        const int t0 = c * g.Lc;
        const int len = min(g.Lc, g.T - t0);
        Tables<RI, RJ> tb;
        if (NU)
            tb.load_rates(p, b, i0, j0);
        else
            tb.load(p, b, i0, j0);
        load_increments(p, liftS, dxs, dys, dts, b, t0, len);
        const size_t slot = ((size_t)b * g.C + c) * g.SW;
        int* flag = p.flags + (size_t)b * g.C + c;
        // elapsed clock from the end of interval t to the end of the path (NU), else a step count
        const float* ck = NU ? p.clock + (size_t)b * (g.T + 1) : nullptr;
        const float clock_end = NU ? ck[g.T] : 0.f;
        const float clock_chunk_end = NU ? ck[t0 + len] : 0.f;
        float ur[RI], uc[RJ];  // rates (NU) or log-flows: exponents are elapsed x these
#pragma unroll
        for (int r = 0; r < RI; ++r) ur[r] = NU ? tb.rr[r] : tb.xr[r];
#pragma unroll
        for (int cc = 0; cc < RJ; ++cc) uc[cc] = NU ? tb.rc[cc] : tb.xc[cc];

        // terminal readout: lambda2_t = E_i E_j g2 with E = e^{(T-1-t) x}; load g once
        float tg1[RI], tg2[RI][RJ];
        if (terminal) read_row<RI, RJ>(p.grad_out + (size_t)b * g.W, tg1, tg2, Nr, i0, j0);

        // ---- 1. zero-carry local adjoint over the chunk (reverse)
        Adj<RI, RJ> mu;
        mu.zero();
        // uniform clock: the pair complements 1 - rho_i rho_j are constant; the basepoint interval (k = 0 of
        // chunk 0) runs apart from the loops
        const bool bpc = basepoint && t0 == 0;
        float dd[RI][RJ];
#pragma unroll
        for (int r = 0; r < RI; ++r)
#pragma unroll
            for (int cc = 0; cc < RJ; ++cc) dd[r][cc] = NU ? 0.f : comp_mul(tb.dr[r], tb.dc[cc]);
        if (!terminal && !rows_in_registers<RI, RJ, NU>()) {
            // gradient rows in blocks of SR, the next block copied in while this one runs
            int slot = 0;
            int cur = stage_span(dxs, g.b_gst, p.grad_out + ((size_t)b * g.T + t0 + max(0, len - g.SR)) * g.W,
                                 (len - max(0, len - g.SR)) * g.W);
            cp_async_commit();
            for (int kb = len; kb > 0; kb -= g.SR) {
                const int k0 = max(0, kb - g.SR);
                int nxt = 0;
                if (k0 > 0) {
                    const int k1 = max(0, k0 - g.SR);
                    nxt = stage_span(dxs, slot ? g.b_gst : g.b_gst2, p.grad_out + ((size_t)b * g.T + t0 + k1) * g.W,
                                     (k0 - k1) * g.W);
                }
                cp_async_commit();
                cp_async_wait<1>();
                __syncwarp();
                const float* rows = dxs + cur;
                const int kl = (bpc && k0 == 0) ? 1 : k0;
                for (int k = kb - 1; k >= kl; --k) {
                    add_grad_row(mu, rows + (k - k0) * g.W, Nr, i0, j0);
                    if (NU) {
                        float fr[RI], fc[RJ];
                        tb.at(p, dts[k]);
                        step_flow(tb, false, fr, fc);
                        adj_step(tb, fr, fc, dys + k * NP, mu, j0, false);
                    } else {
                        adj_step_u(tb, dd, dys + k * NP, mu, j0);
                    }
                }
                if (kl > k0) {
                    add_grad_row(mu, rows, Nr, i0, j0);
                    float fr[RI], fc[RJ];
                    step_flow(tb, true, fr, fc);
                    adj_step(tb, fr, fc, dys, mu, j0, true);
                }
                __syncwarp();
                cur = nxt;
                slot ^= 1;
            }
            cp_async_wait<0>();
            __syncwarp();
        } else if (!terminal) {
            // gradient rows straight into registers, the next row's loads in flight while this step runs
            const float* grow = p.grad_out + ((size_t)b * g.T + t0) * g.W;
            float g1[RI], g2[RI][RJ];
            read_row<RI, RJ>(grow + (size_t)(len - 1) * g.W, g1, g2, Nr, i0, j0);
            const int kl = bpc ? 1 : 0;
            for (int k = len - 1; k >= len - kPrefetchRows && k >= 0; --k) prefetch_span_l2(grow + (size_t)k * g.W, g.W);
#pragma unroll 2
            for (int k = len - 1; k >= kl; --k) {
                if (k >= kPrefetchRows) prefetch_span_l2(grow + (size_t)(k - kPrefetchRows) * g.W, g.W);
                float n1[RI], n2[RI][RJ];
                read_row<RI, RJ>(grow + (size_t)max(k - 1, 0) * g.W, n1, n2, Nr, i0, j0);
                add_grad_vals(mu, g1, g2);
                if (NU) {
                    float fr[RI], fc[RJ];
                    tb.at(p, dts[k]);
                    step_flow(tb, false, fr, fc);
                    adj_step(tb, fr, fc, dys + k * NP, mu, j0, false);
                } else {
                    adj_step_u(tb, dd, dys + k * NP, mu, j0);
                }
                copy_vals<RI, RJ>(g1, g2, n1, n2);
            }
            if (kl) {  // the basepoint interval; g1, g2 hold row 0
                add_grad_vals(mu, g1, g2);
                float fr[RI], fc[RJ];
                step_flow(tb, true, fr, fc);
                adj_step(tb, fr, fc, dys, mu, j0, true);
            }
        } else {
            // lambda1 only (lambda2 is closed form): mu1_{t-1} = rho (mu1_t + lambda2_t s1_t); g1 enters at T-1
            for (int k = len - 1; k >= 0; --k) {
                const int t = t0 + k;
                if (t == g.T - 1) {
#pragma unroll
                    for (int r = 0; r < RI; ++r) mu.L1r[r] += tg1[r];
                }
                if (tj == 0) {
#pragma unroll
                    for (int r = 0; r < RI; ++r) lam1[k * NP + i0 + r] = mu.L1r[r];
                }
                float fr[RI], fc[RJ];
                if (NU) tb.at(p, dts[k]);
                const bool bp = basepoint && (t == 0);
                step_flow(tb, bp, fr, fc);
                const float steps_after = NU ? clock_end - ck[t + 1] : (float)(g.T - 1 - t);
                float ecs[RJ];
#pragma unroll
                for (int cc = 0; cc < RJ; ++cc)
                    ecs[cc] = expf(steps_after * uc[cc]) * (bp ? 1.f : tb.q1c[cc]) * dys[k * NP + j0 + cc];
#pragma unroll
                for (int r = 0; r < RI; ++r) {
                    const float er = expf(steps_after * ur[r]);
                    float wr = 0.f;
#pragma unroll
                    for (int cc = 0; cc < RJ; ++cc) wr = fmaf(er * tg2[r][cc], ecs[cc], wr);
                    wr = row_sum(wr) + mu.L1r[r];
                    mu.L1r[r] = fmaf(-fr[r], wr, wr);
                }
            }
        }

        // ---- 2. look-back over the later chunks for the carry cotangent Lam_in (of S at the chunk's end)
        Adj<RI, RJ> lam_in;
        lam_in.zero();
        Elem<RI, RJ> Gc;
        load_elem(p.fagg + slot, Gc, NP, i0, j0);
        if (c == g.C - 1) {
            store_adj(p.incl + slot, mu, NP, i0, j0, tj);
            if (!(g.flags & EWS_F_TEST_WITHHOLD)) publish(flag, kFlagIncl);
        } else {
            store_adj(p.agg + slot, mu, NP, i0, j0, tj);
            publish(flag, kFlagAgg);
            Adj<RI, RJ> acc;
            acc.zero();
            Elem<RI, RJ> Gacc;
            Gacc.identity();
            int j = c + 1;
            const int want = (g.flags & EWS_F_DETERMINISTIC) ? kFlagIncl : kFlagAgg;
            for (;;) {
                const int f = wait_slot(p.flags + (size_t)b * g.C + j, p.st, g.spin_limit, tile, want);
                if (f < 0) return;
                const size_t sj = ((size_t)b * g.C + j) * g.SW;
                Adj<RI, RJ> X;
                if (f == kFlagIncl) {
                    load_adj(p.incl + sj, X, NP, i0, j0);
                    apply_JT(Gacc, X);
                    adj_add(acc, X);
                    break;
                }
                load_adj(p.agg + sj, X, NP, i0, j0);
                apply_JT(Gacc, X);
                adj_add(acc, X);
                Elem<RI, RJ> Gj;
                load_elem(p.fagg + sj, Gj, NP, i0, j0);
                chen_mul(Gacc, Gj, Gacc);
                ++j;
            }
            lam_in = acc;
            Adj<RI, RJ> out = lam_in;
            apply_JT(Gc, out);
            adj_add(out, mu);
            store_adj(p.incl + slot, out, NP, i0, j0, tj);
            publish(flag, kFlagIncl);
        }

        // ---- 3. exact adjoint from the carry, with the gradients
        Grads<RI, RJ> gr;
        gr.zero();
        if (!terminal) {
            Adj<RI, RJ> a = lam_in;
            const float l1w = tj == 0 ? 1.f : 0.f;
            if (!rows_in_registers<RI, RJ, NU>()) {
            // block [k0, kb): gradient rows t0+k0.. and S_{t-1} rows t0+k0-1.. (row -1 is the zero state),
            // the next block copied in while this one runs
            auto stage = [&](int k0s, int kbs, int sl, int& gs, int& ss) {
                const int ns = kbs - k0s;
                gs = stage_span(dxs, sl ? g.b_gst2 : g.b_gst, p.grad_out + ((size_t)b * g.T + t0 + k0s) * g.W, ns * g.W);
                const int first = t0 + k0s - 1;
                const int soff = sl ? g.b_sst2 : g.b_sst;
                if (first >= 0) {
                    ss = stage_span(dxs, soff, p.out + ((size_t)b * g.T + first) * g.W, ns * g.W);
                } else {
                    // row -1 is zero; rows 0.. follow it, placed at the source's 16-byte phase
                    const int shift = (int)(((uintptr_t)(p.out + (size_t)b * g.T * g.W) & 15u) >> 2);
                    const int lead = (shift - g.W % 4 + 8) % 4;  // so that row 0 has the source's phase
                    ss = soff + lead;
                    for (int e = lane; e < g.W; e += 32) dxs[ss + e] = 0.f;
                    if (ns > 1)
                        warp_load_span_async(dxs + ss + g.W - shift, p.out + (size_t)b * g.T * g.W, (ns - 1) * g.W);
                }
            };
            int slot = 0;
            int gcur, scur, gnxt = 0, snxt = 0;
            stage(max(0, len - g.SR), len, 0, gcur, scur);
            cp_async_commit();
            for (int kb = len; kb > 0; kb -= g.SR) {
                const int k0 = max(0, kb - g.SR);
                if (k0 > 0) stage(max(0, k0 - g.SR), k0, slot ^ 1, gnxt, snxt);
                cp_async_commit();
                cp_async_wait<1>();
                __syncwarp();
                const float* grows = dxs + gcur;
                const float* srows = dxs + scur;
                const int kl = (bpc && k0 == 0) ? 1 : k0;
                for (int k = kb - 1; k >= kl; --k) {
                    add_grad_row(a, grows + (k - k0) * g.W, Nr, i0, j0);
                    float S1p[RI], S2p[RI][RJ];
                    read_row<RI, RJ>(srows + (k - k0) * g.W, S1p, S2p, Nr, i0, j0);
                    if (NU) {
                        float fr[RI], fc[RJ];
                        tb.at(p, dts[k]);
                        step_flow(tb, false, fr, fc);
                        bwd_step<RI, RJ, NU>(p, tb, fr, fc, dys + k * NP, S1p, S2p, a, gr, dyg + k * NP, dts[k],
                                             dtg + k, i0, j0, ti, tj, false);
                    } else {
                        bwd_step_u<RI, RJ>(tb, dd, dys + k * NP, S1p, S2p, a, gr, dyg + k * NP, i0, j0, ti, tj, l1w);
                    }
                }
                if (kl > k0) {
                    add_grad_row(a, grows, Nr, i0, j0);
                    float S1p[RI], S2p[RI][RJ];
                    read_row<RI, RJ>(srows, S1p, S2p, Nr, i0, j0);
                    float fr[RI], fc[RJ];
                    step_flow(tb, true, fr, fc);
                    bwd_step<RI, RJ, NU>(p, tb, fr, fc, dys, S1p, S2p, a, gr, dyg, 0.f, dtg, i0, j0, ti, tj, true);
                }
                __syncwarp();
                gcur = gnxt;
                scur = snxt;
                slot ^= 1;
            }
            cp_async_wait<0>();
            __syncwarp();
            } else {
            // gradient row t and state row t-1 straight into registers, the next pair's loads in flight while
            // this step runs; chunk 0's first interval (state row -1 = 0) runs after the loop
            const size_t rb = (size_t)b * g.T + t0;
            const float* grow = p.grad_out + rb * g.W;
            const int klo = t0 == 0 ? 1 : 0;
            float g1[RI], g2[RI][RJ], s1[RI], s2[RI][RJ];
            for (int k = len - 1; k >= len - kPrefetchRows && k >= klo; --k) {
                prefetch_span_l2(grow + (size_t)k * g.W, g.W);
                prefetch_span_l2(p.out + (rb + k - 1) * g.W, g.W);
            }
            read_row<RI, RJ>(grow + (size_t)(len - 1) * g.W, g1, g2, Nr, i0, j0);
            if (len - 1 >= klo) read_row<RI, RJ>(p.out + (rb + len - 2) * g.W, s1, s2, Nr, i0, j0);
#pragma unroll 2
            for (int k = len - 1; k >= klo; --k) {
                if (k - kPrefetchRows >= klo) {
                    prefetch_span_l2(grow + (size_t)(k - kPrefetchRows) * g.W, g.W);
                    prefetch_span_l2(p.out + (rb + k - kPrefetchRows - 1) * g.W, g.W);
                }
                float n1[RI], n2[RI][RJ], m1[RI], m2[RI][RJ];
                read_row<RI, RJ>(grow + (size_t)max(k - 1, 0) * g.W, n1, n2, Nr, i0, j0);
                read_row<RI, RJ>(p.out + (rb + max(k - 1, klo) - 1) * g.W, m1, m2, Nr, i0, j0);
                add_grad_vals(a, g1, g2);
                if (NU) {
                    float fr[RI], fc[RJ];
                    tb.at(p, dts[k]);
                    step_flow(tb, false, fr, fc);
                    bwd_step<RI, RJ, NU>(p, tb, fr, fc, dys + k * NP, s1, s2, a, gr, dyg + k * NP, dts[k], dtg + k, i0,
                                         j0, ti, tj, false);
                } else {
                    bwd_step_u<RI, RJ>(tb, dd, dys + k * NP, s1, s2, a, gr, dyg + k * NP, i0, j0, ti, tj, l1w);
                }
                copy_vals<RI, RJ>(g1, g2, n1, n2);
                copy_vals<RI, RJ>(s1, s2, m1, m2);
            }
            if (klo) {  // interval 0: g1, g2 hold gradient row 0; the state before it is zero
                add_grad_vals(a, g1, g2);
#pragma unroll
                for (int r = 0; r < RI; ++r) {
                    s1[r] = 0.f;
#pragma unroll
                    for (int cc = 0; cc < RJ; ++cc) s2[r][cc] = 0.f;
                }
                float fr[RI], fc[RJ];
                if (NU) tb.at(p, dts[0]);
                step_flow(tb, bpc, fr, fc);
                if (NU || bpc) {
                    bwd_step<RI, RJ, NU>(p, tb, fr, fc, dys, s1, s2, a, gr, dyg, NU ? dts[0] : 0.f, dtg, i0, j0, ti, tj,
                                         bpc);
                } else {
                    bwd_step_u<RI, RJ>(tb, dd, dys, s1, s2, a, gr, dyg, i0, j0, ti, tj, l1w);
                }
            }
            }
            if (!NU && accumulate_flow_terms<RI, RJ>()) {
                // the flow gradient's level-2 part: rho_i rho_j sum_t lambda2 o S2_{t-1}, credited to i and to j
#pragma unroll
                for (int r = 0; r < RI; ++r)
#pragma unroll
                    for (int cc = 0; cc < RJ; ++cc) {
                        const float fl = fmaf(-dd[r][cc], gr.F[r][cc], gr.F[r][cc]);
                        gr.gxr[r] += fl;
                        gr.gxc[cc] += fl;
                    }
            }
        } else {
            // forward sweep from the carry with lambda2 in closed form and lambda1 = mu1 + rho^{end-t} Lam1_in
            Elem<RI, RJ> S;
            load_elem(p.fcarry + slot, S, NP, i0, j0);
            for (int k = 0; k < len; ++k) {
                const int t = t0 + k;
                const float steps_after = NU ? clock_end - ck[t + 1] : (float)(g.T - 1 - t);
                const float steps_to_end = NU ? clock_chunk_end - ck[t + 1] : (float)(len - 1 - k);
                Adj<RI, RJ> a;
                float ecs[RJ];
#pragma unroll
                for (int cc = 0; cc < RJ; ++cc) ecs[cc] = expf(steps_after * uc[cc]);
#pragma unroll
                for (int r = 0; r < RI; ++r) {
                    const float er = expf(steps_after * ur[r]);
                    a.L1r[r] = lam1[k * NP + i0 + r] + expf(steps_to_end * ur[r]) * lam_in.L1r[r];
#pragma unroll
                    for (int cc = 0; cc < RJ; ++cc) a.L2[r][cc] = er * ecs[cc] * tg2[r][cc];
                }
                float S1p[RI], S2p[RI][RJ];
#pragma unroll
                for (int r = 0; r < RI; ++r) {
                    S1p[r] = S.S1r[r];
#pragma unroll
                    for (int cc = 0; cc < RJ; ++cc) S2p[r][cc] = S.S2[r][cc];
                }
                float fr[RI], fc[RJ];
                if (NU) tb.at(p, dts[k]);
                const bool bp = basepoint && (t == 0);
                step_flow(tb, bp, fr, fc);
                bwd_step<RI, RJ, NU>(p, tb, fr, fc, dys + k * NP, S1p, S2p, a, gr, dyg + k * NP, NU ? dts[k] : 0.f,
                                     dtg + k, i0, j0, ti, tj, bp);
                chen_step(tb, dys + k * NP, i0, j0, S, fr, fc, bp);
            }
        }
        finish_chunk<RI, RJ>(p, liftS, dxs, dyg, dtg, gst, b, t0, len, tile, gr, i0, j0, ti, tj);
    }
}

// Deterministic two-stage reduction of the per-tile partials (fixed summation orders, coalesced reads).
// Stage 1: per sample, over its chunks -> sp (B, stride).
__global__ void reduce_chunks_kernel(Params p, float* sp) {
    const Geom& g = p.g;
    const int NP = g.NP;
    const int stride = 2 * NP + NP * NP + NP * g.d_in;
    const size_t total = (size_t)g.B * stride;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int b = (int)(e / stride), off = (int)(e - (size_t)b * stride);
        float acc = 0.f;
        for (int cr = 0; cr < g.C; ++cr) acc += p.partials[((size_t)cr * g.B + b) * stride + off];
        sp[e] = acc;
    }
}

// Stage 2: per-sample table gradients (compacted to the real dimension N) and the lift gradient summed
// over the samples in order.
__global__ void reduce_samples_kernel(Params p, const float* sp, float* grad_x, float* grad_q1, float* grad_q2,
                                      float* grad_lift) {
    const Geom& g = p.g;
    const int NP = g.NP, N = g.N;
    const int stride = 2 * NP + NP * NP + NP * g.d_in;
    const int per_sample = 2 * N + N * N;
    const int total = g.B * per_sample + (grad_lift ? N * g.d_in : 0);
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < total; e += gridDim.x * blockDim.x) {
        if (e < g.B * per_sample) {
            const int b = e / per_sample, r = e - b * per_sample;
            const float* row = sp + (size_t)b * stride;
            if (r < N) {
                grad_x[(size_t)b * N + r] = row[r];
            } else if (r < 2 * N) {
                if (grad_q1) grad_q1[(size_t)b * N + (r - N)] = row[NP + (r - N)];
            } else {
                const int q = r - 2 * N, i = q / N, j = q - i * N;
                if (grad_q2) grad_q2[(size_t)b * N * N + q] = row[2 * NP + i * NP + j];
            }
        } else {
            const int q = e - g.B * per_sample;
            float acc = 0.f;
            for (int b = 0; b < g.B; ++b) acc += sp[(size_t)b * stride + 2 * NP + NP * NP + q];
            grad_lift[q] = acc;
        }
    }
}

// --------------------------------------------------------------------------------- host side

static int pick_chunk(int B, int T) {
    const int want_tiles = 148 * 16;
    int C = (want_tiles + B - 1) / B;
    if (C < 1) C = 1;
    int Lc = (T + C - 1) / C;
    if (Lc < 16) Lc = 16;
    if (Lc > 64) Lc = 64;
    return Lc;
}

constexpr int kWarpFloatBudget = 4096;  // 16 KB of shared memory per warp

static void carve(Geom* g) {
    const int Lc = g->Lc, NP = g->NP;
    const int SR = g->SR < Lc ? g->SR : Lc;
    g->SR = SR;
    g->lift_n = 2 * align4(NP * g->d_in);  // channel-major and row-major copies
    const int xs = align4(Lc * g->d_in), ys = align4(Lc * NP), ts = g->nu ? align4(Lc) : 0;
    g->f_dys = xs;
    g->f_dts = xs + ys;
    g->f_stage = xs + ys + ts;
    g->f_per_warp = g->f_stage + align4(SR * g->W);
    const bool terminal = g->readout == EWS_READOUT_TERMINAL;
    // SR rows at any 16-byte phase; N <= 16 under a uniform clock reads the backward's rows into registers
    const int span = (NP > 16 || g->nu) ? align4(SR * g->W + 4) : 0;
    const int gst_n = align4(std::max(terminal ? 0 : span, Lc * g->d_in));
    g->b_dys = xs;
    g->b_dts = xs + ys;
    g->b_dtg = g->b_dts + ts;
    g->b_dyg = g->b_dtg + ts;
    g->b_lam1 = g->b_dyg + ys;
    g->b_gst = g->b_lam1 + (terminal ? ys : 0);
    // prefix readouts double-buffer the gradient rows and the S_{t-1} rows (two slots each)
    g->b_gst2 = g->b_gst + gst_n;
    g->b_sst = g->b_gst2 + (terminal ? 0 : span);
    g->b_sst2 = g->b_sst + (terminal ? 0 : span);
    g->b_per_warp = g->b_sst2 + (terminal ? 0 : span);
}

static int make_geom(const ews_diag_args* a, Geom* g) {
    if (!a || a->batch <= 0 || a->steps <= 0 || a->d_in <= 0 || a->dim <= 0) return EWS_ERR_INVALID_ARGUMENT;
    if (a->depth != 2) return EWS_ERR_UNSUPPORTED;
    if (a->dim > 32) return EWS_ERR_UNSUPPORTED;
    const bool nu = !(a->flags & EWS_F_UNIFORM);
    if (nu && (a->flags & EWS_F_BASEPOINT)) return EWS_ERR_INVALID_ARGUMENT;
    if (nu && (a->series_q < 0 || a->series_q >= kQNU)) return EWS_ERR_UNSUPPORTED;
    if (a->readout != EWS_READOUT_PREFIX && a->readout != EWS_READOUT_TERMINAL) return EWS_ERR_INVALID_ARGUMENT;
    if ((a->flags & EWS_F_BF16) && !(a->flags & EWS_F_INCREMENTS)) return EWS_ERR_INVALID_ARGUMENT;
    g->nu = nu ? 1 : 0;
    g->B = a->batch;
    g->T = a->steps;
    g->d_in = a->d_in;
    g->N = a->dim;
    g->NP = (a->dim + 7) / 8 * 8;
    g->Lc = a->chunk > 0 ? a->chunk : pick_chunk(a->batch, a->steps);
    g->C = (g->T + g->Lc - 1) / g->Lc;
    g->W = 1 + g->N + g->N * g->N;
    g->SW = 2 * g->NP + g->NP * g->NP;
    g->readout = a->readout;
    g->flags = a->flags;
    g->spin_limit = a->spin_limit > 0 ? a->spin_limit : kDefaultSpinLimit;
    g->SR = g->W >= 512 ? 1 : (512 + g->W - 1) / g->W;
    // shrink the chunk until the backward's per-warp buffers fit the budget (>= 3 CTAs of kWarps per SM)
    for (;;) {
        carve(g);
        if (a->chunk > 0 || g->b_per_warp <= kWarpFloatBudget || g->Lc <= 8) break;
        g->Lc = g->Lc > 16 ? g->Lc - 8 : 8;
    }
    g->C = (g->T + g->Lc - 1) / g->Lc;
    g->ntiles = g->B * g->C;
    return EWS_OK;
}

static size_t al256(size_t n) { return (n + 255) & ~(size_t)255; }

struct WsLayout {
    size_t status, flags, agg, incl, carry, partials, sample_partials, total;
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
    L.total = o;
    return L;
}

static WsLayout bwd_layout(const Geom& g) {
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
    const size_t stride = 2 * g.NP + g.NP * g.NP + g.NP * g.d_in;
    L.partials = o;
    o += al256(sizeof(float) * (size_t)g.ntiles * stride);
    L.sample_partials = o;
    o += al256(sizeof(float) * (size_t)g.B * stride);
    L.total = o;
    return L;
}

static size_t fwd_smem(const Geom& g) { return sizeof(float) * ((size_t)g.lift_n + (size_t)kWarps * g.f_per_warp); }

static size_t bwd_smem(const Geom& g) { return sizeof(float) * ((size_t)g.lift_n + (size_t)kWarps * g.b_per_warp); }

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

template <int NP, bool NU, bool FULL>
static int launch_fwd_t(const Params& p, cudaStream_t s) {
    const size_t smem = fwd_smem(p.g);
    cudaFuncSetAttribute(fwd_kernel<NP, NU, FULL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int per_sm = 0;
    per_sm = resident_ctas((const void*)fwd_kernel<NP, NU, FULL>, kWarps * 32, smem);
    if (per_sm < 1) return EWS_ERR_UNSUPPORTED;
    int grid = per_sm * num_sms();
    const int need = (p.g.ntiles + kWarps - 1) / kWarps;
    if (grid > need) grid = need;
    fwd_kernel<NP, NU, FULL><<<grid, kWarps * 32, smem, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

template <int NP>
static int launch_fwd(const Params& p, cudaStream_t s) {
    const bool full = p.g.N == NP;
    if (p.g.nu) return full ? launch_fwd_t<NP, true, true>(p, s) : launch_fwd_t<NP, true, false>(p, s);
    return full ? launch_fwd_t<NP, false, true>(p, s) : launch_fwd_t<NP, false, false>(p, s);
}

template <int NP, bool NU, bool FULL>
static int launch_bwd_t(const Params& p, cudaStream_t s) {
    const size_t smem = bwd_smem(p.g);
    cudaFuncSetAttribute(bwd_kernel<NP, NU, FULL>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    int per_sm = 0;
    per_sm = resident_ctas((const void*)bwd_kernel<NP, NU, FULL>, kWarps * 32, smem);
    if (per_sm < 1) return EWS_ERR_UNSUPPORTED;
    int grid = per_sm * num_sms();
    const int need = (p.g.ntiles + kWarps - 1) / kWarps;
    if (grid > need) grid = need;
    bwd_kernel<NP, NU, FULL><<<grid, kWarps * 32, smem, s>>>(p);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

template <int NP>
static int launch_bwd(const Params& p, cudaStream_t s) {
    const bool full = p.g.N == NP;
    if (p.g.nu) return full ? launch_bwd_t<NP, true, true>(p, s) : launch_bwd_t<NP, true, false>(p, s);
    return full ? launch_bwd_t<NP, false, true>(p, s) : launch_bwd_t<NP, false, false>(p, s);
}

// Coefficients of the in-kernel series tables: c1_p / p! = 1 / ((p+1) p!) and
// c2_ab / (a! b!) = 1 / ((a+b+2)(b+1) a! b!) for a + b <= q (ews/core/series_leaf.py:45-66), zero above.
static void series_coefficients(int q, Params* p, const float* leaf_coef) {
    if (leaf_coef) {  // the caller's polynomial coefficients (another leaf, e.g. Van Loan's): k1 | k2 rows
        for (int a = 0; a < kQNU; ++a) p->c1[a] = leaf_coef[a];
        for (int e = 0; e < kQNU * kQNU; ++e) p->c2[e] = leaf_coef[kQNU + e];
        return;
    }
    double fact[kQNU];
    fact[0] = 1.0;
    for (int i = 1; i < kQNU; ++i) fact[i] = fact[i - 1] * i;
    for (int a = 0; a < kQNU; ++a) {
        p->c1[a] = a <= q ? (float)(1.0 / ((a + 1) * fact[a])) : 0.f;
        for (int b = 0; b < kQNU; ++b)
            p->c2[a * kQNU + b] = a + b <= q ? (float)(1.0 / ((double)(a + b + 2) * (b + 1) * fact[a] * fact[b])) : 0.f;
    }
}

}  // namespace diag
}  // namespace ews

using namespace ews;
using namespace ews::diag;

// The closed-form terminal path of the uniform clock (ews_diag_term.cu).
namespace ews {
bool diag_term_applies(const ews_diag_args* a);
void diag_term_workspace(const ews_diag_args* a, size_t* fwd_bytes, size_t* bwd_bytes);
int diag_term_fwd(const ews_diag_args* a, cudaStream_t s);
int diag_term_bwd(const ews_diag_args* a, cudaStream_t s);
}  // namespace ews

extern "C" int ews_diag_workspace_size(const ews_diag_args* a, size_t* fwd_bytes, size_t* bwd_bytes) {
    Geom g;
    const int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (diag_term_applies(a)) {
        diag_term_workspace(a, fwd_bytes, bwd_bytes);
        return EWS_OK;
    }
    if (fwd_bytes) *fwd_bytes = fwd_layout(g).total;
    if (bwd_bytes) *bwd_bytes = bwd_layout(g).total;
    return EWS_OK;
}

extern "C" int ews_diag_fwd(const ews_diag_args* a, ews_stream_t stream) {
    Geom g;
    int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (!a->path || !a->out || !a->tab_x) return EWS_ERR_INVALID_ARGUMENT;
    if (g.nu ? !a->clock : (!a->tab_q1 || !a->tab_q2)) return EWS_ERR_INVALID_ARGUMENT;
    if (!a->lift && a->d_in != a->dim) return EWS_ERR_INVALID_ARGUMENT;
    if (diag_term_applies(a)) return diag_term_fwd(a, (cudaStream_t)stream);
    if (a->flags & EWS_F_LOGSIG) return EWS_ERR_UNSUPPORTED;  // the log epilogue rides on the closed form
    const WsLayout L = fwd_layout(g);
    if (!a->fwd_ws || a->fwd_ws_bytes < L.total) return EWS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    char* ws = (char*)a->fwd_ws;
    if (cudaMemsetAsync(ws, 0, L.agg, s) != cudaSuccess) return EWS_ERR_LAUNCH;
    Params p{};
    p.g = g;
    p.path = a->path;
    p.lift = a->lift;
    p.tab_x = a->tab_x;
    p.tab_q1 = a->tab_q1;
    p.tab_q2 = a->tab_q2;
    p.out = a->out;
    p.st = (DeviceStatus*)(ws + L.status);
    p.flags = (int*)(ws + L.flags);
    p.agg = (float*)(ws + L.agg);
    p.incl = (float*)(ws + L.incl);
    p.carry = (float*)(ws + L.carry);
    p.clock = a->clock;
    series_coefficients(a->series_q, &p, a->leaf_coef);
    switch (g.NP) {
        case 8: return launch_fwd<8>(p, s);
        case 16: return launch_fwd<16>(p, s);
        case 24: return launch_fwd<24>(p, s);
        case 32: return launch_fwd<32>(p, s);
    }
    return EWS_ERR_UNSUPPORTED;
}

extern "C" int ews_diag_bwd(const ews_diag_args* a, ews_stream_t stream) {
    Geom g;
    int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (!a->path || !a->grad_out || !a->grad_dx || !a->grad_x || !a->tab_x) return EWS_ERR_INVALID_ARGUMENT;
    if (g.nu ? (!a->clock || !a->grad_dtheta) : (!a->grad_q1 || !a->grad_q2 || !a->tab_q1 || !a->tab_q2))
        return EWS_ERR_INVALID_ARGUMENT;
    if (g.readout == EWS_READOUT_PREFIX && !a->out) return EWS_ERR_INVALID_ARGUMENT;
    if (!a->lift && a->d_in != a->dim) return EWS_ERR_INVALID_ARGUMENT;
    if (diag_term_applies(a)) return diag_term_bwd(a, (cudaStream_t)stream);
    if (a->flags & EWS_F_LOGSIG) return EWS_ERR_UNSUPPORTED;
    const WsLayout F = fwd_layout(g);
    const WsLayout L = bwd_layout(g);
    if (!a->fwd_ws || a->fwd_ws_bytes < F.total) return EWS_ERR_WORKSPACE;
    if (!a->bwd_ws || a->bwd_ws_bytes < L.total) return EWS_ERR_WORKSPACE;
    cudaStream_t s = (cudaStream_t)stream;
    char* ws = (char*)a->bwd_ws;
    const char* fws = (const char*)a->fwd_ws;
    if (cudaMemsetAsync(ws, 0, L.agg, s) != cudaSuccess) return EWS_ERR_LAUNCH;
    Params p{};
    p.g = g;
    p.path = a->path;
    p.lift = a->lift;
    p.tab_x = a->tab_x;
    p.tab_q1 = a->tab_q1;
    p.tab_q2 = a->tab_q2;
    p.out = a->out;
    p.grad_out = a->grad_out;
    p.grad_dx = a->grad_dx;
    p.partials = (float*)(ws + L.partials);
    p.st = (DeviceStatus*)(ws + L.status);
    p.flags = (int*)(ws + L.flags);
    p.agg = (float*)(ws + L.agg);
    p.incl = (float*)(ws + L.incl);
    p.fagg = (const float*)(fws + F.agg);
    p.fcarry = (const float*)(fws + F.carry);
    p.clock = a->clock;
    p.grad_dtheta = a->grad_dtheta;
    series_coefficients(a->series_q, &p, a->leaf_coef);
    switch (g.NP) {
        case 8: rc = launch_bwd<8>(p, s); break;
        case 16: rc = launch_bwd<16>(p, s); break;
        case 24: rc = launch_bwd<24>(p, s); break;
        case 32: rc = launch_bwd<32>(p, s); break;
        default: rc = EWS_ERR_UNSUPPORTED;
    }
    if (rc != EWS_OK) return rc;
    float* sp = (float*)(ws + L.sample_partials);
    const size_t n1 = (size_t)g.B * (2 * g.NP + g.NP * g.NP + g.NP * g.d_in);
    const int threads = 256;
    reduce_chunks_kernel<<<(int)std::min<size_t>((n1 + threads - 1) / threads, 65535), threads, 0, s>>>(p, sp);
    const int total = g.B * (2 * g.N + g.N * g.N) + (a->grad_lift ? g.N * g.d_in : 0);
    reduce_samples_kernel<<<(total + threads - 1) / threads, threads, 0, s>>>(
        p, sp, a->grad_x, g.nu ? nullptr : a->grad_q1, g.nu ? nullptr : a->grad_q2, a->grad_lift);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------------------------------
// Forward without a caller-provided workspace (see ews_diag_fwd_noalloc in include/ews_b200.h).
//
// Some callers cannot allocate device memory for us: a plugin host that hands a kernel only its input
// and output buffers, or a serving loop that forbids cudaMalloc on its hot path because an allocation
// can synchronise the device. For them the forward's look-back workspace lives in this file-scope
// device array instead, EWS_NOALLOC_SCRATCH_BYTES per GPU, held by every GPU that loads the library until
// the process exits. In host code the array's name is only a host-side stand-in, so its device address
// is looked up once per device with cudaGetSymbolAddress (with that device current) and cached.
namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[EWS_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kMaxDevices] = {};

int noalloc_scratch(void** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return EWS_ERR_LAUNCH;
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (!g_noalloc_addr[dev]) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return EWS_ERR_LAUNCH;
        g_noalloc_addr[dev] = ptr;
    }
    *out = g_noalloc_addr[dev];
    return EWS_OK;
}

}  // namespace

extern "C" int ews_diag_fwd_noalloc(const ews_diag_args* a, ews_stream_t stream) {
    Geom g;
    const int rc = make_geom(a, &g);
    if (rc != EWS_OK) return rc;
    if (fwd_layout(g).total > (size_t)EWS_NOALLOC_SCRATCH_BYTES) return EWS_ERR_WORKSPACE;
    void* scratch = nullptr;
    const int sc = noalloc_scratch(&scratch);
    if (sc != EWS_OK) return sc;
    ews_diag_args b = *a;
    b.fwd_ws = scratch;
    b.fwd_ws_bytes = EWS_NOALLOC_SCRATCH_BYTES;
    b.flags |= EWS_F_TERMINAL_SCAN;  // the scan's workspace is the one sized against the array above
    // ews_diag_fwd clears the status block and flags it needs zeroed before its kernel runs, allocates
    // nothing, and leaves the aggregates and carries in the array until the next call overwrites them.
    return ews_diag_fwd(&b, stream);
}

// The status block at the start of the array, read like any workspace's (ews_read_device_status): the
// caller of the no-alloc forward has no pointer to the array, so this is how it learns of a look-back
// timeout. Uses the current device's array; synchronises the stream.
extern "C" int ews_diag_fwd_noalloc_status(ews_stream_t stream, int* status) {
    if (!status) return EWS_ERR_INVALID_ARGUMENT;
    void* scratch = nullptr;
    const int sc = noalloc_scratch(&scratch);
    if (sc != EWS_OK) return sc;
    return ews_read_device_status(scratch, stream, status);
}
