// The block's clock prologue: the token-gated clock of the block input, in one pass per direction.
//
// theta_0 = 0, theta_{t+1} = (1/c) sum_{tau <= t} relu(<s x_{tau+1} - s x_tau, w> - b)   (ews/clocks.py:409-466,
// mode "token_gated", no mask; the driver is scaled before the difference, as the reference does). The gates'
// dot products run one warp per interval (lane-strided over the driver's channels, warp-reduced) over the whole
// grid; then one CTA per sample scans the increments in tiles of GC_TILE steps, adding each tile to the
// running total. The backward recomputes the gates: dI_t = (1/c) sum_{j > t} dtheta_j (a reverse scan),
// g_t = dI_t [pre_t > 0]; dw = sum_t g_t dx_t, db = -sum_t g_t (per span of intervals, then summed over the spans
// in order), and d x_t = s w (g_{t-1} - g_t) by the adjoint of the difference. The gates run GC_SPAN intervals per
// CTA over the whole grid; only the scans go one CTA per sample.
#include <algorithm>

#include "ews_common.cuh"

namespace ews {
namespace gclock {

constexpr int GC_THREADS = 256;
constexpr int GC_WARPS = GC_THREADS / 32;
constexpr int GC_TILE = 1024;   // steps per scan tile
constexpr int GC_SPAN = 512;    // intervals per CTA of the gate kernels

struct Args {
    int B, L, H;
    float s, inv_c;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// pre_t = <s x_{t+1} - s x_t, w> - b for one interval, by one warp (every lane gets it)
__device__ __forceinline__ float gate_pre(const Args& a, const float* xb, const float* w, float bias, int t) {
    const float* x0 = xb + (size_t)t * a.H;
    const float* x1 = x0 + a.H;
    float acc = 0.f;
    for (int h = threadIdx.x & 31; h < a.H; h += 32) acc = fmaf(x1[h] * a.s - x0[h] * a.s, w[h], acc);
    return warp_sum(acc) - bias;
}

// Inclusive scan of GC_TILE floats in shared memory by the whole CTA (4 per thread, then warp and block scans).
__device__ float block_scan_tile(float* v, int n, float* wsum) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float loc[4];
    float run = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = 4 * tid + k;
        run += i < n ? v[i] : 0.f;
        loc[k] = run;
    }
    float x = run;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) wsum[warp] = x;
    __syncthreads();
    float before = 0.f;
    for (int k = 0; k < warp; ++k) before += wsum[k];
    float total = 0.f;
    for (int k = 0; k < GC_WARPS; ++k) total += wsum[k];
    const float excl = before + x - run;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int i = 4 * tid + k;
        if (i < n) v[i] = excl + loc[k];
    }
    __syncthreads();
    return total;
}

// Gates of GC_SPAN consecutive intervals of one sample per CTA (warp-strided): theta[b][t + 1] = relu(pre_t), the
// increments, turned into the clock by gated_clock_scan_kernel.
__global__ void __launch_bounds__(GC_THREADS) gated_clock_incr_kernel(Args a, const float* __restrict__ x,
                                                                     const float* __restrict__ w,
                                                                     const float* __restrict__ b,
                                                                     float* __restrict__ theta) {
    const int bs = blockIdx.y, warp = threadIdx.x >> 5;
    const int t0 = blockIdx.x * GC_SPAN, t1 = min(a.L - 1, t0 + GC_SPAN);
    const float* xb = x + (size_t)bs * a.L * a.H;
    float* th = theta + (size_t)bs * a.L;
    const float bias = *b;
    if (blockIdx.x == 0 && threadIdx.x == 0) th[0] = 0.f;
    for (int t = t0 + warp; t < t1; t += GC_WARPS) {
        const float pre = gate_pre(a, xb, w, bias, t);
        if ((threadIdx.x & 31) == 0) th[t + 1] = fmaxf(pre, 0.f);
    }
}

// One CTA per sample: theta[1..L-1] <- (1/c) x the running sum of the increments, tile by tile.
__global__ void __launch_bounds__(GC_THREADS) gated_clock_scan_kernel(Args a, float* __restrict__ theta) {
    __shared__ float v[GC_TILE];
    __shared__ float wsum[GC_WARPS];
    float* th = theta + (size_t)blockIdx.x * a.L + 1;
    const int n_int = a.L - 1;
    float carry = 0.f;
    for (int t0 = 0; t0 < n_int; t0 += GC_TILE) {
        const int n = min(GC_TILE, n_int - t0);
        for (int i = threadIdx.x; i < n; i += GC_THREADS) v[i] = th[t0 + i];
        __syncthreads();
        const float total = block_scan_tile(v, n, wsum);
        for (int i = threadIdx.x; i < n; i += GC_THREADS) th[t0 + i] = (carry + v[i]) * a.inv_c;
        carry += total;
        __syncthreads();
    }
}

// One CTA per sample: gbuf[b][t] = dI_t = (1/c) sum_{j = t+1}^{L-1} dtheta_j, by a reverse scan.
__global__ void __launch_bounds__(GC_THREADS) gated_clock_rscan_kernel(Args a, const float* __restrict__ dtheta,
                                                                      float* __restrict__ gbuf) {
    __shared__ float v[GC_TILE];
    __shared__ float wsum[GC_WARPS];
    const float* dth = dtheta + (size_t)blockIdx.x * a.L;
    float* gb = gbuf + (size_t)blockIdx.x * (a.L - 1);
    float carry = 0.f;
    for (int t1 = a.L - 1; t1 > 0; t1 -= GC_TILE) {
        const int n = min(GC_TILE, t1);
        for (int i = threadIdx.x; i < n; i += GC_THREADS) v[i] = dth[t1 - i] * a.inv_c;  // i -> t = t1 - 1 - i
        __syncthreads();
        const float total = block_scan_tile(v, n, wsum);
        for (int i = threadIdx.x; i < n; i += GC_THREADS) gb[t1 - 1 - i] = carry + v[i];
        carry += total;
        __syncthreads();
    }
}

// The gates of GC_SPAN intervals per CTA: gbuf <- g_t = dI_t [pre_t > 0]; the CTA's dw and db partials
// (warp rows summed in warp order) into part[(b, span)].
__global__ void __launch_bounds__(GC_THREADS) gated_clock_gate_kernel(Args a, const float* __restrict__ x,
                                                                     const float* __restrict__ w,
                                                                     const float* __restrict__ b,
                                                                     float* __restrict__ gbuf,
                                                                     float* __restrict__ part) {
    __shared__ float dbw[GC_WARPS];
    extern __shared__ float dws[];  // GC_WARPS x H partial dw
    const int bs = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = blockIdx.x * GC_SPAN, t1 = min(a.L - 1, t0 + GC_SPAN);
    const float* xb = x + (size_t)bs * a.L * a.H;
    float* gb = gbuf + (size_t)bs * (a.L - 1);
    const float bias = *b;
    for (int e = threadIdx.x; e < GC_WARPS * a.H; e += GC_THREADS) dws[e] = 0.f;
    __syncthreads();
    float dbacc = 0.f;
    for (int t = t0 + warp; t < t1; t += GC_WARPS) {
        const float pre = gate_pre(a, xb, w, bias, t);
        const float g = pre > 0.f ? gb[t] : 0.f;
        __syncwarp();
        if (lane == 0) gb[t] = g;
        dbacc -= g;
        if (g != 0.f) {
            const float* x0 = xb + (size_t)t * a.H;
            for (int h = lane; h < a.H; h += 32) dws[warp * a.H + h] += g * (x0[h + a.H] * a.s - x0[h] * a.s);
        }
    }
    if (lane == 0) dbw[warp] = dbacc;
    __syncthreads();
    float* pb = part + ((size_t)bs * gridDim.x + blockIdx.x) * (a.H + 1);
    for (int h = threadIdx.x; h < a.H; h += GC_THREADS) {
        float sum = 0.f;
        for (int k = 0; k < GC_WARPS; ++k) sum += dws[k * a.H + h];
        pb[h] = sum;
    }
    if (threadIdx.x == 0) {
        float sum = 0.f;
        for (int k = 0; k < GC_WARPS; ++k) sum += dbw[k];
        pb[a.H] = sum;
    }
}

// d x_t = s w (g_{t-1} - g_t), g_{-1} = g_{L-1} = 0
__global__ void gated_clock_dx_kernel(Args a, const float* __restrict__ w, const float* __restrict__ gbuf,
                                      float* __restrict__ dx) {
    const size_t total = (size_t)a.B * a.L * a.H;
    for (size_t e = (size_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (size_t)gridDim.x * blockDim.x) {
        const int h = (int)(e % a.H);
        const size_t r = e / a.H;
        const int bs = (int)(r / a.L), t = (int)(r - (size_t)bs * a.L);
        const float* gb = gbuf + (size_t)bs * (a.L - 1);
        const float gp = t >= 1 ? gb[t - 1] : 0.f;
        const float gc = t < a.L - 1 ? gb[t] : 0.f;
        dx[e] = a.s * w[h] * (gp - gc);
    }
}

// dw, db: the (sample, span) partials summed in order
__global__ void gated_clock_reduce_kernel(Args a, const float* __restrict__ part, int nparts, float* __restrict__ dw,
                                          float* __restrict__ db) {
    for (int h = blockIdx.x * blockDim.x + threadIdx.x; h <= a.H; h += gridDim.x * blockDim.x) {
        float sum = 0.f;
        for (int k = 0; k < nparts; ++k) sum += part[(size_t)k * (a.H + 1) + h];
        if (h < a.H) dw[h] = sum;
        else *db = sum;
    }
}

static int make_args(int B, int L, int H, float s, float c, Args* a) {
    if (B < 0 || L < 1 || H < 1 || !(c != 0.f)) return EWS_ERR_INVALID_ARGUMENT;
    if (H > 8192) return EWS_ERR_UNSUPPORTED;
    *a = Args{B, L, H, s, 1.f / c};
    return EWS_OK;
}

}  // namespace gclock
}  // namespace ews

using namespace ews::gclock;

static int gc_spans(int steps) { return steps > 1 ? (steps - 1 + GC_SPAN - 1) / GC_SPAN : 1; }

extern "C" size_t ews_gated_clock_work_size(int batch, int steps, int dim) {
    if (batch <= 0 || steps <= 0 || dim <= 0) return 0;
    return sizeof(float) * ((size_t)batch * (size_t)(steps > 1 ? steps - 1 : 1) +
                            (size_t)batch * gc_spans(steps) * (size_t)(dim + 1));
}

extern "C" int ews_gated_clock_fwd(const float* x, const float* w, const float* b, float in_scale, float norm_constant,
                                   int batch, int steps, int dim, float* theta, ews_stream_t stream) {
    Args a{};
    const int rc = make_args(batch, steps, dim, in_scale, norm_constant, &a);
    if (rc != EWS_OK || batch == 0) return rc;
    if (!x || !w || !b || !theta) return EWS_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    gated_clock_incr_kernel<<<dim3(gc_spans(steps), batch), GC_THREADS, 0, s>>>(a, x, w, b, theta);
    gated_clock_scan_kernel<<<batch, GC_THREADS, 0, s>>>(a, theta);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

extern "C" int ews_gated_clock_bwd(const float* x, const float* w, const float* b, float in_scale, float norm_constant,
                                   const float* dtheta, int batch, int steps, int dim, float* dx, float* dw, float* db,
                                   void* work, size_t work_bytes, ews_stream_t stream) {
    Args a{};
    const int rc = make_args(batch, steps, dim, in_scale, norm_constant, &a);
    if (rc != EWS_OK) return rc;
    if (!dw || !db) return EWS_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    if (batch == 0) {
        if (cudaMemsetAsync(dw, 0, sizeof(float) * dim, s) != cudaSuccess) return EWS_ERR_LAUNCH;
        return cudaMemsetAsync(db, 0, sizeof(float), s) == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
    }
    if (!x || !w || !b || !dtheta || !dx) return EWS_ERR_INVALID_ARGUMENT;
    if (!work || work_bytes < ews_gated_clock_work_size(batch, steps, dim)) return EWS_ERR_WORKSPACE;
    float* gbuf = static_cast<float*>(work);
    float* part = gbuf + (size_t)batch * (size_t)(steps > 1 ? steps - 1 : 1);
    const int spans = gc_spans(steps);
    gated_clock_rscan_kernel<<<batch, GC_THREADS, 0, s>>>(a, dtheta, gbuf);
    const size_t dsm = sizeof(float) * GC_WARPS * (size_t)dim;
    cudaFuncSetAttribute(gated_clock_gate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dsm);
    gated_clock_gate_kernel<<<dim3(spans, batch), GC_THREADS, dsm, s>>>(a, x, w, b, gbuf, part);
    const size_t total = (size_t)batch * steps * dim;
    const unsigned grid = (unsigned)std::min<size_t>((total + 255) / 256, 65535);
    gated_clock_dx_kernel<<<grid, 256, 0, s>>>(a, w, gbuf, dx);
    gated_clock_reduce_kernel<<<(dim + 1 + 255) / 256, 256, 0, s>>>(a, part, batch * spans, dw, db);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}
