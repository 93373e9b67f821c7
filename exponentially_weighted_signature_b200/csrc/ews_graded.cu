// The stream consumer of the block: the EWS prefix rows -> the graded RMS norm's input to c_down, in one pass.
//
// The block drops level 0 of the EWS prefix output, prepends a zero row (the state before the first
// interval) and normalises every level by its own live RMS (ews/block.py:282-306 and :406,
// ews/norms.py:47-135, variant "live_rms"):
//     y[:, 0] = 0,    y[:, t + 1] level k = g_k x_k / (RMS(x_k) + eps_k),    x = flat[:, t, 1:],
// with RMS(x_k) = sqrt(mean(x_k^2)) and 0 for an all-zero level (the zero-safe square root: its derivative
// is 0 there, so dy/dx = g_k / eps_k). One warp per output row; the levels' sums of squares are warp
// reductions. The backward recomputes the statistics from x (nothing is saved) and writes dflat (level-0
// column zero) and the gain gradients, summed per CTA in warp order and then over CTAs in order.
#include "ews_common.cuh"

namespace ews {
namespace graded {

constexpr int GW = 8;      // warps (rows) per CTA
constexpr int GMAXN = 3;   // levels

struct Args {
    int B, L, d, N, D;
    int off[GMAXN + 1];    // level k occupies [off[k], off[k+1]) of the level-0-free row
    float eps[GMAXN];
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void __launch_bounds__(GW * 32) graded_fwd_kernel(Args a, const float* __restrict__ flat,
                                                            const float* __restrict__ gains, float* __restrict__ y) {
    const int lane = threadIdx.x & 31;
    const long row = (long)blockIdx.x * GW + (threadIdx.x >> 5);
    const long rows = (long)a.B * (a.L + 1);
    if (row >= rows) return;
    const int b = (int)(row / (a.L + 1)), t = (int)(row - (long)b * (a.L + 1));
    float* yr = y + row * a.D;
    if (t == 0) {
        for (int e = lane; e < a.D; e += 32) yr[e] = 0.f;
        return;
    }
    const float* x = flat + ((long)b * a.L + (t - 1)) * (a.D + 1) + 1;
    for (int k = 0; k < a.N; ++k) {
        const int s = a.off[k], e1 = a.off[k + 1], n = e1 - s;
        float ss = 0.f;
        for (int e = s + lane; e < e1; e += 32) {
            const float v = x[e];
            ss = fmaf(v, v, ss);
        }
        const float ms = warp_sum(ss) / (float)n;
        const float rms = ms > 0.f ? sqrtf(ms) : 0.f;
        const float sc = gains[k] / (rms + a.eps[k]);
        for (int e = s + lane; e < e1; e += 32) yr[e] = x[e] * sc;
    }
}

// dflat and per-CTA partial gain gradients (work: gridDim.x x N floats).
__global__ void __launch_bounds__(GW * 32) graded_bwd_kernel(Args a, const float* __restrict__ flat,
                                                            const float* __restrict__ gains,
                                                            const float* __restrict__ dy, float* __restrict__ dflat,
                                                            float* __restrict__ work) {
    __shared__ float part[GW][GMAXN];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const long r = (long)blockIdx.x * GW + warp;  // input row: sample b, interval t
    const long rows = (long)a.B * a.L;
    float dgk[GMAXN] = {0.f, 0.f, 0.f};
    if (r < rows) {
        const int b = (int)(r / a.L), t = (int)(r - (long)b * a.L);
        const float* x = flat + r * (a.D + 1) + 1;
        const float* g = dy + ((long)b * (a.L + 1) + t + 1) * a.D;
        float* dx = dflat + r * (a.D + 1);
        if (lane == 0) dx[0] = 0.f;
        dx += 1;
        for (int k = 0; k < a.N; ++k) {
            const int s = a.off[k], e1 = a.off[k + 1], n = e1 - s;
            float ss = 0.f, sd = 0.f;
            for (int e = s + lane; e < e1; e += 32) {
                const float v = x[e];
                ss = fmaf(v, v, ss);
                sd = fmaf(g[e], v, sd);
            }
            const float ms = warp_sum(ss) / (float)n;
            sd = warp_sum(sd);
            const float rms = ms > 0.f ? sqrtf(ms) : 0.f;
            const float den = rms + a.eps[k];
            const float gk = gains[k];
            const float c1 = gk / den;
            // d/dx of rms: x / (n rms) where ms > 0, else 0
            const float c2 = ms > 0.f ? gk * sd / (den * den * (float)n * rms) : 0.f;
            for (int e = s + lane; e < e1; e += 32) dx[e] = c1 * g[e] - c2 * x[e];
            dgk[k] = sd / den;
        }
    }
    if (lane == 0)
        for (int k = 0; k < GMAXN; ++k) part[warp][k] = dgk[k];
    __syncthreads();
    if (threadIdx.x < a.N) {
        float s = 0.f;
        for (int w = 0; w < GW; ++w) s += part[w][threadIdx.x];
        work[(long)blockIdx.x * a.N + threadIdx.x] = s;
    }
}

__global__ void graded_dg_kernel(Args a, const float* __restrict__ work, int nblk, float* __restrict__ dg) {
    // one warp per level: lane-strided partial sums, then a fixed-order warp reduction
    const int k = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (k >= a.N) return;
    float s = 0.f;
    for (int i = lane; i < nblk; i += 32) s += work[(long)i * a.N + k];
    s = warp_sum(s);
    if (lane == 0) dg[k] = s;
}

static int make_args(int B, int L, int d, int N, const float* eps, Args* a) {
    if (B < 0 || L < 0 || d <= 0 || N < 1 || N > GMAXN || !eps) return EWS_ERR_INVALID_ARGUMENT;
    a->B = B;
    a->L = L;
    a->d = d;
    a->N = N;
    int off = 0, p = 1;
    for (int k = 0; k < N; ++k) {
        a->off[k] = off;
        p *= d;
        off += p;
        a->eps[k] = eps[k];
        if (!(eps[k] > 0.f)) return EWS_ERR_INVALID_ARGUMENT;
    }
    a->off[N] = off;
    a->D = off;
    if (off > (1 << 20)) return EWS_ERR_UNSUPPORTED;
    return EWS_OK;
}

}  // namespace graded
}  // namespace ews

using namespace ews::graded;

extern "C" size_t ews_graded_norm_work_size(int batch, int steps, int d, int levels) {
    if (batch <= 0 || steps <= 0 || d <= 0 || levels < 1) return 0;
    const long rows = (long)batch * steps;
    return sizeof(float) * (size_t)((rows + GW - 1) / GW) * (size_t)levels;
}

extern "C" int ews_graded_norm_fwd(const float* flat, const float* gains, const float* eps, int batch, int steps,
                                   int d, int levels, float* y, ews_stream_t stream) {
    Args a{};
    const int rc = make_args(batch, steps, d, levels, eps, &a);
    if (rc != EWS_OK) return rc;
    if (batch == 0) return EWS_OK;
    if (!gains || !y || (steps > 0 && !flat)) return EWS_ERR_INVALID_ARGUMENT;
    const long rows = (long)batch * (steps + 1);
    graded_fwd_kernel<<<(unsigned)((rows + GW - 1) / GW), GW * 32, 0, (cudaStream_t)stream>>>(a, flat, gains, y);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

extern "C" int ews_graded_norm_bwd(const float* flat, const float* gains, const float* eps, const float* dy, int batch,
                                   int steps, int d, int levels, float* dflat, float* dgains, void* work,
                                   size_t work_bytes, ews_stream_t stream) {
    Args a{};
    const int rc = make_args(batch, steps, d, levels, eps, &a);
    if (rc != EWS_OK) return rc;
    if (!dgains) return EWS_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    if (batch == 0 || steps == 0) {
        return cudaMemsetAsync(dgains, 0, sizeof(float) * levels, s) == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
    }
    if (!flat || !gains || !dy || !dflat) return EWS_ERR_INVALID_ARGUMENT;
    if (!work || work_bytes < ews_graded_norm_work_size(batch, steps, d, levels)) return EWS_ERR_WORKSPACE;
    const long rows = (long)batch * steps;
    const int nblk = (int)((rows + GW - 1) / GW);
    float* wk = static_cast<float*>(work);
    graded_bwd_kernel<<<nblk, GW * 32, 0, s>>>(a, flat, gains, dy, dflat, wk);
    graded_dg_kernel<<<1, 32 * GMAXN, 0, s>>>(a, wk, nblk, dgains);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}
