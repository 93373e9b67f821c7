// Flow tables of the dense engine: the batched matrix exponential M = expm(-h A) and its adjoint.
//
// The reference builds the dense flow per interval (or once for a uniform clock) with
// expm_matrix(-h A, method) (ews/core/chen_scan.py:155-168, ews/core/expm_approx.py:34-41; "exact" is
// jax.scipy.linalg.expm). Here one CTA evaluates one matrix in float64 on the device, so building the
// tables never waits on the host: scaling and squaring with a degree-14 Taylor polynomial, the scaling
// chosen in the kernel so that ||X / 2^s||_1 <= 1/2 (truncation error below 3e-17 relative to ||e^X||).
//
// The adjoint d<G, expm(X)>/dX is the Frechet derivative L(X^T, G), read from the upper-right block of
// expm([[X^T, G], [0, X^T]]) (the block-triangular identity for Frechet derivatives of matrix
// functions); G is scaled to unit 1-norm first so that the block's norm, and with it the scaling, does
// not depend on the cotangent's magnitude.

#include <cuda_runtime.h>

#include "../../include/ews_b200.h"

namespace ews {
namespace tables {

constexpr int XT = 256;  // threads per CTA: a 16 x 16 grid of register blocks

// C = A B for padded NP x NP row-major float64 matrices in shared memory; thread (r, c) of the 16 x 16
// grid owns the BS x BS block at rows BS r, columns BS c. The caller synchronises before and after.
template <int NP>
__device__ __forceinline__ void matmul(const double* A, const double* B, double* C) {
    constexpr int BS = NP / 16;
    const int r = threadIdx.x >> 4, c = threadIdx.x & 15;
    double acc[BS][BS];
#pragma unroll
    for (int i = 0; i < BS; ++i)
#pragma unroll
        for (int j = 0; j < BS; ++j) acc[i][j] = 0.0;
#pragma unroll 4
    for (int k = 0; k < NP; ++k) {
        double a[BS], b[BS];
#pragma unroll
        for (int i = 0; i < BS; ++i) a[i] = A[(BS * r + i) * NP + k];
#pragma unroll
        for (int j = 0; j < BS; ++j) b[j] = B[k * NP + BS * c + j];
#pragma unroll
        for (int i = 0; i < BS; ++i)
#pragma unroll
            for (int j = 0; j < BS; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
    }
#pragma unroll
    for (int i = 0; i < BS; ++i)
#pragma unroll
        for (int j = 0; j < BS; ++j) C[(BS * r + i) * NP + BS * c + j] = acc[i][j];
}

// 1-norm (largest column sum of magnitudes) of an NP x NP shared-memory matrix, returned to every thread.
template <int NP>
__device__ double norm1(const double* X, double* red) {
    double s = 0.0;
    if (threadIdx.x < NP)
        for (int i = 0; i < NP; ++i) s += fabs(X[i * NP + threadIdx.x]);
    if (threadIdx.x < NP) red[threadIdx.x] = s;
    __syncthreads();
    double m = 0.0;
    for (int j = 0; j < NP; ++j) {
        const double v = red[j];
        m = (v > m || v != v) ? v : m;  // a NaN column wins, so a NaN input gives a NaN result
    }
    __syncthreads();
    return m;
}

// expm of the NP x NP matrix in X (overwritten with X / 2^s); the result is left in *res (one of Acc or
// Tmp). Every thread calls it.
template <int NP>
__device__ void expm_inplace(double* X, double* Acc, double* Tmp, double* red, double** res) {
    const double nrm = norm1<NP>(X, red);
    int s = 0;
    if (nrm == nrm && nrm <= 1.0e300) {
        double v = nrm;
        while (v > 0.5 && s < 1100) {
            v *= 0.5;
            ++s;
        }
    }
    const double scale = ldexp(1.0, -s);
    constexpr int DEG = 14;
    for (int e = threadIdx.x; e < NP * NP; e += XT) {
        const double x = X[e] * scale;
        X[e] = x;
        Acc[e] = ((e / NP) == (e % NP) ? 1.0 : 0.0) + x / DEG;
    }
    __syncthreads();
    // Horner: Acc <- I + X Acc / k for k = DEG-1 .. 1
    for (int k = DEG - 1; k >= 1; --k) {
        matmul<NP>(X, Acc, Tmp);
        __syncthreads();
        const double inv = 1.0 / k;
        for (int e = threadIdx.x; e < NP * NP; e += XT)
            Acc[e] = ((e / NP) == (e % NP) ? 1.0 : 0.0) + Tmp[e] * inv;
        __syncthreads();
    }
    double* a = Acc;
    double* t = Tmp;
    for (int i = 0; i < s; ++i) {
        matmul<NP>(a, a, t);
        __syncthreads();
        double* sw = a;
        a = t;
        t = sw;
    }
    *res = a;
}

template <int NP>
__global__ void __launch_bounds__(XT) expm_kernel(const double* __restrict__ x, double* __restrict__ out, int n) {
    extern __shared__ double sm[];
    double* X = sm;
    double* Acc = X + NP * NP;
    double* Tmp = Acc + NP * NP;
    double* red = Tmp + NP * NP;
    const double* xb = x + (size_t)blockIdx.x * n * n;
    for (int e = threadIdx.x; e < NP * NP; e += XT) {
        const int i = e / NP, j = e - i * NP;
        X[e] = (i < n && j < n) ? xb[i * n + j] : 0.0;
    }
    __syncthreads();
    double* res;
    expm_inplace<NP>(X, Acc, Tmp, red, &res);
    double* ob = out + (size_t)blockIdx.x * n * n;
    for (int e = threadIdx.x; e < n * n; e += XT) {
        const int i = e / n, j = e - i * n;
        ob[e] = res[i * NP + j];
    }
}

// out = L(X^T, G) for n <= 32, through the 64 x 64 block [[X^T, G/g], [0, X^T]] (zero padded per block).
__global__ void __launch_bounds__(XT) expm_adjoint_kernel(const double* __restrict__ x, const double* __restrict__ g,
                                                          double* __restrict__ out, int n) {
    constexpr int NP = 64, H = 32;
    extern __shared__ double sm[];
    double* X = sm;
    double* Acc = X + NP * NP;
    double* Tmp = Acc + NP * NP;
    double* red = Tmp + NP * NP;
    const double* xb = x + (size_t)blockIdx.x * n * n;
    const double* gb = g + (size_t)blockIdx.x * n * n;
    // the cotangent's 1-norm, staged in Tmp
    for (int e = threadIdx.x; e < H * H; e += XT) {
        const int i = e / H, j = e - i * H;
        Tmp[e] = (i < n && j < n) ? gb[i * n + j] : 0.0;
    }
    __syncthreads();
    double gn = 0.0;
    {
        double s = 0.0;
        if (threadIdx.x < H)
            for (int i = 0; i < H; ++i) s += fabs(Tmp[i * H + threadIdx.x]);
        if (threadIdx.x < H) red[threadIdx.x] = s;
        __syncthreads();
        for (int j = 0; j < H; ++j) {
            const double v = red[j];
            gn = (v > gn || v != v) ? v : gn;
        }
        __syncthreads();
    }
    const double gs = (gn > 0.0) ? 1.0 / gn : 0.0;
    for (int e = threadIdx.x; e < NP * NP; e += XT) {
        const int i = e / NP, j = e - i * NP;
        const int bi = i / H, bj = j / H, ii = i % H, jj = j % H;
        double v = 0.0;
        if (ii < n && jj < n) {
            if (bi == bj) v = xb[jj * n + ii];              // X^T on both diagonal blocks
            else if (bi == 0 && bj == 1) v = Tmp[ii * H + jj] * gs;  // G / ||G||_1
        }
        Acc[e] = v;
    }
    __syncthreads();
    for (int e = threadIdx.x; e < NP * NP; e += XT) X[e] = Acc[e];
    __syncthreads();
    double* res;
    expm_inplace<NP>(X, Acc, Tmp, red, &res);
    double* ob = out + (size_t)blockIdx.x * n * n;
    for (int e = threadIdx.x; e < n * n; e += XT) {
        const int i = e / n, j = e - i * n;
        ob[e] = res[i * NP + H + j] * gn;
    }
}

template <int NP>
static size_t smem_bytes() {
    return sizeof(double) * (3 * NP * NP + NP);
}

}  // namespace tables
}  // namespace ews

using namespace ews::tables;

extern "C" int ews_expm_batched(const double* x, double* out, int batch, int n, ews_stream_t stream) {
    if (batch < 0 || n <= 0 || n > 64) return n > 64 ? EWS_ERR_UNSUPPORTED : EWS_ERR_INVALID_ARGUMENT;
    if (batch == 0) return EWS_OK;
    if (!x || !out) return EWS_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    if (n <= 32) {
        const size_t smem = smem_bytes<32>();
        expm_kernel<32><<<batch, XT, smem, s>>>(x, out, n);
    } else {
        const size_t smem = smem_bytes<64>();
        cudaFuncSetAttribute(expm_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        expm_kernel<64><<<batch, XT, smem, s>>>(x, out, n);
    }
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

extern "C" int ews_expm_adjoint_batched(const double* x, const double* g, double* out, int batch, int n,
                                        ews_stream_t stream) {
    if (batch < 0 || n <= 0 || n > 32) return n > 32 ? EWS_ERR_UNSUPPORTED : EWS_ERR_INVALID_ARGUMENT;
    if (batch == 0) return EWS_OK;
    if (!x || !g || !out) return EWS_ERR_INVALID_ARGUMENT;
    cudaStream_t s = (cudaStream_t)stream;
    const size_t smem = smem_bytes<64>();
    cudaFuncSetAttribute(expm_adjoint_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    expm_adjoint_kernel<<<batch, XT, smem, s>>>(x, g, out, n);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}
