// Shared device helpers of the EWS kernels: look-back flags with bounded waits, warp span copies
// between global memory and shared memory, and input loads.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/ews_b200.h"

namespace ews {

constexpr unsigned kFull = 0xffffffffu;

// Look-back slot states. A chunk publishes its aggregate (AGG) before it knows its carry, then its
// inclusive value (INCL) once it does.
constexpr int kFlagEmpty = 0;
constexpr int kFlagAgg = 1;
constexpr int kFlagIncl = 2;

// Device status block at the start of every workspace: a tile ticket counter and an error word.
struct DeviceStatus {
    int ticket;
    int error;
    int err_tile;
    int pad;
};

constexpr int kDefaultSpinLimit = 1 << 21;

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release(int* p, int v) {
    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Warp-wide: take the next tile ticket (lane 0 increments, all lanes receive it).
__device__ __forceinline__ int next_ticket(DeviceStatus* st) {
    int t = 0;
    if ((threadIdx.x & 31) == 0) t = atomicAdd(&st->ticket, 1);
    return __shfl_sync(kFull, t, 0);
}

// Warp-wide publish: every lane has stored its part of the slot; the warp barrier orders those stores before
// lane 0's release of the flag, whose release is cumulative over them (one fence per publish).
__device__ __forceinline__ void publish(int* flag, int value) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) st_release(flag, value);
}

// Warp-wide bounded wait for a slot's flag to reach at least `want` (kFlagAgg: any published value;
// kFlagIncl: the inclusive value). Returns the flag value, or -1 when the wait ran out (the error word is
// then set) or another tile already failed. Never spins without a limit. Every lane issues the acquire
// load (one request for the warp), so each lane's later reads of the slot are ordered after the
// publisher's writes; the loop follows lane 0's value.
__device__ __forceinline__ int wait_slot(const int* flag, DeviceStatus* st, int limit, int tile, int want = kFlagAgg) {
    int v = kFlagEmpty;
    unsigned ns = 32;
    for (int it = 0; it < limit; ++it) {
        v = __shfl_sync(kFull, ld_acquire(flag), 0);
        if (v >= want) break;
        if (__shfl_sync(kFull, *((volatile int*)&st->error), 0) != 0) {
            v = -1;
            break;
        }
        __nanosleep(ns);
        if (ns < 256) ns <<= 1;
    }
    if (v >= 0 && v < want) {
        if ((threadIdx.x & 31) == 0 && atomicCAS(&st->error, 0, EWS_ERR_LOOKBACK_TIMEOUT) == 0) st->err_tile = tile;
        v = -1;
    }
    return v;
}

// Loads that bypass L1: look-back slots written by other SMs.
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

// Warp copy of n contiguous floats from shared memory to global memory. The global span may start at
// any 4-byte offset: the head up to the first 16-byte boundary and the tail are scalar stores, the body
// 16-byte vector stores (shared memory is read with scalar loads, since its offset need not be aligned).
__device__ __forceinline__ void warp_store_span(float* __restrict__ g, const float* __restrict__ s, int n) {
    const int lane = threadIdx.x & 31;
    int head = (int)(((16u - ((uintptr_t)g & 15u)) & 15u) >> 2);
    if (head > n) head = n;
    if (lane < head) g[lane] = s[lane];
    const int nvec = (n - head) >> 2;
    float4* gv = reinterpret_cast<float4*>(g + head);
    for (int v = lane; v < nvec; v += 32) {
        const float* sp = s + head + 4 * v;
        gv[v] = make_float4(sp[0], sp[1], sp[2], sp[3]);
    }
    const int done = head + 4 * nvec;
    if (lane < n - done) g[done + lane] = s[done + lane];
}

// Warp copy of n contiguous floats from global memory to shared memory (L2-cached loads: the backward
// reads its gradient rows twice).
__device__ __forceinline__ void warp_load_span(float* __restrict__ s, const float* __restrict__ g, int n) {
    const int lane = threadIdx.x & 31;
    int head = (int)(((16u - ((uintptr_t)g & 15u)) & 15u) >> 2);
    if (head > n) head = n;
    if (lane < head) s[lane] = __ldcg(g + lane);
    const int nvec = (n - head) >> 2;
    const float4* gv = reinterpret_cast<const float4*>(g + head);
    for (int v = lane; v < nvec; v += 32) {
        float4 q = __ldcg(gv + v);
        float* sp = s + head + 4 * v;
        sp[0] = q.x;
        sp[1] = q.y;
        sp[2] = q.z;
        sp[3] = q.w;
    }
    const int done = head + 4 * nvec;
    if (lane < n - done) s[done + lane] = __ldcg(g + done + lane);
}

// Asynchronous global -> shared copies (cp.async); each warp tracks its own groups.
__device__ __forceinline__ unsigned smem_addr(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void cp_async4(float* s, const float* g) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(s)), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async16(float* s, const float* g) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(s)), "l"(g) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int K>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(K) : "memory"); }

// Starts a warp copy of n contiguous floats from global memory into buf (16-byte aligned, n + 3 floats):
// the span lands at buf + shift with the same 16-byte phase as the source, so its body moves as 16-byte
// copies and only the head and tail as 4-byte ones. Returns the span's shared-memory start. The caller
// commits the group and waits for it (cp_async_wait, then __syncwarp) before reading.
__device__ __forceinline__ float* warp_load_span_async(float* __restrict__ buf, const float* __restrict__ g, int n) {
    const int lane = threadIdx.x & 31;
    const int shift = (int)(((uintptr_t)g & 15u) >> 2);
    float* s = buf + shift;
    int head = (4 - shift) & 3;
    if (head > n) head = n;
    if (lane < head) cp_async4(s + lane, g + lane);
    const int nvec = (n - head) >> 2;
    for (int v = lane; v < nvec; v += 32) cp_async16(s + head + 4 * v, g + head + 4 * v);
    const int done = head + 4 * nvec;
    if (lane < n - done) cp_async4(s + done + lane, g + done + lane);
    return s;
}

// Asks L2 for the 128-byte lines that hold [p, p + n) (n <= 1024 floats; lane l takes line l). Only lines
// that contain an element of the range are named, so every address lies inside the caller's buffer.
__device__ __forceinline__ void prefetch_span_l2(const float* p, int n) {
    const int lane = threadIdx.x & 31;
    const uintptr_t first = reinterpret_cast<uintptr_t>(p) & ~static_cast<uintptr_t>(127);
    const uintptr_t line = first + 128u * static_cast<uintptr_t>(lane);
    if (line < reinterpret_cast<uintptr_t>(p + n)) asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
}

__device__ __forceinline__ float load_in(const void* p, size_t idx, bool bf16) {
    if (bf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[idx]);
    return reinterpret_cast<const float*>(p)[idx];
}

// Increment dx_t (d_in values) of sample b at interval t, from knots or from stored increments.
__device__ __forceinline__ float input_increment(const void* path, int b, int t, int c, int T, int d_in,
                                                 unsigned flags) {
    const bool bf16 = (flags & EWS_F_BF16) != 0;
    if (flags & EWS_F_INCREMENTS) return load_in(path, ((size_t)b * T + t) * d_in + c, bf16);
    const size_t k0 = ((size_t)b * (T + 1) + t) * d_in + c;
    return load_in(path, k0 + d_in, bf16) - load_in(path, k0, bf16);
}

// CTAs of `kernel` that fit on one SM with `threads` threads and `smem` bytes of dynamic shared memory,
// from the device's register, shared-memory and thread limits (the occupancy query is taken too and the
// larger answer kept: on this part it has answered 1 where 2 CTAs fit). Grids of these kernels take
// work from an ordered ticket and only wait on lower tickets, so a CTA that is not resident never
// blocks a resident one.
inline int resident_ctas(const void* kernel, int threads, size_t smem) {
    int api = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&api, kernel, threads, smem);
    cudaFuncAttributes fa{};
    if (cudaFuncGetAttributes(&fa, kernel) != cudaSuccess) return api;
    int dev = 0, smem_sm = 0, reserved = 0, regs_sm = 0, thr_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
    cudaDeviceGetAttribute(&regs_sm, cudaDevAttrMaxRegistersPerMultiprocessor, dev);
    cudaDeviceGetAttribute(&thr_sm, cudaDevAttrMaxThreadsPerMultiProcessor, dev);
    const long per_cta_smem = (long)smem + (long)fa.sharedSizeBytes + reserved;
    const int by_smem = per_cta_smem > 0 ? (int)(smem_sm / per_cta_smem) : 32;
    const int regs_warp = ((fa.numRegs + 7) / 8) * 8 * 32;  // registers are allocated per warp, 256 at a time
    const int warps = (threads + 31) / 32;
    const int by_regs = regs_warp > 0 ? regs_sm / (regs_warp * warps) : 32;
    const int by_threads = thr_sm / threads;
    int mine = by_smem < by_regs ? by_smem : by_regs;
    if (by_threads < mine) mine = by_threads;
    return api > mine ? api : mine;
}

}  // namespace ews
