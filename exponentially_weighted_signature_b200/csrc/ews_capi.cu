// C ABI utilities shared by the engines: status read-back, error strings, version.
#include "ews_common.cuh"

extern "C" int ews_read_device_status(const void* workspace, ews_stream_t stream, int* status) {
    if (!workspace || !status) return EWS_ERR_INVALID_ARGUMENT;
    ews::DeviceStatus st{};
    cudaStream_t s = (cudaStream_t)stream;
    if (cudaMemcpyAsync(&st, workspace, sizeof(st), cudaMemcpyDeviceToHost, s) != cudaSuccess) return EWS_ERR_LAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return EWS_ERR_LAUNCH;
    *status = st.error;
    return EWS_OK;
}

namespace {
// One thread: fold a workspace's error word into the caller's sticky word (the first error is kept).
__global__ void status_fold_kernel(const ews::DeviceStatus* st, int* sticky) {
    const int e = *((volatile const int*)&st->error);
    if (e != 0) atomicCAS(sticky, 0, e);
}
}  // namespace

extern "C" int ews_status_fold(const void* workspace, int* sticky, ews_stream_t stream) {
    if (!workspace || !sticky) return EWS_ERR_INVALID_ARGUMENT;
    status_fold_kernel<<<1, 1, 0, (cudaStream_t)stream>>>((const ews::DeviceStatus*)workspace, sticky);
    return cudaGetLastError() == cudaSuccess ? EWS_OK : EWS_ERR_LAUNCH;
}

extern "C" const char* ews_error_string(int code) {
    switch (code) {
        case EWS_OK: return "ok";
        case EWS_ERR_INVALID_ARGUMENT: return "invalid argument";
        case EWS_ERR_UNSUPPORTED: return "unsupported configuration";
        case EWS_ERR_WORKSPACE: return "workspace missing or too small";
        case EWS_ERR_LAUNCH: return "CUDA launch failed";
        case EWS_ERR_LOOKBACK_TIMEOUT: return "look-back wait timed out";
    }
    return "unknown error";
}

extern "C" int ews_version(void) { return 1; }
