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
