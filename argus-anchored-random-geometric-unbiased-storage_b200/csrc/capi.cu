// Status codes, error text and version of the C ABI (include/argus_b200.h).
#include <stdio.h>
#include <string.h>

#include "common.cuh"

namespace {
thread_local char g_last_error[512] = "";
}

int argus_set_error(int status, const char* msg) {
    snprintf(g_last_error, sizeof(g_last_error), "%s", msg ? msg : "");
    return status;
}

int argus_set_cuda_error(cudaError_t e) {
    snprintf(g_last_error, sizeof(g_last_error), "CUDA error %d: %s", (int)e, cudaGetErrorString(e));
    return ARGUS_ERR_CUDA;
}

extern "C" {

const char* argus_status_string(int status) {
    switch (status) {
        case ARGUS_OK: return "ok";
        case ARGUS_ERR_INVALID_ARGUMENT: return "invalid argument";
        case ARGUS_ERR_MISALIGNED: return "misaligned pointer or stride";
        case ARGUS_ERR_CUDA: return "CUDA error";
        case ARGUS_ERR_UNSUPPORTED: return "unsupported shape";
        case ARGUS_ERR_TIMEOUT: return "device-side wait timed out";
        case ARGUS_ERR_CAPACITY: return "request exceeds a fixed-size buffer";
        default: return "unknown status";
    }
}

const char* argus_last_error(void) { return g_last_error; }

int argus_version(void) { return 100; /* 0.1.0 */ }

}  // extern "C"

extern "C" int argus_memcpy2d_async(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch, int64_t width,
                                    int64_t height, argus_stream_t stream) {
    if (width < 0 || height < 0 || dst_pitch < width || src_pitch < width)
        return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad 2-D copy");
    if (width == 0 || height == 0) return ARGUS_OK;
    if (!dst || !src) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "null pointer");
    cudaError_t e = cudaMemcpy2DAsync(dst, (size_t)dst_pitch, src, (size_t)src_pitch, (size_t)width, (size_t)height,
                                      cudaMemcpyDefault, (cudaStream_t)stream);
    return e == cudaSuccess ? ARGUS_OK : argus_set_cuda_error(e);
}

extern "C" int argus_memcpy_async(void* dst, const void* src, int64_t bytes, argus_stream_t stream) {
    if (bytes < 0 || (bytes > 0 && (!dst || !src))) return argus_set_error(ARGUS_ERR_INVALID_ARGUMENT, "bad copy");
    if (bytes == 0) return ARGUS_OK;
    cudaError_t e = cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, (cudaStream_t)stream);
    return e == cudaSuccess ? ARGUS_OK : argus_set_cuda_error(e);
}
