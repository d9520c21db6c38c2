// Status strings and ABI version of the C interface.
#include "mmb_common.cuh"

#define MMB_ABI_VERSION 2

extern "C" const char* mmb_status_string(int status) {
    switch (status) {
        case MMB_OK: return "ok";
        case MMB_ERR_NULL: return "a required pointer is NULL";
        case MMB_ERR_SHAPE: return "a size or stride is out of range";
        case MMB_ERR_ALIGN: return "a pointer or stride breaks the required alignment";
        case MMB_ERR_UNSUPPORTED: return "unsupported configuration";
        case MMB_ERR_WORKSPACE: return "workspace missing";
        case MMB_ERR_LAUNCH: return "CUDA launch failed";
        case MMB_ERR_TIMEOUT: return "a bounded device-side wait timed out";
        default: return "unknown status";
    }
}

extern "C" int mmb_abi_version(void) { return MMB_ABI_VERSION; }

static thread_local cudaError_t g_last_cuda_error = cudaSuccess;

void mmb_record_cuda_error(cudaError_t e) { g_last_cuda_error = e; }

extern "C" const char* mmb_last_error(void) {
    if (g_last_cuda_error == cudaSuccess) return "no CUDA error recorded";
    return cudaGetErrorString(g_last_cuda_error);
}
