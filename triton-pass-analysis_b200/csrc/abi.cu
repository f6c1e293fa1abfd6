// Status helpers of the C ABI (snnb200.h).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "common.cuh"

namespace snnb {
namespace {
thread_local char g_last_error[256] = "";
}

bool pdl_enabled() {
    static const bool on = [] {
        const char* v = getenv("SNNB_NO_PDL");
        return !(v && v[0] && v[0] != '0');
    }();
    return on;
}

int record_cuda_error(cudaError_t e) {
    const char* name = cudaGetErrorName(e);
    const char* text = cudaGetErrorString(e);
    snprintf(g_last_error, sizeof(g_last_error), "%s: %s", name ? name : "?", text ? text : "?");
    return SNNB_ERR_CUDA;
}
}  // namespace snnb

extern "C" int snnb_abi_version(void) { return 1; }

extern "C" const char* snnb_status_string(int status) {
    switch (status) {
        case SNNB_OK: return "ok";
        case SNNB_ERR_ARG: return "invalid argument";
        case SNNB_ERR_UNSUPPORTED: return "unsupported combination";
        case SNNB_ERR_CUDA: return "CUDA error";
        case SNNB_ERR_TIMEOUT: return "device wait timed out";
        case SNNB_ERR_DEVICE: return "device-side check failed";
        default: return "unknown status";
    }
}

extern "C" const char* snnb_last_cuda_error(void) { return snnb::g_last_error; }
