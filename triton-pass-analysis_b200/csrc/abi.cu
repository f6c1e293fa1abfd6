// Status helpers of the C ABI (snnb200.h).
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "common.cuh"

namespace snnb {
namespace {
thread_local char g_last_error[256] = "";

std::atomic<int> g_inject_status{0};
std::atomic<int> g_inject_status_count{0};
std::atomic<int> g_inject_stall_count{0};

// Takes one from a pending count; true if there was one.
bool take_one(std::atomic<int>& count) {
    int c = count.load(std::memory_order_relaxed);
    while (c > 0) {
        if (count.compare_exchange_weak(c, c - 1, std::memory_order_acq_rel)) return true;
    }
    return false;
}

struct WaitLimitSetters {
    std::mutex lock;
    std::vector<cudaError_t (*)(unsigned long long)> fns;
};
WaitLimitSetters& wait_limit_setters() {
    static WaitLimitSetters s;      // constructed on first use: safe from any unit's init
    return s;
}
}  // namespace

int take_injected_status() {
    return take_one(g_inject_status_count) ? g_inject_status.load(std::memory_order_acquire) : 0;
}
int take_injected_stall() { return take_one(g_inject_stall_count) ? 1 : 0; }

int register_wait_limit_setter(cudaError_t (*setter)(unsigned long long)) {
    WaitLimitSetters& w = wait_limit_setters();
    std::lock_guard<std::mutex> guard(w.lock);
    w.fns.push_back(setter);
    return 1;
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

extern "C" int snnb_set_wait_limit(int64_t cycles) {
    if (cycles != 0 && cycles < 1000) return SNNB_ERR_ARG;
    const unsigned long long v = cycles == 0 ? 4000000000ull : (unsigned long long)cycles;
    snnb::WaitLimitSetters& w = snnb::wait_limit_setters();
    std::lock_guard<std::mutex> guard(w.lock);
    for (auto fn : w.fns) {
        const cudaError_t e = fn(v);
        if (e != cudaSuccess) return snnb::record_cuda_error(e);
    }
    return SNNB_OK;
}

extern "C" int snnb_debug_inject_status(int status, int count) {
    if (status >= 0 || count < 0) return SNNB_ERR_ARG;
    snnb::g_inject_status.store(status, std::memory_order_release);
    snnb::g_inject_status_count.store(count, std::memory_order_release);
    return SNNB_OK;
}

extern "C" int snnb_debug_inject_stall(int count) {
    if (count < 0) return SNNB_ERR_ARG;
    snnb::g_inject_stall_count.store(count, std::memory_order_release);
    return SNNB_OK;
}
