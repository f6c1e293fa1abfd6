// Shared helpers for the sm_100a kernels of libsnnb200.so.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "snnb200.h"

namespace snnb {

// Records the text of a CUDA error for snnb_last_cuda_error() and maps it to a status.
int record_cuda_error(cudaError_t e);

// Test hooks (snnb_debug_inject_status / snnb_debug_inject_stall): a pending injected status
// is returned (and consumed) by the next entry call; a pending stall is consumed by the next
// launch of the T-sequential conv kernel.  0 when nothing is pending.
int take_injected_status();
int take_injected_stall();

// Each translation unit with tensor-core waits registers the setter of its copy of the
// per-device wait limit (tc_common.cuh); snnb_set_wait_limit calls them all.
int register_wait_limit_setter(cudaError_t (*setter)(unsigned long long));

// Status of the most recent launch on this thread (cudaGetLastError, which also clears it).
inline int launch_status() {
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? SNNB_OK : record_cuda_error(e);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Debug build (-DSNNB_CHECK_BOUNDS, `make check` -> libsnnb200_check.so): index checks on the
// kernels' global accesses that record SNNB_ERR_DEVICE in the device status word and skip the
// access.  The release build compiles them to `true`.
#ifdef SNNB_CHECK_BOUNDS
__device__ __forceinline__ bool check_index(int64_t i, int64_t n, int* status) {
    if (i >= 0 && i < n) return true;
    if (status) atomicExch(status, SNNB_ERR_DEVICE);
    return false;
}
#define SNNB_IN_BOUNDS(i, n, status) (::snnb::check_index((int64_t)(i), (int64_t)(n), (status)))
#else
#define SNNB_IN_BOUNDS(i, n, status) (true)
#endif

// Programmatic dependent launch.  Every kernel of this library is launched with programmatic
// stream serialization allowed (launch_k), so its CTAs may be scheduled while the previous
// kernel on the stream is still finishing.  Each kernel runs pdl_wait() before it touches
// global memory -- it returns once every earlier kernel of the stream has completed and its
// writes are visible -- and pdl_trigger() to let the next kernel be scheduled early.  A
// kernel launched without the attribute sees both as no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// SNNB_NO_PDL=1 in the environment launches without the attribute (plain stream order),
// e.g. under a profiler that replays kernels one by one.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline int launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                    Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
    return e == cudaSuccess ? launch_status() : record_cuda_error(e);
}

// launch_k for thread-block clusters of `cluster_x` CTAs along x.
template <typename... KArgs, typename... Args>
inline int launch_kc(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                     unsigned cluster_x, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster_x;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<Args&&>(args)...);
    return e == cudaSuccess ? launch_status() : record_cuda_error(e);
}

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T> __device__ __forceinline__ T spike_value(bool s);
template <> __device__ __forceinline__ float spike_value<float>(bool s) { return s ? 1.0f : 0.0f; }
template <> __device__ __forceinline__ __half spike_value<__half>(bool s) {
    return __ushort_as_half(s ? (unsigned short)0x3C00 : (unsigned short)0);
}
template <> __device__ __forceinline__ __nv_bfloat16 spike_value<__nv_bfloat16>(bool s) {
    return __ushort_as_bfloat16(s ? (unsigned short)0x3F80 : (unsigned short)0);
}
template <> __device__ __forceinline__ uint8_t spike_value<uint8_t>(bool s) { return s ? 1 : 0; }

// Membrane charge with every product and the sum rounded separately to float32
// (no FMA contraction), matching the reference's eager torch-CPU loop.
__device__ __forceinline__ float charge(float v, float df, float sc, float in) {
    return __fadd_rn(__fmul_rn(df, v), __fmul_rn(sc, in));
}

// Reset after the threshold test.  A compile-time HARD keeps the per-neuron code free of
// branches (a run-time choice here was compiled to a branch per neuron and made the LIF
// epilogues ~3x slower).
template <bool HARD>
__device__ __forceinline__ float reset_v(float v, bool s, float thr, float v_reset) {
    if (HARD) return s ? v_reset : v;
    return s ? __fsub_rn(v, thr) : v;
}

// float32 a as three bf16 terms hi = rn(a), mid = rn(a - hi), lo = rn(a - hi - mid) (each
// subtraction exact in float32; non-finite values keep only hi).  A finite value
// above bf16's largest (rounding would give infinity) takes hi = +-0x7F7F, the largest bf16.
__device__ __forceinline__ void split_bf16x3(float a, __nv_bfloat16& h, __nv_bfloat16& m,
                                       __nv_bfloat16& l) {
    h = __float2bfloat16_rn(a);
    if (isinf(__bfloat162float(h)) && isfinite(a))
        h = __ushort_as_bfloat16(a > 0.0f ? (unsigned short)0x7F7F : (unsigned short)0xFF7F);
    const float fh = __bfloat162float(h);
    if (!isfinite(fh)) {
        m = l = __float2bfloat16_rn(0.0f);
        return;
    }
    const float r1 = __fsub_rn(a, fh);
    m = __float2bfloat16_rn(r1);
    const float r2 = __fsub_rn(r1, __bfloat162float(m));
    l = __float2bfloat16_rn(r2);
}

// split_bf16x3 of two values with |a| <= SPLIT2_FAST_MAX (finite, and their bf16 rounding
// cannot overflow), as bf16x2 words (a0 in the low half): the same roundings and exact
// residuals, with paired conversions.
constexpr float SPLIT2_FAST_MAX = 3.0e38f;
__device__ __forceinline__ void split2_bf16x3_finite(float a0, float a1, uint32_t& h,
                                                     uint32_t& m, uint32_t& l) {
    auto bits = [](__nv_bfloat162 v) -> uint32_t {
        return (uint32_t)__bfloat16_as_ushort(v.x) | ((uint32_t)__bfloat16_as_ushort(v.y) << 16);
    };
    const __nv_bfloat162 h2 = __float22bfloat162_rn(make_float2(a0, a1));
    const float2 fh = __bfloat1622float2(h2);
    const float2 r1 = make_float2(__fsub_rn(a0, fh.x), __fsub_rn(a1, fh.y));
    const __nv_bfloat162 m2 = __float22bfloat162_rn(r1);
    const float2 fm = __bfloat1622float2(m2);
    const __nv_bfloat162 l2 =
        __float22bfloat162_rn(make_float2(__fsub_rn(r1.x, fm.x), __fsub_rn(r1.y, fm.y)));
    h = bits(h2);
    m = bits(m2);
    l = bits(l2);
}

// The same for any two values: those whose bf16 rounding could overflow, and non-finite
// ones, take the scalar path.
__device__ __forceinline__ void split2_bf16x3(float a0, float a1, uint32_t& h, uint32_t& m,
                                              uint32_t& l) {
    auto bits = [](__nv_bfloat162 v) -> uint32_t {
        return (uint32_t)__bfloat16_as_ushort(v.x) | ((uint32_t)__bfloat16_as_ushort(v.y) << 16);
    };
    if (fabsf(a0) <= SPLIT2_FAST_MAX && fabsf(a1) <= SPLIT2_FAST_MAX) {
        split2_bf16x3_finite(a0, a1, h, m, l);
    } else {
        __nv_bfloat16 h0, m0, l0, h1, m1, l1;
        split_bf16x3(a0, h0, m0, l0);
        split_bf16x3(a1, h1, m1, l1);
        h = bits(__halves2bfloat162(h0, h1));
        m = bits(__halves2bfloat162(m0, m1));
        l = bits(__halves2bfloat162(l0, l1));
    }
}

// 8 spike bits -> 8 bf16 values (0.0 / 1.0) packed in 16 bytes, bit i -> element i.
__device__ __forceinline__ uint4 spikes_to_bf16x8(uint32_t bits8) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t lo = ((bits8 >> (2 * i)) & 1u) ? 0x3F80u : 0u;
        const uint32_t hi = ((bits8 >> (2 * i + 1)) & 1u) ? 0x3F800000u : 0u;
        w[i] = lo | hi;
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

}  // namespace snnb
