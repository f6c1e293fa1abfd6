// float32 operands on the bf16 tensor cores without losing float32 precision.
//
// The reference runs F.conv2d / F.linear in the input's dtype (snn_compiler/nn/modules.py:
// 194-206, 241-255, 324-345): a float32 module on a real-valued float32 input convolves in
// float32.  The tcgen05 kernels multiply bf16 x bf16 into float32 accumulators, so a float32
// value a is carried as three bf16 terms
//     a_hi = rn(a),  a_mid = rn(a - a_hi),  a_lo = rn(a - a_hi - a_mid)
// (each subtraction is exact in float32), which represent a to within 2^-24 |a|.  Of the nine
// products of an activation's and a weight's terms the six larger ones are kept,
//     x_hi w_hi + x_hi w_mid + x_hi w_lo + x_mid w_hi + x_mid w_mid + x_lo w_hi,
// each exact in float32; the three dropped ones are together below 2^-23 |x w| (|mid| <=
// 2^-8 |a|, |lo| <= 2^-16 |a|), the order of float32 rounding itself.  The conv then runs on
// six channel groups: activations [hi, hi, hi, mid, mid, lo] against weights
// [hi, mid, lo, hi, mid, hi] (group g holds channels g*Cp .. g*Cp + C - 1; Cp - C zero
// channels pad each group so that 6 * Cp is a multiple of 8, the kernels' 16-byte rows).
// This file writes the activation side; the weights are split once on the host.
#include "common.cuh"

namespace snnb {
namespace {

__device__ __forceinline__ uint2 pack4(const __nv_bfloat16 (&v)[4]) {
    uint2 r;
    r.x = (uint32_t)__bfloat16_as_ushort(v[0]) | ((uint32_t)__bfloat16_as_ushort(v[1]) << 16);
    r.y = (uint32_t)__bfloat16_as_ushort(v[2]) | ((uint32_t)__bfloat16_as_ushort(v[3]) << 16);
    return r;
}

// One thread per (row, 4-channel group of the padded width Cp): reads 4 float32 (zeros past
// C), writes the 4 channels of each of the six groups (8-byte stores).
__global__ void __launch_bounds__(256) split_terms_kernel(const float* __restrict__ x, int64_t rows,
                                                          int64_t C, int64_t Cp,
                                                          __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t q = Cp / 4;
    const int64_t total = rows * q;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / q, c0 = (i - r * q) * 4;
        const float* src = x + r * C;
        float a[4];
        if ((C & 3) == 0 && c0 < C) {               // 4 channels inside the row
            const float4 v = __ldg(reinterpret_cast<const float4*>(src + c0));
            a[0] = v.x; a[1] = v.y; a[2] = v.z; a[3] = v.w;
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k) a[k] = c0 + k < C ? __ldg(src + c0 + k) : 0.0f;
        }
        __nv_bfloat16 h[4], m[4], l[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) split_bf16x3(a[k], h[k], m[k], l[k]);
        const uint2 ph = pack4(h), pm = pack4(m), pl = pack4(l);
        uint2* dst = reinterpret_cast<uint2*>(out + r * 6 * Cp + c0);
        const int64_t g = Cp / 4;                   // one group, in uint2 units
        dst[0] = ph; dst[g] = ph; dst[2 * g] = ph;  // hi, hi, hi
        dst[3 * g] = pm; dst[4 * g] = pm;           // mid, mid
        dst[5 * g] = pl;                            // lo
    }
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_split_bf16_terms(const float* x, int64_t rows, int64_t C, int64_t Cp,
                                     void* out, snnb_stream_t stream) {
    if (const int inj = take_injected_status()) return inj;
    if (!x || !out || rows < 0 || C <= 0 || Cp < C || (Cp & 3) != 0) return SNNB_ERR_ARG;
    if ((C & 3) == 0 && !aligned16(x)) return SNNB_ERR_ARG;
    if ((reinterpret_cast<uintptr_t>(out) & 7u) != 0) return SNNB_ERR_ARG;
    if (rows > ((int64_t)1 << 40) / (6 * Cp)) return SNNB_ERR_ARG;
    if (rows == 0) return SNNB_OK;
    const int64_t total = rows * (Cp / 4);
    const int64_t blocks = (total + 255) / 256;
    const int grid = (int)(blocks < 148 * 16 ? blocks : 148 * 16);
    return launch_k(split_terms_kernel, dim3(grid), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), x, rows, C, Cp,
                    static_cast<__nv_bfloat16*>(out));
}
