// Classifier head of a spiking network: logits = spikes @ W^T + b for a small number
// of classes, averaged over T (or kept per step).
//
// Replaces the last nn.Linear of VGGSNN (snn_compiler/zoo/vgg.py:84, run at :111-114)
// and the caller's mean over T (examples/vgg16_snn/vgg16_test.py:243).  With N <= 64
// outputs the product is a few dot products per sample -- far too narrow for a
// tensor-core tile -- so it runs on the CUDA cores: one CTA per sample and one warp
// per output, 16-byte loads of the bf16 spike row and of the weight row, warp-shuffle
// reductions.  Per step
// y_t = dot + b (float32); mean = (((y_0 + y_1) + y_2) + ...) * (1/T).
#include "common.cuh"

namespace snnb {
namespace {


__device__ __forceinline__ void bf16x8_to_f32(uint4 q, float (&o)[8]) {
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        o[2 * i] = __uint_as_float(w[i] << 16);
        o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

// One CTA per sample, one warp per output (N <= 32 warps): for every step the warp
// takes the dot product of the sample's spike row with its weight row (16-byte loads,
// each lane a strided slice of K), reduces it with shuffles, and lane 0 keeps the
// running per-step sum.  No block-wide synchronisation.
__global__ void linear_head_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int B, int K, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ bias, int N, int per_step, float* __restrict__ out) {
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K8 = K / 8;
    for (int n = warp; n < N; n += blockDim.x >> 5) {
        const uint4* wr = reinterpret_cast<const uint4*>(w + (int64_t)n * K);
        const float bn = __ldg(bias + n);
        float mean_acc = 0.0f;
        for (int t = 0; t < T; ++t) {
            const uint4* xr = reinterpret_cast<const uint4*>(x + ((int64_t)t * B + b) * K);
            float acc = 0.0f;
            for (int k8 = lane; k8 < K8; k8 += 32) {
                float xv[8], wv[8];
                bf16x8_to_f32(__ldg(xr + k8), xv);
                bf16x8_to_f32(__ldg(wr + k8), wv);
#pragma unroll
                for (int i = 0; i < 8; ++i) acc = __fmaf_rn(xv[i], wv[i], acc);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            const float y = __fadd_rn(acc, bn);
            if (per_step) {
                if (lane == 0) out[((int64_t)t * B + b) * N + n] = y;
            } else {
                mean_acc = __fadd_rn(mean_acc, y);
            }
        }
        if (!per_step && lane == 0) out[(int64_t)b * N + n] = __fmul_rn(mean_acc, 1.0f / (float)T);
    }
}

int run_head(const void* x, int64_t T, int64_t B, int64_t K, const void* w, const float* bias,
             int64_t N, float* out, int per_step, cudaStream_t s) {
    if (!x || !w || !bias || !out) return SNNB_ERR_ARG;
    if (T <= 0 || B <= 0 || K <= 0 || N <= 0 || N > 64) return SNNB_ERR_ARG;
    if (K % 8 || !aligned16(x) || !aligned16(w)) return SNNB_ERR_ARG;
    if (B > 0x7fffffff || T > 0x7fffffff || K > 0x7fffffff) return SNNB_ERR_ARG;
    const int threads = 32 * (int)(N < 32 ? N : 32);
    linear_head_kernel<<<(unsigned)B, threads, 0, s>>>(
        static_cast<const __nv_bfloat16*>(x), (int)T, (int)B, (int)K,
        static_cast<const __nv_bfloat16*>(w), bias, (int)N, per_step, out);
    return launch_status();
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_linear_mean(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                                const float* bias, int64_t N, float* out, snnb_stream_t stream) {
    return run_head(x, T, B, K, w, bias, N, out, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int snnb_linear_out(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                               const float* bias, int64_t N, float* out, snnb_stream_t stream) {
    return run_head(x, T, B, K, w, bias, N, out, 1, static_cast<cudaStream_t>(stream));
}
