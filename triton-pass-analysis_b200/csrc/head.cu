// Classifier head of a spiking network: logits = spikes @ W^T + b for a small number
// of classes, averaged over T (or kept per step).
//
// Replaces the last nn.Linear of VGGSNN (snn_compiler/zoo/vgg.py:84, run at :111-114)
// and the caller's mean over T (examples/vgg16_snn/vgg16_test.py:243).  With N <= 64
// outputs the product is a few dot products per sample -- far too narrow for a
// tensor-core tile -- so it runs on the CUDA cores.
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

// One CTA of 256 threads per sample.  A pass covers up to TC steps x NC outputs: every
// thread takes a strided set of 8-element K slices, loads the TC spike slices and NC weight
// slices at once (16-byte loads), and keeps TC x NC independent float32 partial sums; the
// partials are reduced with shuffles within warps and through shared memory across the
// 8 warps.  Per step y_t = dot + b; mean = (((y_0 + y_1) + y_2) + ...) * (1/T).
constexpr int HEAD_THREADS = 256;
constexpr int TC = 4, NC = 8;

__global__ void __launch_bounds__(HEAD_THREADS) linear_head_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int B, int K, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ bias, int N, int per_step, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[HEAD_THREADS / 32][TC * NC];
    __shared__ float mean_acc[64];
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K8 = K / 8;
    if (threadIdx.x < 64) mean_acc[threadIdx.x] = 0.0f;
    for (int t0 = 0; t0 < T; t0 += TC) {
        for (int n0 = 0; n0 < N; n0 += NC) {
            float acc[TC][NC];
#pragma unroll
            for (int i = 0; i < TC; ++i)
#pragma unroll
                for (int j = 0; j < NC; ++j) acc[i][j] = 0.0f;
            for (int k8 = threadIdx.x; k8 < K8; k8 += HEAD_THREADS) {
                uint4 xq[TC], wq[NC];
#pragma unroll
                for (int i = 0; i < TC; ++i)
                    xq[i] = t0 + i < T ? __ldg(reinterpret_cast<const uint4*>(
                                             x + ((int64_t)(t0 + i) * B + b) * K) + k8)
                                       : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int j = 0; j < NC; ++j)
                    wq[j] = n0 + j < N ? __ldg(reinterpret_cast<const uint4*>(
                                             w + (int64_t)(n0 + j) * K) + k8)
                                       : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int i = 0; i < TC; ++i) {
                    float xv[8];
                    bf16x8_to_f32(xq[i], xv);
#pragma unroll
                    for (int j = 0; j < NC; ++j) {
                        float wv[8];
                        bf16x8_to_f32(wq[j], wv);
#pragma unroll
                        for (int e = 0; e < 8; ++e) acc[i][j] = __fmaf_rn(xv[e], wv[e], acc[i][j]);
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < TC; ++i)
#pragma unroll
                for (int j = 0; j < NC; ++j) {
                    float a = acc[i][j];
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
                    if (lane == 0) red[warp][i * NC + j] = a;
                }
            __syncthreads();
            if (threadIdx.x < TC * NC) {
                const int i = threadIdx.x / NC, j = threadIdx.x % NC;
                const int t = t0 + i, n = n0 + j;
                if (t < T && n < N) {
                    float d = red[0][threadIdx.x];
#pragma unroll
                    for (int k = 1; k < HEAD_THREADS / 32; ++k) d += red[k][threadIdx.x];
                    const float y = __fadd_rn(d, __ldg(bias + n));
                    if (per_step) out[((int64_t)t * B + b) * N + n] = y;
                    else red[0][threadIdx.x] = y;
                }
            }
            __syncthreads();
            if (!per_step && threadIdx.x < NC && n0 + threadIdx.x < N) {
                // steps in order, so the running sum matches (((y_0 + y_1) + y_2) + ...)
                float m = mean_acc[n0 + threadIdx.x];
                for (int i = 0; i < TC && t0 + i < T; ++i) m = __fadd_rn(m, red[0][i * NC + threadIdx.x]);
                mean_acc[n0 + threadIdx.x] = m;
            }
            __syncthreads();
        }
    }
    if (!per_step && threadIdx.x < N)
        out[(int64_t)b * N + threadIdx.x] = __fmul_rn(mean_acc[threadIdx.x], 1.0f / (float)T);
}

// One 128-thread CTA per (class n, sample b) -- B x N small CTAs in flight together instead of
// B CTAs looping over the classes: each thread takes every 128th 8-element K slice, keeps the
// partial dot products of up to 4 steps, and the CTA reduces them (shuffles, then the 4 warps
// in order).  Per step y_t = dot + b; mean = (((y_0 + y_1) + y_2) + ...) * (1/T).
constexpr int HEAD2_THREADS = 128;

__global__ void __launch_bounds__(HEAD2_THREADS) linear_head_nb_kernel(
    const __nv_bfloat16* __restrict__ x, int T, int B, int K, const __nv_bfloat16* __restrict__ w,
    const float* __restrict__ bias, int N, int per_step, float* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    __shared__ float red[HEAD2_THREADS / 32][TC];
    const int n = blockIdx.x, b = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int K8 = K / 8;
    const uint4* wrow = reinterpret_cast<const uint4*>(w + (int64_t)n * K);
    const float bn = __ldg(bias + n);
    float mean = 0.0f;
    for (int t0 = 0; t0 < T; t0 += TC) {
        float acc[TC];
#pragma unroll
        for (int i = 0; i < TC; ++i) acc[i] = 0.0f;
        for (int k8 = threadIdx.x; k8 < K8; k8 += HEAD2_THREADS) {
            float wv[8];
            bf16x8_to_f32(__ldg(wrow + k8), wv);
            uint4 xq[TC];
#pragma unroll
            for (int i = 0; i < TC; ++i)           // the step slices' loads in flight together
                xq[i] = t0 + i < T ? __ldg(reinterpret_cast<const uint4*>(
                                         x + ((int64_t)(t0 + i) * B + b) * K) + k8)
                                   : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int i = 0; i < TC; ++i) {
                float xv[8];
                bf16x8_to_f32(xq[i], xv);
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[i] = __fmaf_rn(xv[e], wv[e], acc[i]);
            }
        }
#pragma unroll
        for (int i = 0; i < TC; ++i) {
            float a = acc[i];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            if (lane == 0) red[warp][i] = a;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            for (int i = 0; i < TC && t0 + i < T; ++i) {
                float d = red[0][i];
#pragma unroll
                for (int k = 1; k < HEAD2_THREADS / 32; ++k) d += red[k][i];
                const float y = __fadd_rn(d, bn);
                if (per_step) out[((int64_t)(t0 + i) * B + b) * N + n] = y;
                else mean = __fadd_rn(mean, y);           // steps in order
            }
        }
        __syncthreads();
    }
    if (!per_step && threadIdx.x == 0)
        out[(int64_t)b * N + n] = __fmul_rn(mean, 1.0f / (float)T);
}

int run_head(const void* x, int64_t T, int64_t B, int64_t K, const void* w, const float* bias,
             int64_t N, float* out, int per_step, cudaStream_t s) {
    if (!x || !w || !bias || !out) return SNNB_ERR_ARG;
    if (T <= 0 || B <= 0 || K <= 0 || N <= 0 || N > 64) return SNNB_ERR_ARG;
    if (K % 8 || !aligned16(x) || !aligned16(w)) return SNNB_ERR_ARG;
    if (B > 0x7fffffff || T > 0x7fffffff || K > 0x7fffffff) return SNNB_ERR_ARG;
    if (B <= 65535)
        return launch_k(linear_head_nb_kernel, dim3((unsigned)N, (unsigned)B), dim3(HEAD2_THREADS),
                        0, s, static_cast<const __nv_bfloat16*>(x), (int)T, (int)B, (int)K,
                        static_cast<const __nv_bfloat16*>(w), bias, (int)N, per_step, out);
    return launch_k(linear_head_kernel, dim3((unsigned)B), dim3(HEAD_THREADS), 0, s,
                    static_cast<const __nv_bfloat16*>(x), (int)T, (int)B, (int)K,
                    static_cast<const __nv_bfloat16*>(w), bias, (int)N, per_step, out);
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_linear_mean(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                                const float* bias, int64_t N, float* out, snnb_stream_t stream) {
    if (const int inj = snnb::take_injected_status()) return inj;
    return run_head(x, T, B, K, w, bias, N, out, 0, static_cast<cudaStream_t>(stream));
}

extern "C" int snnb_linear_out(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                               const float* bias, int64_t N, float* out, snnb_stream_t stream) {
    if (const int inj = snnb::take_injected_status()) return inj;
    return run_head(x, T, B, K, w, bias, N, out, 1, static_cast<cudaStream_t>(stream));
}
