// First layer of a spiking CNN: the input is a real-valued image (not exact in bf16),
// so the conv runs in float32 on the CUDA cores; it is <1% of the network's FLOPs.
//
// Replaces the first FusedConvBNNeuron of VGGSNN (snn_compiler/zoo/vgg.py:88-94 ->
// nn/modules.py:347-357): F.conv2d(x, W') + fused_bias_if_lif(..., b').
//
// Thread = one output pixel x 64 output channels (one 2x2 pooled pixel x 16 channels
// when pooling).  The folded weights sit in shared memory as [tap][cout] and are read
// as warp-wide broadcasts, each input value is loaded once per thread, and the
// membrane potentials stay in registers across the T loop.  With direct encoding (Ti == 1) the conv runs once and every
// step reuses it.  Spikes leave as bf16 NHWC, 32 bytes per pixel per step.
#include "common.cuh"

namespace snnb {
namespace {

constexpr int THREADS = 128;

template <bool POOL, int CG, bool HARD>
__global__ void __launch_bounds__(THREADS) first_conv_lif_kernel(
    const float* __restrict__ x, int Ti, int T, int B, int Cin, int H, int W,
    const float* __restrict__ w, const float* __restrict__ bias, int Cout,
    float df, float sc, float thr, float v_reset, __nv_bfloat16* __restrict__ out) {
    extern __shared__ float sw[];                    // [Cin*9][Cout]
    const int K = Cin * 9;
    for (int i = threadIdx.x; i < K * Cout; i += THREADS) {
        const int co = i % Cout, k = i / Cout;       // k = ci*9 + kh*3 + kw (torch order)
        sw[i] = w[(int64_t)co * K + k];
    }
    __syncthreads();
    constexpr int NP = POOL ? 4 : 1;
    const int groups = Cout / CG;
    const int Ho = POOL ? H / 2 : H, Wo = POOL ? W / 2 : W;
    const int64_t total = (int64_t)B * Ho * Wo * groups;
    const int64_t gid = (int64_t)blockIdx.x * THREADS + threadIdx.x;
    if (gid >= total) return;
    const int g = (int)(gid % groups);
    int64_t r = gid / groups;
    const int ow = (int)(r % Wo);
    r /= Wo;
    const int oh = (int)(r % Ho);
    const int b = (int)(r / Ho);
    float bb[CG];
#pragma unroll
    for (int j = 0; j < CG; ++j) bb[j] = __ldg(bias + g * CG + j);
    float v[NP][CG], y[NP][CG];
#pragma unroll
    for (int q = 0; q < NP; ++q)
#pragma unroll
        for (int j = 0; j < CG; ++j) v[q][j] = 0.0f;
    for (int t = 0; t < T; ++t) {
        if (t == 0 || Ti != 1) {
            const int ti = Ti == 1 ? 0 : t;
#pragma unroll
            for (int q = 0; q < NP; ++q) {
                const int h = POOL ? 2 * oh + (q >> 1) : oh;
                const int ww = POOL ? 2 * ow + (q & 1) : ow;
#pragma unroll
                for (int j = 0; j < CG; ++j) y[q][j] = 0.0f;
                for (int ci = 0; ci < Cin; ++ci) {
                    const float* xc = x + (((int64_t)ti * B + b) * Cin + ci) * H * W;
#pragma unroll
                    for (int kh = 0; kh < 3; ++kh) {
                        const int ih = h + kh - 1;
#pragma unroll
                        for (int kw = 0; kw < 3; ++kw) {
                            const int iw = ww + kw - 1;
                            const float xv = (ih >= 0 && ih < H && iw >= 0 && iw < W)
                                                 ? __ldg(xc + ih * W + iw) : 0.0f;
                            const float* wk = sw + (ci * 9 + kh * 3 + kw) * Cout + g * CG;
#pragma unroll
                            for (int j = 0; j < CG; ++j) y[q][j] = __fmaf_rn(xv, wk[j], y[q][j]);
                        }
                    }
                }
            }
        }
        uint32_t bits[(CG + 31) / 32];
#pragma unroll
        for (int k = 0; k < (CG + 31) / 32; ++k) bits[k] = 0u;
#pragma unroll
        for (int q = 0; q < NP; ++q) {
#pragma unroll
            for (int j = 0; j < CG; ++j) {
                const float in = __fadd_rn(y[q][j], bb[j]);
                float vv = charge(v[q][j], df, sc, in);
                const bool s = vv >= thr;
                v[q][j] = reset_v<HARD>(vv, s, thr, v_reset);
                bits[j / 32] |= (s ? 1u : 0u) << (j % 32);
            }
        }
        const int64_t o = ((((int64_t)t * B + b) * Ho + oh) * Wo + ow) * Cout + g * CG;
        uint4* dst = reinterpret_cast<uint4*>(out + o);
#pragma unroll
        for (int k = 0; k < CG / 8; ++k) dst[k] = spikes_to_bf16x8(bits[k / 4] >> (8 * (k % 4)) & 0xffu);
    }
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_first_conv_lif(const float* x, int64_t Ti, int64_t T, int64_t B, int64_t Cin,
                                   int64_t H, int64_t W, const float* w, const float* bias,
                                   int64_t Cout, float decay, float input_scale,
                                   float v_threshold, float v_reset, int hard_reset, int pool,
                                   void* out, snnb_stream_t stream) {
    if (!x || !w || !bias || !out) return SNNB_ERR_ARG;
    if (T <= 0 || B <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0) return SNNB_ERR_ARG;
    if (Ti != 1 && Ti != T) return SNNB_ERR_ARG;
    if (Cout % 16 || !aligned16(out)) return SNNB_ERR_ARG;
    const int CG = (!pool && Cout % 64 == 0) ? 64 : 16;
    if (pool && ((H % 2) || (W % 2))) return SNNB_ERR_UNSUPPORTED;
    const int64_t smem = Cin * 9 * Cout * 4;
    if (smem > 200 * 1024) return SNNB_ERR_UNSUPPORTED;
    if (T * B * Cin * H * W > ((int64_t)1 << 40) || T > 0x7fffffff) return SNNB_ERR_ARG;
    const int Ho = pool ? (int)H / 2 : (int)H, Wo = pool ? (int)W / 2 : (int)W;
    const int64_t total = B * Ho * Wo * (Cout / CG);
    const int64_t blocks = (total + THREADS - 1) / THREADS;
    if (blocks > 0x7fffffffll) return SNNB_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto* o = static_cast<__nv_bfloat16*>(out);
    auto run = [&](auto kernel) -> int {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return record_cuda_error(e);
        kernel<<<(unsigned)blocks, THREADS, smem, s>>>(
            x, (int)Ti, (int)T, (int)B, (int)Cin, (int)H, (int)W, w, bias, (int)Cout, decay,
            input_scale, v_threshold, v_reset, o);
        return launch_status();
    };
    if (pool)
        return hard_reset ? run(first_conv_lif_kernel<true, 16, true>)
                          : run(first_conv_lif_kernel<true, 16, false>);
    if (CG == 64)
        return hard_reset ? run(first_conv_lif_kernel<false, 64, true>)
                          : run(first_conv_lif_kernel<false, 64, false>);
    return hard_reset ? run(first_conv_lif_kernel<false, 16, true>)
                      : run(first_conv_lif_kernel<false, 16, false>);
}
