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
    pdl_wait();
    pdl_trigger();
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

// Band form for the common case (no pooling, 128 % W == 0, Cout % 16 == 0, Cout <= 128):
// a CTA owns a band of R = 128 / W whole rows of one image; its input patch (R + 2 rows with
// the zero halo, all Cin channels) and the weights ([tap][cout]) are staged in shared
// memory, and thread = (pixel, 16 output channels) -- the 16-channel group is warp-uniform,
// so weight reads are broadcasts.  Few registers per thread keep many warps resident to
// hide the staging and store latency.
constexpr int BAND_CG = 16;

template <bool HARD>
__global__ void __launch_bounds__(1024) first_conv_band_kernel(
    const float* __restrict__ x, int Ti, int T, int B, int Cin, int H, int W,
    const float* __restrict__ w, const float* __restrict__ bias, int Cout,
    float df, float sc, float thr, float v_reset, __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float smf[];
    const int K = Cin * 9;
    const int R = 128 / W;
    const int PW = W + 2, PH = R + 2;
    float* sw = smf;                                  // [K][Cout]
    float* sb = smf + K * Cout;                       // [Cout]
    float* sx = sb + Cout;                            // [Cin][PH][PW]
    const int nb = (H + R - 1) / R;
    const int b = blockIdx.x / nb, h0 = (blockIdx.x % nb) * R;
    for (int i = threadIdx.x; i < K * Cout; i += blockDim.x) {
        const int co = i % Cout, k = i / Cout;       // k = ci*9 + kh*3 + kw (torch order)
        sw[i] = __ldg(w + (int64_t)co * K + k);
    }
    for (int i = threadIdx.x; i < Cout; i += blockDim.x) sb[i] = __ldg(bias + i);
    const int p = threadIdx.x & 127, g = threadIdx.x >> 7;
    const int py = p / W, px = p % W;
    const int c0 = g * BAND_CG;
    const bool live = h0 + py < H;
    float v[BAND_CG], y[BAND_CG];
#pragma unroll
    for (int j = 0; j < BAND_CG; ++j) v[j] = 0.0f;
    for (int t = 0; t < T; ++t) {
        if (t == 0 || Ti != 1) {
            const int ti = Ti == 1 ? 0 : t;
            if (t > 0) __syncthreads();               // previous step done with sx
            for (int i = threadIdx.x; i < Cin * PH * PW; i += blockDim.x) {
                const int ci = i / (PH * PW), rem = i % (PH * PW);
                const int ih = h0 + rem / PW - 1, iw = rem % PW - 1;
                sx[i] = (ih >= 0 && ih < H && iw >= 0 && iw < W)
                            ? __ldg(x + (((int64_t)ti * B + b) * Cin + ci) * H * W + ih * W + iw)
                            : 0.0f;
            }
            __syncthreads();
#pragma unroll
            for (int j = 0; j < BAND_CG; ++j) y[j] = 0.0f;
            for (int ci = 0; ci < Cin; ++ci) {
#pragma unroll
                for (int kh = 0; kh < 3; ++kh) {
#pragma unroll
                    for (int kw = 0; kw < 3; ++kw) {
                        const float xv = sx[(ci * PH + py + kh) * PW + px + kw];
                        const float4* wk = reinterpret_cast<const float4*>(
                            sw + (ci * 9 + kh * 3 + kw) * Cout + c0);
#pragma unroll
                        for (int q = 0; q < BAND_CG / 4; ++q) {
                            const float4 w4 = wk[q];
                            y[4 * q] = __fmaf_rn(xv, w4.x, y[4 * q]);
                            y[4 * q + 1] = __fmaf_rn(xv, w4.y, y[4 * q + 1]);
                            y[4 * q + 2] = __fmaf_rn(xv, w4.z, y[4 * q + 2]);
                            y[4 * q + 3] = __fmaf_rn(xv, w4.w, y[4 * q + 3]);
                        }
                    }
                }
            }
        }
        uint32_t bits = 0;
#pragma unroll
        for (int j = 0; j < BAND_CG; ++j) {
            const float in = __fadd_rn(y[j], sb[c0 + j]);
            float vv = charge(v[j], df, sc, in);
            const bool s = vv >= thr;
            v[j] = reset_v<HARD>(vv, s, thr, v_reset);
            bits |= (s ? 1u : 0u) << j;
        }
        if (live) {
            uint4* dst = reinterpret_cast<uint4*>(
                out + ((((int64_t)t * B + b) * H + h0 + py) * W + px) * Cout + c0);
            dst[0] = spikes_to_bf16x8(bits & 0xffu);
            dst[1] = spikes_to_bf16x8(bits >> 8);
        }
    }
}

// Quad form (no pooling, W % 4 == 0, Cout % 16 == 0): thread = 4 horizontally adjacent
// pixels x 16 output channels, so each weight read from shared memory feeds 4 pixels and
// each 6-value input row segment feeds 3 taps x 4 pixels (shared-memory instructions per
// FMA drop ~3x against one pixel per thread, which was load/store-unit bound).  Channel
// pairs go through the packed float32x2 FMA / add / mul of sm_100 (each component rounded
// as the scalar __fmaf_rn / __fadd_rn / __fmul_rn), halving the arithmetic instructions.
// With direct encoding the scaled input current sc * (conv + b) is computed once and
// reused at every step.
constexpr int QUAD_THREADS = 128;

template <bool HARD, bool DIRECT>
__global__ void __launch_bounds__(QUAD_THREADS, DIRECT ? 4 : 3) first_conv_quad_kernel(
    const float* __restrict__ x, int Ti, int T, int B, int Cin, int H, int W, int R,
    const float* __restrict__ w, const float* __restrict__ bias, int Cout,
    float df, float sc, float thr, float v_reset, __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ float smf[];
    const int K = Cin * 9;
    const int PW = W + 2, PH = R + 2;
    float* sw = smf;                                  // [K][Cout]
    float* sb = smf + K * Cout;                       // [Cout]
    // [Cin][PH][PW] pixels, each stored twice (x, x) so that one 8-byte load gives the
    // broadcast operand of a packed FMA
    float2* sx = reinterpret_cast<float2*>(sb + Cout);
    const int nb = (H + R - 1) / R;
    const int b = blockIdx.x / nb, h0 = (blockIdx.x % nb) * R;
    for (int i = threadIdx.x; i < K * Cout; i += QUAD_THREADS) {
        const int co = i % Cout, k = i / Cout;       // k = ci*9 + kh*3 + kw (torch order)
        sw[i] = __ldg(w + (int64_t)co * K + k);
    }
    for (int i = threadIdx.x; i < Cout; i += QUAD_THREADS) sb[i] = __ldg(bias + i);
    // thread = (4-pixel quad, channel group g): the Cout/16 groups of a quad are adjacent
    // lanes, and group g owns channels 8g..8g+7 and Cout/2+8g..Cout/2+8g+7, so that one
    // 16-byte spike store per lane fills whole 32-byte sectors (the quad's groups write
    // channels 0..Cout/2-1, then Cout/2..Cout-1, contiguously)
    const int quads = R * (W / 4);
    const int G = Cout / 16;
    const int g = threadIdx.x % G, qd = threadIdx.x / G;
    const int py = qd / (W / 4), px0 = 4 * (qd % (W / 4));
    const int c_lo = 8 * g, c_hi = Cout / 2 + 8 * g;
    const bool live = qd < quads && h0 + py < H;
    const float2 df2 = make_float2(df, df), sc2 = make_float2(sc, sc);
    float2 u[4][8];                                   // sc * (conv + b), channel pairs
    float2 v[4][8];
    // stage frame ti of the input and compute u = sc * (conv + b) for this thread's pixels
    auto conv = [&](int ti) {
        for (int i = threadIdx.x; i < Cin * PH * PW; i += QUAD_THREADS) {
            const int ci = i / (PH * PW), rem = i % (PH * PW);
            const int ih = h0 + rem / PW - 1, iw = rem % PW - 1;
            const float xv = (ih >= 0 && ih < H && iw >= 0 && iw < W)
                        ? __ldg(x + (((int64_t)ti * B + b) * Cin + ci) * H * W + ih * W + iw)
                        : 0.0f;
            sx[i] = make_float2(xv, xv);
        }
        __syncthreads();
        if (!live) return;
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int j = 0; j < 8; ++j) u[p][j] = make_float2(0.0f, 0.0f);
        for (int ci = 0; ci < Cin; ++ci) {
#pragma unroll
            for (int kh = 0; kh < 3; ++kh) {
                const float2* row = sx + (ci * PH + py + kh) * PW + px0;
                float2 xr[6];
#pragma unroll
                for (int e = 0; e < 6; ++e) xr[e] = row[e];
#pragma unroll
                for (int kw = 0; kw < 3; ++kw) {
                    const float* wrow = sw + (ci * 9 + kh * 3 + kw) * Cout;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float4 w4 = *reinterpret_cast<const float4*>(
                            wrow + (q < 2 ? c_lo + 4 * q : c_hi + 4 * (q - 2)));
                        const float2 wlo = make_float2(w4.x, w4.y);
                        const float2 whi = make_float2(w4.z, w4.w);
#pragma unroll
                        for (int p = 0; p < 4; ++p) {
                            u[p][2 * q] = __ffma2_rn(xr[p + kw], wlo, u[p][2 * q]);
                            u[p][2 * q + 1] = __ffma2_rn(xr[p + kw], whi, u[p][2 * q + 1]);
                        }
                    }
                }
            }
        }
        const float2* b2lo = reinterpret_cast<const float2*>(sb + c_lo);
        const float2* b2hi = reinterpret_cast<const float2*>(sb + c_hi);
#pragma unroll
        for (int p = 0; p < 4; ++p)
#pragma unroll
            for (int j = 0; j < 8; ++j)
                u[p][j] = __fmul2_rn(sc2, __fadd2_rn(u[p][j], j < 4 ? b2lo[j] : b2hi[j - 4]));
    };
    // one LIF step of this thread's 64 neurons and the spike stores of frame t
    auto lif = [&](int t) {
        if (!live) return;
        __nv_bfloat16* dst = out + ((((int64_t)t * B + b) * H + h0 + py) * W + px0) * Cout;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            uint32_t bits = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                // v = df * v + sc * in, each product and the sum rounded separately
                const float2 vv = __fadd2_rn(__fmul2_rn(df2, v[p][j]), u[p][j]);
                const bool s0 = vv.x >= thr, s1 = vv.y >= thr;
                v[p][j] = make_float2(reset_v<HARD>(vv.x, s0, thr, v_reset),
                                      reset_v<HARD>(vv.y, s1, thr, v_reset));
                bits |= (s0 ? 1u : 0u) << (2 * j);
                bits |= (s1 ? 1u : 0u) << (2 * j + 1);
            }
            *reinterpret_cast<uint4*>(dst + p * Cout + c_lo) = spikes_to_bf16x8(bits & 0xffu);
            *reinterpret_cast<uint4*>(dst + p * Cout + c_hi) = spikes_to_bf16x8(bits >> 8);
        }
    };
    if (DIRECT) {
        // one input frame for every step: each pixel's 16 neurons run their whole T
        // recurrence at once (v for 16 neurons live, not 64: the kernel fits 4 CTAs per SM)
        // and each (pixel, step) leaves as two 16-byte stores
        conv(0);
        if (!live) return;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            float2 vp[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) vp[j] = make_float2(0.0f, 0.0f);
            for (int t = 0; t < T; ++t) {
                uint32_t bits = 0;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float2 vv = __fadd2_rn(__fmul2_rn(df2, vp[j]), u[p][j]);
                    const bool s0 = vv.x >= thr, s1 = vv.y >= thr;
                    vp[j] = make_float2(reset_v<HARD>(vv.x, s0, thr, v_reset),
                                        reset_v<HARD>(vv.y, s1, thr, v_reset));
                    bits |= ((s0 ? 1u : 0u) | (s1 ? 2u : 0u)) << (2 * j);
                }
                __nv_bfloat16* dst =
                    out + ((((int64_t)t * B + b) * H + h0 + py) * W + px0 + p) * Cout;
                *reinterpret_cast<uint4*>(dst + c_lo) = spikes_to_bf16x8(bits & 0xffu);
                *reinterpret_cast<uint4*>(dst + c_hi) = spikes_to_bf16x8(bits >> 8);
            }
        }
        return;
    }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[p][j] = make_float2(0.0f, 0.0f);
    for (int t = 0; t < T; ++t) {
        if (!DIRECT) {
            if (t > 0) __syncthreads();               // previous step done with sx
            conv(t);
        }
        lif(t);
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
    if (const int inj = snnb::take_injected_status()) return inj;
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
    if (!pool && W % 4 == 0 && W <= 4 * QUAD_THREADS && Cout % 16 == 0 && Cin <= 16) {
        // rows per CTA so that R x (W/4) quads x (Cout/16) groups fill the CTA
        const int per_row = (int)(W / 4) * (int)(Cout / 16);
        const int R = per_row <= QUAD_THREADS ? QUAD_THREADS / per_row : 0;
        const int64_t nblk = B * ((H + (R ? R : 1) - 1) / (R ? R : 1));
        const int64_t qsmem = (9 * Cin * Cout + Cout + 2 * Cin * (R + 2) * (W + 2)) * 4;
        if (R >= 1 && nblk <= 0x7fffffffll && qsmem <= 64 * 1024) {
            auto quad = [&](auto kernel) -> int {
                cudaError_t e = cudaFuncSetAttribute(
                    kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)qsmem);
                if (e != cudaSuccess) return record_cuda_error(e);
                return launch_k(kernel, dim3((unsigned)nblk), dim3(QUAD_THREADS), qsmem, s, x,
                                (int)Ti, (int)T, (int)B, (int)Cin, (int)H, (int)W, R, w, bias,
                                (int)Cout, decay, input_scale, v_threshold, v_reset, o);
            };
            if (Ti == 1)
                return hard_reset ? quad(first_conv_quad_kernel<true, true>)
                                  : quad(first_conv_quad_kernel<false, true>);
            return hard_reset ? quad(first_conv_quad_kernel<true, false>)
                              : quad(first_conv_quad_kernel<false, false>);
        }
    }
    if (!pool && W >= 8 && W <= 128 && 128 % W == 0 && Cout % BAND_CG == 0 && Cout <= 128 &&
        Cin <= 16) {
        const int R = 128 / (int)W;
        const int64_t nblk = B * ((H + R - 1) / R);
        const int64_t bsmem = (9 * Cin * Cout + Cout + Cin * (R + 2) * (W + 2)) * 4;
        if (nblk <= 0x7fffffffll && bsmem <= 200 * 1024) {
            const int threads = 128 * (int)(Cout / BAND_CG);
            auto band = [&](auto kernel) -> int {
                cudaError_t e = cudaFuncSetAttribute(
                    kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bsmem);
                if (e != cudaSuccess) return record_cuda_error(e);
                return launch_k(kernel, dim3((unsigned)nblk), dim3(threads), bsmem, s, x, (int)Ti,
                                (int)T, (int)B, (int)Cin, (int)H, (int)W, w, bias, (int)Cout,
                                decay, input_scale, v_threshold, v_reset, o);
            };
            return hard_reset ? band(first_conv_band_kernel<true>)
                              : band(first_conv_band_kernel<false>);
        }
    }
    auto run = [&](auto kernel) -> int {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return record_cuda_error(e);
        return launch_k(kernel, dim3((unsigned)blocks), dim3(THREADS), smem, s, x, (int)Ti, (int)T,
                        (int)B, (int)Cin, (int)H, (int)W, w, bias, (int)Cout, decay, input_scale,
                        v_threshold, v_reset, o);
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
