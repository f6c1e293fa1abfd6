// First layer of a spiking CNN on the tensor cores: the real-valued image convolved in
// float32 precision by tcgen05 bf16 MMAs, then the multi-step neuron.
//
// Replaces, like first_layer.cu, the first FusedConvBNNeuron of VGGSNN
// (snn_compiler/zoo/vgg.py:88-94 -> nn/modules.py:347-357): F.conv2d(x, W') in float32 +
// fused_bias_if_lif(..., b').  Direct encoding (the same image at every step) makes the conv
// T-invariant: each pixel's Cout sums are computed once, into TMEM, and the T steps of the
// neuron run from that accumulator in registers.
//
// Precision: both operands are carried as three bf16 terms (hi, mid, lo; see split.cu) and
// the six larger products are summed: activation groups [hi, hi, hi, mid, mid, lo] against
// weight groups [hi, mid, lo, hi, mid, hi], each group K0 = 9 * Cin wide in torch's weight
// order (ci, ky, kx), zero-padded to KP (a multiple of 64).  Every product is exact in
// float32 and the dropped ones are below 2^-23 of it, so the sums are float32-accurate.
//
// A CTA owns 128 consecutive output pixels (flattened b, h, w) and all Cout channels:
//   1. its threads copy the split weights [Cout][KP] (host-prepared) into shared memory and
//      build the A tile -- thread = pixel: the K0 input values of its 3x3 window (zeros
//      outside the image), split into terms, written as 16-byte chunks in the 128-byte-
//      swizzled K-major layout the MMA descriptor reads (one 1024-byte atom per 8 rows);
//   2. one thread issues KP / 16 MMAs (M = 128, N = Cout, K = 16) and commits to an
//      mbarrier;
//   3. thread = TMEM lane = pixel: per 32-channel slice, bias + T steps of the neuron; each
//      step's 32 spikes leave as bf16 (64 bytes per pixel), a pixel pair's lanes splitting
//      the stores so that each instruction writes whole 32-byte sectors.
// Several CTAs share an SM (about 72 KB of shared memory each), so one CTA's MMA and
// stores overlap another's A build.
#include "tc_common.cuh"

namespace snnb {
namespace {

constexpr int FT_THREADS = 256;     // warps 0-3 build A, 4-7 copy the weights; all 8 run the epilogue

template <int CIN, int KP, int COUT>
struct FirstTcSmem {
    static constexpr int K0 = 9 * CIN;
    static constexpr int SLABS = KP / 64;
    static constexpr int A_SLAB = 128 * 128;             // 128 rows x 128 bytes
    static constexpr int B_SLAB = COUT * 128;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = SLABS * A_SLAB;
    static constexpr int BAR_OFF = B_OFF + SLABS * B_SLAB;
    static constexpr int TMEM_OFF = BAR_OFF + 8;
    static constexpr int TOTAL = TMEM_OFF + 8;
    static constexpr int DYN = TOTAL + 1024;              // slack for 1024-byte alignment
    static constexpr uint32_t TMEM_COLS = COUT < 32 ? 32 : COUT;
};

// Byte offset of 16-byte chunk c (K elements 8c .. 8c+7) of row r in a K-major operand of
// 64-element slabs stored with the 128-byte swizzle (slab_bytes per slab).
__device__ __forceinline__ uint32_t sw128_chunk(int r, int c, int slab_bytes) {
    const int slab = c >> 3, cc = c & 7;
    return (uint32_t)(slab * slab_bytes + r * 128 + ((cc ^ (r & 7)) << 4));
}

template <int CIN, int KP, int COUT, bool HARD>
__global__ void __launch_bounds__(FT_THREADS)
first_conv_tc_kernel(const float* __restrict__ x, int T, int B, int H, int W,
                     const __nv_bfloat16* __restrict__ wsplit, const float* __restrict__ bias,
                     float df, float sc, float thr, float v_reset,
                     __nv_bfloat16* __restrict__ out, int* status) {
    using S = FirstTcSmem<CIN, KP, COUT>;
    constexpr int K0 = S::K0;
    static_assert(6 * K0 <= KP && KP % 64 == 0, "K layout");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    const uint32_t bar = sbase + S::BAR_OFF;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + S::TMEM_OFF);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        tc::mbar_init(bar, 1);
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(sbase + S::TMEM_OFF, S::TMEM_COLS);
        tc::tmem_relinquish();
    }
    const int64_t npix = (int64_t)B * H * W;
    if (tid >= 128) {
        // weights: [COUT][KP] bf16 rows -> swizzled B slabs (no kernel writes them: before
        // the dependency wait)
        constexpr int BCH = COUT * (KP / 8);              // 16-byte chunks
        for (int i = tid - 128; i < BCH; i += 128) {
            const int r = i / (KP / 8), c = i - r * (KP / 8);
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(wsplit) + i);
            *reinterpret_cast<uint4*>(smem + S::B_OFF + sw128_chunk(r, c, S::B_SLAB)) = v;
        }
    }
    pdl_wait();                                           // the image is the stream's input
    pdl_trigger();
    if (tid < 128) {
    // A tile: this thread's pixel, its 3x3 window over CIN channels in torch order
    // (ci, ky, kx), each value split into three bf16 terms
    const int64_t pix = (int64_t)blockIdx.x * 128 + tid;
    const bool inside = pix < npix;
    uint16_t th[K0], tm[K0], tl[K0];
    {
        const int64_t pp = inside ? pix : 0;
        const int w0 = (int)(pp % W);
        const int h0 = (int)((pp / W) % H);
        const int64_t b0 = pp / ((int64_t)W * H);
#pragma unroll
        for (int ci = 0; ci < CIN; ++ci) {
            const float* plane = x + (b0 * CIN + ci) * (int64_t)H * W;
#pragma unroll
            for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const int hh = h0 + ky - 1, ww = w0 + kx - 1;
                    const bool ok = inside && hh >= 0 && hh < H && ww >= 0 && ww < W;
                    const float a = ok ? __ldg(plane + (int64_t)hh * W + ww) : 0.0f;
                    const int j = ci * 9 + ky * 3 + kx;
                    __nv_bfloat16 hb, mb, lb;
                    split_bf16x3(a, hb, mb, lb);
                    th[j] = __bfloat16_as_ushort(hb);
                    tm[j] = __bfloat16_as_ushort(mb);
                    tl[j] = __bfloat16_as_ushort(lb);
                }
            }
        }
    }
    // K element k: group g = k / K0 (terms hi, hi, hi, mid, mid, lo), value k % K0; zero
    // past 6 * K0.  Compile-time indices: the chunks are register moves.
    auto elem = [&](int k) -> uint32_t {
        if (k >= 6 * K0) return 0u;
        const int g = k / K0, j = k - g * K0;
        return g < 3 ? th[j] : (g < 5 ? tm[j] : tl[j]);
    };
#pragma unroll
    for (int c = 0; c < KP / 8; ++c) {
        uint4 v;
        v.x = elem(8 * c + 0) | (elem(8 * c + 1) << 16);
        v.y = elem(8 * c + 2) | (elem(8 * c + 3) << 16);
        v.z = elem(8 * c + 4) | (elem(8 * c + 5) << 16);
        v.w = elem(8 * c + 6) | (elem(8 * c + 7) << 16);
        *reinterpret_cast<uint4*>(smem + S::A_OFF + sw128_chunk(tid, c, S::A_SLAB)) = v;
    }
    }
    tc::fence_proxy_async_smem();                          // generic writes -> tensor core
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (tid == 0) {
        constexpr uint32_t IDESC = tc::idesc_bf16_f32(128, COUT);
        constexpr int KSTEPS = (6 * K0 + 15) / 16;        // k-steps past 6 * K0 are all zero
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ++ks) {
            const int slab = ks >> 2, k = ks & 3;
            const uint64_t da = tc::sdesc_k_sw128(sbase + S::A_OFF + slab * S::A_SLAB);
            const uint64_t db = tc::sdesc_k_sw128(sbase + S::B_OFF + slab * S::B_SLAB);
            tc::umma_bf16(tmem, da + 2 * k, db + 2 * k, IDESC, ks != 0);
        }
        tc::umma_commit(bar);
    }
    __syncwarp();
    // the MMAs read only this CTA's shared memory: they complete on their own (drain limit)
    const uint32_t ok = tc::mbar_wait_warp<true>(bar, 0, 0);
    tc::tc_fence_after();
    if (!ok) {
        if (lane == 0) atomicExch(status, SNNB_ERR_TIMEOUT);
    } else {
        // epilogue: TMEM lane = pixel row of the warp's quadrant (warp & 3); the two warp sets
        // (warp >> 2) take alternate 32-channel slices
        const int q = warp & 3;
        const int64_t pix = (int64_t)blockIdx.x * 128 + 32 * q + lane;
        const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16);
        const int64_t step_stride = npix * COUT;
#pragma unroll 1
        for (int c = warp >> 2; c < COUT / 32; c += 2) {
            float r[32];
            tc::tmem_ld32(tbase + c * 32, r);
            float bb[32];
            const float4* b4 = reinterpret_cast<const float4*>(bias + c * 32);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float4 f = __ldg(b4 + j);
                bb[4 * j] = f.x; bb[4 * j + 1] = f.y; bb[4 * j + 2] = f.z; bb[4 * j + 3] = f.w;
            }
            tc::tmem_wait_ld();
            // direct encoding: the input current, and its scaled form, is the same at every
            // step (sc * in rounded once, as the charge rounds it every step)
            float sin_[32], v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                sin_[j] = __fmul_rn(sc, __fadd_rn(r[j], bb[j]));
                v[j] = 0.0f;
            }
            // the lanes of pixels 2i and 2i + 1 store both pixels' 64 bytes: the even lane the
            // 16-byte chunks 0 and 2, the odd one 1 and 3, so that every store instruction
            // fills whole 32-byte sectors (a lane storing its own pixel alone wrote half
            // sectors)
            const int par = lane & 1;
            const int64_t pbase = pix & ~(int64_t)1;
            const bool pair_in = pbase < npix;
            __nv_bfloat16* dst = out + pbase * COUT + c * 32;
            for (int t = 0; t < T; ++t) {
                uint32_t mask = 0;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    float vv = __fadd_rn(__fmul_rn(df, v[j]), sin_[j]);   // charge()
                    const bool s = vv >= thr;
                    v[j] = reset_v<HARD>(vv, s, thr, v_reset);
                    mask |= (s ? 1u : 0u) << j;
                }
                const uint32_t other = __shfl_xor_sync(0xffffffffu, mask, 1);
                if (pair_in) {
                    __nv_bfloat16* d0 = dst + (int64_t)t * step_stride;
#pragma unroll
                    for (int pi = 0; pi < 2; ++pi) {
                        if (pbase + pi >= npix) continue;
                        if (!SNNB_IN_BOUNDS((int64_t)t * step_stride + (pbase + pi) * COUT + c * 32 + 31,
                                            (int64_t)T * step_stride, status))
                            continue;
                        const uint32_t mm = pi == par ? mask : other;
                        uint4* d = reinterpret_cast<uint4*>(d0 + pi * COUT);
#pragma unroll
                        for (int i = 0; i < 2; ++i) {
                            const int q = 2 * i + par;
                            d[q] = spikes_to_bf16x8((mm >> (8 * q)) & 0xffu);
                        }
                    }
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, S::TMEM_COLS);
    }
}

template <int CIN, int KP, int COUT>
int launch_first_tc(const float* x, int T, int B, int H, int W, const __nv_bfloat16* ws,
                    const float* bias, float df, float sc, float thr, float vr, int hard,
                    __nv_bfloat16* out, int* status, cudaStream_t s) {
    using S = FirstTcSmem<CIN, KP, COUT>;
    const int64_t tiles = ((int64_t)B * H * W + 127) / 128;
    if (tiles > 0x7fffffffll) return SNNB_ERR_ARG;
    auto go = [&](auto kernel) -> int {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             S::DYN);
        if (e != cudaSuccess) return record_cuda_error(e);
        return launch_k(kernel, dim3((unsigned)tiles), dim3(FT_THREADS), S::DYN, s, x, T, B, H,
                        W, ws, bias, df, sc, thr, vr, out, status);
    };
    return hard ? go(first_conv_tc_kernel<CIN, KP, COUT, true>)
                : go(first_conv_tc_kernel<CIN, KP, COUT, false>);
}

}  // namespace

int* device_status_ptr();

}  // namespace snnb

using namespace snnb;

extern "C" int64_t snnb_first_conv_tc_weight_k(int64_t Cin) {
    if (Cin < 1 || Cin > 4) return -1;
    return (6 * 9 * Cin + 63) / 64 * 64;
}

extern "C" int snnb_first_conv_lif_tc(const float* x, int64_t T, int64_t B, int64_t Cin,
                                      int64_t H, int64_t W, const void* w_split,
                                      const float* bias, int64_t Cout, float decay,
                                      float input_scale, float v_threshold, float v_reset,
                                      int hard_reset, void* out, snnb_stream_t stream) {
    if (const int inj = take_injected_status()) return inj;
    if (!x || !w_split || !bias || !out) return SNNB_ERR_ARG;
    if (T <= 0 || B <= 0 || H <= 0 || W <= 0 || T > 0x7fffffff) return SNNB_ERR_ARG;
    if (H > 0x7fffffff || W > 0x7fffffff || B > 0x7fffffff) return SNNB_ERR_ARG;
    if ((int64_t)B * H * W > ((int64_t)1 << 40) / (T * (Cout > 0 ? Cout : 1)))
        return SNNB_ERR_ARG;
    if (!aligned16(w_split) || !aligned16(out)) return SNNB_ERR_ARG;
    int* status = device_status_ptr();
    if (!status) return SNNB_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto* ws = static_cast<const __nv_bfloat16*>(w_split);
    auto* o = static_cast<__nv_bfloat16*>(out);
    const int hard = hard_reset ? 1 : 0;
#define SNNB_FIRST_TC(CIN, COUT)                                                                \
    if (Cin == CIN && Cout == COUT)                                                             \
        return launch_first_tc<CIN, (6 * 9 * CIN + 63) / 64 * 64, COUT>(                        \
            x, (int)T, (int)B, (int)H, (int)W, ws, bias, decay, input_scale, v_threshold,       \
            v_reset, hard, o, status, s);
    SNNB_FIRST_TC(1, 32) SNNB_FIRST_TC(1, 64) SNNB_FIRST_TC(1, 128)
    SNNB_FIRST_TC(2, 32) SNNB_FIRST_TC(2, 64) SNNB_FIRST_TC(2, 128)
    SNNB_FIRST_TC(3, 32) SNNB_FIRST_TC(3, 64) SNNB_FIRST_TC(3, 128)
    SNNB_FIRST_TC(4, 32) SNNB_FIRST_TC(4, 64) SNNB_FIRST_TC(4, 128)
#undef SNNB_FIRST_TC
    return SNNB_ERR_UNSUPPORTED;
}
