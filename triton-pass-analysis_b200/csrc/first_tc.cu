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
// The kernel is persistent (one CTA per SM) and walks 128-pixel tiles (flattened b, h, w)
// with two stages, each an A tile in shared memory and an accumulator [128 x Cout] in TMEM:
//   - the CTA copies the split weights [Cout][KP] (host-prepared) into shared memory once;
//   - warps 0-3 build the A tile of their next tile -- thread = pixel: the K0 input values of
//     its 3x3 window (zeros outside the image; the loads are issued before the wait for a
//     free stage), split into terms and written as 16-byte chunks in the 128-byte-swizzled
//     K-major layout the MMA descriptor reads -- and warp 0's elected lane issues KP / 16
//     MMAs (M = 128, N = Cout, K = 16) into the stage's accumulator and commits them to the
//     stage's full barrier;
//   - warps 4-11 (TMEM lane quadrant = warp % 4, two sets taking alternate 32-channel
//     slices) run bias + the T steps of the neuron from the accumulator, storing each step's
//     spikes as bf16 (a pixel pair's lanes split the stores so that every instruction writes
//     whole 32-byte sectors), then free the stage on its empty barrier.
// So one tile's neuron steps and stores overlap the next tile's loads, split and MMAs.
#include "tc_common.cuh"

namespace snnb {

int sm_count();

namespace {

constexpr int FT_THREADS = 384;     // warps 0-3 build A / issue MMAs, 4-11 run the neuron
constexpr int FT_STAGES = 2;

template <int CIN, int KP, int COUT>
struct FirstTcSmem {
    static constexpr int K0 = 9 * CIN;
    static constexpr int SLABS = KP / 64;
    static constexpr int A_SLAB = 128 * 128;             // 128 rows x 128 bytes
    static constexpr int A_STAGE = SLABS * A_SLAB;
    static constexpr int B_SLAB = COUT * 128;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = FT_STAGES * A_STAGE;
    static constexpr int BAR_OFF = B_OFF + SLABS * B_SLAB;  // full[FT_STAGES], empty[FT_STAGES]
    static constexpr int TMEM_OFF = BAR_OFF + 16 * FT_STAGES;
    static constexpr int TOTAL = TMEM_OFF + 8;
    static constexpr int DYN = TOTAL + 1024;              // slack for 1024-byte alignment
    static constexpr uint32_t ACC_COLS = COUT < 32 ? 32 : COUT;
    static constexpr uint32_t TMEM_COLS = FT_STAGES * ACC_COLS;
};

// Byte offset of 16-byte chunk c (K elements 8c .. 8c+7) of row r in a K-major operand of
// 64-element slabs stored with the 128-byte swizzle (slab_bytes per slab).
__device__ __forceinline__ uint32_t sw128_chunk(int r, int c, int slab_bytes) {
    const int slab = c >> 3, cc = c & 7;
    return (uint32_t)(slab * slab_bytes + r * 128 + ((cc ^ (r & 7)) << 4));
}

// The 3x3 window of pixel `pix` over CIN channels in torch's weight order (ci, ky, kx);
// zeros outside the image and for pixels past the end.
template <int CIN, typename I>
__device__ __forceinline__ void load_window(const float* __restrict__ x, int64_t pix,
                                            int64_t npix, int H, int W, float (&a)[9 * CIN]) {
    const bool inside = pix < npix;
    const I pp = inside ? (I)pix : (I)0;
    const int w0 = (int)(pp % (I)W);
    const int h0 = (int)((pp / (I)W) % (I)H);
    const int64_t b0 = (int64_t)(pp / ((I)W * (I)H));
#pragma unroll
    for (int ci = 0; ci < CIN; ++ci) {
        const float* plane = x + (b0 * CIN + ci) * (int64_t)H * W;
#pragma unroll
        for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
            for (int kx = 0; kx < 3; ++kx) {
                const int hh = h0 + ky - 1, ww = w0 + kx - 1;
                const bool ok = inside && hh >= 0 && hh < H && ww >= 0 && ww < W;
                a[ci * 9 + ky * 3 + kx] = ok ? __ldg(plane + (int64_t)hh * W + ww) : 0.0f;
            }
        }
    }
}

template <int CIN, int KP, int COUT, bool HARD>
__global__ void __launch_bounds__(FT_THREADS, 1)
first_conv_tc_kernel(const float* __restrict__ x, int T, int B, int H, int W,
                     const __nv_bfloat16* __restrict__ wsplit, const float* __restrict__ bias,
                     float df, float sc, float thr, float v_reset,
                     __nv_bfloat16* __restrict__ out, int* status) {
    using S = FirstTcSmem<CIN, KP, COUT>;
    constexpr int K0 = S::K0;
    static_assert(6 * K0 <= KP && KP % 64 == 0, "K layout");
    static_assert(S::DYN <= 227 * 1024, "shared memory");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    const uint32_t full0 = sbase + S::BAR_OFF;             // + 8 * stage
    const uint32_t empty0 = full0 + 8 * FT_STAGES;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + S::TMEM_OFF);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
#pragma unroll
        for (int s = 0; s < FT_STAGES; ++s) {
            tc::mbar_init(full0 + 8 * s, 1);
            tc::mbar_init(empty0 + 8 * s, 8);             // one arrival per neuron warp
        }
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(sbase + S::TMEM_OFF, S::TMEM_COLS);
        tc::tmem_relinquish();
    }
    {
        // weights: [COUT][KP] bf16 rows -> swizzled B slabs, once per CTA (no kernel writes
        // them: before the dependency wait)
        constexpr int BCH = COUT * (KP / 8);              // 16-byte chunks
        for (int i = tid; i < BCH; i += FT_THREADS) {
            const int r = i / (KP / 8), c = i - r * (KP / 8);
            const uint4 v = __ldg(reinterpret_cast<const uint4*>(wsplit) + i);
            *reinterpret_cast<uint4*>(smem + S::B_OFF + sw128_chunk(r, c, S::B_SLAB)) = v;
        }
    }
    tc::fence_proxy_async_smem();                          // generic writes -> tensor core
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();                                           // the image is the stream's input
    pdl_trigger();

    const int64_t npix = (int64_t)B * H * W;
    const int64_t ntiles = (npix + 127) / 128;
    const bool narrow = npix < 0x7fffffffll;

    if (warp < 4) {
        // ---- A builders; warp 0's elected lane issues the MMAs ----
        uint32_t failed = 0, committed = 0, last_bar = 0, last_par = 0;
        int i = 0;
        for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
            const int s = i % FT_STAGES;
            const uint32_t u = (uint32_t)(i / FT_STAGES);
            float a[K0];
            if (narrow) load_window<CIN, uint32_t>(x, tile * 128 + tid, npix, H, W, a);
            else load_window<CIN, int64_t>(x, tile * 128 + tid, npix, H, W, a);
            // stage s's A tile is free once the MMAs of local tile i - FT_STAGES completed
            // (they read only this CTA's shared memory: the drain limit)
            if (i >= FT_STAGES && !tc::mbar_wait_warp<true>(full0 + 8 * s, (u - 1) & 1, failed))
                failed = 1;
            uint16_t th[K0], tm[K0], tl[K0];
#pragma unroll
            for (int j = 0; j < K0; ++j) {
                __nv_bfloat16 hb, mb, lb;
                split_bf16x3(a[j], hb, mb, lb);
                th[j] = __bfloat16_as_ushort(hb);
                tm[j] = __bfloat16_as_ushort(mb);
                tl[j] = __bfloat16_as_ushort(lb);
            }
            // K element k: group g = k / K0 (terms hi, hi, hi, mid, mid, lo), value k % K0;
            // zero past 6 * K0.  Compile-time indices: the chunks are register moves.
            auto elem = [&](int k) -> uint32_t {
                if (k >= 6 * K0) return 0u;
                const int g = k / K0, j = k - g * K0;
                return g < 3 ? th[j] : (g < 5 ? tm[j] : tl[j]);
            };
            if (!failed) {
                uint8_t* as = smem + S::A_OFF + s * S::A_STAGE;
#pragma unroll
                for (int c = 0; c < KP / 8; ++c) {
                    uint4 v;
                    v.x = elem(8 * c + 0) | (elem(8 * c + 1) << 16);
                    v.y = elem(8 * c + 2) | (elem(8 * c + 3) << 16);
                    v.z = elem(8 * c + 4) | (elem(8 * c + 5) << 16);
                    v.w = elem(8 * c + 6) | (elem(8 * c + 7) << 16);
                    *reinterpret_cast<uint4*>(as + sw128_chunk(tid, c, S::A_SLAB)) = v;
                }
            }
            tc::fence_proxy_async_smem();
            if (tc::named_bar_any(1, 128, failed != 0)) {
                failed = 1;
                break;
            }
            if (warp == 0) {
                // stage s's accumulator is free once the neuron warps have read local tile
                // i - FT_STAGES
                if (i >= FT_STAGES && !tc::mbar_wait_warp(empty0 + 8 * s, (u - 1) & 1, 0)) {
                    failed = 1;                           // the builders abort at the next tile
                } else {
                    tc::tc_fence_after();
                    if (lane == 0) {
                        constexpr uint32_t IDESC = tc::idesc_bf16_f32(128, COUT);
                        constexpr int KSTEPS = (6 * K0 + 15) / 16;   // past 6 * K0: all zero
                        const uint32_t acc = tmem + (uint32_t)s * S::ACC_COLS;
                        const uint32_t abase = sbase + S::A_OFF + s * S::A_STAGE;
#pragma unroll
                        for (int ks = 0; ks < KSTEPS; ++ks) {
                            const int slab = ks >> 2, k = ks & 3;
                            const uint64_t da = tc::sdesc_k_sw128(abase + slab * S::A_SLAB);
                            const uint64_t db = tc::sdesc_k_sw128(sbase + S::B_OFF + slab * S::B_SLAB);
                            tc::umma_bf16(acc, da + 2 * k, db + 2 * k, IDESC, ks != 0);
                        }
                        tc::umma_commit(full0 + 8 * s);
                    }
                    __syncwarp();
                    committed = 1;
                    last_bar = full0 + 8 * s;
                    last_par = u & 1;
                }
            }
        }
        // the MMAs still in flight (only after an abort) finish before TMEM is freed
        if (warp == 0 && committed) tc::mbar_wait_warp<true>(last_bar, last_par, 0);
        if (failed && lane == 0) atomicExch(status, SNNB_ERR_TIMEOUT);
    } else {
        // ---- neuron warps: TMEM lane quadrant warp % 4, channel slices set, set + 2, ... ----
        const int q = warp & 3, set = (warp - 4) >> 2;
        const int64_t step_stride = npix * COUT;
        const float2 df2 = make_float2(df, df), sc2 = make_float2(sc, sc);
        uint32_t failed = 0;
        int i = 0;
        for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
            const int s = i % FT_STAGES;
            const uint32_t u = (uint32_t)(i / FT_STAGES);
            if (!tc::mbar_wait_warp(full0 + 8 * s, u & 1, failed)) {
                failed = 1;
                break;
            }
            tc::tc_fence_after();
            const int64_t pix = tile * 128 + 32 * q + lane;
            const uint32_t tacc = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)s * S::ACC_COLS;
#pragma unroll 1
            for (int c = set; c < COUT / 32; c += 2) {
                float r[32];
                tc::tmem_ld32(tacc + c * 32, r);
                float2 bb[16];
                const float4* b4 = reinterpret_cast<const float4*>(bias + c * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 f = __ldg(b4 + j);
                    bb[2 * j] = make_float2(f.x, f.y);
                    bb[2 * j + 1] = make_float2(f.z, f.w);
                }
                tc::tmem_wait_ld();
                // direct encoding: the input current, and its scaled form, is the same at
                // every step (sc * in rounded once, as the charge rounds it every step);
                // packed f32x2 operations round each component as the scalar ones do
                float2 sin2[16], v2[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    sin2[j] = __fmul2_rn(sc2, __fadd2_rn(make_float2(r[2 * j], r[2 * j + 1]), bb[j]));
                    v2[j] = make_float2(0.0f, 0.0f);
                }
                // the lanes of pixels 2i and 2i + 1 store both pixels' 64 bytes: the even lane
                // the 16-byte chunks 0 and 2, the odd one 1 and 3
                const int par = lane & 1;
                const int64_t pbase = pix & ~(int64_t)1;
                const bool pair_in = pbase < npix;
                __nv_bfloat16* dst = out + pbase * COUT + c * 32;
                for (int t = 0; t < T; ++t) {
                    uint32_t mask = 0;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float2 vv = __fadd2_rn(__fmul2_rn(df2, v2[j]), sin2[j]);  // charge()
                        const bool s0 = vv.x >= thr, s1 = vv.y >= thr;
                        v2[j] = make_float2(reset_v<HARD>(vv.x, s0, thr, v_reset),
                                            reset_v<HARD>(vv.y, s1, thr, v_reset));
                        mask |= (s0 ? 1u : 0u) << (2 * j);
                        mask |= (s1 ? 1u : 0u) << (2 * j + 1);
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
                            for (int h = 0; h < 2; ++h) {
                                const int qq = 2 * h + par;
                                d[qq] = spikes_to_bf16x8((mm >> (8 * qq)) & 0xffu);
                            }
                        }
                    }
                }
            }
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(empty0 + 8 * s);
        }
        if (failed && lane == 0) atomicExch(status, SNNB_ERR_TIMEOUT);
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
        const int64_t grid = tiles < sm_count() ? tiles : sm_count();
        return launch_k(kernel, dim3((unsigned)grid), dim3(FT_THREADS), S::DYN, s, x, T, B, H,
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
