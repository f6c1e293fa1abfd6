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
// weight groups [hi, mid, lo, hi, mid, hi], each group the K0 = 9 * Cin values in torch's
// weight order (ci, ky, kx) padded with a zero to an even width G (so that value pairs are
// 32-bit words of the operand), zero-padded to KP (a multiple of 64).  Every product is
// exact in float32 and the dropped ones are below 2^-23 of it, so the sums are
// float32-accurate.
//
// The kernel is persistent (one CTA per SM) and walks 128-pixel tiles (flattened b, h, w)
// with two stages, each an A tile in shared memory and an accumulator [128 x Cout] in TMEM:
//   - the split weights [Cout][KP] (host-prepared) come into shared memory once per CTA, by
//     TMA, before the dependency wait;
//   - warps 0-3 build the A tile of their next tile -- thread = pixel: the K0 input values of
//     its 3x3 window (zeros outside the image; the loads are issued before the wait for a
//     free stage), split into terms two values at a time (bf16x2 conversions) and written as
//     16-byte chunks in the 128-byte-swizzled K-major layout the MMA descriptor reads;
//   - warp 12's elected lane, once a stage's A tile is written and its accumulator free,
//     issues the MMAs (M = 128, N = Cout, K = 16) into it and commits them to the stage's
//     full barrier (a warp of its own: the builders go on to their next tile at once);
//   - warps 4-11 (TMEM lane quadrant = warp % 4, two sets taking the two 32-channel
//     halves of each 64-channel panel) read the accumulator, free the stage on its empty
//     barrier and run bias + the T steps of the neuron; each compare yields its spike's
//     bf16 half-word directly.  Each warp writes its own [32 pixels x 32 channels] block of
//     a step: into a 64-byte-swizzled staging buffer of its own (conflict-free 16-byte
//     shared stores, a ring of buffers) and out with a TMA tiled store issued by its lane 0
//     -- whole segments to L2 instead of per-lane sector writes, and no synchronisation
//     between warps.  Pixels past the end are clipped by the tensor map
//     ([T][pixels][Cout]).
// The builders load the next tile's windows before splitting the current one, so one tile's
// neuron steps and stores overlap the next tile's loads, split and MMAs.
#include "tc_common.cuh"

namespace snnb {

int sm_count();

namespace {

constexpr int FT_THREADS = 416;     // warps 0-3 build A, 4-11 run the neuron, 12 issues MMAs
constexpr int FT_STAGES = 2;

template <int CIN, int KP, int COUT>
struct FirstTcSmem {
    static constexpr int K0 = 9 * CIN;
    static constexpr int G = K0 + (K0 & 1);              // group width: K0 values, even
    static constexpr int SLABS = KP / 64;
    static constexpr int A_SLAB = 128 * 128;             // 128 rows x 128 bytes
    static constexpr int A_STAGE = SLABS * A_SLAB;
    static constexpr int B_SLAB = COUT * 128;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = FT_STAGES * A_STAGE;
    static constexpr int STG_BYTES = 32 * 64;            // a warp's block: 32 rows x 32 channels
    static constexpr int STG_OFF = B_OFF + SLABS * B_SLAB;
    // staging buffers per neuron warp: 4 where they fit, else 2
    static constexpr int NSTG = STG_OFF + 8 * 4 * STG_BYTES + 64 + 1024 <= 227 * 1024 ? 4 : 2;
    // barriers: full[FT_STAGES], empty[FT_STAGES], weights, afull[FT_STAGES]
    static constexpr int BAR_OFF = STG_OFF + 8 * NSTG * STG_BYTES;
    static constexpr int TMEM_OFF = BAR_OFF + 24 * FT_STAGES + 8;
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
// zeros outside the image, for pixels past the end and for the group's pad entry.
template <int CIN, typename I>
__device__ __forceinline__ void load_window(const float* __restrict__ x, int64_t pix,
                                            int64_t npix, int H, int W,
                                            float (&a)[9 * CIN + (CIN & 1)]) {
    if (CIN & 1) a[9 * CIN] = 0.0f;
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
first_conv_tc_kernel(const __grid_constant__ CUtensorMap tmO, const __grid_constant__ CUtensorMap tmW,
                     const float* __restrict__ x, int T, int B, int H, int W,
                     const __nv_bfloat16* __restrict__ wsplit, const float* __restrict__ bias,
                     float df, float sc, float thr, float v_reset,
                     __nv_bfloat16* __restrict__ out, int* status) {
    using S = FirstTcSmem<CIN, KP, COUT>;
    constexpr int G = S::G, WPG = G / 2;                  // words per group
    static_assert(6 * G <= KP && KP % 64 == 0, "K layout");
    static_assert(S::DYN <= 227 * 1024, "shared memory");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    const uint32_t full0 = sbase + S::BAR_OFF;             // + 8 * stage
    const uint32_t empty0 = full0 + 8 * FT_STAGES;
    const uint32_t wbar = full0 + 16 * FT_STAGES;          // the weights' TMA loads
    const uint32_t afull0 = wbar + 8;                       // + 8 * stage: A tile written
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + S::TMEM_OFF);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
#pragma unroll
        for (int s = 0; s < FT_STAGES; ++s) {
            tc::mbar_init(full0 + 8 * s, 1);
            tc::mbar_init(empty0 + 8 * s, 8);             // one arrival per neuron warp
            tc::mbar_init(afull0 + 8 * s, 1);             // the builders, after their barrier
        }
        tc::mbar_init(wbar, 1);
        tc::fence_mbar_init();
        // weights [COUT][KP] bf16 -> B slabs (128-byte swizzle), once per CTA; no kernel
        // writes them, so before the dependency wait
        tc::prefetch_tmap(&tmW);
        tc::prefetch_tmap(&tmO);
        tc::mbar_expect_tx(wbar, (uint32_t)(S::SLABS * S::B_SLAB));
#pragma unroll
        for (int sl = 0; sl < S::SLABS; ++sl)
            tc::tma_load_2d(sbase + S::B_OFF + sl * S::B_SLAB, &tmW, wbar, sl * 64, 0);
    }
    if (warp == 0) {
        tc::tmem_alloc(sbase + S::TMEM_OFF, S::TMEM_COLS);
        tc::tmem_relinquish();
    }
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
        // ---- A builders ----
        uint32_t failed = 0;
        auto load = [&](int64_t t, float (&v)[G]) {
            if (narrow) load_window<CIN, uint32_t>(x, t * 128 + tid, npix, H, W, v);
            else load_window<CIN, int64_t>(x, t * 128 + tid, npix, H, W, v);
        };
        float a[G];
        if ((int64_t)blockIdx.x < ntiles) load(blockIdx.x, a);
        int i = 0;
        for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
            const int s = i % FT_STAGES;
            const uint32_t u = (uint32_t)(i / FT_STAGES);
            // the next tile's window loads are in flight while this one is split and written
            float an[G];
            if (tile + gridDim.x < ntiles) load(tile + gridDim.x, an);
            // stage s's A tile is free once the MMAs of local tile i - FT_STAGES completed
            // (they read only this CTA's shared memory: the drain limit)
            if (i >= FT_STAGES && !tc::mbar_wait_warp<true>(full0 + 8 * s, (u - 1) & 1, failed))
                failed = 1;
            uint32_t wh[WPG], wm[WPG], wl[WPG];
            // one warp-uniform test per tile: the paired split without a branch per pair
            bool fast = true;
#pragma unroll
            for (int j = 0; j < G; ++j) fast &= fabsf(a[j]) <= SPLIT2_FAST_MAX;
            if (__all_sync(0xffffffffu, fast)) {
#pragma unroll
                for (int j = 0; j < WPG; ++j)
                    split2_bf16x3_finite(a[2 * j], a[2 * j + 1], wh[j], wm[j], wl[j]);
            } else {
#pragma unroll
                for (int j = 0; j < WPG; ++j)
                    split2_bf16x3(a[2 * j], a[2 * j + 1], wh[j], wm[j], wl[j]);
            }
            // 32-bit word kw of the row (K elements 2kw, 2kw + 1): group g = kw / WPG (terms
            // hi, hi, hi, mid, mid, lo), value pair kw % WPG; zero past 6 groups.
            // Compile-time indices: the chunks are register moves.
            auto word = [&](int kw) -> uint32_t {
                if (kw >= 6 * WPG) return 0u;
                const int g = kw / WPG, j = kw - g * WPG;
                return g < 3 ? wh[j] : (g < 5 ? wm[j] : wl[j]);
            };
            if (!failed) {
                uint8_t* as = smem + S::A_OFF + s * S::A_STAGE;
#pragma unroll
                for (int c = 0; c < KP / 8; ++c) {
                    const uint4 v = make_uint4(word(4 * c), word(4 * c + 1), word(4 * c + 2),
                                               word(4 * c + 3));
                    *reinterpret_cast<uint4*>(as + sw128_chunk(tid, c, S::A_SLAB)) = v;
                }
            }
            tc::fence_proxy_async_smem();
#pragma unroll
            for (int j = 0; j < G; ++j) a[j] = an[j];
            if (tc::named_bar_any(1, 128, failed != 0)) {
                failed = 1;
                break;
            }
            // A tile i is written (every builder passed the barrier): the MMA warp may read it
            if (tid == 0) tc::mbar_arrive(afull0 + 8 * s);
        }
        if (failed && lane == 0) atomicExch(status, SNNB_ERR_TIMEOUT);
    } else if (warp == 12) {
        // ---- MMA issuer: per local tile, once its A tile is written and its accumulator
        //      stage is free, KP / 16 MMAs from the elected lane, committed to full[s] ----
        uint32_t failed = 0, committed = 0, last_bar = 0, last_par = 0;
        if (!tc::mbar_wait_warp(wbar, 0, 0)) failed = 1;   // the weights
        int i = 0;
        for (int64_t tile = blockIdx.x; tile < ntiles && !failed; tile += gridDim.x, ++i) {
            const int s = i % FT_STAGES;
            const uint32_t u = (uint32_t)(i / FT_STAGES);
            if (!tc::mbar_wait_warp(afull0 + 8 * s, u & 1, failed)) failed = 1;
            // the accumulator stage is free once the neuron warps have read local tile
            // i - FT_STAGES
            if (i >= FT_STAGES && !tc::mbar_wait_warp(empty0 + 8 * s, (u - 1) & 1, failed))
                failed = 1;
            if (failed) break;
            tc::tc_fence_after();
            if (lane == 0) {
                constexpr uint32_t IDESC = tc::idesc_bf16_f32(128, COUT);
                constexpr int KSTEPS = (6 * G + 15) / 16;    // past 6 * G: all zero
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
        // the MMAs still in flight (only after an abort) finish before TMEM is freed, and the
        // weight copies before the CTA exits
        if (committed) tc::mbar_wait_warp<true>(last_bar, last_par, 0);
        tc::mbar_wait_warp<true>(wbar, 0, 0);
        if (failed && lane == 0) atomicExch(status, SNNB_ERR_TIMEOUT);
    } else {
        // ---- neuron warps: TMEM lane quadrant warp % 4, 32-channel slices set, set + 2, ...
        const int q = warp & 3, set = (warp - 4) >> 2;
        const uint32_t stg = sbase + S::STG_OFF + (uint32_t)(warp - 4) * S::NSTG * S::STG_BYTES;
        const float2 df2 = make_float2(df, df), sc2 = make_float2(sc, sc);
        constexpr int NSL = (COUT / 32 + 1) / 2;           // slices per set
        uint32_t failed = 0, unit = 0;
        int i = 0;
        for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++i) {
            const int s = i % FT_STAGES;
            const uint32_t u = (uint32_t)(i / FT_STAGES);
            if (!tc::mbar_wait_warp(full0 + 8 * s, u & 1, failed)) {
                failed = 1;
                break;
            }
            tc::tc_fence_after();
            const uint32_t tacc = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)s * S::ACC_COLS;
#pragma unroll 1
            for (int k = 0; k < NSL; ++k) {
                const int c = set + 2 * k;                // 32-channel slice
                const bool active = c < COUT / 32;        // Cout = 32: set 1 has none
                float r[32];
                if (active) tc::tmem_ld32(tacc + c * 32, r);
                float2 bb[16];
                const float4* b4 = reinterpret_cast<const float4*>(bias + (active ? c : 0) * 32);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 f = __ldg(b4 + j);
                    bb[2 * j] = make_float2(f.x, f.y);
                    bb[2 * j + 1] = make_float2(f.z, f.w);
                }
                tc::tmem_wait_ld();
                if (k == NSL - 1) {
                    // the accumulator stage is read: the MMAs of local tile i + FT_STAGES may
                    // overwrite it while these neurons run
                    tc::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) tc::mbar_arrive(empty0 + 8 * s);
                }
                if (!active) continue;
                // direct encoding: the input current, and its scaled form, is the same at
                // every step (sc * in rounded once, as the charge rounds it every step);
                // packed f32x2 operations round each component as the scalar ones do
                float2 sin2[16], v2[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    sin2[j] = __fmul2_rn(sc2, __fadd2_rn(make_float2(r[2 * j], r[2 * j + 1]), bb[j]));
                    v2[j] = make_float2(0.0f, 0.0f);
                }
                for (int t = 0; t < T; ++t, ++unit) {
                    // each compare gives its spike's bf16 half-word (1.0 = 0x3F80)
                    uint32_t wd[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float2 vv = __fadd2_rn(__fmul2_rn(df2, v2[j]), sin2[j]);  // charge()
                        const bool s0 = vv.x >= thr, s1 = vv.y >= thr;
                        v2[j] = make_float2(reset_v<HARD>(vv.x, s0, thr, v_reset),
                                            reset_v<HARD>(vv.y, s1, thr, v_reset));
                        wd[j] = (s0 ? 0x3F80u : 0u) | (s1 ? 0x3F800000u : 0u);
                    }
                    // buffer unit % NSTG was last read by the store of unit - NSTG: lane 0
                    // (which issued it) waits until at most NSTG - 1 stores still read
                    const uint32_t buf = stg + (unit % S::NSTG) * S::STG_BYTES;
                    if (lane == 0) tc::bulk_wait_group_read<S::NSTG - 1>();
                    __syncwarp();
                    // row = lane (64 bytes), 16-byte chunk j at its 64-byte-swizzle position
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint32_t dst = buf + lane * 64 + ((((uint32_t)j) ^ ((lane >> 1) & 3)) << 4);
                        asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(dst),
                                     "r"(wd[4 * j]), "r"(wd[4 * j + 1]), "r"(wd[4 * j + 2]),
                                     "r"(wd[4 * j + 3])
                                     : "memory");
                    }
                    tc::fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tc::tma_store_3d(&tmO, buf, 32 * c, (int)(tile * 128) + 32 * q, t);
                        tc::bulk_commit_group();
                    }
                }
            }
        }
        if (lane == 0) tc::bulk_wait_group<0>();          // this warp's stores are complete
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
    // output [T][B*H*W][Cout] bf16, stored as 32-channel x 32-pixel boxes of one step (int32
    // box coordinates); weights [Cout][KP] bf16 loaded as 64-element K slabs
    if ((int64_t)B * H * W > 0x7fffffffll) return SNNB_ERR_ARG;
    CUtensorMap tmo, tmw;
    {
        const uint64_t npix = (uint64_t)B * H * W;
        const uint64_t dims[3] = {(uint64_t)COUT, npix, (uint64_t)T};
        const uint64_t str[2] = {(uint64_t)COUT * 2, npix * COUT * 2};
        const uint32_t box[3] = {32, 32, 1};
        int rc = encode_tmap(&tmo, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, out, dims, str, box,
                             CU_TENSOR_MAP_SWIZZLE_64B);
        if (rc != SNNB_OK) return rc;
        const uint64_t wdims[2] = {(uint64_t)KP, (uint64_t)COUT};
        const uint64_t wstr[1] = {(uint64_t)KP * 2};
        const uint32_t wbox[2] = {64, (uint32_t)COUT};
        rc = encode_tmap(&tmw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ws, wdims, wstr, wbox,
                         CU_TENSOR_MAP_SWIZZLE_128B);
        if (rc != SNNB_OK) return rc;
    }
    auto go = [&](auto kernel) -> int {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             S::DYN);
        if (e != cudaSuccess) return record_cuda_error(e);
        const int64_t grid = tiles < sm_count() ? tiles : sm_count();
        return launch_k(kernel, dim3((unsigned)grid), dim3(FT_THREADS), S::DYN, s, tmo, tmw, x, T,
                        B, H, W, ws, bias, df, sc, thr, vr, out, status);
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
    return (6 * (9 * Cin + (Cin & 1)) + 63) / 64 * 64;
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
    if (!aligned16(w_split) || (reinterpret_cast<uintptr_t>(out) & 31) != 0) return SNNB_ERR_ARG;
    int* status = device_status_ptr();
    if (!status) return SNNB_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto* ws = static_cast<const __nv_bfloat16*>(w_split);
    auto* o = static_cast<__nv_bfloat16*>(out);
    const int hard = hard_reset ? 1 : 0;
#define SNNB_FIRST_TC(CIN, COUT)                                                                \
    if (Cin == CIN && Cout == COUT)                                                             \
        return launch_first_tc<CIN, (6 * (9 * CIN + (CIN & 1)) + 63) / 64 * 64, COUT>(         \
            x, (int)T, (int)B, (int)H, (int)W, ws, bias, decay, input_scale, v_threshold,       \
            v_reset, hard, o, status, s);
    SNNB_FIRST_TC(1, 32) SNNB_FIRST_TC(1, 64) SNNB_FIRST_TC(1, 128)
    SNNB_FIRST_TC(2, 32) SNNB_FIRST_TC(2, 64) SNNB_FIRST_TC(2, 128)
    SNNB_FIRST_TC(3, 32) SNNB_FIRST_TC(3, 64) SNNB_FIRST_TC(3, 128)
    SNNB_FIRST_TC(4, 32) SNNB_FIRST_TC(4, 64) SNNB_FIRST_TC(4, 128)
#undef SNNB_FIRST_TC
    return SNNB_ERR_UNSUPPORTED;
}
