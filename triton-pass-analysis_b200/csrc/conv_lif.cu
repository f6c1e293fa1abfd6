// K1 -- fused implicit-GEMM conv3x3 (or linear) + folded-BN bias + multi-step LIF
//       (+ 2x2 max-pool) on the 5th-generation tensor cores.
//
// Replaces, per layer, the reference's F.conv2d / F.linear library call followed by
// _bias_if_lif_kernel (snn_compiler/nn/modules.py:324-357 -> kernels/fused.py:50-114)
// and the ATen max-pool (snn_compiler/zoo/vgg.py:100-104); the fused-pool precedent is
// the AvgPool epilogue prototype snn_compiler/explore/large_T/pool_epilogue_proto.py:40-130,
// here with max-pool, which on {0,1} spikes is an OR of the 2x2 window.
//
// GEMM view per time step t: M = output pixels, N = output channels, K = taps * Cin,
// with activations NHWC bf16 [T*B, H, W, Cin] (frame f = t*B + b) and folded weights
// bf16 [Cout, taps, Cin] (K-major).  One CTA owns a 128-pixel block (bn images x bh
// rows x bw columns, 2x2-aligned so pooling windows stay inside) and BN channels,
// and walks t = 0..T-1 itself, so the membrane potential never leaves registers.
//
// Warp roles (192 threads):
//   warp 0  TMA producer: for each (t, tap, 64-channel slab) one 4-D tiled load of the
//           activation box at (c0, w0+s-1, h0+r-1, f0) -- the conv halo and padding come
//           from the hardware's zero fill of out-of-range coordinates -- and one 2-D load
//           of the weight slab, into a STAGES-deep ring (128-byte swizzle).
//   warp 1  MMA issuer: allocates 2*BN TMEM columns (two accumulators), issues
//           tcgen05.mma kind::f16 (M=128, N=BN, K=16) x4 per slab, frees ring slots with
//           tcgen05.commit, and signals "accumulator t ready"; accumulator t+1 fills
//           while the epilogue drains t.
//   warps 2-5  epilogue: thread = TMEM lane = pixel; tcgen05.ld 32 columns at a time,
//           v = decay*v + scale*(acc + bias) (float32, no FMA contraction), threshold,
//           reset, spike bits into shared memory; then (optionally pooled) bf16 spikes
//           NHWC stored with 16-byte writes.  Only spikes reach HBM.
// Every mbarrier wait is bounded; on timeout the CTA records SNNB_ERR_TIMEOUT, drains
// its in-flight copies, frees its TMEM and returns.
#include <mutex>
#include <type_traits>

#include "conv_tm.cuh"

namespace snnb {

__device__ int g_device_status = 0;

namespace {

// Producer drain after a failed wait: wait (bounded, whole warp) for the copies still in
// flight -- the last min(stages, issued) stages before ring position (stage, phase).
__device__ __forceinline__ void drain_ring_warp(uint32_t bar0, int stages, int stage,
                                                uint32_t phase, uint32_t issued) {
    for (uint32_t k = 0; k < (uint32_t)stages && k < issued; ++k) {
        if (--stage < 0) { stage = stages - 1; phase ^= 1u; }
        tc::mbar_wait_warp<true>(bar0 + 8u * stage, phase, 0);
    }
}

// Spikes of one (step, pixel) of a pixel block, stored by the thread that owns the pixel
// (TMEM lane m; the block is bn images x bh rows x bw columns, row-major): unpooled, its BN
// channels as 16-byte stores; pooled, the 2x2 OR formed with shuffles (column pairs are
// adjacent lanes, row pairs lanes bw apart when bw < 32) or through shared memory (row pair
// in another warp), stored by the window's top-left thread.  Every epilogue thread calls it
// (shuffles, barrier); `sm` is this step's half of the double-buffered exchange area.
template <int NCH>
__device__ __forceinline__ void store_pixel(const ConvParams& p, const Tile& tl, int t, int m,
                                            uint32_t (&mk)[NCH], uint32_t* sm) {
    const int x = m % p.bw, y = (m / p.bw) % p.bh, n = m / (p.bw * p.bh);
    const int ow = tl.w0 + x, oh = tl.h0 + y, on = tl.img0 + n;
    const bool inside = ow < p.W && oh < p.H && on < p.B;
    const int64_t frame = (int64_t)t * p.B + on;
    if (!p.pool) {
        if (inside) {
            uint4* dst = reinterpret_cast<uint4*>(p.out + ((frame * p.H + oh) * p.W + ow) * p.Cout + tl.n0);
#pragma unroll
            for (int c = 0; c < NCH; ++c)
#pragma unroll
                for (int k = 0; k < 4; ++k) dst[c * 4 + k] = spikes_to_bf16x8((mk[c] >> (8 * k)) & 0xffu);
        }
        return;
    }
#pragma unroll
    for (int c = 0; c < NCH; ++c) mk[c] |= __shfl_xor_sync(0xffffffffu, mk[c], 1);
    if (p.bw < 32) {
#pragma unroll
        for (int c = 0; c < NCH; ++c) mk[c] |= __shfl_xor_sync(0xffffffffu, mk[c], p.bw);
    } else {
#pragma unroll
        for (int c = 0; c < NCH; ++c) sm[c * 128 + m] = mk[c];
        tc::named_bar_sync(1, 128);
#pragma unroll
        for (int c = 0; c < NCH; ++c) mk[c] |= sm[c * 128 + (m ^ p.bw)];
    }
    if (((x | y) & 1) == 0 && inside) {
        const int Ho = p.H / 2, Wo = p.W / 2;
        uint4* dst = reinterpret_cast<uint4*>(p.out + ((frame * Ho + oh / 2) * Wo + ow / 2) * p.Cout + tl.n0);
#pragma unroll
        for (int c = 0; c < NCH; ++c)
#pragma unroll
            for (int k = 0; k < 4; ++k) dst[c * 4 + k] = spikes_to_bf16x8((mk[c] >> (8 * k)) & 0xffu);
    }
}

// LIF over one 32-column slice of a thread's accumulator row: v = decay*v + scale*(acc + b),
// threshold, reset; returns the spike bits.
template <bool HARD>
__device__ __forceinline__ uint32_t lif_slice(const float (&r)[32], const float* bias, float* v,
                                              const ConvParams& p) {
    uint32_t mask = 0;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
        const float in = __fadd_rn(r[j], bias[j]);
        float vv = charge(v[j], p.df, p.sc, in);
        const bool s = vv >= p.thr;
        v[j] = reset_v<HARD>(vv, s, p.thr, p.v_reset);
        mask |= (s ? 1u : 0u) << j;
    }
    return mask;
}

// ---- variant 1: T sequential inside the CTA ---------------------------------------------
// Persistent: CTA c handles tiles c, c + gridDim.x, ...  Every (tile, step) is one
// accumulation into one of two TMEM accumulators used alternately, so the epilogue of
// step i (LIF + stores) overlaps the MMAs of step i + 1 -- across tile boundaries too.
// Producer and MMA roles are whole warps that wait together (mbar_wait_warp) and issue
// from one elected lane; a failed wait follows the protocol of the band kernel below.
template <int BN, int STAGES>
struct Smem {
    static constexpr int B_TILE = BN * 128;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = STAGES * A_TILE_BYTES;
    static constexpr int MASK_OFF = B_OFF + STAGES * B_TILE;          // 2 x (BN/32) x 128 u32
    static constexpr int BAR_OFF = MASK_OFF + 2 * (BN / 32) * 128 * 4;
    static constexpr int NBARS = 2 * STAGES + 5;
    static constexpr int TMEM_OFF = BAR_OFF + NBARS * 8;
    static constexpr int ABORT_OFF = TMEM_OFF + 4;
    static constexpr int TOTAL = ABORT_OFF + 4;
    static constexpr int DYN = TOTAL + 1024;     // slack for 1024-byte alignment
};

// GEN: general tap coordinates (conv stride p.stride, k x k kernel p.ksize) for the strided
// and 5x5 / 7x7 convs; without it the stride-1 3x3 / 1x1 coordinates only (as the T-folded
// kernel's GEN).
template <int BN, int STAGES, bool HARD, bool GEN = false>
__global__ void __launch_bounds__(THREADS, 1)
conv_lif_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const ConvParams p) {
    using S = Smem<BN, STAGES>;
    constexpr int NCH = BN / 32;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    uint32_t* smask = reinterpret_cast<uint32_t*>(smem + S::MASK_OFF);
    const uint32_t bar0 = sbase + S::BAR_OFF;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto accf_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto acce_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
    const uint32_t done_bar = bar0 + 8u * (2 * STAGES + 4);
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + S::TMEM_OFF);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::ABORT_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = p.taps * p.cin_blocks;
    constexpr uint32_t STAGE_TX = A_TILE_BYTES + S::B_TILE;
    constexpr uint32_t TMEM_COLS = 2 * BN < 32 ? 32 : 2 * BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(full_bar(s), 1);
            tc::mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(accf_bar(a), 1);
            tc::mbar_init(acce_bar(a), 128);
        }
        tc::mbar_init(done_bar, 1);
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmA);
        tc::prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tc::tmem_alloc(sbase + S::TMEM_OFF, TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 64 && p.wq) prefetch_weights_l2(p);
    // Programmatic dependent launch: the producer waits for the previous kernel only before
    // its first activation load (see conv_lif_tm_kernel).
    pdl_trigger();

    if (warp == 0) {
        // ------------------------------------------------------------- TMA producer
        int stage = 0, istage = 0;
        uint32_t phase = 0, iphase = 0, issued = 0, failed = 0;
        bool dep_ready = false;                 // griddepcontrol.wait done
        // Test hook (snnb_debug_inject_stall): CTA 0's producer -- the CTA's only issuer of
        // copies -- withholds every stage, so that the MMA warp's wait for the first stage
        // runs out (SNNB_ERR_TIMEOUT) with nothing in flight in the CTA.
        const int tile0 = (p.stall && blockIdx.x == 0) ? p.num_tiles : (int)blockIdx.x;
        const int cst = GEN ? p.stride : 1;             // the boxes' traversal stride
        const int kk = GEN ? p.ksize : 3;
        for (int tile = tile0; tile < p.num_tiles; tile += gridDim.x) {
            const Tile tl = decode_tile(tile, p, BN);
            for (int t = 0; t < p.T; ++t) {
                const int f0 = t * p.B + tl.img0;
                for (int kb = 0; kb < KB; ++kb) {
                    failed |= 1u - tc::mbar_wait_warp(empty_bar(stage), phase ^ 1u, failed);
                    const int tap = kb / p.cin_blocks;
                    const int cb = kb - tap * p.cin_blocks;
                    int r, s;                   // input offset of the tap from the pixel
                    if constexpr (GEN) {
                        r = tap / kk;
                        s = tap - r * kk - (kk >> 1);
                        r -= kk >> 1;
                    } else {
                        r = p.taps == 9 ? tap / 3 - 1 : 0;
                        s = p.taps == 9 ? tap % 3 - 1 : 0;
                    }
                    if (!failed && tc::elect_one()) {
                        tc::mbar_expect_tx(full_bar(stage), STAGE_TX);
                        tc::tma_load_3d(sbase + S::B_OFF + stage * S::B_TILE, &tmB, full_bar(stage),
                                        cb * 64, tap, tl.n0);
                    }
                    __syncwarp();
                    if (!dep_ready) {
                        pdl_wait();
                        dep_ready = true;
                    }
                    if (!failed && tc::elect_one())
                        tc::tma_load_4d(sbase + S::A_OFF + stage * A_TILE_BYTES, &tmA,
                                        full_bar(stage), cb * 64, tl.w0 * cst + s,
                                        tl.h0 * cst + r, f0);
                    __syncwarp();
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                    if (!failed) {
                        ++issued;
                        istage = stage;
                        iphase = phase;
                    }
                }
            }
        }
        if (failed) {
            drain_ring_warp(bar0, STAGES, istage, iphase, issued);
            if (lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        constexpr uint32_t IDESC = tc::idesc_bf16_f32(128, BN);
        int stage = 0;
        uint32_t phase = 0, it = 0, failed = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            for (int t = 0; t < p.T; ++t, ++it) {
                const int a = it & 1;
                failed |= 1u - tc::mbar_wait_warp(acce_bar(a), ((it >> 1) & 1u) ^ 1u, failed);
                tc::tc_fence_after();
                const uint32_t dcol = tmem + a * BN;
                for (int kb = 0; kb < KB; ++kb) {
                    int nstage = stage + 1;
                    uint32_t nphase = phase;
                    if (nstage == STAGES) { nstage = 0; nphase ^= 1u; }
                    // the issuing lane alone waits, for the next stage before committing this
                    // one (a wait queued behind a commit returns only once the pipe drained)
                    if (tc::elect_one()) {
                        if (kb == 0) {
                            failed |= 1u - tc::mbar_wait_lane(full_bar(stage), phase, failed);
                            tc::tc_fence_after();
                        }
                        const uint64_t da = tc::sdesc_k_sw128(sbase + S::A_OFF + stage * A_TILE_BYTES);
                        const uint64_t db = tc::sdesc_k_sw128(sbase + S::B_OFF + stage * S::B_TILE);
#pragma unroll
                        for (int k = 0; k < 4; ++k)   // 4 x K=16 inside the 128-byte swizzle atom
                            tc::umma_bf16(dcol, da + 2 * k, db + 2 * k, IDESC, (kb | k) != 0);
                        if (kb + 1 < KB) {
                            failed |= 1u - tc::mbar_wait_lane(full_bar(nstage), nphase, failed);
                            tc::tc_fence_after();
                        }
                        tc::umma_commit(empty_bar(stage));
                    }
                    __syncwarp();
                    stage = nstage;
                    phase = nphase;
                }
                if (tc::elect_one()) tc::umma_commit(accf_bar(a));
                __syncwarp();
                failed = __shfl_sync(0xffffffffu, failed, 0);
            }
        }
        if (tc::elect_one()) tc::umma_commit(done_bar);
        __syncwarp();
        failed |= 1u - tc::mbar_wait_warp<true>(done_bar, 0, 0);
        if (failed && lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
    } else {
        // ------------------------------------------------------------- epilogue
        const int q = warp & 3;                  // TMEM lane quadrant of this warp
        const int m = 32 * q + lane;             // pixel row of the block
        uint32_t it = 0, failed = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            const Tile tl = decode_tile(tile, p, BN);
            const float4* bias4 = reinterpret_cast<const float4*>(p.bias + tl.n0);
            float v[BN];
#pragma unroll
            for (int j = 0; j < BN; ++j) v[j] = 0.0f;
            for (int t = 0; t < p.T; ++t, ++it) {
                const int a = it & 1;
                failed |= 1u - tc::mbar_wait_warp(accf_bar(a), (it >> 1) & 1u, failed);
                tc::tc_fence_after();
                const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + a * BN;
                uint32_t mk[NCH];
#pragma unroll
                for (int c = 0; c < NCH; ++c) {
                    float r[32], bb[32];
                    tc::tmem_ld32(tbase + c * 32, r);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 b4 = __ldg(bias4 + c * 8 + j);
                        bb[4 * j] = b4.x; bb[4 * j + 1] = b4.y; bb[4 * j + 2] = b4.z; bb[4 * j + 3] = b4.w;
                    }
                    tc::tmem_wait_ld();
                    // residual input: block_n <= 64 only (with v[128] in registers the
                    // extra operands would spill)
                    if (BN <= 64 && p.res) {
                        const int x = m % p.bw, y = (m / p.bw) % p.bh, n = m / (p.bw * p.bh);
                        const int ow = tl.w0 + x, oh = tl.h0 + y, on = tl.img0 + n;
                        if (ow < p.W && oh < p.H && on < p.B)
                            add_res_slice(p, res_index(p, t, on, oh, ow, tl.n0 + c * 32), r, bb);
                    }
                    mk[c] = lif_slice<HARD>(r, bb, v + c * 32, p);
                }
                tc::tc_fence_before();
                tc::mbar_arrive(acce_bar(a));
                store_pixel<NCH>(p, tl, t, m, mk, smask + (it & 1) * (NCH * 128));
            }
        }
        if (failed && lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}


// ---- variant 3: row bands, halo reuse, resident weights ------------------------------------
// For 3x3 layers whose width W divides 128 (W in 8..64): a tile is a band of bh = 128 / W
// whole rows of one image, walked over t as in variant 1 (two TMEM accumulators, v in the
// epilogue's registers).  Per (step, 64-channel slab) the producer loads the band plus one
// halo row above and below three times, shifted by one column each (dx = 0, 1, 2; columns
// outside the image read zeros).  The 128-row A operand of tap (dy, dx) is copy dx from
// row dy*W on -- an offset of dy*W*128 bytes, a multiple of the 1024-byte swizzle atom --
// so one load serves the three taps of a column: 3 loads of (bh+2)*W rows per slab
// instead of 9 loads of 128 rows.  The weights of the CTA's channel block (9 taps x Cin x
// BN, <= 108 KB) stay in shared memory; tiles are ordered channel-block-major so a CTA
// reloads them only when its next tile belongs to another block.  Weight slab (cb, dx)
// holds taps dy = 0..2 as [dy][BN rows][64 channels] (XS below: slab (cb, dy) holds
// dx = 0..2).
constexpr int BAND_MAX_STAGES = 8;

template <int BN>
struct SmemBand {
    static constexpr int MASK_BYTES = 2 * (BN / 32) * 128 * 4;     // double-buffered pool exchange
    static constexpr int NBARS = 2 * BAND_MAX_STAGES + 7;
    // layout (runtime sizes): weights [w_bytes] | A ring [ring x a_bytes] | masks | barriers |
    // TMEM slot | abort flag
    static int dyn_bytes(int w_bytes, int ring, int a_bytes, int copies = 3) {
        return w_bytes + ring * copies * a_bytes + MASK_BYTES + NBARS * 8 + 8 + 1024;
    }
};

__device__ __forceinline__ Tile decode_band(int tile, const ConvParams& p, int BN) {
    const int nb = tile / p.mtiles;
    const int mt = tile - nb * p.mtiles;
    const int img = mt / p.tiles_h;
    const int band = mt - img * p.tiles_h;
    return Tile{0, band * p.bh, img, nb * BN};
}

// XS (variant 7, W <= 32): the column taps are shifted on the OUTPUT side instead.  A stage
// holds ONE copy of the band (columns 0..W-1, no column halo), and tap (dy, dx) multiplies
// rows dy*W .. dy*W + 127 of it into accumulator dx of the tile: D_dx[m] is then the dx tap's
// share of output pixel m + 1 - dx (same image row).  The epilogue adds the three,
// out[m] = D_1[m] + D_0[m - 1] + D_2[m + 1], with one-lane shuffles inside each row's W
// lanes; a row's first (last) column takes no D_0 (D_2) term -- it would come from the
// zero padding.  Stages are a third of the size, so the ring is three times deeper and the
// operand copies' round trips hide behind the MMAs; TMEM holds 2 x 3 accumulators.  The
// three column taps of a tap row run as ONE MMA of N = 3 x BN (their weights adjacent in
// shared memory, their accumulators adjacent in TMEM): per (step, slab) 12 MMAs reading
// 120 KB of operands instead of 36 reading 216 KB, and one band copy (a third of the TMA
// bytes) -- shared-memory bandwidth, not the tensor pipe, bounds the N = 64 MMAs.
constexpr int BAND_THREADS = 320;   // producer, MMA issuer, 2 x 4 epilogue warps

template <int BN, bool HARD, bool XS>
__global__ void __launch_bounds__(BAND_THREADS, 1)
conv_lif_band_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const ConvParams p) {
    using S = SmemBand<BN>;
    constexpr int NCH = BN / 32;
    constexpr uint32_t TAP_BYTES = BN * 128;
    constexpr int NACC = XS ? 3 : 1;                     // accumulators per (tile, step)
    constexpr uint32_t ACC_COLS = NACC * BN;             // TMEM columns of one buffer
    constexpr uint32_t TMEM_COLS = 2 * ACC_COLS <= 32 ? 32 : (2 * ACC_COLS <= 64 ? 64
                                 : (2 * ACC_COLS <= 128 ? 128 : (2 * ACC_COLS <= 256 ? 256 : 512)));
    static_assert(2 * ACC_COLS <= 512, "accumulators exceed TMEM");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    const int nst = p.ring;
    const uint32_t a_off = (uint32_t)p.w_bytes;
    const uint32_t a_bytes = (uint32_t)p.a_bytes;        // one (column-shifted) copy
    const uint32_t st_bytes = (XS ? 1u : 3u) * a_bytes;  // a stage: the copies of a slab
    const uint32_t mask_off = a_off + (uint32_t)nst * st_bytes;
    uint32_t* smask = reinterpret_cast<uint32_t*>(smem + mask_off);
    const uint32_t bar_off = mask_off + S::MASK_BYTES;
    const uint32_t bar0 = sbase + bar_off;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (BAND_MAX_STAGES + s); };
    auto accf_bar = [&](int a) { return bar0 + 8u * (2 * BAND_MAX_STAGES + a); };
    auto acce_bar = [&](int a) { return bar0 + 8u * (2 * BAND_MAX_STAGES + 2 + a); };
    const uint32_t wfull_bar = bar0 + 8u * (2 * BAND_MAX_STAGES + 4);
    const uint32_t wempty_bar = bar0 + 8u * (2 * BAND_MAX_STAGES + 5);
    const uint32_t done_bar = bar0 + 8u * (2 * BAND_MAX_STAGES + 6);
    const uint32_t tmem_off = bar_off + S::NBARS * 8;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + tmem_off);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + tmem_off + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int CB = p.cin_blocks;
    // weight slot of tap (dy, dx) of slab cb: [cb][dx][dy] (the A copy dx serves taps
    // dy = 0..2), or with XS [cb][dy][dx], so that a tap row's three column taps are one
    // B operand of 3 x BN rows
    auto wslot = [](int cb, int dx, int dy) -> uint32_t {
        return (uint32_t)(XS ? (cb * 3 + dy) * 3 + dx : (cb * 3 + dx) * 3 + dy);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < nst; ++s) {
            tc::mbar_init(full_bar(s), 1);
            tc::mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(accf_bar(a), 1);
            tc::mbar_init(acce_bar(a), 256);             // every thread of both epilogue sets
        }
        tc::mbar_init(wfull_bar, 1);
        tc::mbar_init(wempty_bar, 1);
        tc::mbar_init(done_bar, 1);
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmA);
        tc::prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        tc::tmem_alloc(sbase + tmem_off, TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 64 && p.wq) prefetch_weights_l2(p);
    // Programmatic dependent launch: the producer waits for the previous kernel only before
    // its first activation load (the resident weights are loaded before that); everything
    // this kernel writes follows those loads through the barriers.
    pdl_trigger();

    // Failure protocol: every role walks the whole schedule; a bounded wait that gives up
    // sets the role's `failed`, after which its waits return at once (no branch on the wait
    // results inside the loops -- see mbar_wait_warp).  The producer stops issuing copies,
    // drains the ones in flight, and the CTA records SNNB_ERR_TIMEOUT at the end.
    if (warp == 0) {
        // ------------------------------------------------------------- TMA producer
        int stage = 0, cur_nb = -1, istage = 0;
        uint32_t phase = 0, wloads = 0, failed = 0, issued = 0, iphase = 0, wissued = 0;
        bool dep_ready = false;                 // griddepcontrol.wait done
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            const Tile tl = decode_band(tile, p, BN);
            const int nb = tile / p.mtiles;
            if (nb != cur_nb) {
                // the previous block's weights are free once every MMA reading them is done
                if (wloads > 0) failed |= 1u - tc::mbar_wait_warp(wempty_bar, (wloads - 1) & 1u, failed);
                if (!failed && tc::elect_one()) {
                    tc::mbar_expect_tx(wfull_bar, (uint32_t)p.w_bytes);
                    for (int cb = 0; cb < CB; ++cb)
                        for (int dx = 0; dx < 3; ++dx)
                            for (int dy = 0; dy < 3; ++dy)
                                tc::tma_load_3d(sbase + wslot(cb, dx, dy) * TAP_BYTES, &tmB,
                                                wfull_bar, cb * 64, dy * 3 + dx, tl.n0);
                }
                __syncwarp();
                wissued += failed ? 0u : 1u;
                ++wloads;
                cur_nb = nb;
            }
            for (int t = 0; t < p.T; ++t) {
                const int f = t * p.B + tl.img0;
                for (int cb = 0; cb < CB; ++cb) {
                    failed |= 1u - tc::mbar_wait_warp(empty_bar(stage), phase ^ 1u, failed);
                    if (!dep_ready) {
                        pdl_wait();
                        dep_ready = true;
                    }
                    if (!failed && tc::elect_one()) {
                        tc::mbar_expect_tx(full_bar(stage), st_bytes);
                        const uint32_t dst = sbase + a_off + (uint32_t)stage * st_bytes;
                        if constexpr (XS) {
                            tc::tma_load_4d(dst, &tmA, full_bar(stage), cb * 64, 0, tl.h0 - 1, f);
                        } else {
                            for (int dx = 0; dx < 3; ++dx)
                                tc::tma_load_4d(dst + dx * a_bytes, &tmA, full_bar(stage),
                                                cb * 64, dx - 1, tl.h0 - 1, f);
                        }
                    }
                    __syncwarp();
                    if (++stage == nst) { stage = 0; phase ^= 1u; }
                    if (!failed) {            // ring position after the last issued stage
                        ++issued;
                        istage = stage;
                        iphase = phase;
                    }
                }
            }
        }
        if (failed) {
            // wait (bounded) for the copies still in flight: the last min(nst, issued) stages
            // issued and the last weight load
            int st = istage;
            uint32_t ph = iphase;
            for (uint32_t k = 0; k < (uint32_t)nst && k < issued; ++k) {
                if (--st < 0) { st = nst - 1; ph ^= 1u; }
                tc::mbar_wait_warp<true>(full_bar(st), ph, 0);
            }
            if (wissued > 0) tc::mbar_wait_warp<true>(wfull_bar, (wissued - 1) & 1u, 0);
            if (lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        // The whole warp walks the schedule; one elected lane waits and issues.  A wait that
        // the issuing thread places behind a tcgen05.commit returns only once the tensor pipe
        // has drained, so the waits for the next step -- its accumulator and its first stage
        // -- are made before this step's commits (unless the next step belongs to another
        // channel block, whose weights are loaded only after this block's last MMAs): with
        // Cin = 64 a step is one stage of 36 MMAs, and a drain per step cost ~40% of them.
        constexpr uint32_t IDESC = tc::idesc_bf16_f32(128, BN);
        constexpr uint32_t IDESC3 = tc::idesc_bf16_f32(128, XS ? 3 * BN : BN);
        static_assert(!XS || (3 * BN <= 256 && (3 * BN) % 16 == 0), "MMA N of the XS form");
        const uint32_t row_step = (uint32_t)p.W * 128u;         // one image row of the band copy
        int stage = 0, cur_nb = -1;
        uint32_t phase = 0, it = 0, wl = 0, failed = 0, ready = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            const int nb = tile / p.mtiles;
            if (nb != cur_nb) {
                if (wl > 0) {
                    if (tc::elect_one()) tc::umma_commit(wempty_bar);
                    __syncwarp();
                }
                failed |= 1u - tc::mbar_wait_warp(wfull_bar, wl & 1u, failed);
                tc::tc_fence_after();
                ++wl;
                cur_nb = nb;
            }
            const int ntile = tile + (int)gridDim.x;
            const bool next_same_block = ntile < p.num_tiles && ntile / p.mtiles == nb;
            for (int t = 0; t < p.T; ++t, ++it) {
                const int a = it & 1;
                const bool has_next = (t + 1 < p.T) || next_same_block;
                const uint32_t dcol = tmem + a * ACC_COLS;
                for (int cb = 0; cb < CB; ++cb) {
                    int nstage = stage + 1;
                    uint32_t nphase = phase;
                    if (nstage == nst) { nstage = 0; nphase ^= 1u; }
                    const uint32_t sb = sbase + a_off + (uint32_t)stage * st_bytes;
                    if (tc::elect_one()) {
                        if (cb == 0 && !ready) {
                            failed |= 1u - tc::mbar_wait_lane(acce_bar(a), ((it >> 1) & 1u) ^ 1u,
                                                              failed);
                            failed |= 1u - tc::mbar_wait_lane(full_bar(stage), phase, failed);
                            tc::tc_fence_after();
                        }
                        if constexpr (XS) {
                            // one MMA per (dy, k) with N = 3 x BN: the three column taps'
                            // weights are adjacent rows of the B operand and their sums land
                            // in the adjacent accumulators D_0 | D_1 | D_2, so each A row is
                            // read from shared memory once for all three
#pragma unroll
                            for (int dy = 0; dy < 3; ++dy) {
                                const uint64_t da = tc::sdesc_k_sw128(sb + dy * row_step);
                                const uint64_t db =
                                    tc::sdesc_k_sw128(sbase + wslot(cb, 0, dy) * TAP_BYTES);
#pragma unroll
                                for (int k = 0; k < 4; ++k)
                                    tc::umma_bf16(dcol, da + 2 * k, db + 2 * k, IDESC3,
                                                  (cb | dy | k) != 0);
                            }
                        } else {
#pragma unroll
                            for (int dx = 0; dx < 3; ++dx) {
                                const uint32_t abase = sb + dx * a_bytes;
#pragma unroll
                                for (int dy = 0; dy < 3; ++dy) {
                                    const uint64_t da = tc::sdesc_k_sw128(abase + dy * row_step);
                                    const uint64_t db =
                                        tc::sdesc_k_sw128(sbase + wslot(cb, dx, dy) * TAP_BYTES);
#pragma unroll
                                    for (int k = 0; k < 4; ++k)
                                        tc::umma_bf16(dcol, da + 2 * k, db + 2 * k, IDESC,
                                                      (cb | dx | dy | k) != 0);
                                }
                            }
                        }
                        if (cb + 1 < CB) {
                            failed |= 1u - tc::mbar_wait_lane(full_bar(nstage), nphase, failed);
                            tc::tc_fence_after();
                        } else if (has_next) {
                            const uint32_t na = (it + 1) & 1u;
                            failed |= 1u - tc::mbar_wait_lane(acce_bar((int)na),
                                                              (((it + 1) >> 1) & 1u) ^ 1u, failed);
                            failed |= 1u - tc::mbar_wait_lane(full_bar(nstage), nphase, failed);
                            tc::tc_fence_after();
                        }
                        tc::umma_commit(empty_bar(stage));
                        if (cb + 1 == CB) tc::umma_commit(accf_bar(a));
                    }
                    __syncwarp();
                    stage = nstage;
                    phase = nphase;
                }
                ready = has_next ? 1u : 0u;
                failed = __shfl_sync(0xffffffffu, failed, 0);
            }
        }
        // every MMA issued must be complete before the CTA frees its TMEM
        if (tc::elect_one()) tc::umma_commit(done_bar);
        __syncwarp();
        failed |= 1u - tc::mbar_wait_warp<true>(done_bar, 0, 0);
        if (failed && lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
    } else {
        // ------------------------------------------------------------- epilogue
        // Two sets of 4 warps (warps 2-5 and 6-9): thread = TMEM lane = band pixel m (row
        // y = m / W, column x = m % W), set s taking the 32-channel slices c = s, s + 2, ...
        // (one warp per SM sub-partition was too few: a step's neurons, loads and stores of
        // a single warp outlasted the step's MMAs).  The bias of the slices stays in
        // registers for the tile, v across t; shared memory is touched only to pool across
        // warps (W >= 32).
        const int q = warp & 3;
        const int set = (warp - 2) >> 2;
        constexpr int NCS = (NCH + 1) / 2;                  // slices per set
        const int m = 32 * q + lane;
        const int W = p.W;
        const int x = m % W, y = m / W;
        const int Ho = p.pool ? p.H / 2 : p.H, Wo = p.pool ? W / 2 : W;
        uint32_t it = 0, failed = 0;
        for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
            const Tile tl = decode_band(tile, p, BN);
            // channel pairs: the neuron runs on packed f32x2 operations (each component
            // rounded as the scalar operation: the same values, half the instructions)
            float2 bias2[16 * NCS];
#pragma unroll
            for (int cs = 0; cs < NCS; ++cs) {
                const int c = set + 2 * cs;
                const float4* bias4 = reinterpret_cast<const float4*>(p.bias + tl.n0 + 32 * c);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 b4 = c < NCH ? __ldg(bias4 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
                    bias2[16 * cs + 2 * j] = make_float2(b4.x, b4.y);
                    bias2[16 * cs + 2 * j + 1] = make_float2(b4.z, b4.w);
                }
            }
            float2 v2[16 * NCS];
#pragma unroll
            for (int j = 0; j < 16 * NCS; ++j) v2[j] = make_float2(0.0f, 0.0f);
            const float2 df2 = make_float2(p.df, p.df), sc2 = make_float2(p.sc, p.sc);
            const int hy = tl.h0 + y;                         // image row of this pixel
            for (int t = 0; t < p.T; ++t, ++it) {
                const int a = it & 1;
                failed |= 1u - tc::mbar_wait_warp(accf_bar(a), (it >> 1) & 1u, failed);
                tc::tc_fence_after();
                const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + a * ACC_COLS;
                uint32_t mk[NCS];
                // the accumulator goes back to the MMA warp as soon as its last columns are in
                // registers: the MMAs of step t + 2 then overlap this step's neurons
                bool released = false;
                auto release = [&]() {
                    tc::tc_fence_before();
                    tc::mbar_arrive(acce_bar(a));
                    released = true;
                };
#pragma unroll
                for (int cs = 0; cs < NCS; ++cs) {
                    const int c = set + 2 * cs;
                    mk[cs] = 0;
                    if (c >= NCH) continue;
                    float r[32];
                    tc::tmem_ld32(tbase + (XS ? BN : 0) + c * 32, r);
                    tc::tmem_wait_ld();
                    if (!XS && cs == NCS - 1) release();
                    float2 r2[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) r2[j] = make_float2(r[2 * j], r[2 * j + 1]);
                    if constexpr (XS) {
                        // out[m] = D_1[m] + D_0[m - 1] + D_2[m + 1] within the image row
                        // (W lanes; W <= 32 divides the warp)
                        float e[32];
                        tc::tmem_ld32(tbase + c * 32, e);
                        tc::tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float u0 = __shfl_up_sync(0xffffffffu, e[2 * j], 1, W);
                            const float u1 = __shfl_up_sync(0xffffffffu, e[2 * j + 1], 1, W);
                            r2[j] = __fadd2_rn(r2[j], x > 0 ? make_float2(u0, u1)
                                                            : make_float2(0.0f, 0.0f));
                        }
                        tc::tmem_ld32(tbase + 2 * BN + c * 32, e);
                        tc::tmem_wait_ld();
                        if (cs == NCS - 1) release();
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const float d0 = __shfl_down_sync(0xffffffffu, e[2 * j], 1, W);
                            const float d1 = __shfl_down_sync(0xffffffffu, e[2 * j + 1], 1, W);
                            r2[j] = __fadd2_rn(r2[j], x < W - 1 ? make_float2(d0, d1)
                                                                : make_float2(0.0f, 0.0f));
                        }
                    }
                    uint32_t mask = 0;
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        // charge(): decay * v + input_scale * (acc + bias), each rounded
                        const float2 in2 = __fadd2_rn(r2[j], bias2[16 * cs + j]);
                        const float2 vv = __fadd2_rn(__fmul2_rn(df2, v2[16 * cs + j]),
                                                     __fmul2_rn(sc2, in2));
                        const bool s0 = vv.x >= p.thr, s1 = vv.y >= p.thr;
                        v2[16 * cs + j] = make_float2(reset_v<HARD>(vv.x, s0, p.thr, p.v_reset),
                                                      reset_v<HARD>(vv.y, s1, p.thr, p.v_reset));
                        mask |= (s0 ? 1u : 0u) << (2 * j);
                        mask |= (s1 ? 1u : 0u) << (2 * j + 1);
                    }
                    mk[cs] = mask;
                }
                if (!released) release();                     // (a set without a last slice)
                if (set >= NCH) continue;                     // no slice for this set (BN 32)
                const int64_t frame = (int64_t)t * p.B + tl.img0;
                if (!p.pool) {
                    // the lanes of pixels x and x ^ 1 (same row: W is even) store both pixels,
                    // 16-byte chunk 2i of a slice by the even lane and 2i + 1 by the odd one,
                    // so that every store instruction fills whole 32-byte sectors
                    uint32_t ok[NCS];
#pragma unroll
                    for (int cs = 0; cs < NCS; ++cs) ok[cs] = __shfl_xor_sync(0xffffffffu, mk[cs], 1);
                    if (hy < p.H) {
                        const int par = x & 1;
#pragma unroll
                        for (int pi = 0; pi < 2; ++pi) {
                            const int64_t e0 = ((frame * Ho + hy) * Wo + ((x & ~1) | pi)) * p.Cout + tl.n0;
                            uint4* dst = reinterpret_cast<uint4*>(p.out + e0);
#pragma unroll
                            for (int cs = 0; cs < NCS; ++cs) {
                                const int c = set + 2 * cs;
                                if (c >= NCH) continue;
                                if (!SNNB_IN_BOUNDS(e0 + 32 * c + 31, out_elems(p), p.status)) continue;
                                const uint32_t mm = pi == par ? mk[cs] : ok[cs];
#pragma unroll
                                for (int i = 0; i < 2; ++i) {
                                    const int j = 2 * i + par;      // 16-byte chunk of the slice
                                    dst[4 * c + j] = spikes_to_bf16x8((mm >> (8 * j)) & 0xffu);
                                }
                            }
                        }
                    }
                } else {
                    // 2x2 max-pool = OR: column pairs are adjacent lanes; row pairs are lanes
                    // W apart (W < 32) or the same lane of another warp of the set (W >= 32)
#pragma unroll
                    for (int cs = 0; cs < NCS; ++cs) mk[cs] |= __shfl_xor_sync(0xffffffffu, mk[cs], 1);
                    if (W < 32) {
#pragma unroll
                        for (int cs = 0; cs < NCS; ++cs)
                            mk[cs] |= __shfl_xor_sync(0xffffffffu, mk[cs], W);
                    } else {
                        uint32_t* sm = smask + (it & 1) * (NCH * 128);
#pragma unroll
                        for (int cs = 0; cs < NCS; ++cs)
                            if (set + 2 * cs < NCH) sm[(set + 2 * cs) * 128 + m] = mk[cs];
                        tc::named_bar_sync(1 + set, 128);
#pragma unroll
                        for (int cs = 0; cs < NCS; ++cs)
                            if (set + 2 * cs < NCH) mk[cs] |= sm[(set + 2 * cs) * 128 + (m ^ W)];
                    }
                    if ((y & 1) == 0 && hy < p.H) {
                        // both column lanes of the window hold its OR: the even one stores
                        // chunks 2i and the odd one 2i + 1 (whole 32-byte sectors per store)
                        const int64_t e0 = ((frame * Ho + hy / 2) * Wo + x / 2) * p.Cout + tl.n0;
                        uint4* dst = reinterpret_cast<uint4*>(p.out + e0);
                        const int par = x & 1;
#pragma unroll
                        for (int cs = 0; cs < NCS; ++cs) {
                            const int c = set + 2 * cs;
                            if (c >= NCH) continue;
                            if (!SNNB_IN_BOUNDS(e0 + 32 * c + 31, out_elems(p), p.status)) continue;
#pragma unroll
                            for (int i = 0; i < 2; ++i) {
                                const int j = 2 * i + par;
                                dst[4 * c + j] = spikes_to_bf16x8((mk[cs] >> (8 * j)) & 0xffu);
                            }
                        }
                    }
                }
            }
        }
        if (failed && lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---- split-K reduction + bias + multi-step LIF (+ 2x2 max-pool) -------------------------
// splitsum_kernel<S>: thread = (step, pixel, 8 channels); adds the S partial sums in the
// order s = 0..S-1 and the bias, in place of split 0 (S = 1: the bias add of the
// float32-output linear).  splitsum_lif_kernel (below) finishes split-K conv layers.
template <int S>
__global__ void __launch_bounds__(256) splitsum_kernel(float* __restrict__ partial, int64_t rows,
                                                       int C, const float* __restrict__ bias) {
    pdl_wait();
    pdl_trigger();
    const int groups = C / 8;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= rows * groups) return;
    const int g = (int)(gid % groups);
    const int64_t row = gid / groups;                 // t * npix + pixel
    const int64_t stride = rows * C;                  // one split
    float4 v[S][2];
#pragma unroll
    for (int s = 0; s < S; ++s) {
        const float4* src = reinterpret_cast<const float4*>(partial + s * stride + row * C + g * 8);
        v[s][0] = __ldcs(src);
        v[s][1] = __ldcs(src + 1);
    }
    float acc[8];
    acc[0] = v[0][0].x; acc[1] = v[0][0].y; acc[2] = v[0][0].z; acc[3] = v[0][0].w;
    acc[4] = v[0][1].x; acc[5] = v[0][1].y; acc[6] = v[0][1].z; acc[7] = v[0][1].w;
#pragma unroll
    for (int s = 1; s < S; ++s) {
        acc[0] = __fadd_rn(acc[0], v[s][0].x); acc[1] = __fadd_rn(acc[1], v[s][0].y);
        acc[2] = __fadd_rn(acc[2], v[s][0].z); acc[3] = __fadd_rn(acc[3], v[s][0].w);
        acc[4] = __fadd_rn(acc[4], v[s][1].x); acc[5] = __fadd_rn(acc[5], v[s][1].y);
        acc[6] = __fadd_rn(acc[6], v[s][1].z); acc[7] = __fadd_rn(acc[7], v[s][1].w);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], __ldg(bias + g * 8 + j));
    float4* dst = reinterpret_cast<float4*>(partial + row * C + g * 8);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
}

// Split-K finish in one pass: thread = (pixel, 4 channels).  Per step it adds the S partial
// sums of its pixel in the order s = 0..S-1 (the loads of step t+1 are in flight while step t
// is computed), adds the bias (and the residual input), runs the neuron with v in registers
// and stores bf16 spikes [T][B][Ho][Wo][C].  With pooling the four pixels of a 2x2 window are
// four adjacent lanes that OR their spike bits by shuffles; the first of them stores the
// pooled spikes.
__device__ __forceinline__ void load_res4(const void* res, int res_f32, int64_t idx,
                                          float (&o)[4]) {
    if (res_f32) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(res) + idx));
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    } else {
        const uint2 q = __ldg(reinterpret_cast<const uint2*>(
            static_cast<const __nv_bfloat16*>(res) + idx));
        o[0] = __uint_as_float(q.x << 16); o[1] = __uint_as_float(q.x & 0xffff0000u);
        o[2] = __uint_as_float(q.y << 16); o[3] = __uint_as_float(q.y & 0xffff0000u);
    }
}

template <int S, bool POOL, bool HARD>
__global__ void __launch_bounds__(256) splitsum_lif_kernel(
    const float* __restrict__ partial, int T, int B, int H, int W, int C,
    const float* __restrict__ bias, float df, float sc, float thr, float v_reset,
    const void* __restrict__ res, int res_f32, __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    constexpr int NP = POOL ? 4 : 1;
    const int Ho = POOL ? H / 2 : H, Wo = POOL ? W / 2 : W;
    const int groups = C / 4;
    const int64_t total = (int64_t)B * Ho * Wo * groups * NP;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    // out-of-range lanes stay (no early exit) so the window shuffles see full warps; total
    // is a multiple of 4, so a window's four lanes are all in range or all out
    const bool valid = gid < total;
    const int q = POOL ? (int)(gid & 3) : 0;
    int64_t r = POOL ? (gid >> 2) : gid;
    const int g = (int)(r % groups);
    r /= groups;
    const int ow = (int)(r % Wo);
    r /= Wo;
    const int oh = (int)(r % Ho);
    const int b = (int)(r / Ho);
    const int h = POOL ? 2 * oh + (q >> 1) : oh;
    const int w = POOL ? 2 * ow + (q & 1) : ow;
    const int64_t npix = (int64_t)B * H * W;
    const int64_t pix = ((int64_t)b * H + h) * W + w;
    const int64_t split4 = (int64_t)T * npix * C / 4;        // one split, in float4
    float bb[4] = {0.f, 0.f, 0.f, 0.f}, v[4] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
        const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias + g * 4));
        bb[0] = b0.x; bb[1] = b0.y; bb[2] = b0.z; bb[3] = b0.w;
    }
    auto load_step = [&](int t, float4 (&dst)[S]) {
        const float4* src = reinterpret_cast<const float4*>(partial + ((int64_t)t * npix + pix) * C) + g;
#pragma unroll
        for (int k = 0; k < S; ++k) dst[k] = __ldcs(src + k * split4);
    };
    float4 cur[S], nxt[S];
    if (valid) load_step(0, cur);
    for (int t = 0; t < T; ++t) {
        if (valid && t + 1 < T) load_step(t + 1, nxt);
        uint32_t bits = 0;
        if (valid) {
            float y[4] = {cur[0].x, cur[0].y, cur[0].z, cur[0].w};
#pragma unroll
            for (int k = 1; k < S; ++k) {
                y[0] = __fadd_rn(y[0], cur[k].x); y[1] = __fadd_rn(y[1], cur[k].y);
                y[2] = __fadd_rn(y[2], cur[k].z); y[3] = __fadd_rn(y[3], cur[k].w);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) y[j] = __fadd_rn(y[j], bb[j]);
            if (!POOL && res) {              // residual input after the bias (no pooling then)
                float rr[4];
                load_res4(res, res_f32, (((int64_t)t * B + b) * H * W + (int64_t)h * W + w) * C + g * 4, rr);
#pragma unroll
                for (int j = 0; j < 4; ++j) y[j] = __fadd_rn(y[j], rr[j]);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float vv = charge(v[j], df, sc, y[j]);
                const bool sp = vv >= thr;
                v[j] = reset_v<HARD>(vv, sp, thr, v_reset);
                bits |= (sp ? 1u : 0u) << j;
            }
        }
        if (POOL) {
            bits |= __shfl_xor_sync(0xffffffffu, bits, 1);
            bits |= __shfl_xor_sync(0xffffffffu, bits, 2);
        }
        if (valid && q == 0) {
            const int64_t o = ((((int64_t)t * B + b) * Ho + oh) * Wo + ow) * C + g * 4;
            store_bits_bf16<4>(out + o, bits);
        }
#pragma unroll
        for (int k = 0; k < S; ++k) cur[k] = nxt[k];
    }
}

template <int S>
int launch_splitsum_lif_s(const float* partial, int T, int B, int H, int W, int C,
                          const float* bias, float df, float sc, float thr, float v_reset,
                          int hard, int pool, const void* res, int res_f32,
                          __nv_bfloat16* out, cudaStream_t s) {
    const int Ho = pool ? H / 2 : H, Wo = pool ? W / 2 : W;
    const int64_t threads = (int64_t)B * Ho * Wo * (C / 4) * (pool ? 4 : 1);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    if (pool) {
        if (hard) return launch_k(splitsum_lif_kernel<S, true, true>, dim3(blocks), dim3(256), 0, s, partial, T, B, H, W, C, bias, df, sc, thr, v_reset, res, res_f32, out);
        else return launch_k(splitsum_lif_kernel<S, true, false>, dim3(blocks), dim3(256), 0, s, partial, T, B, H, W, C, bias, df, sc, thr, v_reset, res, res_f32, out);
    } else {
        if (hard) return launch_k(splitsum_lif_kernel<S, false, true>, dim3(blocks), dim3(256), 0, s, partial, T, B, H, W, C, bias, df, sc, thr, v_reset, res, res_f32, out);
        else return launch_k(splitsum_lif_kernel<S, false, false>, dim3(blocks), dim3(256), 0, s, partial, T, B, H, W, C, bias, df, sc, thr, v_reset, res, res_f32, out);
    }
    return launch_status();
}

int launch_splitsum_lif(const float* partial, int S, int T, int B, int H, int W, int C,
                        const float* bias, float df, float sc, float thr, float v_reset, int hard,
                        int pool, const void* res, int res_f32, __nv_bfloat16* out,
                        cudaStream_t s) {
    switch (S) {
        case 2: return launch_splitsum_lif_s<2>(partial, T, B, H, W, C, bias, df, sc, thr, v_reset, hard, pool, res, res_f32, out, s);
        case 3: return launch_splitsum_lif_s<3>(partial, T, B, H, W, C, bias, df, sc, thr, v_reset, hard, pool, res, res_f32, out, s);
        case 4: return launch_splitsum_lif_s<4>(partial, T, B, H, W, C, bias, df, sc, thr, v_reset, hard, pool, res, res_f32, out, s);
        case 5: return launch_splitsum_lif_s<5>(partial, T, B, H, W, C, bias, df, sc, thr, v_reset, hard, pool, res, res_f32, out, s);
        case 6: return launch_splitsum_lif_s<6>(partial, T, B, H, W, C, bias, df, sc, thr, v_reset, hard, pool, res, res_f32, out, s);
        case 7: return launch_splitsum_lif_s<7>(partial, T, B, H, W, C, bias, df, sc, thr, v_reset, hard, pool, res, res_f32, out, s);
        case 8: return launch_splitsum_lif_s<8>(partial, T, B, H, W, C, bias, df, sc, thr, v_reset, hard, pool, res, res_f32, out, s);
        default: return SNNB_ERR_UNSUPPORTED;
    }
}

int launch_splitsum(float* partial, int S, int64_t rows, int C, const float* bias, cudaStream_t s) {
    const int64_t threads = rows * (C / 8);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    if (S != 1) return SNNB_ERR_UNSUPPORTED;
    return launch_k(splitsum_kernel<1>, dim3(blocks), dim3(256), 0, s, partial, rows, C, bias);
}

}  // namespace

// SM count of the current device (cached per device); also used by first_tc.cu.
int sm_count() {
    static int n[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!n[dev]) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
            v = 148;
        n[dev] = v;
    }
    return n[dev];
}

namespace {

template <typename K>
int launch_persistent(K kernel, int smem, const CUtensorMap& ta, const CUtensorMap& tb,
                      const ConvParams& p, cudaStream_t s, int threads = THREADS) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return record_cuda_error(e);
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kernel, threads, smem);
    if (e != cudaSuccess) return record_cuda_error(e);
    if (occ < 1) return SNNB_ERR_UNSUPPORTED;
    const int64_t cap = (int64_t)sm_count() * occ;
    const int64_t items = (int64_t)p.num_tiles * (p.splits > 1 ? p.splits : 1);
    const int grid = (int)(items < cap ? items : cap);
    return launch_k(kernel, dim3(grid), dim3(threads), smem, s, ta, tb, p);
}

// Persistent launch of a CTA-pair kernel: clusters of 2, as many as can be resident at
// once (pairs sit on the two SMs of a TPC, so this can be below half the SM count).
template <typename K>
int launch_persistent_pair(K kernel, int smem, const CUtensorMap& ta, const CUtensorMap& tb,
                           const ConvParams& p, cudaStream_t s, int threads) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return record_cuda_error(e);
    const int64_t items = (int64_t)p.num_tiles * (p.splits > 1 ? p.splits : 1);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * (sm_count() / 2)));
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg);
    if (e != cudaSuccess) return record_cuda_error(e);
    if (clusters < 1) return SNNB_ERR_UNSUPPORTED;
    const int pairs = (int)(items < clusters ? items : clusters);
    return launch_kc(kernel, dim3(2 * pairs), dim3(threads), smem, s, 2u, ta, tb, p);
}

// Ring depths fill the ~227 KB of shared memory: at these tile sizes one k-slab of MMAs
// (0.1-0.4 us) is far shorter than a TMA round trip, so depth is what keeps the tensor
// pipe fed.
template <int BN, int STAGES, bool GEN = false>
int launch_conv(const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p, cudaStream_t s) {
    return p.hard ? launch_persistent(conv_lif_kernel<BN, STAGES, true, GEN>, Smem<BN, STAGES>::DYN, ta, tb, p, s)
                  : launch_persistent(conv_lif_kernel<BN, STAGES, false, GEN>, Smem<BN, STAGES>::DYN, ta, tb, p, s);
}

template <int BN, int STAGES, int TS, int MH = 1>
int launch_conv_tm(const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
                   cudaStream_t s) {
    constexpr int dyn = SmemTM<BN, STAGES, TS, MH>::DYN;
    constexpr int NP = BN == 256 ? 2 : (BN == 64 ? 4 : 3);
    constexpr int threads = THREADS + 32 * (NP - 1) + 128;
    if (MH == 1 && p.res)
        return p.hard ? launch_persistent(conv_lif_tm_kernel<BN, STAGES, TS, true, NP, MH, 1, MH == 1>, dyn, ta, tb, p, s, threads)
                      : launch_persistent(conv_lif_tm_kernel<BN, STAGES, TS, false, NP, MH, 1, MH == 1>, dyn, ta, tb, p, s, threads);
    if (p.res) return SNNB_ERR_UNSUPPORTED;
    return p.hard ? launch_persistent(conv_lif_tm_kernel<BN, STAGES, TS, true, NP, MH, 1, false>, dyn, ta, tb, p, s, threads)
                  : launch_persistent(conv_lif_tm_kernel<BN, STAGES, TS, false, NP, MH, 1, false>, dyn, ta, tb, p, s, threads);
}

// CTA-pair form: each CTA stages A (16 KB) + BN/2 weight rows per k-slab.
template <int BN, int STAGES, int TS>
int launch_conv_tm_pair(const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
                        cudaStream_t s) {
    constexpr int dyn = SmemTM<BN, STAGES, TS, 1, 2>::DYN;
    constexpr int NP = BN == 256 ? 2 : 3;
    constexpr int threads = THREADS + 32 * (NP - 1) + 128;
    if (p.res) return SNNB_ERR_UNSUPPORTED;
    return p.hard ? launch_persistent_pair(conv_lif_tm_kernel<BN, STAGES, TS, true, NP, 1, 2, false>, dyn, ta, tb, p, s, threads)
                  : launch_persistent_pair(conv_lif_tm_kernel<BN, STAGES, TS, false, NP, 1, 2, false>, dyn, ta, tb, p, s, threads);
}

template <int TS>
int launch_tm_bn(int BN, const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
                 cudaStream_t s, int mh = 1, int cg = 1) {
    if (cg == 2) {
        switch (BN) {
            case 256: return launch_conv_tm_pair<256, 6, TS>(ta, tb, p, s);
            case 128: return launch_conv_tm_pair<128, 8, TS>(ta, tb, p, s);
            case 64: return launch_conv_tm_pair<64, 9, TS>(ta, tb, p, s);
            default: return SNNB_ERR_UNSUPPORTED;
        }
    }
    if (mh == 2) {
        switch (BN) {
            case 128: return launch_conv_tm<128, 4, TS, 2>(ta, tb, p, s);
            case 64: return launch_conv_tm<64, 5, TS, 2>(ta, tb, p, s);
            case 32: return launch_conv_tm<32, 5, TS, 2>(ta, tb, p, s);
            default: return SNNB_ERR_UNSUPPORTED;
        }
    }
    switch (BN) {
        case 256: return launch_conv_tm<256, 4, TS>(ta, tb, p, s);
        case 128: return launch_conv_tm<128, 7, TS>(ta, tb, p, s);
        case 64: return launch_conv_tm<64, 9, TS>(ta, tb, p, s);
        default: return launch_conv_tm<32, 10, TS>(ta, tb, p, s);
    }
}

// Pixel block of P rows (P = 128, or 128 / T when T is folded into M) for an H x W
// image batch: bw columns x bh rows x bn images with bw * bh * bn == P.  Exact tilings
// are preferred; otherwise power-of-two block sides leave partial blocks at the right /
// bottom / last-image edges, whose out-of-range rows the TMA zero-fills and the
// epilogue never stores.  With pooling bw and bh are even so that every 2x2 window
// lies inside one block.
static int pow2_floor(int v) {
    int r = 1;
    while (r * 2 <= v) r *= 2;
    return r;
}

bool choose_block(int H, int W, int P, bool pool, int& bw, int& bh, int& bn) {
    if (W >= P && W % P == 0 && !pool) {
        bw = P; bh = 1; bn = 1;
        return true;
    }
    if (W >= P / 2 && pool) {
        bw = P / 2; bh = 2; bn = 1;
    } else if (W < P && P % W == 0) {
        bw = W;
    } else {
        bw = pow2_floor(W < P ? W : P);
        if (pool && bw < 2) return false;
    }
    const int rows = P / bw;
    if (pool && bw == P / 2) {
        bh = 2; bn = 1;
    } else if (H >= rows) {
        bh = rows; bn = 1;
    } else if (rows % H == 0) {
        bh = H; bn = rows / H;
    } else {
        bh = pow2_floor(H);
        bn = rows / bh;
    }
    if (bw * bh * bn != P) return false;
    return !pool || ((bw % 2 == 0) && (bh % 2 == 0));
}

}  // namespace

int* device_status_ptr() {
    static int* ptrs[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!ptrs[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
        ptrs[dev] = static_cast<int*>(p);
    }
    return ptrs[dev];
}

int encode_tmap(CUtensorMap* map, CUtensorMapDataType dtype, int rank, const void* base,
                const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                CUtensorMapSwizzle swizzle, const uint32_t* elem_strides) {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* f = nullptr;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f) {
            if (e != cudaSuccess) return record_cuda_error(e);
            return SNNB_ERR_CUDA;
        }
        fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    cuuint64_t d[5], st[4];
    cuuint32_t b[5], es[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        // traversal stride: a box of box[i] elements along dimension i loads every
        // es[i]-th of them (ceil(box[i] / es[i]) elements)
        es[i] = elem_strides ? elem_strides[i] : 1;
        if (i < rank - 1) st[i] = strides_bytes[i];
    }
    CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? SNNB_OK : SNNB_ERR_ARG;
}

namespace {

// ---- variant 3 host path -----------------------------------------------------------------
constexpr int BAND_W_MAX = 108 * 1024;          // resident weights per CTA (3 band copies)
constexpr int BAND_XS_W_MAX = 160 * 1024;       // the XS form: one copy per stage

int smem_optin() {
    static int v[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 227 * 1024;
    if (!v[dev]) {
        int x = 0;
        if (cudaDeviceGetAttribute(&x, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
            x <= 0)
            x = 227 * 1024;
        v[dev] = x;
    }
    return v[dev];
}

// Channel-block width for the band kernel, or 0 if the layer does not qualify.  The XS
// form's stages hold one band copy instead of three, which leaves room for larger resident
// weights (its ring still gets >= 2 stages: run_band_layer checks).
int band_block_n(int W, int Cin, int Cout, int block_n, bool xs) {
    if (!(W == 8 || W == 16 || W == 32 || W == 64)) return 0;
    if (xs && W > 32) return 0;
    const int CB = (Cin + 63) / 64;
    const int wmax = xs ? BAND_XS_W_MAX : BAND_W_MAX;
    auto fits = [&](int bn) { return Cout % bn == 0 && 9 * CB * bn * 128 <= wmax; };
    if (block_n) return (block_n == 32 || block_n == 64) && fits(block_n) ? block_n : 0;
    if (fits(64)) return 64;
    return fits(32) ? 32 : 0;
}

int run_band_layer(const void* x, int T, int B, int H, int W, int Cin, const void* w,
                   const float* bias, int Cout, int BN, float df, float sc, float thr,
                   float v_reset, int hard, int pool, const void* res, int res_f32, void* out,
                   int* status, cudaStream_t s, bool xs = false) {
    const int bh = 128 / W;
    if (pool && (bh % 2)) return SNNB_ERR_UNSUPPORTED;
    if (xs && W > 32) return SNNB_ERR_UNSUPPORTED;       // a row's lanes must share a warp
    const int CB = (Cin + 63) / 64;
    const int a_bytes = (bh + 2) * W * 128;
    const int w_bytes = 9 * CB * BN * 128;
    const int copies = xs ? 1 : 3;
    const int fixed = BN == 64 ? SmemBand<64>::dyn_bytes(w_bytes, 0, a_bytes, copies)
                               : SmemBand<32>::dyn_bytes(w_bytes, 0, a_bytes, copies);
    int ring = (smem_optin() - fixed) / (copies * a_bytes);
    if (ring > BAND_MAX_STAGES) ring = BAND_MAX_STAGES;
    if (ring < 2) return SNNB_ERR_UNSUPPORTED;
    // activation map: dims (Cin, W, H, T*B), box (64, W, bh + 2, 1): the band and its halo
    CUtensorMap ta, tb;
    const uint64_t adims[4] = {(uint64_t)Cin, (uint64_t)W, (uint64_t)H, (uint64_t)T * B};
    const uint64_t astr[3] = {(uint64_t)Cin * 2, (uint64_t)W * Cin * 2, (uint64_t)H * W * Cin * 2};
    const uint32_t abox[4] = {64, (uint32_t)W, (uint32_t)(bh + 2), 1};
    int rc = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, x, adims, astr, abox,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SNNB_OK) return rc;
    // weight map: dims (Cin, 9 taps, Cout), box (64, 1, BN): one tap's slab of the block
    const uint64_t bdims[3] = {(uint64_t)Cin, 9, (uint64_t)Cout};
    const uint64_t bstr[2] = {(uint64_t)Cin * 2, (uint64_t)9 * Cin * 2};
    const uint32_t bbox[3] = {64, 1, (uint32_t)BN};
    rc = encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, w, bdims, bstr, bbox,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SNNB_OK) return rc;
    ConvParams p = {};
    p.T = T; p.B = B; p.H = H; p.W = W; p.Cin = Cin; p.Cout = Cout;
    p.bw = W; p.bh = bh; p.bn = 1;
    p.tiles_w = 1; p.tiles_h = (H + bh - 1) / bh;
    p.n_tiles_n = Cout / BN;
    p.mtiles = B * p.tiles_h;
    const int64_t ntiles = (int64_t)p.mtiles * p.n_tiles_n;
    if (ntiles > 0x7fffffff) return SNNB_ERR_ARG;
    p.num_tiles = (int)ntiles;
    p.taps = 9; p.cin_blocks = CB; p.pool = pool;
    p.df = df; p.sc = sc; p.thr = thr; p.v_reset = v_reset; p.hard = hard ? 1 : 0;
    p.bias = bias; p.out = static_cast<__nv_bfloat16*>(out); p.status = status;
    p.wq = w; p.wq_bytes = (int64_t)Cout * p.taps * Cin * 2;
    p.res = res; p.res_f32 = res_f32;
    p.splits = 1; p.partial = nullptr;
    p.ring = ring; p.a_bytes = a_bytes; p.w_bytes = w_bytes;
    const int dyn = BN == 64 ? SmemBand<64>::dyn_bytes(w_bytes, ring, a_bytes, copies)
                             : SmemBand<32>::dyn_bytes(w_bytes, ring, a_bytes, copies);
    if (xs) {
        if (BN == 64)
            return hard ? launch_persistent(conv_lif_band_kernel<64, true, true>, dyn, ta, tb, p, s, BAND_THREADS)
                        : launch_persistent(conv_lif_band_kernel<64, false, true>, dyn, ta, tb, p, s, BAND_THREADS);
        return hard ? launch_persistent(conv_lif_band_kernel<32, true, true>, dyn, ta, tb, p, s, BAND_THREADS)
                    : launch_persistent(conv_lif_band_kernel<32, false, true>, dyn, ta, tb, p, s, BAND_THREADS);
    }
    if (BN == 64)
        return hard ? launch_persistent(conv_lif_band_kernel<64, true, false>, dyn, ta, tb, p, s, BAND_THREADS)
                    : launch_persistent(conv_lif_band_kernel<64, false, false>, dyn, ta, tb, p, s, BAND_THREADS);
    return hard ? launch_persistent(conv_lif_band_kernel<32, true, false>, dyn, ta, tb, p, s, BAND_THREADS)
                : launch_persistent(conv_lif_band_kernel<32, false, false>, dyn, ta, tb, p, s, BAND_THREADS);
}

// Bytes of the split-K partial sums, splits * T * B * H * W * Cout float32 values, or -1
// when a factor is negative or the product overflows int64 (each factor may be as large as
// 2^31 - 1, so the product of six of them can wrap).
static int64_t split_partial_bytes(int64_t splits, int64_t T, int64_t B, int64_t H, int64_t W,
                                   int64_t Cout) {
    const int64_t f[6] = {splits, T, B, H, W, Cout};
    int64_t n = 4;
    for (int i = 0; i < 6; ++i) {
        if (f[i] < 0 || __builtin_mul_overflow(n, f[i], &n)) return -1;
    }
    return n;
}

// Shared host path of the conv / linear entries.
// variant: 0 = choose, 1 = T sequential inside the CTA (128-pixel blocks),
//          2 = T folded into M (128/T-pixel blocks, T in {2, 4, 8}),
//          3 = row bands with halo reuse and resident weights (W in {8, 16, 32, 64}),
//          4 = as 2 with two M-tiles per CTA, 5 = as 2 on CTA pairs (cta_group::2),
//          6 = as 2 with the K range split across a cluster (conv_cluster.cu).
// block_n: 0 = choose, else 32 / 64 / 128 (/ 256 with variant 2) output channels per CTA.
// splits : > 1 splits the K range (variants 2 and 6): with variant 2 partial sums go to
//          `workspace` ([splits][T][B*H*W][Cout] f32, caller-owned) and
//          splitsum_lif_kernel finishes; with variant 6 the cluster reduces them itself.
int run_tc_layer(const void* x, int T, int B, int H, int W, int Cin, const void* w,
                 const float* bias, int Cout, int taps, float df, float sc, float thr,
                 float v_reset, int hard, int pool, int variant, int block_n, int splits,
                 void* workspace, int64_t workspace_bytes, void* out, cudaStream_t s,
                 const void* res = nullptr, int res_f32 = 0, int x_packed = 0,
                 int out_packed = 0, int stride = 1, int f32_out = 0) {
    if (const int inj = take_injected_status()) return inj;
    if (!x || !w || !out || !bias) return SNNB_ERR_ARG;
    // stride 2 (k x k / padding k / 2, k odd): H, W are the input's sizes here and the
    // output's from the shape checks on, (H - 1) / 2 + 1 x (W - 1) / 2 + 1; the activation
    // boxes traverse the input with stride 2.  T-sequential and T-folded kernels only.
    if (stride != 1 && stride != 2) return SNNB_ERR_ARG;
    // k x k kernels, padding k / 2: 1, 3 (taps 1 / 9) and 5, 7 (T-sequential / T-folded)
    const int ksize = taps == 1 ? 1 : taps == 9 ? 3 : taps == 25 ? 5 : taps == 49 ? 7 : 0;
    if (!ksize) return SNNB_ERR_ARG;
    // general tap coordinates (stride 2 or a 5x5 / 7x7 kernel): the T-sequential kernel and
    // the single-CTA T-folded kernel (any splits) -- not the band, two-tile, CTA-pair,
    // cluster split-K, packed or dense forms
    const bool gen = stride != 1 || ksize > 3;
    if (gen && (x_packed || out_packed || pool == 2 || variant >= 3))
        return SNNB_ERR_UNSUPPORTED;
    // f32_out: no neuron -- out is float32 [T*B, H, W, Cout] = conv + bias (the T-folded
    // kernel's raw sums, then the bias added in place), e.g. a downsample branch
    if (f32_out) {
        if (pool || res || x_packed || out_packed || splits > 1) return SNNB_ERR_UNSUPPORTED;
        if (variant != 0 && variant != 2) return SNNB_ERR_UNSUPPORTED;
        variant = 2;
    }
    if (H <= 0 || W <= 0) return SNNB_ERR_ARG;
    const int Hin = H, Win = W;
    if (stride == 2) {
        H = (H - 1) / 2 + 1;
        W = (W - 1) / 2 + 1;
    }
    // packed spikes in / out: the T-folded kernel (variant 2), one launch (no split-K), no
    // residual; packed input for 3x3 convs with Cin % 64 == 0
    if (x_packed || out_packed) {
        if (variant == 0) variant = 2;
        if (variant != 2 || splits > 1 || res || pool == 2) return SNNB_ERR_UNSUPPORTED;
        if (x_packed && (taps != 9 || Cin % 64 != 0)) return SNNB_ERR_UNSUPPORTED;
        if (x_packed && block_n == 32) return SNNB_ERR_UNSUPPORTED;
        if (reinterpret_cast<uintptr_t>(out) & 3u) return SNNB_ERR_ARG;
    }
    if (res && (pool || !aligned16(res))) return res && pool ? SNNB_ERR_UNSUPPORTED : SNNB_ERR_ARG;
    // pool == 2: OR over groups of 4 consecutive output columns (the dense form of a pooled
    // 2x2-image conv, snnb_conv3x3_lif_dense); T-folded epilogues only
    const bool gpool = pool == 2;
    if (pool < 0 || pool > 2) return SNNB_ERR_ARG;
    if (gpool) {
        if (taps != 1 || H != 1 || W != 1 || Cout % 128 != 0) return SNNB_ERR_UNSUPPORTED;
        if ((variant != 0 && variant != 2) || splits > 1) return SNNB_ERR_UNSUPPORTED;
        variant = 2;
    }
    if (T <= 0 || B <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0) return SNNB_ERR_ARG;
    if (Cin % 8 != 0 || Cout % 32 != 0) return SNNB_ERR_UNSUPPORTED;
    if (!aligned16(x) || !aligned16(w) || (!out_packed && !aligned16(out))) return SNNB_ERR_ARG;
    if (pool == 1 && ((H % 2) || (W % 2))) return SNNB_ERR_UNSUPPORTED;
    if ((int64_t)T * B > 0x7fffffff / 2) return SNNB_ERR_ARG;
    if (variant < 0 || variant > 7) return SNNB_ERR_ARG;
    // variant 6: T folded into M, the K range split across a cluster of `splits` CTAs that
    // reduce through distributed shared memory (conv_cluster.cu); no workspace
    const bool ck = variant == 6;
    if (ck) {
        if (splits != 2 && splits != 4 && splits != 8) return SNNB_ERR_UNSUPPORTED;
        if (block_n == 0) block_n = splits == 8 ? 256 : 128;
        if (block_n != 128 && block_n != 256) return SNNB_ERR_UNSUPPORTED;
        if (splits == 8 && block_n != 256) return SNNB_ERR_UNSUPPORTED;
        variant = 2;
    }
    // variant 4: T folded into M with two M-tiles per CTA sharing each weight stage
    const int mh = variant == 4 ? 2 : 1;
    if (variant == 4) {
        if (block_n == 256) return SNNB_ERR_UNSUPPORTED;      // 2 x 2 x 256 TMEM columns
        variant = 2;
    }
    // variant 5: T folded into M, CTA pairs with M = 256 MMAs (cta_group::2)
    const int cg = variant == 5 ? 2 : 1;
    if (variant == 5) {
        if (block_n == 32) return SNNB_ERR_UNSUPPORTED;       // 16 weight rows per CTA
        variant = 2;
    }
    if (block_n != 0 && block_n != 32 && block_n != 64 && block_n != 128 && block_n != 256)
        return SNNB_ERR_ARG;
    if (block_n && Cout % block_n) return SNNB_ERR_ARG;
    if (splits < 1) splits = 1;
    if (splits > 8) return SNNB_ERR_UNSUPPORTED;
    const int KB = taps * ((Cin + 63) / 64);
    if (splits > KB) return SNNB_ERR_ARG;
    if (variant == 3 || variant == 7) {
        if (taps != 9 || splits > 1 || res) return SNNB_ERR_UNSUPPORTED;
        const int BN3 = band_block_n(W, Cin, Cout, block_n, variant == 7);
        if (!BN3) return SNNB_ERR_UNSUPPORTED;
        int* st = device_status_ptr();
        if (!st) return SNNB_ERR_CUDA;
        return run_band_layer(x, T, B, H, W, Cin, w, bias, Cout, BN3, df, sc, thr, v_reset, hard,
                              pool, res, res_f32, out, st, s, variant == 7);
    }
    const bool tm_ok = (T == 2 || T == 4 || T == 8);
    if (variant == 2 && !tm_ok) return SNNB_ERR_UNSUPPORTED;
    if (splits > 1 && (variant == 1 || !tm_ok)) return SNNB_ERR_UNSUPPORTED;
    if (splits > 1) variant = 2;
    if (mh == 2 && variant != 2) return SNNB_ERR_UNSUPPORTED;
    const int bn_max = (Cout % 128 == 0) ? 128 : (Cout % 64 == 0 ? 64 : 32);
    int bw, bh, bn;
    if (variant == 0) {
        // sequential kernel unless its grid leaves SMs idle and folding T is possible
        variant = 1;
        if (tm_ok && choose_block(H, W, 128, pool == 1, bw, bh, bn)) {
            const int64_t seq_grid = ((int64_t)((W + bw - 1) / bw) * ((H + bh - 1) / bh) *
                                      ((B + bn - 1) / bn)) * (Cout / (block_n ? block_n : bn_max));
            if (seq_grid < 2 * 148) variant = 2;
        } else if (tm_ok) {
            variant = 2;
        }
    }
    if (variant == 1 && block_n == 256) return SNNB_ERR_UNSUPPORTED;   // v[] would not fit
    if (variant == 1 && res && block_n == 128) return SNNB_ERR_UNSUPPORTED;
    const int P = variant == 2 ? 128 / T : 128;
    if (!choose_block(H, W, P, pool == 1, bw, bh, bn)) return SNNB_ERR_UNSUPPORTED;
    const int64_t mtiles = (int64_t)((W + bw - 1) / bw) * ((H + bh - 1) / bh) * ((B + bn - 1) / bn);
    int BN = block_n;
    if (!BN) {
        BN = bn_max;
        // narrower channel blocks until the grid covers the SMs
        if (mh == 2 && BN > 128) BN = 128;
        const int bn_min = (cg == 2 || x_packed) ? 64 : 32;
        while (BN > bn_min && ((mtiles + mh * cg - 1) / (mh * cg)) * (Cout / BN) * splits * cg < 148)
            BN /= 2;
    }
    if (cg == 2 && BN < 64) return SNNB_ERR_UNSUPPORTED;
    if (variant == 1 && res && BN > 64) BN = 64;     // residual operands: see conv_lif_kernel
    if (splits > 1 && !ck) {
        const int64_t need = split_partial_bytes(splits, T, B, H, W, Cout);
        if (need < 0 || !workspace || workspace_bytes < need || !aligned16(workspace))
            return SNNB_ERR_ARG;
    }
    int pk_px = 0, pk_ps = 0;
    if (x_packed) {
        // the kernel's patch: T planes of bn*(bh+2)*(bw+2) pixel slots -- of Cin/32 + 2 words
        // and 8 more words per plane (fewer bank conflicts) when that fits, else unpadded
        const int64_t npx = (int64_t)bn * (bh + 2) * (bw + 2);
        pk_px = Cin / 32 + 2;
        pk_ps = (int)(npx * pk_px + 8);
        if ((int64_t)T * pk_ps * 4 > packed_patch_limit()) {
            pk_px = Cin / 32;
            pk_ps = (int)(npx * pk_px);
        }
        if ((int64_t)T * npx * (Cin / 32) * 4 > packed_patch_limit()) return SNNB_ERR_UNSUPPORTED;
    }
    int* status = device_status_ptr();
    if (!status) return SNNB_ERR_CUDA;
    CUtensorMap ta, tb;
    int rc = SNNB_OK;
    if (x_packed) {
        // no activation tensor map: the kernel reads the packed patch itself
    } else if (variant == 2) {
        // activation map: dims (Cin, T, W, H, B) of the input, box (64, T, bw, bh, bn) of
        // loaded elements: one box = the pixel block at every step, rows ordered (pixel, t)
        // -- a pixel's T steps are adjacent accumulator rows, i.e. adjacent lanes of one
        // epilogue warp.  Stride 2: the box spans 2 bw x 2 bh input pixels, every second one
        // loaded (traversal stride 2).
        const uint64_t adims[5] = {(uint64_t)Cin, (uint64_t)T, (uint64_t)Win, (uint64_t)Hin,
                                   (uint64_t)B};
        const uint64_t astr[4] = {(uint64_t)B * Hin * Win * Cin * 2, (uint64_t)Cin * 2,
                                  (uint64_t)Win * Cin * 2, (uint64_t)Hin * Win * Cin * 2};
        const uint32_t abox[5] = {64, (uint32_t)T, (uint32_t)(bw * stride), (uint32_t)(bh * stride),
                                  (uint32_t)bn};
        const uint32_t aes[5] = {1, 1, (uint32_t)stride, (uint32_t)stride, 1};
        rc = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, x, adims, astr, abox,
                         CU_TENSOR_MAP_SWIZZLE_128B, aes);
    } else {
        // activation map: dims (Cin, W, H, T*B) of the input, box (64, bw, bh, bn) of loaded
        // elements (traversal stride as above)
        const uint64_t adims[4] = {(uint64_t)Cin, (uint64_t)Win, (uint64_t)Hin, (uint64_t)T * B};
        const uint64_t astr[3] = {(uint64_t)Cin * 2, (uint64_t)Win * Cin * 2,
                                  (uint64_t)Hin * Win * Cin * 2};
        const uint32_t abox[4] = {64, (uint32_t)(bw * stride), (uint32_t)(bh * stride), (uint32_t)bn};
        const uint32_t aes[4] = {1, (uint32_t)stride, (uint32_t)stride, 1};
        rc = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, x, adims, astr, abox,
                         CU_TENSOR_MAP_SWIZZLE_128B, aes);
    }
    if (rc != SNNB_OK) return rc;
    // weight map: dims (Cin, taps, Cout), box (64, 1, BN): channels past Cin read as zero
    const uint64_t bdims[3] = {(uint64_t)Cin, (uint64_t)taps, (uint64_t)Cout};
    const uint64_t bstr[2] = {(uint64_t)Cin * 2, (uint64_t)taps * Cin * 2};
    const uint32_t bbox[3] = {64, 1, (uint32_t)(BN / cg)};   // a pair: half the rows per CTA
    rc = encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, w, bdims, bstr, bbox,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SNNB_OK) return rc;
    if (x_packed) ta = tb;                // unused by the packed-input kernel
    ConvParams p = {};
    p.T = T; p.B = B; p.H = H; p.W = W; p.Cin = Cin; p.Cout = Cout;
    p.bw = bw; p.bh = bh; p.bn = bn;
    p.tiles_w = (W + bw - 1) / bw; p.tiles_h = (H + bh - 1) / bh;
    p.n_tiles_n = Cout / BN;
    p.taps = taps; p.cin_blocks = (Cin + 63) / 64; p.pool = pool;
    p.df = df; p.sc = sc; p.thr = thr; p.v_reset = v_reset; p.hard = hard ? 1 : 0;
    p.bias = bias; p.out = static_cast<__nv_bfloat16*>(out); p.status = status;
    p.wq = w; p.wq_bytes = (int64_t)Cout * p.taps * Cin * 2;
    p.res = res; p.res_f32 = res_f32;
    p.xq = x_packed ? static_cast<const uint32_t*>(x) : nullptr;
    p.pk_px = pk_px; p.pk_ps = pk_ps;
    p.out_packed = out_packed ? 1 : 0;
    p.splits = ck ? 1 : splits;
    p.partial = splits > 1 && !ck ? static_cast<float*>(workspace) : nullptr;
    if (f32_out) {
        p.out = nullptr;
        p.partial = static_cast<float*>(out);     // one split: the raw sums are the result
    }
    p.stride = stride;
    p.ksize = ksize;
    const int64_t ntiles = ((mtiles + mh * cg - 1) / (mh * cg)) * p.n_tiles_n;
    p.mtiles = (int)mtiles;
    if (ntiles * splits > 0x7fffffff) return SNNB_ERR_ARG;
    p.num_tiles = (int)ntiles;
    if (ck) return launch_tm_cluster(T, BN, splits, ta, tb, p, s);
    if (x_packed || out_packed) return launch_tm_packed(T, BN, x_packed, out_packed, ta, tb, p, s);
    if (gpool) return launch_tm_cpool(T, BN, ta, tb, p, s);
    if (variant == 2) {
        if (gen) {
            rc = launch_tm_general(T, BN, ta, tb, p, s);
        } else {
            switch (T) {
                case 2: rc = launch_tm_bn<2>(BN, ta, tb, p, s, mh, cg); break;
                case 4: rc = launch_tm_bn<4>(BN, ta, tb, p, s, mh, cg); break;
                default: rc = launch_tm_bn<8>(BN, ta, tb, p, s, mh, cg); break;
            }
        }
        if (rc != SNNB_OK) return rc;
        if (f32_out)
            return launch_splitsum(p.partial, 1, (int64_t)T * B * H * W, Cout, bias, s);
        if (splits == 1) return rc;
        return launch_splitsum_lif(p.partial, splits, T, B, H, W, Cout, bias, df, sc, thr, v_reset,
                                   p.hard, pool, res, res_f32, p.out, s);
    }
    p.stall = take_injected_stall();
    if (gen) {
        switch (BN) {
            case 128: return launch_conv<128, 6, true>(ta, tb, p, s);
            case 64: return launch_conv<64, 8, true>(ta, tb, p, s);
            default: return launch_conv<32, 10, true>(ta, tb, p, s);
        }
    }
    switch (BN) {
        case 128: return launch_conv<128, 6>(ta, tb, p, s);
        case 64: return launch_conv<64, 8>(ta, tb, p, s);
        default: return launch_conv<32, 10>(ta, tb, p, s);
    }
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_conv3x3_lif(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                                int64_t Cin, const void* w, const float* bias, int64_t Cout,
                                float decay, float input_scale, float v_threshold, float v_reset,
                                int hard_reset, int pool, int variant, int block_n, int splits,
                                void* workspace, int64_t workspace_bytes, void* out,
                                snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || H > 0x7fffffff || W > 0x7fffffff ||
        Cin > 0x7fffffff || Cout > 0x7fffffff)
        return SNNB_ERR_ARG;
    return run_tc_layer(x, (int)T, (int)B, (int)H, (int)W, (int)Cin, w, bias, (int)Cout, 9, decay,
                        input_scale, v_threshold, v_reset, hard_reset, pool, variant, block_n,
                        splits, workspace, workspace_bytes, out, static_cast<cudaStream_t>(stream));
}

extern "C" int snnb_conv3x3_lif_res(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                                    int64_t Cin, const void* w, const float* bias, int64_t Cout,
                                    float decay, float input_scale, float v_threshold,
                                    float v_reset, int hard_reset, const void* residual,
                                    int residual_dtype, int variant, int block_n, int splits,
                                    void* workspace, int64_t workspace_bytes, void* out,
                                    snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || H > 0x7fffffff || W > 0x7fffffff ||
        Cin > 0x7fffffff || Cout > 0x7fffffff)
        return SNNB_ERR_ARG;
    if (!residual || (residual_dtype != SNNB_BF16 && residual_dtype != SNNB_F32))
        return SNNB_ERR_ARG;
    return run_tc_layer(x, (int)T, (int)B, (int)H, (int)W, (int)Cin, w, bias, (int)Cout, 9, decay,
                        input_scale, v_threshold, v_reset, hard_reset, 0, variant, block_n,
                        splits, workspace, workspace_bytes, out, static_cast<cudaStream_t>(stream),
                        residual, residual_dtype == SNNB_F32 ? 1 : 0);
}

extern "C" int snnb_conv_lif_strided(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                                     int64_t Cin, const void* w, const float* bias, int64_t Cout,
                                     int ksize, int stride, float decay, float input_scale,
                                     float v_threshold, float v_reset, int hard_reset,
                                     const void* residual, int residual_dtype, int variant,
                                     int block_n, int splits, void* workspace,
                                     int64_t workspace_bytes, void* out, snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || H > 0x7fffffff || W > 0x7fffffff ||
        Cin > 0x7fffffff || Cout > 0x7fffffff)
        return SNNB_ERR_ARG;
    if ((ksize != 1 && ksize != 3 && ksize != 5 && ksize != 7) || (stride != 1 && stride != 2))
        return SNNB_ERR_ARG;
    if (residual && residual_dtype != SNNB_BF16 && residual_dtype != SNNB_F32) return SNNB_ERR_ARG;
    return run_tc_layer(x, (int)T, (int)B, (int)H, (int)W, (int)Cin, w, bias, (int)Cout,
                        ksize * ksize, decay, input_scale, v_threshold, v_reset, hard_reset, 0,
                        variant, block_n, splits, workspace, workspace_bytes, out,
                        static_cast<cudaStream_t>(stream), residual,
                        residual && residual_dtype == SNNB_F32 ? 1 : 0, 0, 0, stride, 0);
}

extern "C" int snnb_conv_f32(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                             int64_t Cin, const void* w, const float* bias, int64_t Cout,
                             int ksize, int stride, float* out, snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || H > 0x7fffffff || W > 0x7fffffff ||
        Cin > 0x7fffffff || Cout > 0x7fffffff)
        return SNNB_ERR_ARG;
    if ((ksize != 1 && ksize != 3 && ksize != 5 && ksize != 7) || (stride != 1 && stride != 2))
        return SNNB_ERR_ARG;
    return run_tc_layer(x, (int)T, (int)B, (int)H, (int)W, (int)Cin, w, bias, (int)Cout,
                        ksize * ksize, 0.0f, 0.0f, 0.0f, 0.0f, 1, 0, 2, 0, 1, nullptr, 0, out,
                        static_cast<cudaStream_t>(stream), nullptr, 0, 0, 0, stride, 1);
}

extern "C" int snnb_linear_lif(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                               const float* bias, int64_t N, float decay, float input_scale,
                               float v_threshold, float v_reset, int hard_reset, int variant,
                               int block_n, int splits, void* workspace, int64_t workspace_bytes,
                               void* out, snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || K > 0x7fffffff || N > 0x7fffffff) return SNNB_ERR_ARG;
    // a linear layer is a 1x1 "conv" over B images of 1 x 1 pixels
    return run_tc_layer(x, (int)T, (int)B, 1, 1, (int)K, w, bias, (int)N, 1, decay, input_scale,
                        v_threshold, v_reset, hard_reset, 0, variant, block_n, splits, workspace,
                        workspace_bytes, out, static_cast<cudaStream_t>(stream));
}

// Linear layer with a float32 result (no neuron): out[t*B + b, n] = x[t*B + b] @ w[n]^T + bias[n].
// Runs the T-folded tensor-core kernel with its raw-accumulator epilogue (one split, the
// output buffer as the partial-sum array), then adds the bias in place.
extern "C" int snnb_linear_f32(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                               const float* bias, int64_t N, float* out, snnb_stream_t stream) {
    if (!x || !w || !bias || !out) return SNNB_ERR_ARG;
    if (T <= 0 || B <= 0 || K <= 0 || N <= 0) return SNNB_ERR_ARG;
    if (T > 0x7fffffff || B > 0x7fffffff || K > 0x7fffffff || N > 0x7fffffff) return SNNB_ERR_ARG;
    if (!(T == 2 || T == 4 || T == 8)) return SNNB_ERR_UNSUPPORTED;
    if (K % 8 || N % 32) return SNNB_ERR_UNSUPPORTED;
    if (!aligned16(x) || !aligned16(w) || !aligned16(out)) return SNNB_ERR_ARG;
    int* status = device_status_ptr();
    if (!status) return SNNB_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int iT = (int)T, iB = (int)B, iK = (int)K, iN = (int)N;
    int bw, bh, bn;
    if (!choose_block(1, 1, 128 / iT, false, bw, bh, bn)) return SNNB_ERR_UNSUPPORTED;
    const int64_t mtiles = (iB + bn - 1) / bn;
    int BN = (iN % 128 == 0) ? 128 : (iN % 64 == 0 ? 64 : 32);
    while (BN > 32 && mtiles * (iN / BN) < 148) BN /= 2;
    CUtensorMap ta, tb;
    const uint64_t adims[5] = {(uint64_t)K, (uint64_t)T, 1, 1, (uint64_t)B};
    const uint64_t astr[4] = {(uint64_t)B * K * 2, (uint64_t)K * 2, (uint64_t)K * 2,
                              (uint64_t)K * 2};
    const uint32_t abox[5] = {64, (uint32_t)T, 1, 1, (uint32_t)bn};
    int rc = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, x, adims, astr, abox,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SNNB_OK) return rc;
    const uint64_t bdims[3] = {(uint64_t)K, 1, (uint64_t)N};
    const uint64_t bstr[2] = {(uint64_t)K * 2, (uint64_t)K * 2};
    const uint32_t bbox[3] = {64, 1, (uint32_t)BN};
    rc = encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, w, bdims, bstr, bbox,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SNNB_OK) return rc;
    ConvParams p = {};
    p.T = iT; p.B = iB; p.H = 1; p.W = 1; p.Cin = iK; p.Cout = iN;
    p.bw = bw; p.bh = bh; p.bn = bn;
    p.tiles_w = 1; p.tiles_h = 1;
    p.n_tiles_n = iN / BN;
    p.taps = 1; p.cin_blocks = (iK + 63) / 64; p.pool = 0;
    p.df = 0.f; p.sc = 0.f; p.thr = 0.f; p.v_reset = 0.f; p.hard = 1;
    p.bias = bias; p.out = nullptr; p.status = status;
    p.wq = w; p.wq_bytes = (int64_t)iN * iK * 2;
    p.res = nullptr; p.res_f32 = 0;
    p.splits = 1;
    p.partial = out;
    p.mtiles = (int)mtiles;
    p.num_tiles = (int)(mtiles * p.n_tiles_n);
    switch (iT) {
        case 2: rc = launch_tm_bn<2>(BN, ta, tb, p, s); break;
        case 4: rc = launch_tm_bn<4>(BN, ta, tb, p, s); break;
        default: rc = launch_tm_bn<8>(BN, ta, tb, p, s); break;
    }
    if (rc != SNNB_OK) return rc;
    return launch_splitsum(out, 1, (int64_t)T * B, iN, bias, s);
}

extern "C" int snnb_conv3x3_lif_packed(const void* x, int x_packed, int64_t T, int64_t B,
                                       int64_t H, int64_t W, int64_t Cin, const void* w,
                                       const float* bias, int64_t Cout, float decay,
                                       float input_scale, float v_threshold, float v_reset,
                                       int hard_reset, int pool, int out_packed, int block_n,
                                       void* out, snnb_stream_t stream) {
    if (T <= 0 || B <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0 || T > 0x7fffffff ||
        B > 0x7fffffff || H > 0x7fffffff || W > 0x7fffffff || Cin > 0x7fffffff ||
        Cout > 0x7fffffff)
        return SNNB_ERR_ARG;
    if (pool != 0 && pool != 1) return SNNB_ERR_ARG;
    return run_tc_layer(x, (int)T, (int)B, (int)H, (int)W, (int)Cin, w, bias, (int)Cout, 9, decay,
                        input_scale, v_threshold, v_reset, hard_reset, pool, 2, block_n, 1,
                        nullptr, 0, out, static_cast<cudaStream_t>(stream), nullptr, 0,
                        x_packed ? 1 : 0, out_packed ? 1 : 0);
}
extern "C" int snnb_conv3x3_lif_dense(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                                      int64_t Cin, const void* wd, const float* bias_d,
                                      int64_t Cout, float decay, float input_scale,
                                      float v_threshold, float v_reset, int hard_reset, int pool,
                                      int variant, int block_n, int splits, void* workspace,
                                      int64_t workspace_bytes, void* out, snnb_stream_t stream) {
    if (H < 1 || H > 2 || W < 1 || W > 2 || Cin <= 0 || Cout <= 0 || T <= 0 || B <= 0 ||
        T > 0x7fffffff || B > 0x7fffffff || Cin > 0x7fffffff || Cout > 0x7fffffff)
        return SNNB_ERR_ARG;
    if (pool && (H != 2 || W != 2)) return SNNB_ERR_UNSUPPORTED;
    // one image = one "pixel" of a linear layer with K = H*W*Cin inputs and H*W*Cout outputs
    return run_tc_layer(x, (int)T, (int)B, 1, 1, (int)(H * W * Cin), wd, bias_d,
                        (int)(H * W * Cout), 1, decay, input_scale, v_threshold, v_reset,
                        hard_reset, pool ? 2 : 0, variant, block_n, splits, workspace,
                        workspace_bytes, out, static_cast<cudaStream_t>(stream));
}
extern "C" int64_t snnb_split_workspace_bytes(int64_t T, int64_t B, int64_t H, int64_t W,
                                              int64_t Cout, int splits) {
    if (splits <= 1) return 0;
    return split_partial_bytes(splits, T, B, H, W, Cout);
}

extern "C" int snnb_read_device_status(snnb_stream_t stream, int* status_out) {
    if (!status_out) return SNNB_ERR_ARG;
    int* d = device_status_ptr();
    if (!d) return SNNB_ERR_CUDA;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, d, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess) e = cudaMemsetAsync(d, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return record_cuda_error(e);
    *status_out = h;
    return SNNB_OK;
}

// ---- split-K conv without any allocation ------------------------------------------------
// Some callers cannot hand this library a workspace: a plugin interface whose enqueue call
// offers no scratch buffer, a runtime whose device memory is fixed at start-up and that
// forbids cudaMalloc afterwards, or code that must not risk the implicit device
// synchronisation cudaMalloc / cudaFree can cause.  For them the split-K path of
// snnb_conv3x3_lif can use the fixed scratch array below instead of a caller buffer.
//
// The array lives in the library image: every GPU that loads libsnnb200.so holds these
// SNNB_STATIC_SCRATCH_BYTES until the process exits.  Host code must not use the symbol
// itself as a device address (on the host it only names a stand-in); the address is looked
// up once per device with cudaGetSymbolAddress and handed to the kernels.
#define SNNB_STATIC_SCRATCH_BYTES (16ll << 20)
static __device__ __align__(256) float g_static_scratch[SNNB_STATIC_SCRATCH_BYTES / 4];

namespace {
std::mutex g_static_scratch_lock;
void* g_static_scratch_ptr[64] = {nullptr};
}  // namespace

extern "C" int snnb_conv3x3_lif_static_scratch(
    const void* x, int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin, const void* w,
    const float* bias, int64_t Cout, float decay, float input_scale, float v_threshold,
    float v_reset, int hard_reset, int pool, int block_n, int splits, void* out,
    snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || H > 0x7fffffff || W > 0x7fffffff ||
        Cin > 0x7fffffff || Cout > 0x7fffffff || T <= 0 || B <= 0 || H <= 0 || W <= 0 ||
        Cout <= 0 || splits < 1 || splits > 8)
        return SNNB_ERR_ARG;
    const int64_t need = snnb_split_workspace_bytes(T, B, H, W, Cout, splits);
    // negative: the size overflows int64; above the array: exceeds the fixed scratch
    if (need < 0 || need > SNNB_STATIC_SCRATCH_BYTES) return SNNB_ERR_ARG;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return record_cuda_error(e);
    if (dev < 0 || dev >= 64) return SNNB_ERR_UNSUPPORTED;
    void* scratch = nullptr;
    {
        // first call on this device: resolve the array's device address (device current)
        std::lock_guard<std::mutex> guard(g_static_scratch_lock);
        if (!g_static_scratch_ptr[dev]) {
            void* ptr = nullptr;
            e = cudaGetSymbolAddress(&ptr, g_static_scratch);
            if (e != cudaSuccess) return record_cuda_error(e);
            g_static_scratch_ptr[dev] = ptr;
        }
        scratch = g_static_scratch_ptr[dev];
    }
    // Every element of the partial sums that is read was first written by this call, so
    // nothing in the scratch has to start at zero.
    return run_tc_layer(x, (int)T, (int)B, (int)H, (int)W, (int)Cin, w, bias, (int)Cout, 9,
                        decay, input_scale, v_threshold, v_reset, hard_reset, pool,
                        splits > 1 ? 2 : 0, block_n, splits, scratch, need > 0 ? need : 0, out,
                        static_cast<cudaStream_t>(stream));
}
