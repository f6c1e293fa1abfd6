// The T-folded fused conv + LIF kernel (variant 2 of csrc/conv_lif.cu) and the parameter
// block shared by every implicit-GEMM conv kernel.  Included by conv_lif.cu (single-CTA,
// CTA-pair and split-K forms) and conv_cluster.cu (cluster split-K form), so that the two
// translation units compile their instantiations in parallel.
#pragma once
#include <type_traits>

#include "tc_common.cuh"

namespace snnb {

constexpr int THREADS = 192;
constexpr int A_TILE_BYTES = 128 * 128;          // 128 rows x 64 bf16

struct ConvParams {
    int T, B, H, W, Cin, Cout;
    int bw, bh, bn;               // pixel block: bn images x bh rows x bw columns
    int tiles_w, tiles_h, n_tiles_n, num_tiles;
    int taps;                     // 9 (3x3 conv) or 1 (linear / 1x1)
    int cin_blocks;               // Cin / 64
    int pool;
    float df, sc, thr, v_reset;
    int hard;
    const float* bias;
    __nv_bfloat16* out;
    int* status;
    int splits;                   // k-range splits (T-folded kernel); 1 = none
    float* partial;               // split-K: f32 partial sums [splits][T][B*H*W][Cout]
    int mtiles;                   // pixel tiles per channel block (band kernel)
    int ring, a_bytes, w_bytes;   // band kernel: A ring depth, bytes per A stage, weight bytes
    const void* wq;               // the layer's weights in global memory, wq_bytes long
    int64_t wq_bytes;
    const void* res;              // residual input of the neuron or nullptr (no pooling then)
    int res_f32;                  // residual dtype: float32 (1) or bf16 (0)
    const uint32_t* xq;           // packed-spike input [T*B][H][W][Cin/32] (T-folded kernel)
    int out_packed;               // spikes stored packed, [T*B][Ho][Wo][Cout/32] uint32
    int pk_px, pk_ps;             // packed-input patch: words per pixel slot / per step plane
    int stall;                    // test hook (snnb_debug_inject_stall): CTA 0's producer of
                                  // the T-sequential kernel withholds every stage
    int stride;                   // conv stride (T-sequential and T-folded kernels): output
                                  // pixel (h, w) reads input (stride*h + dy - k/2, stride*w +
                                  // dx - k/2) for tap (dy, dx) of a k x k kernel; H, W above
                                  // are the OUTPUT sizes.  0 reads as 1.
    int ksize;                    // k of the k x k kernel (taps = k * k)
};

struct Tile {
    int w0, h0, img0, n0;
};

namespace {
// Residual input of the neuron, added after the bias as the reference's fused kernel does
// (x = y + b; x = x + residual: fused.py:97-108).  NHWC [T*B, H, W, Cout] of bf16 or
// float32 -- the unpooled output's layout.  8 consecutive channels from element idx
// (idx % 8 == 0: 16-byte aligned loads).
__device__ __forceinline__ void load_res8(const void* res, int res_f32, int64_t idx,
                                          float (&o)[8]) {
    if (res_f32) {
        const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(res) + idx);
        const float4 a = __ldg(q), b = __ldg(q + 1);
        o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
        o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
    } else {
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(
            static_cast<const __nv_bfloat16*>(res) + idx));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            o[2 * i] = __uint_as_float(w[i] << 16);
            o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
}
__device__ __forceinline__ float load_res1(const ConvParams& p, int64_t idx) {
    return p.res_f32 ? __ldg(static_cast<const float*>(p.res) + idx)
                     : __bfloat162float(static_cast<const __nv_bfloat16*>(p.res)[idx]);
}
__device__ __forceinline__ int64_t res_index(const ConvParams& p, int t, int on, int oh, int ow,
                                             int ch) {
    return ((((int64_t)t * p.B + on) * p.H + oh) * p.W + ow) * p.Cout + ch;
}
// r[j] = (r[j] + bias[j]) + residual[j] over one 32-channel slice of one output pixel; the
// bias is then consumed (set to 0) so the neuron's own "+ bias" adds nothing.
__device__ __forceinline__ void add_res_slice(const ConvParams& p, int64_t idx, float (&r)[32],
                                              float (&bias)[32]) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
        float rr[8];
        load_res8(p.res, p.res_f32, idx + 8 * u, rr);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            r[8 * u + k] = __fadd_rn(__fadd_rn(r[8 * u + k], bias[8 * u + k]), rr[k]);
            bias[8 * u + k] = 0.0f;
        }
    }
}

// Before waiting for the previous kernel: pull this CTA's share of the layer's weights
// (which no kernel writes) into L2, so the first weight stages of every CTA hit L2 instead
// of DRAM.  One thread, up to 64 KB per bulk prefetch.
__device__ __forceinline__ void prefetch_weights_l2(const ConvParams& p) {
    const int64_t per = ((p.wq_bytes + gridDim.x - 1) / gridDim.x + 15) & ~int64_t(15);
    const int64_t b0 = per * blockIdx.x;
    const int64_t b1 = b0 + per < p.wq_bytes ? b0 + per : p.wq_bytes;
    for (int64_t b = b0; b + 16 <= b1; b += 65536) {
        const int64_t n = (b1 - b < 65536 ? b1 - b : 65536) & ~int64_t(15);
        tc::prefetch_l2(static_cast<const uint8_t*>(p.wq) + b, (uint32_t)n);
    }
}


// bf16 elements of the spike output [T, B, Ho, Wo, Cout] (pool 0 / 1) -- the debug build's
// bound for the epilogue stores.
__device__ __forceinline__ int64_t out_elems(const ConvParams& p) {
    const int64_t hw = p.pool == 1 ? (int64_t)(p.H / 2) * (p.W / 2) : (int64_t)p.H * p.W;
    return (int64_t)p.T * p.B * hw * p.Cout;
}

__device__ __forceinline__ Tile decode_tile(int tile, const ConvParams& p, int BN) {
    const int nt = tile % p.n_tiles_n;
    const int mt = tile / p.n_tiles_n;
    const int tw = mt % p.tiles_w;
    const int th = (mt / p.tiles_w) % p.tiles_h;
    const int tn = mt / (p.tiles_w * p.tiles_h);
    return Tile{tw * p.bw, th * p.bh, tn * p.bn, nt * BN};
}


// NPT spikes (bits 0..NPT-1) as bf16 0/1 values at dst (2 * NPT bytes, aligned to them).
template <int NPT>
__device__ __forceinline__ void store_bits_bf16(__nv_bfloat16* dst, uint32_t bits) {
    auto two = [](uint32_t b2) {
        return ((b2 & 1u) ? 0x3F80u : 0u) | ((b2 & 2u) ? 0x3F800000u : 0u);
    };
    if constexpr (NPT == 8) {
        *reinterpret_cast<uint4*>(dst) = spikes_to_bf16x8(bits);
    } else if constexpr (NPT == 4) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(two(bits), two(bits >> 2));
    } else {
        *reinterpret_cast<uint32_t*>(dst) = two(bits);
    }
}

// ---- variant 2: T folded into M -----------------------------------------------------------
// For layers whose pixel count is too small to fill the GPU with 128-pixel blocks: the
// 128 accumulator rows of a tile are P = 128/TS pixels x TS steps (row p*TS + t), so the
// grid is TS times larger and each tile runs the K loop once.  One 5-D TMA box per k-slab
// (channels, step, w, h, image) lands each pixel's TS steps in consecutive rows of the A
// tile.  The epilogue (two sets of 4 warps, each taking 16 columns of every 32-column slice)
// finds a pixel's steps in TS adjacent lanes, transposes them in registers with shuffles so
// that a lane owns 16/TS columns at every step, runs the T recurrence there and stores the
// spikes directly (a warp's store of one step covers whole 32-byte sectors); 2x2 pooling ORs
// the column neighbour by a shuffle and the row neighbour through one shared-memory word.  Persistent, with two TMEM accumulators alternating between
// consecutive work items of a CTA.
//
// Split-K (p.partial != nullptr): work item = (tile, split); the split's k-slab range is
// accumulated and written as float32 partial sums [split][t][pixel][channel]; the neuron
// then runs in splitsum_lif_kernel, which adds the splits in a fixed order.
// Packed output of one epilogue slice: the TS lanes of a pixel (lane kq holds NPT columns of
// the set's 16 at every step, bit t * NPT + e of lb) gather the 16-channel half-word of every
// step, and lane kq stores step kq's at dst (already offset to step kq).
template <int TS, int NPT>
__device__ __forceinline__ void store_packed_halfword(unsigned short* dst, uint32_t lb, int kq,
                                                   bool ok) {
    uint32_t hw[TS];
#pragma unroll
    for (int t = 0; t < TS; ++t) hw[t] = ((lb >> (t * NPT)) & ((1u << NPT) - 1u)) << (kq * NPT);
#pragma unroll
    for (int bb = 1; bb < TS; bb <<= 1)
#pragma unroll
        for (int t = 0; t < TS; ++t) hw[t] |= __shfl_xor_sync(0xffffffffu, hw[t], bb);
    uint32_t mine = hw[0];
#pragma unroll
    for (int t = 1; t < TS; ++t) mine = kq == t ? hw[t] : mine;
    if (ok) *dst = (unsigned short)mine;
}

// PATCH: bytes of the packed-spike input patch (packed-input form; 0 otherwise)
template <int BN, int STAGES, int TS, int MH, int CG = 1, int PATCH = 0>
struct SmemTM {
    static constexpr int P = 128 / TS;
    static constexpr int NCH = BN / 32;
    static constexpr int B_TILE = BN / CG * 128;       // weight rows this CTA stages
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = STAGES * MH * A_TILE_BYTES;
    static constexpr int PATCH_OFF = B_OFF + STAGES * B_TILE;
    static constexpr int MASK_OFF = PATCH_OFF + PATCH;                 // 2 x 128 u32 (pool)
    static constexpr int SB_OFF = MASK_OFF + 256 * 4;                  // BN f32 (bias)
    static constexpr int BAR_OFF = (SB_OFF + BN * 4 + 7) & ~7;
    static constexpr int NBARS = 2 * STAGES + 4 * MH + 1 + 2;         // + cluster split-K
    static constexpr int TMEM_OFF = BAR_OFF + NBARS * 8;
    static constexpr int ABORT_OFF = TMEM_OFF + 4;
    static constexpr int TOTAL = ABORT_OFF + 4;
    static constexpr int DYN = TOTAL + 1024;
};

// NP producer warps (warp 0 and warps 6 ..) take the k-slab stages round-robin: each TMA
// issue occupies its thread for ~250 cycles whatever the box size, so one issuing thread
// cannot keep up with 4 MMAs per stage.
// MH M-tiles per work item (MH = 2: two 128-row tiles of the same channel block share each
// weight stage, so every weight byte brought into shared memory feeds twice the MMAs --
// these layers are bound by the L2 -> shared-memory stream of ~55 B/cycle per SM).  Each
// tile has its own pair of TMEM accumulators (slot = (item & 1) * MH + h).
// CG = 2: CTA pairs (clusters of 2) with M = 256 MMAs (cta_group::2).  A work item is two
// consecutive M-tiles (one per CTA) x BN channels; each CTA stages its own A tile and half
// of the BN weight rows, so per MMA cycle a CTA streams 2/3 (BN = 128) or 1/2 (BN = 256)
// of the bytes of the single-CTA form.  The even CTA waits for both CTAs' bytes on its
// full barrier and issues the MMAs; its commits arrive on both CTAs' barriers (stage free,
// accumulator ready); both epilogues hand the accumulator back on the even CTA's barrier.
// RES: the neuron input also takes p.res (a separate instantiation: the residual loads in
// the epilogue cost the plain form ~4% when compiled in behind a run-time test).
// Two sets of 4 epilogue warps (warps 2-5 and 5+NP .. 8+NP) split every 32-column slice of
// the accumulator into halves: the epilogue of a CTA's last work item, which no MMA
// overlaps, takes half as long (measured: 4.3 us of a conv9 launch's 21.5 us with one set).
// PKO: spikes stored packed; CPOOL: the column-group pool of the dense 2x2 form (pool == 2).
// Both are compile-time choices: a run-time test in the epilogue's loop cost epilogue-bound
// launches ~5%.  GEN: general tap coordinates -- conv stride p.stride and k x k kernels
// (p.ksize) -- for the strided / 5x5 / 7x7 convs (conv_strided.cu); without it the producers
// compute the stride-1 3x3 / 1x1 coordinates only (the general arithmetic in the same loop
// cost the VGG16 layers ~1%, measured A/B on one box).
template <int BN, int STAGES, int TS, bool HARD, int NP, int MH, int CG, bool RES, int SK = 1,
          int PATCH = 0, bool PKO = false, bool CPOOL = false, bool GEN = false>
__global__ void __launch_bounds__(THREADS + 32 * (NP - 1) + 128, 1)
conv_lif_tm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const ConvParams p) {
    constexpr bool PAIR = CG == 2;
    constexpr bool CK = SK > 1;
    constexpr bool PKI = PATCH > 0;                 // packed-spike input (see below)
    static_assert(!PKI || (MH == 1 && CG == 1 && !RES && SK == 1 && NP == 4),
                  "packed input: single CTA, one M-tile, four producer warps");
    // Producer warps taking the k-slabs round-robin must be no more than the ring's stages:
    // a warp then never runs two ring rounds ahead of the stage releases, the only case in
    // which the one-bit phase parity of its empty-slot wait could pass early.
    constexpr int NRR = PKI ? (NP < STAGES ? NP : STAGES) : NP;
    static_assert(PKI || NP <= STAGES, "more round-robin producers than ring stages");
    static_assert(!PAIR || MH == 1, "CTA pairs take one M-tile each");
    static_assert(!CK || (MH == 1 && CG == 1), "cluster split-K: one M-tile, single CTA");
    static_assert(!RES || (MH == 1 && CG == 1), "residual input: one M-tile, single CTA");
    using S = SmemTM<BN, STAGES, TS, MH, CG, PATCH>;
    constexpr int P = S::P, NCH = S::NCH;
    static_assert(!CK || NCH % SK == 0, "cluster split-K: whole 32-column slices per CTA");
    static_assert(!CK || BN * 128 * 4 <= STAGES * (MH * A_TILE_BYTES + S::B_TILE),
                  "cluster split-K: the partial sums fit in the drained ring");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    uint32_t* smask = reinterpret_cast<uint32_t*>(smem + S::MASK_OFF);
    float* sbias = reinterpret_cast<float*>(smem + S::SB_OFF);
    const uint32_t bar0 = sbase + S::BAR_OFF;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto accf_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto acce_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 * MH + a); };
    const uint32_t done_bar = bar0 + 8u * (2 * STAGES + 4 * MH);
    // cluster split-K: "every CTA's partial sums of epilogue set `set` are staged"
    auto staged_bar = [&](int set) { return bar0 + 8u * (2 * STAGES + 4 * MH + 1 + set); };
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + S::TMEM_OFF);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::ABORT_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = p.taps * p.cin_blocks;
    // cluster split-K: one work item (tile) per cluster, the CTA's cluster rank is its split
    const int splits = CK ? 1 : p.splits;
    const int num_items = p.num_tiles * splits;
    // work items of this CTA (a pair or a split-K cluster walks its items together)
    constexpr int CL = PAIR ? 2 : SK;
    const int item0 = (int)(blockIdx.x / CL);
    const int item_step = (int)(gridDim.x / CL);
    // bytes that complete a stage: this CTA's tiles, or both CTAs' for a pair
    constexpr uint32_t STAGE_TX = CG * (MH * A_TILE_BYTES + S::B_TILE);
    constexpr uint32_t TMEM_COLS = 2 * MH * BN < 32 ? 32 : 2 * MH * BN;
    static_assert(2 * MH * BN <= 512, "accumulators exceed TMEM");
    const uint32_t crank = (PAIR || CK) ? tc::cluster_rank() : 0u;
    const uint32_t rank = PAIR ? crank : 0u;         // a pair's M-tile offset
    // M-tile h of a work item; false when the item's last tile lies past the layer (odd
    // tile count) -- its box reads zeros and the epilogue stores nothing
    auto half_tile = [&](int item, int h, Tile& tl) {
        const int tile2 = item / splits;
        const int nt = tile2 % p.n_tiles_n;
        const int mt = (tile2 / p.n_tiles_n) * (MH * CG) + h + (int)rank;
        tl = decode_tile(mt * p.n_tiles_n + nt, p, BN);
        return mt < p.mtiles;
    };
    auto krange = [&](int item, int& k0, int& k1) {
        const int ns = CK ? SK : splits;
        const int s = CK ? (int)crank : item % splits;
        k0 = (int)((int64_t)KB * s / ns);
        k1 = (int)((int64_t)KB * (s + 1) / ns);
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            // packed input: the weight copy's expect_tx plus the arrival of the producer warp
            // that wrote the stage's A tile
            tc::mbar_init(full_bar(s), PKI ? 2 : 1);
            tc::mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2 * MH; ++a) {
            tc::mbar_init(accf_bar(a), 1);
            // single CTA: every epilogue thread arrives (2 sets of 128); pair: one arrival
            // per epilogue warp of either CTA, on the even CTA's barrier
            tc::mbar_init(acce_bar(a), PAIR ? 16 : 256);
        }
        tc::mbar_init(done_bar, 1);
        tc::mbar_init(staged_bar(0), SK);
        tc::mbar_init(staged_bar(1), SK);
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmA);
        tc::prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            tc::tmem_alloc_pair(sbase + S::TMEM_OFF, TMEM_COLS);
            tc::tmem_relinquish_pair();
        } else {
            tc::tmem_alloc(sbase + S::TMEM_OFF, TMEM_COLS);
            tc::tmem_relinquish();
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    // a cluster: every CTA's barriers initialised before any signals another's
    if constexpr (PAIR || CK) tc::cluster_sync();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    if (threadIdx.x == 64 && p.wq) prefetch_weights_l2(p);
    // Programmatic dependent launch: only the activation loads read what the previous
    // kernel wrote, so each producer waits for it just before its first activation load --
    // the tile decode, the first weight loads and every other role's setup overlap the
    // previous kernel's tail.  Everything this kernel writes follows those loads (through
    // the full / accumulator barriers).
    pdl_trigger();

    constexpr int W1 = 5 + NP;                    // first warp of the second epilogue set
    if (PKI && (warp == 0 || (warp >= 6 && warp < W1))) {
        // ------------------------------------------------ packed-input producers (NP == 4)
        // Per tile the four warps stage the packed spikes of the tile's pixels and their
        // 1-pixel halo at every step in shared memory ([t][image][PH][PW][Cin/32] words,
        // padded, zero outside the layer: the conv padding).  They then take the k-slabs (tap,
        // 64-channel block) round-robin (over min(4, STAGES) warps, see NRR): the slab's warp
        // copies its weight rows by TMA and
        // expands the 128 A rows (row = pixel * TS + step, the pixel shifted by the tap; lane
        // l writes rows l, l+32, l+64, l+96) to bf16 {0, 1} in the 128-byte-swizzled layout a
        // TMA box would have produced.
        if constexpr (PKI) {
            const int pi = warp == 0 ? 0 : warp - 5;
            const int prow = pi * 32 + lane;                 // this thread's patch-copy index
            const int PW = p.bw + 2, PH = p.bh + 2, CW = p.Cin >> 5;
            // patch layout in words (host-chosen): pixel slots of PX >= CW and step planes of
            // PS >= bn * PH * PW * PX -- padded when it fits, so that the 32 rows a warp reads
            // spread over the banks
            const int PX = p.pk_px, PS = p.pk_ps;
            // the patch word offset of each of this lane's 4 rows (tap (0, 0))
            int roff[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int rr = lane + 32 * i;
                const int px = rr / TS, pt = rr % TS;
                const int lw = px % p.bw, lh = (px / p.bw) % p.bh, ln = px / (p.bw * p.bh);
                roff[i] = pt * PS + ((ln * PH + lh) * PW + lw) * PX;
            }
            uint32_t* patch = reinterpret_cast<uint32_t*>(smem + S::PATCH_OFF);
            const int units = TS * p.bn * PH * PW * (CW >> 1);      // 8-byte units
            uint32_t g = 0, issued = 0, last_g = 0, failed = 0;
            bool dep_ready = false;
            for (int item = item0; item < num_items; item += item_step) {
                Tile tl;
                half_tile(item, 0, tl);
                int k0, k1;
                krange(item, k0, k1);
                if (!dep_ready) {
                    pdl_wait();                      // the patch is the previous kernel's output
                    dep_ready = true;
                }
                tc::named_bar_sync(4, NP * 32);      // the last tile's expansions are done
                // every unit an asynchronous 8-byte copy (zero fill outside the layer), all
                // in flight at once
                for (int u = prow; u < units; u += NP * 32) {
                    int q = u / (CW >> 1);
                    const int cu = u - q * (CW >> 1);
                    const int pw = q % PW; q /= PW;
                    const int ph = q % PH; q /= PH;
                    const int pn = q % p.bn;
                    const int t = q / p.bn;
                    const int gw = tl.w0 - 1 + pw, gh = tl.h0 - 1 + ph, gn = tl.img0 + pn;
                    const bool in = gw >= 0 && gw < p.W && gh >= 0 && gh < p.H && gn < p.B;
                    const uint32_t* src = in ? p.xq + ((((int64_t)t * p.B + gn) * p.H + gh) *
                                                           p.W + gw) * CW + 2 * cu
                                             : p.xq;
                    const int dw = t * PS + ((pn * PH + ph) * PW + pw) * PX + 2 * cu;
                    tc::cp_async_8(sbase + S::PATCH_OFF + (uint32_t)dw * 4u, src, in ? 8u : 0u);
                }
                tc::cp_async_wait_all();
                tc::named_bar_sync(4, NP * 32);      // patch complete
                for (int kb = k0; kb < k1; ++kb, ++g) {
                    if (g % NRR != (uint32_t)pi) continue;     // pi >= NRR: patch copies only
                    const int stage = (int)(g % STAGES);
                    const uint32_t phase = (g / STAGES) & 1u;
                    failed |= 1u - tc::mbar_wait_warp(empty_bar(stage), phase ^ 1u, failed);
                    const int tap = kb / p.cin_blocks;
                    const int cb = kb - tap * p.cin_blocks;
                    const int r = tap / 3, s = tap % 3;
                    if (!failed && tc::elect_one()) {
                        tc::mbar_expect_tx(full_bar(stage), (uint32_t)S::B_TILE);
                        tc::tma_load_3d(sbase + S::B_OFF + stage * S::B_TILE, &tmB,
                                        full_bar(stage), cb * 64, tap, tl.n0);
                    }
                    __syncwarp();
                    const int shift = (r * PW + s) * PX + cb * 2;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        if (failed) break;
                        const int prow = lane + 32 * i;          // A row written
                        const uint2 bits = *reinterpret_cast<const uint2*>(patch + roff[i] + shift);
                        uint8_t* rowp = smem + S::A_OFF + stage * A_TILE_BYTES + prow * 128;
                        // channel pairs (2i, 2i+1) of each 8-channel chunk -> one word of two
                        // bf16: the even and odd bits of the chunk's byte are brought to bytes
                        // 0 and 2 of v (one byte permute), (v >> 2i) & 0x10001 keeps the pair,
                        // and the multiply by 0x3F80 (bf16 1.0) writes both halves
                        const uint32_t ev[2] = {bits.x & 0x55555555u, bits.y & 0x55555555u};
                        const uint32_t od[2] = {(bits.x >> 1) & 0x55555555u,
                                                (bits.y >> 1) & 0x55555555u};
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const uint32_t k = (uint32_t)(j & 3);
                            const uint32_t v = __byte_perm(ev[j >> 2], od[j >> 2],
                                                           k | (k << 4) | ((k + 4) << 8) |
                                                               ((k + 4) << 12));
                            uint4 o;
                            o.x = (v & 0x10001u) * 0x3F80u;
                            o.y = ((v >> 2) & 0x10001u) * 0x3F80u;
                            o.z = ((v >> 4) & 0x10001u) * 0x3F80u;
                            o.w = ((v >> 6) & 0x10001u) * 0x3F80u;
                            *reinterpret_cast<uint4*>(rowp + ((j ^ (prow & 7)) << 4)) = o;
                        }
                    }
                    if (!failed) tc::fence_proxy_async_smem();   // visible to the tensor core
                    __syncwarp();
                    if (!failed) {
                        if (lane == 0) tc::mbar_arrive(full_bar(stage));
                        ++issued;
                        last_g = g;
                    }
                }
            }
            if (failed) {
                // this warp's weight copies still in flight: bounded waits
                uint32_t gg = last_g;
                for (uint32_t k = 0; k < issued && k * NRR < (uint32_t)STAGES; ++k, gg -= NRR)
                    tc::mbar_wait_warp<true>(full_bar((int)(gg % STAGES)), (gg / STAGES) & 1u, 0);
                if (lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
            }
        }
    } else if (warp == 0 || (warp >= 6 && warp < W1)) {
        // ------------------------------------------------------------- TMA producers
        // producer pi issues the stages g with g % NP == pi (g counts k-slabs over the
        // whole schedule, as the MMA warp does)
        const uint32_t pi = warp == 0 ? 0u : (uint32_t)(warp - 5);
        uint32_t g = 0, issued = 0, last_g = 0, failed = 0;
        bool dep_ready = false;                 // griddepcontrol.wait done (this warp)
        // GEN: the boxes traverse the input with the conv's stride; tap (r, s) of a k x k
        // kernel reads input (stride * h0 + r - k/2, stride * w0 + s - k/2)
        const int cst = GEN ? p.stride : 1;
        const int kk = GEN ? p.ksize : 3;
        for (int item = item0; item < num_items; item += item_step) {
            Tile tl[MH];
#pragma unroll
            for (int h = 0; h < MH; ++h) half_tile(item, h, tl[h]);
            int k0, k1;
            krange(item, k0, k1);
            for (int kb = k0; kb < k1; ++kb, ++g) {
                if (g % NP != pi) continue;
                const int stage = (int)(g % STAGES);
                const uint32_t phase = (g / STAGES) & 1u;
                failed |= 1u - tc::mbar_wait_warp(empty_bar(stage), phase ^ 1u, failed);
                const int tap = kb / p.cin_blocks;
                const int cb = kb - tap * p.cin_blocks;
                int r, s;                       // input offset of the tap from the pixel
                if constexpr (GEN) {
                    r = tap / kk;
                    s = tap - r * kk - (kk >> 1);
                    r -= kk >> 1;
                } else {
                    r = p.taps == 9 ? tap / 3 - 1 : 0;
                    s = p.taps == 9 ? tap % 3 - 1 : 0;
                }
                // the stage's weight rows first (no kernel writes them), then, once the
                // previous kernel has completed, its activation box(es)
                if (!failed && tc::elect_one()) {
                    if constexpr (PAIR) {
                        // both CTAs' bytes complete the even CTA's full barrier
                        const uint32_t fb = tc::map_to_rank(full_bar(stage), 0);
                        if (rank == 0) tc::mbar_expect_tx(full_bar(stage), STAGE_TX);
                        tc::tma_load_3d_pair(sbase + S::B_OFF + stage * S::B_TILE, &tmB, fb,
                                             cb * 64, tap, tl[0].n0 + (int)rank * (BN / 2));
                    } else {
                        tc::mbar_expect_tx(full_bar(stage), STAGE_TX);
                        tc::tma_load_3d(sbase + S::B_OFF + stage * S::B_TILE, &tmB,
                                        full_bar(stage), cb * 64, tap, tl[0].n0);
                    }
                }
                __syncwarp();
                if (!dep_ready) {
                    pdl_wait();
                    dep_ready = true;
                }
                if (!failed && tc::elect_one()) {
                    if constexpr (PAIR) {
                        const uint32_t fb = tc::map_to_rank(full_bar(stage), 0);
                        tc::tma_load_5d_pair(sbase + S::A_OFF + stage * A_TILE_BYTES, &tmA, fb,
                                             cb * 64, 0, tl[0].w0 * cst + s,
                                             tl[0].h0 * cst + r, tl[0].img0);
                    } else {
#pragma unroll
                        for (int h = 0; h < MH; ++h)
                            tc::tma_load_5d(sbase + S::A_OFF + (stage * MH + h) * A_TILE_BYTES,
                                            &tmA, full_bar(stage), cb * 64, 0,
                                            tl[h].w0 * cst + s, tl[h].h0 * cst + r,
                                            tl[h].img0);
                    }
                }
                __syncwarp();
                if (!failed) {
                    ++issued;
                    last_g = g;
                }
            }
        }
        if (failed) {
            // wait (bounded) for this producer's copies still in flight: on the full barrier,
            // or for the odd CTA of a pair (whose copies complete on the even CTA's barrier)
            // on the stage's release, which follows the MMAs that read them
            uint32_t gg = last_g;
            for (uint32_t k = 0; k < issued && k * NP < (uint32_t)STAGES; ++k, gg -= NP) {
                if (PAIR && rank != 0)
                    tc::mbar_wait_warp<true>(empty_bar((int)(gg % STAGES)), (gg / STAGES) & 1u, 0);
                else
                    tc::mbar_wait_warp<true>(full_bar((int)(gg % STAGES)), (gg / STAGES) & 1u, 0);
            }
            if (lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
        }
    } else if (warp == 1 && PAIR && rank != 0) {
        // odd CTA of a pair: the even CTA issues every MMA; its last commit says that this
        // CTA's TMEM and shared memory are no longer in use by the tensor pipe
        if (!tc::mbar_wait_warp<true>(done_bar, 0, 0) && lane == 0) {
            atomicExch(p.status, SNNB_ERR_TIMEOUT);
            *abort_flag = 1;
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        constexpr uint32_t IDESC = tc::idesc_bf16_f32(128 * CG, BN);
        int stage = 0;
        uint32_t phase = 0, it = 0, failed = 0;
        for (int item = item0; item < num_items; item += item_step, ++it) {
            int k0, k1;
            krange(item, k0, k1);
            const int a0 = (it & 1) * MH;            // this item's first accumulator slot
#pragma unroll
            for (int h = 0; h < MH; ++h)
                failed |= 1u - tc::mbar_wait_warp(acce_bar(a0 + h), ((it >> 1) & 1u) ^ 1u, failed);
            tc::tc_fence_after();
            for (int kb = k0; kb < k1; ++kb) {
                int nstage = stage + 1;
                uint32_t nphase = phase;
                if (nstage == STAGES) { nstage = 0; nphase ^= 1u; }
                // only the issuing lane waits for stages (the others meet it at __syncwarp),
                // and it waits for the next stage before committing this one: a wait queued
                // behind a commit would not return until the tensor pipe had drained
                if (tc::elect_one()) {
                    if (kb == k0) {
                        failed |= 1u - tc::mbar_wait_lane(full_bar(stage), phase, failed);
                        tc::tc_fence_after();
                    }
                    const uint64_t db = tc::sdesc_k_sw128(sbase + S::B_OFF + stage * S::B_TILE);
#pragma unroll
                    for (int h = 0; h < MH; ++h) {
                        const uint64_t da = tc::sdesc_k_sw128(sbase + S::A_OFF +
                                                              (stage * MH + h) * A_TILE_BYTES);
                        const uint32_t dcol = tmem + (a0 + h) * BN;
#pragma unroll
                        for (int k = 0; k < 4; ++k) {
                            if constexpr (PAIR)
                                tc::umma_bf16_pair(dcol, da + 2 * k, db + 2 * k, IDESC,
                                                   (kb > k0) || (k > 0));
                            else
                                tc::umma_bf16(dcol, da + 2 * k, db + 2 * k, IDESC,
                                              (kb > k0) || (k > 0));
                        }
                    }
                    if (kb + 1 < k1) {
                        failed |= 1u - tc::mbar_wait_lane(full_bar(nstage), nphase, failed);
                        tc::tc_fence_after();
                    }
                    if constexpr (PAIR) tc::umma_commit_pair(empty_bar(stage), 3);
                    else tc::umma_commit(empty_bar(stage));
                }
                __syncwarp();
                stage = nstage;
                phase = nphase;
            }
            if (tc::elect_one()) {
#pragma unroll
                for (int h = 0; h < MH; ++h) {
                    if constexpr (PAIR) tc::umma_commit_pair(accf_bar(a0 + h), 3);
                    else tc::umma_commit(accf_bar(a0 + h));
                }
            }
            __syncwarp();
            // lane 0 (the elected lane) owns the failure flag of the stage waits; the warp-wide
            // waits need the same skip value in every lane
            failed = __shfl_sync(0xffffffffu, failed, 0);
        }
        if (tc::elect_one()) {
            if constexpr (PAIR) tc::umma_commit_pair(done_bar, 3);
            else tc::umma_commit(done_bar);
        }
        __syncwarp();
        failed |= 1u - tc::mbar_wait_warp<true>(done_bar, 0, 0);
        if (failed && lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
    } else {
        const int set = warp >= W1 ? 1 : 0;             // which half of each slice
        const int q = warp & 3;                         // TMEM lane quadrant
        const int row = 32 * q + lane;                  // accumulator row = pixel * TS + step
        const int et = threadIdx.x - (set ? 32 * W1 : 64);   // 0..127 within the set
        const int et2 = set * 128 + et;                 // 0..255 over both sets
        constexpr int HC = 16;                          // columns of a slice per set
        constexpr int NPT = HC / TS;                    // columns per thread after the transpose
        // After the in-register transpose the TS lanes of a pixel (rows px*TS .. px*TS+TS-1)
        // hold its TS steps of NPT consecutive columns each: lane k of the group owns columns
        // k*NPT .. k*NPT+NPT-1 (of this set's 16) at every step.
        const int lx = row / TS, kq = row % TS;
        const int64_t npix_total = (int64_t)p.B * p.H * p.W;
        uint32_t it = 0, failed = 0;
        // hand accumulator a back to the MMA issuer (of the even CTA, for a pair)
        auto release_acc = [&](int a) {
            tc::tc_fence_before();
            if constexpr (PAIR) {
                __syncwarp();
                if (lane == 0) tc::mbar_arrive_cluster(tc::map_to_rank(acce_bar(a), 0));
            } else {
                tc::mbar_arrive(acce_bar(a));
            }
        };
        for (int item = item0; item < num_items; item += item_step, ++it) {
          if (!p.partial) {
            // the channel block's bias into shared memory before the accumulator is ready
            Tile t0;
            half_tile(item, 0, t0);
            tc::named_bar_sync(3, 256);              // both sets done with the last item's bias
            for (int i = et2; i < BN; i += 256) sbias[i] = __ldg(p.bias + t0.n0 + i);
            tc::named_bar_sync(3, 256);
          }
          for (int h = 0; h < MH; ++h) {
            Tile tl;
            half_tile(item, h, tl);
            const int a = (int)(it & 1) * MH + h;
            // (before the accumulator is ready) this lane's pixel in the layer
            const int lw = lx % p.bw, lh = (lx / p.bw) % p.bh, ln = lx / (p.bw * p.bh);
            const int ow = tl.w0 + lw, oh = tl.h0 + lh, on = tl.img0 + ln;
            const bool inside = ow < p.W && oh < p.H && on < p.B;
            const int Ho = p.H >> 1, Wo = p.W >> 1;
            // pooled: the window's top-left pixel stores (window inside the layer)
            const bool pool_store = ((lw | lh) & 1) == 0 && (ow >> 1) < Wo && (oh >> 1) < Ho &&
                                    on < p.B;
            failed |= 1u - tc::mbar_wait_warp(accf_bar(a), (it >> 1) & 1u, failed);
            tc::tc_fence_after();
            // transpose across the TS lanes of the pixel: block j (NPT columns) of the lane
            // with step t moves to the lane with k = j, slot t (butterfly over the bits of t;
            // each stage swaps half of the blocks with the partner lane).  Afterwards
            // r[t * NPT + e] = step t of column kq * NPT + e.
            auto transpose = [&](float (&r)[HC]) {
#pragma unroll
                for (int bb = TS / 2; bb >= 1; bb >>= 1) {
                    const bool hi = (kq & bb) != 0;
#pragma unroll
                    for (int j0 = 0; j0 < TS; ++j0) {
                        if (j0 & bb) continue;
                        const int j1 = j0 | bb;
#pragma unroll
                        for (int e = 0; e < NPT; ++e) {
                            const float snd = hi ? r[j0 * NPT + e] : r[j1 * NPT + e];
                            const float rcv = __shfl_xor_sync(0xffffffffu, snd, bb);
                            if (hi) r[j0 * NPT + e] = rcv;
                            else r[j1 * NPT + e] = rcv;
                        }
                    }
                }
            };
            int c_lo = 0, c_hi = NCH;
            if constexpr (CK) {
                // ---- cluster split-K, phase 1: this split's partial sums into the drained
                // ring, [slice][set][row][16 floats], the four float4 of a row rotated by
                // (row >> 1) & 3 so that 8 consecutive rows' 16-byte accesses hit distinct
                // banks; then this set's staged barrier in every CTA of the cluster
                float* stg = reinterpret_cast<float*>(smem + S::A_OFF);
                const int sw = (row >> 1) & 3;
#pragma unroll 1
                for (int c = 0; c < NCH; ++c) {
                    float r[HC];
                    tc::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + a * BN + c * 32 + set * HC, r);
                    tc::tmem_wait_ld();
                    float4* d = reinterpret_cast<float4*>(stg + ((c * 2 + set) * 128 + row) * HC);
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        d[j ^ sw] = make_float4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
                }
                release_acc(a);
                tc::named_bar_sync(1 + set, 128);       // the set's rows all staged
                if (et == 0) {
                    tc::fence_acq_rel_cluster();
                    for (int s = 0; s < SK; ++s)
                        tc::mbar_arrive_cluster(tc::map_to_rank(staged_bar(set), (uint32_t)s));
                }
                __syncwarp();
                failed |= 1u - tc::mbar_wait_warp_cluster(staged_bar(set), 0, failed);
                // phase 2: this CTA finishes slices c_lo .. c_hi-1 of the tile
                c_lo = (int)crank * (NCH / SK);
                c_hi = c_lo + NCH / SK;
            }
            if (p.partial) {
                // ---- split-K: raw float32 partial sums of this split, transposed like the
                // neuron path so that a warp's store of one step covers whole sectors
                const int split = item % splits;
                const int64_t gpix = ((int64_t)on * p.H + oh) * p.W + ow;
#pragma unroll 1
                for (int c = 0; c < NCH; ++c) {
                    float r[HC];
                    tc::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + a * BN + c * 32 + set * HC, r);
                    tc::tmem_wait_ld();
                    transpose(r);
                    if (inside) {
#pragma unroll
                        for (int t = 0; t < TS; ++t) {
                            float* d = p.partial + (((int64_t)split * p.T + t) * npix_total + gpix) * p.Cout +
                                       tl.n0 + c * 32 + set * HC + kq * NPT;
#pragma unroll
                            for (int e = 0; e < NPT; e += 2)
                                *reinterpret_cast<float2*>(d + e) = make_float2(r[t * NPT + e], r[t * NPT + e + 1]);
                        }
                    }
                }
                release_acc(a);
                continue;
            }
            // (not cluster split-K) the next slice's columns are loaded from TMEM while this
            // slice's neurons run
            float rn[HC];
            if constexpr (!CK)
                tc::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + a * BN + c_lo * 32 + set * HC, rn);
#pragma unroll 1
            for (int c = c_lo; c < c_hi; ++c) {
                float r[HC];
                if constexpr (CK) {
                    // the SK splits' partial sums of this row, added in split order
                    const uint32_t src = sbase + S::A_OFF +
                                         (uint32_t)(((c * 2 + set) * 128 + row) * HC * 4);
                    const int sw = (row >> 1) & 3;
#pragma unroll
                    for (int s = 0; s < SK; ++s) {
                        const uint32_t ra = tc::map_to_rank(src, (uint32_t)s);
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const float4 v4 = tc::ld_dsmem_f4(ra + 16u * (uint32_t)(j ^ sw));
                            if (s == 0) {
                                r[4 * j] = v4.x; r[4 * j + 1] = v4.y;
                                r[4 * j + 2] = v4.z; r[4 * j + 3] = v4.w;
                            } else {
                                r[4 * j] = __fadd_rn(r[4 * j], v4.x);
                                r[4 * j + 1] = __fadd_rn(r[4 * j + 1], v4.y);
                                r[4 * j + 2] = __fadd_rn(r[4 * j + 2], v4.z);
                                r[4 * j + 3] = __fadd_rn(r[4 * j + 3], v4.w);
                            }
                        }
                    }
                } else {
                    tc::tmem_wait_ld();
                    tc::reg_fence16(rn);                // rn is valid only after the wait
#pragma unroll
                    for (int e = 0; e < HC; ++e) r[e] = rn[e];
                    if (c + 1 < c_hi)
                        tc::tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + a * BN + (c + 1) * 32 +
                                      set * HC, rn);
                    if (c == NCH - 1) release_acc(a);   // accumulator fully read: hand it back
                }
                transpose(r);
                const int ch0 = c * 32 + set * HC + kq * NPT;        // column within the block
                uint32_t lb = 0;                    // bit t * NPT + e
                // column pairs on packed f32x2 operations (each component rounded as the
                // scalar operation: the same values, half the instructions)
                auto lif_cols = [&](auto with_res) {
                    constexpr bool WITH_RES = decltype(with_res)::value;
                    constexpr int NP2 = NPT / 2;
                    static_assert(NPT % 2 == 0, "column pairs");
                    const float2 df2 = make_float2(p.df, p.df), sc2 = make_float2(p.sc, p.sc);
                    float2 in[TS][NP2], v[NP2];
#pragma unroll
                    for (int e = 0; e < NP2; ++e) {
                        const float2 bb = *reinterpret_cast<const float2*>(sbias + ch0 + 2 * e);
                        v[e] = make_float2(0.0f, 0.0f);
#pragma unroll
                        for (int t = 0; t < TS; ++t)
                            in[t][e] = __fadd2_rn(make_float2(r[t * NPT + 2 * e],
                                                              r[t * NPT + 2 * e + 1]), bb);
                    }
                    if constexpr (WITH_RES) {
                        if (inside) {
#pragma unroll
                            for (int t = 0; t < TS; ++t)
#pragma unroll
                                for (int e = 0; e < NP2; ++e) {
                                    in[t][e].x = __fadd_rn(in[t][e].x, load_res1(p, res_index(
                                        p, t, on, oh, ow, tl.n0 + ch0 + 2 * e)));
                                    in[t][e].y = __fadd_rn(in[t][e].y, load_res1(p, res_index(
                                        p, t, on, oh, ow, tl.n0 + ch0 + 2 * e + 1)));
                                }
                        }
                    }
#pragma unroll
                    for (int t = 0; t < TS; ++t) {
#pragma unroll
                        for (int e = 0; e < NP2; ++e) {
                            // charge(): decay * v + input_scale * in, each product rounded
                            const float2 vv = __fadd2_rn(__fmul2_rn(df2, v[e]),
                                                         __fmul2_rn(sc2, in[t][e]));
                            const bool s0 = vv.x >= p.thr, s1 = vv.y >= p.thr;
                            v[e] = make_float2(reset_v<HARD>(vv.x, s0, p.thr, p.v_reset),
                                               reset_v<HARD>(vv.y, s1, p.thr, p.v_reset));
                            lb |= (s0 ? 1u : 0u) << (t * NPT + 2 * e);
                            lb |= (s1 ? 1u : 0u) << (t * NPT + 2 * e + 1);
                        }
                    }
                };
                lif_cols(std::integral_constant<bool, RES>{});
                const int ch = tl.n0 + ch0;
                // packed output: the TS lanes of a pixel gather the set's 16 channels of every
                // step (bit = channel within the half-word) and lane kq stores step kq
                auto store_packed = [&](bool ok, int y, int x, int Hs, int Ws) {
                    store_packed_halfword<TS, NPT>(
                        reinterpret_cast<unsigned short*>(p.out) +
                            ((((int64_t)kq * p.B + on) * Hs + y) * Ws + x) * (p.Cout >> 4) +
                            ((tl.n0 + c * 32) >> 4) + set,
                        lb, kq, ok);
                };
                if constexpr (CPOOL) {
                    // dense form of a pooled 2x2-image layer (taps == 1, H == W == 1): the
                    // columns are ordered (channel, pixel), so the 2x2 max-pool is an OR over
                    // 4 consecutive columns -- NPT / 4 groups per lane, or (NPT == 2) half a
                    // group, completed by the neighbouring lane
                    if constexpr (NPT == 2) lb |= __shfl_xor_sync(0xffffffffu, lb, 1);
                    if (inside && (NPT >= 4 || (kq & 1) == 0)) {
                        constexpr int G = NPT >= 4 ? NPT / 4 : 1;
                        constexpr uint32_t GM = NPT >= 4 ? 0xfu : 0x3u;
                        unsigned short* o = reinterpret_cast<unsigned short*>(p.out) +
                                            (int64_t)on * (p.Cout >> 2) + (ch >> 2);
                        const int64_t tstride = (int64_t)p.B * (p.Cout >> 2);
#pragma unroll
                        for (int t = 0; t < TS; ++t)
#pragma unroll
                            for (int gi = 0; gi < G; ++gi)
                                o[t * tstride + gi] =
                                    ((lb >> (t * NPT + 4 * gi)) & GM) ? 0x3F80u : 0u;
                    }
                } else if (PKO && !p.pool) {
                    store_packed(inside, oh, ow, p.H, p.W);
                } else if (!p.pool) {
                    if (inside) {
#pragma unroll
                        for (int t = 0; t < TS; ++t) {
                            const int64_t e = ((((int64_t)t * p.B + on) * p.H + oh) * p.W + ow) *
                                                  p.Cout + ch;
                            if (SNNB_IN_BOUNDS(e + NPT - 1, out_elems(p), p.status))
                                store_bits_bf16<NPT>(p.out + e, (lb >> (t * NPT)) & ((1u << NPT) - 1u));
                        }
                    }
                } else {
                    // 2x2 max-pool = OR: the column neighbour is TS lanes away; the row
                    // neighbour (bw pixels away, possibly in another warp) through shared memory
                    lb |= __shfl_xor_sync(0xffffffffu, lb, TS);
                    smask[set * 128 + row] = lb;
                    tc::named_bar_sync(1 + set, 128);    // row neighbours' bits visible
                    lb |= smask[set * 128 + (row ^ (TS * p.bw))];
                    if (PKO) {
                        store_packed(pool_store, oh >> 1, ow >> 1, Ho, Wo);
                    } else if (pool_store) {
#pragma unroll
                        for (int t = 0; t < TS; ++t) {
                            const int64_t e = ((((int64_t)t * p.B + on) * Ho + (oh >> 1)) * Wo +
                                               (ow >> 1)) * p.Cout + ch;
                            if (SNNB_IN_BOUNDS(e + NPT - 1, out_elems(p), p.status))
                                store_bits_bf16<NPT>(p.out + e, (lb >> (t * NPT)) & ((1u << NPT) - 1u));
                        }
                    }
                    tc::named_bar_sync(1 + set, 128);    // smask free for the next slice
                }
            }
          }
        }
        if (failed && lane == 0) { atomicExch(p.status, SNNB_ERR_TIMEOUT); *abort_flag = 1; }
    }
    tc::tc_fence_before();
    __syncthreads();
    // a pair: neither CTA leaves (or frees TMEM) while the other may still signal its
    // barriers or have its shared memory read by the tensor pipe; a split-K cluster: while
    // another CTA may still read its partial sums
    if constexpr (PAIR || CK) tc::cluster_sync();
    if (warp == 1) {
        tc::tc_fence_after();
        if constexpr (PAIR) tc::tmem_dealloc_pair(tmem, TMEM_COLS);
        else tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

}  // namespace

// Cluster split-K launch of conv_lif_tm_kernel (conv_cluster.cu): the SK k-range splits of
// a tile run as one thread-block cluster and reduce their partial sums through distributed
// shared memory, so the neuron runs in the same launch.
int launch_tm_cluster(int TS, int BN, int SK, const CUtensorMap& ta, const CUtensorMap& tb,
                      const ConvParams& p, cudaStream_t s);

// Strided and k x k (k in {1, 3, 5, 7}) convs on conv_lif_tm_kernel with general tap
// coordinates (GEN; conv_strided.cu): single-CTA T-folded form, any split count, residual
// or not.
int launch_tm_general(int TS, int BN, const CUtensorMap& ta, const CUtensorMap& tb,
                      const ConvParams& p, cudaStream_t s);

// Packed-spike launches of conv_lif_tm_kernel (conv_packed.cu): packed input (PATCH > 0)
// and / or packed output (PKO); packed_patch_limit() is the largest input patch (bytes) one
// CTA stages.
int launch_tm_packed(int TS, int BN, int x_packed, int out_packed, const CUtensorMap& ta,
                     const CUtensorMap& tb, const ConvParams& p, cudaStream_t s);
int packed_patch_limit();
// The dense form of a pooled 2x2-image layer (CPOOL; conv_packed.cu): plain T-folded kernel
// whose epilogue ORs groups of 4 consecutive columns.
int launch_tm_cpool(int TS, int BN, const CUtensorMap& ta, const CUtensorMap& tb,
                    const ConvParams& p, cudaStream_t s);

}  // namespace snnb
