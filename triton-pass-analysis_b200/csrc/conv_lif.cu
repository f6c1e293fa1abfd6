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
#include "tc_common.cuh"

namespace snnb {

__device__ int g_device_status = 0;

namespace {

constexpr int THREADS = 192;
constexpr int A_TILE_BYTES = 128 * 128;          // 128 rows x 64 bf16

struct ConvParams {
    int T, B, H, W, Cin, Cout;
    int bw, bh, bn;               // pixel block: bn images x bh rows x bw columns (product 128)
    int tiles_w, tiles_h, n_tiles_n;
    int taps;                     // 9 (3x3 conv) or 1 (linear / 1x1)
    int cin_blocks;               // Cin / 64
    int pool;
    int mode;                     // 0: LIF spikes bf16;  1: mean over T of (acc + bias), f32;
                                  // 2: per-step (acc + bias), f32 [T*B, Cout]
    float df, sc, thr, v_reset;
    int hard;
    const float* bias;
    void* out;
    int* status;
};

template <int BN, int STAGES>
struct Smem {
    static constexpr int B_TILE = BN * 128;
    static constexpr int A_OFF = 0;
    static constexpr int B_OFF = STAGES * A_TILE_BYTES;
    static constexpr int MASK_OFF = B_OFF + STAGES * B_TILE;          // (BN/32) x 128 u32
    static constexpr int BIAS_OFF = MASK_OFF + (BN / 32 > 0 ? BN / 32 : 1) * 128 * 4;
    static constexpr int BAR_OFF = BIAS_OFF + BN * 4;
    static constexpr int NBARS = 2 * STAGES + 4;
    static constexpr int TMEM_OFF = BAR_OFF + NBARS * 8;
    static constexpr int ABORT_OFF = TMEM_OFF + 4;
    static constexpr int TOTAL = ABORT_OFF + 4;
    static constexpr int DYN = TOTAL + 1024;     // slack for 1024-byte alignment
};

__device__ __forceinline__ uint4 spikes_to_bf16x8(uint32_t bits8) {
    uint4 r;
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t lo = ((bits8 >> (2 * i)) & 1u) ? 0x3F80u : 0u;
        const uint32_t hi = ((bits8 >> (2 * i + 1)) & 1u) ? 0x3F800000u : 0u;
        w[i] = lo | hi;
    }
    r.x = w[0]; r.y = w[1]; r.z = w[2]; r.w = w[3];
    return r;
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(THREADS, 1)
conv_lif_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const ConvParams p) {
    using S = Smem<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    uint32_t* smask = reinterpret_cast<uint32_t*>(smem + S::MASK_OFF);
    float* sbias = reinterpret_cast<float*>(smem + S::BIAS_OFF);
    const uint32_t bar0 = sbase + S::BAR_OFF;
    // barrier addresses
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto accf_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + a); };
    auto acce_bar = [&](int a) { return bar0 + 8u * (2 * STAGES + 2 + a); };
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + S::TMEM_OFF);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + S::ABORT_OFF);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nt = blockIdx.x % p.n_tiles_n;
    const int mt = blockIdx.x / p.n_tiles_n;
    const int tw = mt % p.tiles_w;
    const int th = (mt / p.tiles_w) % p.tiles_h;
    const int tn = mt / (p.tiles_w * p.tiles_h);
    const int w0 = tw * p.bw, h0 = th * p.bh, img0 = tn * p.bn, n0 = nt * BN;
    const int KB = p.taps * p.cin_blocks;
    constexpr uint32_t STAGE_TX = A_TILE_BYTES + S::B_TILE;
    constexpr uint32_t TMEM_COLS = (2 * BN < 32) ? 32 : 2 * BN;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            tc::mbar_init(full_bar(s), 1);
            tc::mbar_init(empty_bar(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            tc::mbar_init(accf_bar(a), 1);
            tc::mbar_init(acce_bar(a), 128);
        }
        *abort_flag = 0;
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmA);
        tc::prefetch_tmap(&tmB);
    }
    for (int i = threadIdx.x; i < BN; i += THREADS) {
        const int c = n0 + i;
        sbias[i] = (p.bias && c < p.Cout) ? p.bias[c] : 0.0f;
    }
    if (warp == 1) {
        tc::tmem_alloc(sbase + S::TMEM_OFF, TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------- TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            int issued = 0;
            bool ok = true;
            for (int t = 0; t < p.T && ok; ++t) {
                const int f0 = t * p.B + img0;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!tc::mbar_wait(empty_bar(stage), phase ^ 1u, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    const int tap = kb / p.cin_blocks;
                    const int cb = kb - tap * p.cin_blocks;
                    const int r = p.taps == 9 ? tap / 3 : 1;
                    const int s = p.taps == 9 ? tap % 3 : 1;
                    tc::mbar_expect_tx(full_bar(stage), STAGE_TX);
                    tc::tma_load_4d(sbase + S::A_OFF + stage * A_TILE_BYTES, &tmA, full_bar(stage),
                                    cb * 64, w0 + s - 1, h0 + r - 1, f0);
                    tc::tma_load_2d(sbase + S::B_OFF + stage * S::B_TILE, &tmB, full_bar(stage),
                                    tap * p.Cin + cb * 64, n0);
                    ++issued;
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
            }
            if (!ok) {
                // drain: wait (bounded) for the copies still in flight in every ring slot
                for (int k = 0; k < STAGES && k < issued; ++k) {
                    if (--stage < 0) { stage = STAGES - 1; phase ^= 1u; }
                    const long long t0 = clock64();
                    while (!tc::mbar_try_wait(full_bar(stage), phase) &&
                           clock64() - t0 < tc::WAIT_LIMIT_CYCLES) {
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t IDESC = tc::idesc_bf16_f32(128, BN);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = 0; t < p.T && ok; ++t) {
                const int a = t & 1;
                if (!tc::mbar_wait(acce_bar(a), ((t >> 1) & 1) ^ 1u, abort_flag, p.status)) break;
                tc::tc_fence_after();
                const uint32_t dcol = tmem + a * BN;
                for (int kb = 0; kb < KB; ++kb) {
                    if (!tc::mbar_wait(full_bar(stage), phase, abort_flag, p.status)) {
                        ok = false;
                        break;
                    }
                    tc::tc_fence_after();
                    const uint32_t sa = sbase + S::A_OFF + stage * A_TILE_BYTES;
                    const uint32_t sb = sbase + S::B_OFF + stage * S::B_TILE;
                    const uint64_t da = tc::sdesc_k_sw128(sa);
                    const uint64_t db = tc::sdesc_k_sw128(sb);
#pragma unroll
                    for (int k = 0; k < 4; ++k)   // 4 x K=16 inside the 128-byte swizzle atom
                        tc::umma_bf16(dcol, da + 2 * k, db + 2 * k, IDESC, (kb | k) != 0);
                    tc::umma_commit(empty_bar(stage));
                    if (++stage == STAGES) { stage = 0; phase ^= 1u; }
                }
                if (ok) tc::umma_commit(accf_bar(a));
            }
        }
    } else {
        // ------------------------------------------------------------- epilogue
        const int q = warp & 3;                  // TMEM lane quadrant of this warp
        const int m = 32 * q + lane;             // pixel row of the tile
        const int et = threadIdx.x - 64;         // 0..127
        const int mw = m % p.bw, mh = (m / p.bw) % p.bh, mn = m / (p.bw * p.bh);
        const int gw = w0 + mw, gh = h0 + mh, gimg = img0 + mn;
        const bool row_valid = gw < p.W && gh < p.H && gimg < p.B;
        float v[BN];
#pragma unroll
        for (int j = 0; j < BN; ++j) v[j] = 0.0f;
        for (int t = 0; t < p.T; ++t) {
            const int a = t & 1;
            if (!tc::mbar_wait(accf_bar(a), (t >> 1) & 1, abort_flag, p.status)) break;
            tc::tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + a * BN;
            if (BN >= 32) {
#pragma unroll
                for (int c = 0; c < BN / 32; ++c) {
                    float r[32];
                    tc::tmem_ld32(tbase + c * 32, r);
                    tc::tmem_wait_ld();
                    uint32_t mask = 0;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float in = __fadd_rn(r[j], sbias[c * 32 + j]);
                        if (p.mode == 0) {
                            float vv = charge(v[c * 32 + j], p.df, p.sc, in);
                            const bool s = vv >= p.thr;
                            vv = p.hard ? (s ? p.v_reset : vv) : (s ? __fsub_rn(vv, p.thr) : vv);
                            v[c * 32 + j] = vv;
                            mask |= (s ? 1u : 0u) << j;
                        } else {
                            v[c * 32 + j] = p.mode == 1 ? __fadd_rn(v[c * 32 + j], in) : in;
                        }
                    }
                    smask[c * 128 + m] = mask;
                }
            } else {
                float r[16];
                tc::tmem_ld16(tbase, r);
                tc::tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < BN && j < 16; ++j) {
                    const float in = __fadd_rn(r[j], sbias[j]);
                    v[j] = p.mode == 1 ? __fadd_rn(v[j], in) : in;   // BN < 32: head modes only
                }
            }
            tc::tc_fence_before();
            tc::mbar_arrive(acce_bar(a));
            if (p.mode == 2) {
                if (row_valid) {
                    float* outf = static_cast<float*>(p.out);
                    const int64_t row = (int64_t)t * p.B + gimg;
#pragma unroll
                    for (int j = 0; j < BN; ++j) {
                        const int c = n0 + j;
                        if (c < p.Cout) outf[row * p.Cout + c] = v[j];
                    }
                }
                continue;
            }
            if (p.mode != 0) continue;
            tc::named_bar_sync(1, 128);
            // ---- store the spikes of step t
            const int nchunks = BN / 32;
            __nv_bfloat16* out = static_cast<__nv_bfloat16*>(p.out);
            if (p.pool) {
                const int pw = p.bw / 2, ph = p.bh / 2;
                const int npix = pw * ph * p.bn;
                const int Ho = p.H / 2, Wo = p.W / 2;
                for (int item = et; item < npix * nchunks; item += 128) {
                    const int pix = item / nchunks, c = item - pix * nchunks;
                    const int xw = pix % pw, xh = (pix / pw) % ph, xn = pix / (pw * ph);
                    const int m00 = 2 * xw + p.bw * (2 * xh + p.bh * xn);
                    const uint32_t bits = smask[c * 128 + m00] | smask[c * 128 + m00 + 1] |
                                          smask[c * 128 + m00 + p.bw] |
                                          smask[c * 128 + m00 + p.bw + 1];
                    const int ow = w0 / 2 + xw, oh = h0 / 2 + xh, on = img0 + xn;
                    if (ow >= Wo || oh >= Ho || on >= p.B) continue;
                    const int64_t base =
                        ((((int64_t)t * p.B + on) * Ho + oh) * Wo + ow) * p.Cout + n0 + c * 32;
                    uint4* dst = reinterpret_cast<uint4*>(out + base);
#pragma unroll
                    for (int k = 0; k < 4; ++k) dst[k] = spikes_to_bf16x8((bits >> (8 * k)) & 0xffu);
                }
            } else {
                for (int item = et; item < 128 * nchunks; item += 128) {
                    const int pix = item / nchunks, c = item - pix * nchunks;
                    const int xw = pix % p.bw, xh = (pix / p.bw) % p.bh, xn = pix / (p.bw * p.bh);
                    const int ow = w0 + xw, oh = h0 + xh, on = img0 + xn;
                    if (ow >= p.W || oh >= p.H || on >= p.B) continue;
                    const uint32_t bits = smask[c * 128 + pix];
                    const int64_t base =
                        ((((int64_t)t * p.B + on) * p.H + oh) * p.W + ow) * p.Cout + n0 + c * 32;
                    uint4* dst = reinterpret_cast<uint4*>(out + base);
#pragma unroll
                    for (int k = 0; k < 4; ++k) dst[k] = spikes_to_bf16x8((bits >> (8 * k)) & 0xffu);
                }
            }
            tc::named_bar_sync(1, 128);
        }
        if (p.mode == 1 && row_valid) {
            // mean over T of (acc + bias): f32 [B, Cout] (linear layers: pixel = image)
            float* out = static_cast<float*>(p.out);
            const float inv = 1.0f / (float)p.T;
            const int64_t row = (int64_t)gimg;
#pragma unroll
            for (int j = 0; j < BN; ++j) {
                const int c = n0 + j;
                if (c < p.Cout) out[row * p.Cout + c] = __fmul_rn(v[j], inv);
            }
        }
        (void)row_valid;
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// ---- first layer: real-valued image, Cin = 3, fp32 SIMT ------------------------------
// Direct 3x3 conv in float32 (the image is not exact in bf16) + bias + multi-step LIF.
// x: f32 NCHW [Ti, B, Cin, H, W] with Ti = T, or Ti = 1 for direct encoding (the same
// image at every step: the conv is computed once).  w: f32 [Cout, Cin, 3, 3] (torch
// layout).  out: bf16 NHWC spikes [T*B, Ho, Wo, Cout] (pooled if requested).
// Thread = one output pixel x 8 output channels; the LIF state lives in registers.
__global__ void __launch_bounds__(256) first_conv_lif_kernel(
    const float* __restrict__ x, int Ti, int T, int B, int Cin, int H, int W,
    const float* __restrict__ w, const float* __restrict__ bias, int Cout,
    float df, float sc, float thr, float v_reset, int hard, int pool,
    __nv_bfloat16* __restrict__ out) {
    const int groups = Cout / 8;
    const int Ho = pool ? H / 2 : H, Wo = pool ? W / 2 : W;
    const int64_t total = (int64_t)B * Ho * Wo * groups;
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= total) return;
    const int g = (int)(gid % groups);
    int64_t r = gid / groups;
    const int ow = (int)(r % Wo); r /= Wo;
    const int oh = (int)(r % Ho);
    const int b = (int)(r / Ho);
    const int npix = pool ? 4 : 1;
    float v[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
    float y[4][8];
    for (int t = 0; t < T; ++t) {
        const int ti = Ti == 1 ? 0 : t;
        if (ti == t || t == 0) {
            for (int pi = 0; pi < npix; ++pi) {
                const int h = pool ? 2 * oh + (pi >> 1) : oh;
                const int ww = pool ? 2 * ow + (pi & 1) : ow;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int co = g * 8 + j;
                    float acc = 0.0f;
                    for (int ci = 0; ci < Cin; ++ci) {
                        const float* xc = x + (((int64_t)ti * B + b) * Cin + ci) * H * W;
                        const float* wc = w + ((int64_t)co * Cin + ci) * 9;
#pragma unroll
                        for (int kh = 0; kh < 3; ++kh) {
                            const int ih = h + kh - 1;
                            if (ih < 0 || ih >= H) continue;
#pragma unroll
                            for (int kw = 0; kw < 3; ++kw) {
                                const int iw = ww + kw - 1;
                                if (iw < 0 || iw >= W) continue;
                                acc = __fmaf_rn(__ldg(xc + ih * W + iw), __ldg(wc + kh * 3 + kw), acc);
                            }
                        }
                    }
                    y[pi][j] = acc;
                }
            }
        }
        uint32_t bits = 0;
        for (int pi = 0; pi < npix; ++pi) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float in = __fadd_rn(y[pi][j], __ldg(bias + g * 8 + j));
                float vv = charge(v[pi][j], df, sc, in);
                const bool s = vv >= thr;
                vv = hard ? (s ? v_reset : vv) : (s ? __fsub_rn(vv, thr) : vv);
                v[pi][j] = vv;
                bits |= (s ? 1u : 0u) << j;
            }
        }
        const int64_t o = ((((int64_t)t * B + b) * Ho + oh) * Wo + ow) * Cout + g * 8;
        *reinterpret_cast<uint4*>(out + o) = spikes_to_bf16x8(bits & 0xffu);
    }
}

template <int BN, int STAGES>
int launch_conv(const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p, int grid,
                cudaStream_t s) {
    using S = Smem<BN, STAGES>;
    cudaError_t e = cudaFuncSetAttribute(conv_lif_kernel<BN, STAGES>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, S::DYN);
    if (e != cudaSuccess) return record_cuda_error(e);
    conv_lif_kernel<BN, STAGES><<<grid, THREADS, S::DYN, s>>>(ta, tb, p);
    return launch_status();
}

// Pixel block of 128 rows for an H x W image batch: full rows when W <= 128, pairs
// of rows / columns kept even for pooling.
bool choose_block(int H, int W, int& bw, int& bh, int& bn) {
    if (W >= 128) {
        if (W % 128) return false;
        bw = 128; bh = 1; bn = 1;
        return true;
    }
    if (128 % W) return false;
    bw = W;
    const int rows = 128 / W;
    if (H >= rows) {
        if (H % rows) return false;
        bh = rows; bn = 1;
    } else {
        if (rows % H) return false;
        bh = H; bn = rows / H;
    }
    return true;
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
                CUtensorMapSwizzle swizzle) {
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
        es[i] = 1;
        if (i < rank - 1) st[i] = strides_bytes[i];
    }
    CUresult r = fn(map, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, st, b, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? SNNB_OK : SNNB_ERR_ARG;
}

namespace {

// Shared host path of the conv / linear entries.
int run_tc_layer(const void* x, int T, int B, int H, int W, int Cin, const void* w,
                 const float* bias, int Cout, int taps, float df, float sc, float thr,
                 float v_reset, int hard, int pool, int mode, void* out, cudaStream_t s) {
    if (!x || !w || !out) return SNNB_ERR_ARG;
    if (T <= 0 || B <= 0 || H <= 0 || W <= 0 || Cin <= 0 || Cout <= 0) return SNNB_ERR_ARG;
    if (Cin % 64 != 0) return SNNB_ERR_UNSUPPORTED;
    if (!aligned16(x) || !aligned16(w) || !aligned16(out)) return SNNB_ERR_ARG;
    int bw, bh, bn;
    if (!choose_block(H, W, bw, bh, bn)) return SNNB_ERR_UNSUPPORTED;
    if (pool && ((H % 2) || (W % 2) || (bw % 2) || (bh % 2))) return SNNB_ERR_UNSUPPORTED;
    if ((int64_t)T * B > 0x7fffffff / 2) return SNNB_ERR_ARG;
    int BN;
    if (mode != 0) {
        BN = Cout <= 16 ? 16 : (Cout <= 32 ? 32 : 64);
    } else {
        if (Cout % 32) return SNNB_ERR_UNSUPPORTED;
        BN = (Cout % 128 == 0) ? 128 : (Cout % 64 == 0 ? 64 : 32);
    }
    int* status = device_status_ptr();
    if (!status) return SNNB_ERR_CUDA;
    // activation map: dims (Cin, W, H, T*B), box (64, bw, bh, bn)
    CUtensorMap ta, tb;
    const uint64_t adims[4] = {(uint64_t)Cin, (uint64_t)W, (uint64_t)H, (uint64_t)T * B};
    const uint64_t astr[3] = {(uint64_t)Cin * 2, (uint64_t)W * Cin * 2, (uint64_t)H * W * Cin * 2};
    const uint32_t abox[4] = {64, (uint32_t)bw, (uint32_t)bh, (uint32_t)bn};
    int rc = encode_tmap(&ta, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, x, adims, astr, abox,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SNNB_OK) return rc;
    // weight map: dims (taps*Cin, Cout), box (64, BN)
    const uint64_t bdims[2] = {(uint64_t)taps * Cin, (uint64_t)Cout};
    const uint64_t bstr[1] = {(uint64_t)taps * Cin * 2};
    const uint32_t bbox[2] = {64, (uint32_t)BN};
    rc = encode_tmap(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, bdims, bstr, bbox,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SNNB_OK) return rc;
    ConvParams p;
    p.T = T; p.B = B; p.H = H; p.W = W; p.Cin = Cin; p.Cout = Cout;
    p.bw = bw; p.bh = bh; p.bn = bn;
    p.tiles_w = (W + bw - 1) / bw; p.tiles_h = (H + bh - 1) / bh;
    const int tiles_n = (B + bn - 1) / bn;
    p.n_tiles_n = (Cout + BN - 1) / BN;
    p.taps = taps; p.cin_blocks = Cin / 64; p.pool = pool; p.mode = mode;
    p.df = df; p.sc = sc; p.thr = thr; p.v_reset = v_reset; p.hard = hard ? 1 : 0;
    p.bias = bias; p.out = out; p.status = status;
    const int64_t grid = (int64_t)p.tiles_w * p.tiles_h * tiles_n * p.n_tiles_n;
    if (grid > 0x7fffffff) return SNNB_ERR_ARG;
    switch (BN) {
        case 128: return launch_conv<128, 4>(ta, tb, p, (int)grid, s);
        case 64: return launch_conv<64, 6>(ta, tb, p, (int)grid, s);
        case 32: return launch_conv<32, 6>(ta, tb, p, (int)grid, s);
        default: return launch_conv<16, 6>(ta, tb, p, (int)grid, s);
    }
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_conv3x3_lif(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                                int64_t Cin, const void* w, const float* bias, int64_t Cout,
                                float decay, float input_scale, float v_threshold, float v_reset,
                                int hard_reset, int pool, void* out, snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || H > 0x7fffffff || W > 0x7fffffff ||
        Cin > 0x7fffffff || Cout > 0x7fffffff)
        return SNNB_ERR_ARG;
    return run_tc_layer(x, (int)T, (int)B, (int)H, (int)W, (int)Cin, w, bias, (int)Cout, 9, decay,
                        input_scale, v_threshold, v_reset, hard_reset, pool, 0, out,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int snnb_linear_lif(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                               const float* bias, int64_t N, float decay, float input_scale,
                               float v_threshold, float v_reset, int hard_reset, void* out,
                               snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || K > 0x7fffffff || N > 0x7fffffff) return SNNB_ERR_ARG;
    // a linear layer is a 1x1 "conv" over B images of 1 x 1 pixels
    return run_tc_layer(x, (int)T, (int)B, 1, 1, (int)K, w, bias, (int)N, 1, decay, input_scale,
                        v_threshold, v_reset, hard_reset, 0, 0, out,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int snnb_linear_mean(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                                const float* bias, int64_t N, float* out, snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || K > 0x7fffffff || N > 64) return SNNB_ERR_ARG;
    return run_tc_layer(x, (int)T, (int)B, 1, 1, (int)K, w, bias, (int)N, 1, 0.f, 0.f, 0.f, 0.f, 0,
                        0, 1, out, static_cast<cudaStream_t>(stream));
}

extern "C" int snnb_linear_out(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                               const float* bias, int64_t N, float* out, snnb_stream_t stream) {
    if (T > 0x7fffffff || B > 0x7fffffff || K > 0x7fffffff || N > 64) return SNNB_ERR_ARG;
    return run_tc_layer(x, (int)T, (int)B, 1, 1, (int)K, w, bias, (int)N, 1, 0.f, 0.f, 0.f, 0.f, 0,
                        0, 2, out, static_cast<cudaStream_t>(stream));
}

extern "C" int snnb_first_conv_lif(const float* x, int64_t Ti, int64_t T, int64_t B, int64_t Cin,
                                   int64_t H, int64_t W, const float* w, const float* bias,
                                   int64_t Cout, float decay, float input_scale,
                                   float v_threshold, float v_reset, int hard_reset, int pool,
                                   void* out, snnb_stream_t stream) {
    if (!x || !w || !bias || !out) return SNNB_ERR_ARG;
    if (T <= 0 || B <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0) return SNNB_ERR_ARG;
    if (Ti != 1 && Ti != T) return SNNB_ERR_ARG;
    if (Cout % 8 || !aligned16(out)) return SNNB_ERR_ARG;
    if (pool && ((H % 2) || (W % 2))) return SNNB_ERR_UNSUPPORTED;
    if (T * B * Cin * H * W > ((int64_t)1 << 40)) return SNNB_ERR_ARG;
    const int Ho = pool ? (int)H / 2 : (int)H, Wo = pool ? (int)W / 2 : (int)W;
    const int64_t total = B * Ho * Wo * (Cout / 8);
    const int64_t blocks = (total + 255) / 256;
    first_conv_lif_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, (int)Ti, (int)T, (int)B, (int)Cin, (int)H, (int)W, w, bias, (int)Cout, decay,
        input_scale, v_threshold, v_reset, hard_reset, pool, static_cast<__nv_bfloat16*>(out));
    return launch_status();
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
