// Linear layers over few rows in the transposed form: D^T = W X^T, + bias, multi-step LIF.
//
// Replaces, for the classifier (FusedLinearNeuron, snn_compiler/nn/modules.py:241-255) and
// the dense form of 3x3 layers on 2x2 images (FusedConvBNNeuron, modules.py:347-357), the
// F.linear + fused_bias_if_lif pair of the reference when the layer has few rows: at VGG16's
// B = 64 per GPU a linear layer multiplies M = T x B = 256 rows by a K x N weight, and the
// row-major tiling (128 rows x N/… channels per CTA) re-reads the whole activation tile for
// every channel block.  Here the roles swap: M = 128 output features per CTA, N = the
// T x nb rows of one column tile (T * nb = 256, tcgen05 N = 256: every row at once), and the
// K range is split across a cluster of S CTAs so that the grid still covers the SMs.  The
// weights are read once, the activations once per 128 features.
//
//   grid (N / 128 feature tiles, ceil(B / nb) column tiles, S splits), cluster (1, 1, S)
//   warp 0     TMA producer: per 64-wide k-slab one weight box (64 x 128 features, loaded
//              before the previous kernel has finished: no kernel writes weights) and one
//              activation box (64 x T x nb over X [T, B, K]: rows ordered (sample, step))
//   warp 1     MMA issuer: tcgen05.mma M = 128, N = 256, K = 16, accumulator in TMEM
//   warps 2-5  epilogue, thread = TMEM lane = output feature
// S == 1: each thread adds the bias and runs the neuron over the T steps of each sample from
// its accumulator row, and stores the spikes.  S > 1: each CTA stores its float32 partial
// sums [256 columns][feature] to the workspace (coalesced: a warp's 32 features per column), the cluster synchronises (release /
// acquire at cluster scope), and CTA r finishes columns [r * 256 / S, (r + 1) * 256 / S):
// it adds the S partial sums in split order, the bias, runs the neuron and stores.
// pool4: OR over 4 consecutive features (the dense form of a pooled 2x2 layer, rows ordered
// (channel, pixel)); output feature f / 4.
#include "tc_common.cuh"

namespace snnb {

int* device_status_ptr();

namespace {

constexpr int LT_THREADS = 192;
constexpr int LT_STAGES = 4;
constexpr int LT_COLS = 256;                 // columns (rows of X) per tile

struct LtParams {
    int T, B, K, N, nb, splits, kslabs, nbt;
    int pool4;
    float df, sc, thr, v_reset;
    const float* bias;
    __nv_bfloat16* out;
    float* partial;                          // [splits][nbt][256][N] float32 when splits > 1
    int* status;
};

struct LtSmem {
    static constexpr int A_TILE = 128 * 128;                 // 128 features x 64 k (bf16)
    static constexpr int B_TILE = LT_COLS * 128;             // 256 rows x 64 k
    static constexpr int STAGE = A_TILE + B_TILE;
    static constexpr int BAR_OFF = LT_STAGES * STAGE;
    static constexpr int NBARS = 2 * LT_STAGES + 2;
    static constexpr int TMEM_OFF = BAR_OFF + NBARS * 8;
    static constexpr int TOTAL = TMEM_OFF + 8;
    static constexpr int DYN = TOTAL + 1024;
};

// Neuron over the TS steps of one sample: y[t] (+ bias) -> spike bits (bit t).
template <bool HARD, int TS>
__device__ __forceinline__ uint32_t lif_steps(const float* y, float bias, const LtParams& p) {
    float v = 0.0f;
    uint32_t bits = 0;
#pragma unroll
    for (int t = 0; t < TS; ++t) {
        float vv = charge(v, p.df, p.sc, __fadd_rn(y[t], bias));
        const bool s = vv >= p.thr;
        v = reset_v<HARD>(vv, s, p.thr, p.v_reset);
        bits |= (s ? 1u : 0u) << t;
    }
    return bits;
}

// Spikes of one sample's TS steps for this lane's feature; with pool4 the OR over the four
// features of a group (lanes 4i .. 4i + 3), stored by the group's first lane.
template <int TS>
__device__ __forceinline__ void store_sample(const LtParams& p, int feature, int b,
                                             uint32_t bits, int lane) {
    if (p.pool4) {
        bits |= __shfl_xor_sync(0xffffffffu, bits, 1);
        bits |= __shfl_xor_sync(0xffffffffu, bits, 2);
    }
    if (b >= p.B || feature >= p.N) return;
    const int No = p.pool4 ? p.N / 4 : p.N;
    if (p.pool4 && (lane & 3)) return;
    const int f = p.pool4 ? feature / 4 : feature;
#pragma unroll
    for (int t = 0; t < TS; ++t) {
        const int64_t e = ((int64_t)t * p.B + b) * No + f;
        if (SNNB_IN_BOUNDS(e, (int64_t)p.T * p.B * No, p.status))
            p.out[e] = spike_value<__nv_bfloat16>(((bits >> t) & 1u) != 0);
    }
}

template <bool HARD, int TS>
__global__ void __launch_bounds__(LT_THREADS, 1)
linear_t_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX,
                const LtParams p) {
    using S = LtSmem;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = tc::smem_u32(smem);
    const uint32_t bar0 = sbase + S::BAR_OFF;
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (LT_STAGES + s); };
    const uint32_t accf_bar = bar0 + 8u * (2 * LT_STAGES);
    const uint32_t done_bar = accf_bar + 8u;
    volatile uint32_t* tmem_slot = reinterpret_cast<volatile uint32_t*>(smem + S::TMEM_OFF);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.x * 128;
    const int bt = blockIdx.y;
    const int split = blockIdx.z;
    const int b0 = bt * p.nb;
    const int s0 = (int)((int64_t)p.kslabs * split / p.splits);
    const int s1 = (int)((int64_t)p.kslabs * (split + 1) / p.splits);
    const int nsl = s1 - s0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < LT_STAGES; ++s) {
            tc::mbar_init(full_bar(s), 1);
            tc::mbar_init(empty_bar(s), 1);
        }
        tc::mbar_init(accf_bar, 1);
        tc::mbar_init(done_bar, 1);
        tc::fence_mbar_init();
        tc::prefetch_tmap(&tmW);
        tc::prefetch_tmap(&tmX);
    }
    if (warp == 1) {
        tc::tmem_alloc(sbase + S::TMEM_OFF, LT_COLS);
        tc::tmem_relinquish();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_trigger();
    uint32_t failed = 0;

    if (warp == 0) {
        // ------------------------------------------------------------- TMA producer
        uint32_t issued = 0;
        bool dep_ready = false;
        for (int g = 0; g < nsl; ++g) {
            const int stage = g % LT_STAGES;
            const uint32_t phase = (uint32_t)(g / LT_STAGES) & 1u;
            failed |= 1u - tc::mbar_wait_warp(empty_bar(stage), phase ^ 1u, failed);
            const uint32_t dst = sbase + (uint32_t)stage * S::STAGE;
            if (!failed && tc::elect_one()) {
                tc::mbar_expect_tx(full_bar(stage), (uint32_t)S::STAGE);
                tc::tma_load_2d(dst, &tmW, full_bar(stage), (s0 + g) * 64, m0);
            }
            __syncwarp();
            if (!dep_ready) {
                pdl_wait();                  // the activations are the previous layer's output
                dep_ready = true;
            }
            if (!failed && tc::elect_one())
                tc::tma_load_3d(dst + S::A_TILE, &tmX, full_bar(stage), (s0 + g) * 64, 0, b0);
            __syncwarp();
            if (!failed) ++issued;
        }
        if (failed) {
            // copies still in flight: wait (bounded) for the last min(stages, issued) stages
            for (uint32_t k = 0; k < issued && k < (uint32_t)LT_STAGES; ++k) {
                const int g = (int)issued - 1 - (int)k;
                tc::mbar_wait_warp<true>(full_bar(g % LT_STAGES), (uint32_t)(g / LT_STAGES) & 1u, 0);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------- MMA issuer
        constexpr uint32_t IDESC = tc::idesc_bf16_f32(128, LT_COLS);
        if (tc::elect_one()) {
            for (int g = 0; g < nsl; ++g) {
                const int stage = g % LT_STAGES;
                if (g == 0) {
                    failed |= 1u - tc::mbar_wait_lane(full_bar(0), 0, failed);
                    tc::tc_fence_after();
                }
                const uint32_t a = sbase + (uint32_t)stage * S::STAGE;
                const uint64_t da = tc::sdesc_k_sw128(a);
                const uint64_t db = tc::sdesc_k_sw128(a + S::A_TILE);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    tc::umma_bf16(tmem, da + 2 * k, db + 2 * k, IDESC, (g | k) != 0);
                // the next stage before this one's commit: a wait behind a commit returns only
                // once the tensor pipe has drained
                if (g + 1 < nsl) {
                    const int ns = (g + 1) % LT_STAGES;
                    failed |= 1u - tc::mbar_wait_lane(full_bar(ns), (uint32_t)((g + 1) / LT_STAGES) & 1u,
                                                      failed);
                    tc::tc_fence_after();
                }
                tc::umma_commit(empty_bar(stage));
            }
            tc::umma_commit(accf_bar);
            tc::umma_commit(done_bar);
        }
        __syncwarp();
        failed = __shfl_sync(0xffffffffu, failed, 0);
        failed |= 1u - tc::mbar_wait_warp<true>(done_bar, 0, 0);
    } else {
        // ------------------------------------------------------------- epilogue
        const int q = warp & 3;
        const int feature = m0 + 32 * q + lane;
        failed |= 1u - tc::mbar_wait_warp(accf_bar, 0, 0);
        tc::tc_fence_after();
        const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16);
        if (!failed) {
            if (p.splits == 1) {
                const float bias = feature < p.N ? __ldg(p.bias + feature) : 0.0f;
#pragma unroll 1
                for (int c = 0; c < LT_COLS / 32; ++c) {
                    float r[32];
                    tc::tmem_ld32(tbase + c * 32, r);
                    tc::tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32 / TS; ++j) {
                        const int b = b0 + c * (32 / TS) + j;
                        const uint32_t bits = lif_steps<HARD, TS>(r + j * TS, bias, p);
                        store_sample<TS>(p, feature, b, bits, lane);
                    }
                }
            } else {
                // this split's partial sums, [256 columns][feature] float32: for each column
                // a warp writes 32 consecutive features (128 bytes)
                float* dst = p.partial + ((int64_t)split * p.nbt + bt) * LT_COLS * p.N + feature;
#pragma unroll 1
                for (int c = 0; c < LT_COLS / 32; ++c) {
                    float r[32];
                    tc::tmem_ld32(tbase + c * 32, r);
                    tc::tmem_wait_ld();
                    if (feature < p.N) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) dst[(int64_t)(c * 32 + j) * p.N] = r[j];
                    }
                }
            }
        }
    }
    if (failed && lane == 0) atomicExch(p.status, SNNB_ERR_TIMEOUT);
    if (p.splits > 1) {
        // every split's partial sums stored (release) and visible (acquire) in the cluster
        tc::cluster_sync();
        if (warp >= 2) {
            const int q = warp & 3;
            const int feature = m0 + 32 * q + lane;
            const int wc = LT_COLS / p.splits;                // columns this CTA finishes
            const int c0 = split * wc;
            const float bias = feature < p.N ? __ldg(p.bias + feature) : 0.0f;
            const float* src = p.partial + ((int64_t)bt * LT_COLS + c0) * p.N + feature;
            const int64_t sstride = (int64_t)p.nbt * LT_COLS * p.N;
            for (int cc = 0; cc < wc; cc += 8) {
                float y[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) y[e] = 0.0f;
                if (feature < p.N) {
                    // every split's 8 values in flight at once (one L2 round trip per 8
                    // columns, not one per split), then added in split order
                    float in[8][8];
#pragma unroll
                    for (int s = 0; s < 8; ++s) {
                        if (s < p.splits) {
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                in[s][e] = __ldcg(src + s * sstride + (int64_t)(cc + e) * p.N);
                        }
                    }
#pragma unroll
                    for (int e = 0; e < 8; ++e) y[e] = in[0][e];
#pragma unroll
                    for (int s = 1; s < 8; ++s) {
                        if (s < p.splits) {
#pragma unroll
                            for (int e = 0; e < 8; ++e) y[e] = __fadd_rn(y[e], in[s][e]);
                        }
                    }
                }
#pragma unroll
                for (int j = 0; j < 8 / TS; ++j) {
                    const int b = b0 + (c0 + cc) / TS + j;
                    const uint32_t bits = lif_steps<HARD, TS>(y + j * TS, bias, p);
                    store_sample<TS>(p, feature, b, bits, lane);
                }
            }
        }
    }
    tc::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc::tc_fence_after();
        tc::tmem_dealloc(tmem, LT_COLS);
    }
}

template <bool HARD, int TS>
int launch_linear_t(const CUtensorMap& tw, const CUtensorMap& tx, const LtParams& p,
                    cudaStream_t s) {
    auto kernel = linear_t_kernel<HARD, TS>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         LtSmem::DYN);
    if (e != cudaSuccess) return record_cuda_error(e);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.N / 128), (unsigned)p.nbt, (unsigned)p.splits);
    cfg.blockDim = dim3(LT_THREADS);
    cfg.dynamicSmemBytes = LtSmem::DYN;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = (unsigned)p.splits;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    e = cudaLaunchKernelEx(&cfg, kernel, tw, tx, p);
    return e == cudaSuccess ? launch_status() : record_cuda_error(e);
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int64_t snnb_linear_t_workspace_bytes(int64_t T, int64_t B, int64_t N, int splits) {
    if (splits <= 1) return 0;
    if (T < 1 || T > 8 || B < 1 || N < 1 || splits > 8) return -1;
    const int64_t nb = LT_COLS / T;
    const int64_t nbt = (B + nb - 1) / nb;
    int64_t n = 4;
    const int64_t f[4] = {splits, nbt, N, LT_COLS};
    for (int i = 0; i < 4; ++i)
        if (__builtin_mul_overflow(n, f[i], &n)) return -1;
    return n;
}

extern "C" int snnb_linear_lif_t(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                                 const float* bias, int64_t N, float decay, float input_scale,
                                 float v_threshold, float v_reset, int hard_reset, int pool4,
                                 int splits, void* workspace, int64_t workspace_bytes, void* out,
                                 snnb_stream_t stream) {
    if (const int inj = take_injected_status()) return inj;
    if (!x || !w || !bias || !out) return SNNB_ERR_ARG;
    if (T != 1 && T != 2 && T != 4 && T != 8) return SNNB_ERR_UNSUPPORTED;
    if (B < 1 || B > 0x7fffffff || K < 8 || K > 0x7fffffff || N < 128 || N > 0x7fffffff)
        return SNNB_ERR_ARG;
    if (K % 8 != 0 || N % 128 != 0) return SNNB_ERR_UNSUPPORTED;
    if (splits != 1 && splits != 2 && splits != 4 && splits != 8) return SNNB_ERR_ARG;
    const int kslabs = (int)((K + 63) / 64);
    if (splits > kslabs) return SNNB_ERR_ARG;
    if (!aligned16(x) || !aligned16(w) || (reinterpret_cast<uintptr_t>(out) & 1u))
        return SNNB_ERR_ARG;
    const int nb = LT_COLS / (int)T;
    const int64_t nbt = (B + nb - 1) / nb;
    if (nbt > 65535) return SNNB_ERR_ARG;
    if (splits > 1) {
        const int64_t need = snnb_linear_t_workspace_bytes(T, B, N, splits);
        if (need < 0 || !workspace || workspace_bytes < need || !aligned16(workspace))
            return SNNB_ERR_ARG;
    }
    int* status = device_status_ptr();
    if (!status) return SNNB_ERR_CUDA;
    // weights [N, K]: box 64 k x 128 features; activations [T, B, K] as dims (K, T, B):
    // box 64 k x T steps x nb samples, rows ordered (sample, step)
    CUtensorMap tw, tx;
    const uint64_t wdims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t wstr[1] = {(uint64_t)K * 2};
    const uint32_t wbox[2] = {64, 128};
    int rc = encode_tmap(&tw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, wdims, wstr, wbox,
                         CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SNNB_OK) return rc;
    const uint64_t xdims[3] = {(uint64_t)K, (uint64_t)T, (uint64_t)B};
    const uint64_t xstr[2] = {(uint64_t)B * K * 2, (uint64_t)K * 2};
    const uint32_t xbox[3] = {64, (uint32_t)T, (uint32_t)nb};
    rc = encode_tmap(&tx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, x, xdims, xstr, xbox,
                     CU_TENSOR_MAP_SWIZZLE_128B);
    if (rc != SNNB_OK) return rc;
    LtParams p = {};
    p.T = (int)T; p.B = (int)B; p.K = (int)K; p.N = (int)N; p.nb = nb; p.splits = splits;
    p.kslabs = kslabs; p.nbt = (int)nbt; p.pool4 = pool4 ? 1 : 0;
    p.df = decay; p.sc = input_scale; p.thr = v_threshold; p.v_reset = v_reset;
    p.bias = bias; p.out = static_cast<__nv_bfloat16*>(out);
    p.partial = static_cast<float*>(workspace); p.status = status;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const bool hard = hard_reset != 0;
#define SNNB_LT(TS)                                                                        \
    if (T == TS) return hard ? launch_linear_t<true, TS>(tw, tx, p, s)                     \
                             : launch_linear_t<false, TS>(tw, tx, p, s);
    SNNB_LT(1) SNNB_LT(2) SNNB_LT(4) SNNB_LT(8)
#undef SNNB_LT
    return SNNB_ERR_UNSUPPORTED;
}
