// K3 -- spiking self-attention core: kv = K^T V, a = Q kv, then a multi-step LIF on
// a * scale, with the membrane potential kept in registers across T.
//
// Replaces the reference's
//   spike_ktv / spike_ktv_popcount   snn_compiler/kernels/attention.py:143-258
//                                    (_pack_N_kernel + _ktv_popcount_kernel)
//   spike_av_lif                     snn_compiler/kernels/attention.py:49-137
//   the K^T V bmm + spike_av_lif of FusedSpikeAttention.forward (nn/attention.py:149-150)
// in one launch.  Q, K, V are {0,1} spikes, so K^T V is an integer <= N and Q (K^T V)
// an integer <= N*d, exact in float32; (Q K^T) V, the order the benchmark describes,
// equals Q (K^T V) exactly.
//
// One CTA per (batch, head), 256 threads, looping over t:
//   1. a warp per 32-token block: each lane reads its token's Q, K and V rows with 16-byte
//      loads and keeps them as d-bit masks; one ballot per feature turns the K and V
//      columns into 32-bit words packed along tokens (bit l of word w = token 32w + l);
//   2. kv[i][j] = sum_w popc(Kbits[i][w] & Vbits[j][w]) -- d*d entries, AND + popcount;
//   3. each thread owns fixed (token, 4 features) groups across t: a = sum of the kv rows
//      selected by the token's Q mask (float4 shared-memory reads), then
//      v = decay*v + input_scale*(a*scale) (float32, no FMA contraction), spike, reset,
//      and one 8-byte store of 4 bf16 spikes.
// Strides are general so the same kernel reads a fused QKV projection output
// [T, B, N, 3D] or separate [T, B, H, N, d] tensors.
#include "common.cuh"

namespace snnb {
namespace {

constexpr int THREADS = 256;
constexpr int MAX_D = 32;
constexpr int MAX_W = 8;            // tokens <= 256


struct AttnParams {
    const __nv_bfloat16* q;
    const __nv_bfloat16* k;
    const __nv_bfloat16* v;
    int64_t st, sb, sh, sn;         // element strides of q / k / v (feature axis contiguous)
    const float* kv_in;             // optional [T, B, H, d, d] f32 (used instead of K, V)
    float* kv_out;                  // optional [T, B, H, d, d] f32
    __nv_bfloat16* out;             // spikes, strides ot, ob, oh, on
    int64_t ot, ob, oh, on;
    int T, B, H, N, d;
    float df, sc, scale, thr, v_reset;
    int hard, do_av;
};

__device__ __forceinline__ bool nz(__nv_bfloat16 x) {
    return (__bfloat16_as_ushort(x) & 0x7fffu) != 0;
}

// Row loads: the d features of one token as a bit mask (bit i = feature i nonzero).
// 16-byte loads when the row is 16-byte aligned and d % 8 == 0, else element loads.
__device__ __forceinline__ uint32_t row_mask(const __nv_bfloat16* row, int d, bool vec) {
    uint32_t m = 0;
    if (vec) {
        const uint4* r4 = reinterpret_cast<const uint4*>(row);
#pragma unroll
        for (int c = 0; c < MAX_D / 8; ++c) {
            if (c * 8 >= d) break;
            const uint4 u = __ldg(r4 + c);
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                if (w[e] & 0x7fffu) m |= 1u << (c * 8 + 2 * e);
                if (w[e] & 0x7fff0000u) m |= 1u << (c * 8 + 2 * e + 1);
            }
        }
    } else {
        for (int i = 0; i < d; ++i)
            if (nz(row[i])) m |= 1u << i;
    }
    return m;
}

// x = row `lane` of a 32 x 32 bit matrix (bit c = column c); afterwards x = column `lane`
// (bit r = row r).  Stage s swaps the off-diagonal s x s blocks of every 2s x 2s block.
__device__ __forceinline__ void transpose32(uint32_t& x, int lane) {
    const uint32_t masks[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
    for (int k = 0; k < 5; ++k) {
        const int sft = 16 >> k;
        const uint32_t m = masks[k];
        const uint32_t y = __shfl_xor_sync(0xffffffffu, x, sft);
        x = (lane & sft) ? ((x & ~m) | ((y >> sft) & m)) : ((x & m) | ((y & m) << sft));
    }
}

constexpr int JG = 4;                    // features per work item in the Q kv stage
constexpr int MAX_ITEMS = 8;             // work items per thread: N * d / JG <= 2048

template <bool HARD>
__global__ void __launch_bounds__(THREADS) attention_core_kernel(const AttnParams p) {
    pdl_wait();
    pdl_trigger();
    __shared__ uint32_t kbits[MAX_D][MAX_W];
    __shared__ uint32_t vbits[MAX_D][MAX_W];
    __shared__ __align__(16) float kv[MAX_D][MAX_D];
    __shared__ uint32_t qmask[MAX_W * 32];
    const int bh = blockIdx.x;
    const int b = bh / p.H, h = bh % p.H;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = p.d, N = p.N;
    const int W = (N + 31) / 32;
    const bool vec = (d % 8 == 0) && ((p.sn % 8) == 0) && ((p.st % 8) == 0) &&
                     ((p.sb % 8) == 0) && ((p.sh % 8) == 0);
    const bool vec4 = (d % JG == 0);
    const int ngroups = vec4 ? d / JG : d;            // groups of JG features (or singles)
    const int items = N * ngroups;
    float vm[MAX_ITEMS][JG];
#pragma unroll
    for (int k = 0; k < MAX_ITEMS; ++k)
#pragma unroll
        for (int j = 0; j < JG; ++j) vm[k][j] = 0.0f;

    for (int t = 0; t < p.T; ++t) {
        const int64_t base = (int64_t)t * p.st + (int64_t)b * p.sb + (int64_t)h * p.sh;
        // ---- 1. per 32-token block: row masks; K and V columns packed along tokens
        for (int w = warp; w < W; w += THREADS / 32) {
            const int n = 32 * w + lane;
            const bool in = n < N;
            const int64_t row = base + (int64_t)n * p.sn;
            uint32_t km = 0, vmk = 0, qm = 0;
            if (in) {
                if (p.kv_in == nullptr) {
                    km = row_mask(p.k + row, d, vec);
                    vmk = row_mask(p.v + row, d, vec);
                }
                if (p.do_av) qm = row_mask(p.q + row, d, vec);
            }
            if (p.kv_in == nullptr) {
                // 32 x 32 bit-matrix transpose across the warp (lane = token, bit = feature
                // -> lane = feature, bit = token): five shuffle stages swapping off-diagonal
                // blocks, instead of one ballot per feature
                transpose32(km, lane);
                transpose32(vmk, lane);
                if (lane < d) {
                    kbits[lane][w] = km;
                    vbits[lane][w] = vmk;
                }
            }
            qmask[n] = qm;
        }
        __syncthreads();
        // ---- 2. kv = K^T V
        const int64_t kvo = (((int64_t)t * p.B + b) * p.H + h) * d * d;
        for (int e = threadIdx.x; e < d * d; e += THREADS) {
            const int i = e / d, j = e % d;
            float val;
            if (p.kv_in) {
                val = p.kv_in[kvo + e];
            } else {
                uint32_t c = 0;
                for (int w = 0; w < W; ++w) c += __popc(kbits[i][w] & vbits[j][w]);
                val = (float)c;
            }
            kv[i][j] = val;
            if (p.kv_out) p.kv_out[kvo + e] = val;
        }
        __syncthreads();
        // ---- 3. a = Q kv over the set bits of each token's Q mask, LIF on a * scale
        if (p.do_av) {
            const int64_t obase = (int64_t)t * p.ot + (int64_t)b * p.ob + (int64_t)h * p.oh;
#pragma unroll
            for (int k = 0; k < MAX_ITEMS; ++k) {
                const int it = threadIdx.x + k * THREADS;
                if (it >= items) break;
                const int n = it / ngroups, gq = it % ngroups;
                uint32_t m = qmask[n];
                float a[JG] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (vec4) {
                    while (m) {
                        const int i = __ffs(m) - 1;
                        m &= m - 1;
                        const float4 r = *reinterpret_cast<const float4*>(&kv[i][gq * JG]);
                        a[0] = __fadd_rn(a[0], r.x);
                        a[1] = __fadd_rn(a[1], r.y);
                        a[2] = __fadd_rn(a[2], r.z);
                        a[3] = __fadd_rn(a[3], r.w);
                    }
                } else {
                    while (m) {
                        const int i = __ffs(m) - 1;
                        m &= m - 1;
                        a[0] = __fadd_rn(a[0], kv[i][gq]);
                    }
                }
                const int nj = vec4 ? JG : 1;
                uint32_t bits = 0;
#pragma unroll
                for (int j = 0; j < JG; ++j) {
                    if (j >= nj) break;
                    const float in = __fmul_rn(a[j], p.scale);
                    float vv = charge(vm[k][j], p.df, p.sc, in);
                    const bool s = vv >= p.thr;
                    vv = reset_v<HARD>(vv, s, p.thr, p.v_reset);
                    vm[k][j] = vv;
                    bits |= (s ? 1u : 0u) << j;
                }
                __nv_bfloat16* dst = p.out + obase + (int64_t)n * p.on + gq * nj;
                if (vec4 && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
                    const uint32_t lo = ((bits & 1u) ? 0x3F80u : 0u) | ((bits & 2u) ? 0x3F800000u : 0u);
                    const uint32_t hi = ((bits & 4u) ? 0x3F80u : 0u) | ((bits & 8u) ? 0x3F800000u : 0u);
                    *reinterpret_cast<uint2*>(dst) = make_uint2(lo, hi);
                } else {
                    for (int j = 0; j < nj; ++j) dst[j] = spike_value<__nv_bfloat16>((bits >> j) & 1u);
                }
            }
        }
        __syncthreads();
    }
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_spike_attention_core(
    const void* q, const void* k, const void* v, int64_t st, int64_t sb, int64_t sh, int64_t sn,
    const float* kv_in, float* kv_out, void* out, int64_t ot, int64_t ob, int64_t oh, int64_t on,
    int64_t T, int64_t B, int64_t H, int64_t N, int64_t d, float decay, float input_scale,
    float scale, float v_threshold, float v_reset, int hard_reset, snnb_stream_t stream) {
    if (const int inj = snnb::take_injected_status()) return inj;
    if (T <= 0 || B <= 0 || H <= 0 || N <= 0 || d <= 0) return SNNB_ERR_ARG;
    const int64_t work = (d % 4 == 0) ? N * (d / 4) : N * d;
    if (d > MAX_D || N > MAX_W * 32 || work > (int64_t)MAX_ITEMS * THREADS)
        return SNNB_ERR_UNSUPPORTED;
    if (B * H > 0x7fffffff || T > 0x7fffffff) return SNNB_ERR_ARG;
    const int do_av = out != nullptr;
    if (do_av && !q) return SNNB_ERR_ARG;
    if (!kv_in && (!k || !v)) return SNNB_ERR_ARG;
    if (!do_av && !kv_out) return SNNB_ERR_ARG;
    AttnParams p;
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.k = static_cast<const __nv_bfloat16*>(k);
    p.v = static_cast<const __nv_bfloat16*>(v);
    p.st = st; p.sb = sb; p.sh = sh; p.sn = sn;
    p.kv_in = kv_in; p.kv_out = kv_out;
    p.out = static_cast<__nv_bfloat16*>(out);
    p.ot = ot; p.ob = ob; p.oh = oh; p.on = on;
    p.T = (int)T; p.B = (int)B; p.H = (int)H; p.N = (int)N; p.d = (int)d;
    p.df = decay; p.sc = input_scale; p.scale = scale; p.thr = v_threshold; p.v_reset = v_reset;
    p.hard = hard_reset ? 1 : 0; p.do_av = do_av;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    return p.hard ? launch_k(attention_core_kernel<true>, dim3((unsigned)(B * H)), dim3(THREADS), 0, s, p)
                  : launch_k(attention_core_kernel<false>, dim3((unsigned)(B * H)), dim3(THREADS), 0, s, p);
}
