// K4 -- bit packing and the AND / XOR + popcount binary GEMM.
//
// Replaces the reference's bit-pack kernel (snn_compiler/kernels/attention.py:195-214)
// and popcount K^T V kernel (attention.py:217-233), generalised to a tiled GEMM
// over packed rows with three products:
//   MODE 0  {0,1} x {0,1}   C = sum_w popc(a & b)
//   MODE 1  {0,1} x {-1,+1} C = 2 * sum_w popc(a & b) - popc(a)     (b bit 1 <=> +1)
//   MODE 2  {-1,+1}^2       C = K - 2 * sum_w popc(a ^ b)            (XNOR form)
// Operands are K-major packed rows: A [M, ldw] and B [N, ldw] uint32, element k of
// a row in bit (k % 32) of word k / 32 (LSB first); words beyond ceil(K/32) are 0.
//
// Design (B200, SIMT integer pipe): 128 x 128 output tile per 256-thread CTA, each
// thread an 8 x 8 register block (rows ty + 16 i, columns tx + 16 j so that a warp's
// shared-memory reads fall in distinct banks), 32-word (1024-bit) k-slabs streamed
// into a 3-stage cp.async ring with 16-byte copies and hardware zero-fill at the
// edges.  Per 4-word step a thread issues 16 LDS.128 and 256 AND+POPC+ADD.  The
// popcount of A's rows (MODE 1) is reduced in the prologue with warp shuffles.  When
// the MxN tile grid cannot fill the 148 SMs the k range is split over gridDim.z and
// the partial sums are combined with integer atomics (order-independent, exact).
#include "common.cuh"

namespace snnb {
namespace {

constexpr int BM = 128, BN = 128, BKW = 32, LDSW = BKW + 4, STAGES = 3, THREADS = 256;
constexpr int STAGE_WORDS = (BM + BN) * LDSW;
constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_WORDS * 4 + BM * 4;

__device__ __forceinline__ void cp_async16(uint32_t* dst, const uint32_t* src, int src_bytes) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src),
                 "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

// Load one k-slab (words [w0, w0+32) of rows r0..r0+127) of a packed operand.
__device__ __forceinline__ void load_slab(uint32_t* s, const uint32_t* G, int64_t rows, int64_t r0,
                                          int64_t ldw, int64_t w0, int64_t wend, int tid) {
#pragma unroll
    for (int c = 0; c < (BM * BKW / 4) / THREADS; ++c) {
        const int chunk = tid + c * THREADS;
        const int row = chunk >> 3;          // 8 chunks of 4 words per row
        const int q = chunk & 7;
        const int64_t gr = r0 + row;
        const int64_t gw = w0 + q * 4;
        int bytes = 0;
        if (gr < rows && gw < wend) bytes = (int)((wend - gw) < 4 ? (wend - gw) : 4) * 4;
        const uint32_t* src = bytes ? G + gr * ldw + gw : G;
        cp_async16(s + row * LDSW + q * 4, src, bytes);
    }
}

template <int MODE>
__global__ void __launch_bounds__(THREADS) bgemm_kernel(const uint32_t* __restrict__ A,
                                                        const uint32_t* __restrict__ B,
                                                        int32_t* __restrict__ C, int64_t M,
                                                        int64_t N, int64_t ldw, int64_t kbits,
                                                        int64_t w_per_split, int atomic) {
    pdl_wait();
    pdl_trigger();
    extern __shared__ __align__(16) uint32_t sm[];
    uint32_t* rowpop = sm + STAGES * STAGE_WORDS;
    const int tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    const int64_t m0 = (int64_t)blockIdx.y * BM, n0 = (int64_t)blockIdx.x * BN;
    const int64_t wtot = (kbits + 31) / 32;
    const int64_t wbeg = (int64_t)blockIdx.z * w_per_split;
    const int64_t wend = (wbeg + w_per_split) < wtot ? (wbeg + w_per_split) : wtot;
    const int nk = wend > wbeg ? (int)((wend - wbeg + BKW - 1) / BKW) : 0;

    if (MODE == 1) {
        // popc of A's 128 rows over the full k range: 2 threads per row, shuffle-combined
        const int row = tid >> 1, half = tid & 1;
        uint32_t pc = 0;
        if (m0 + row < M && blockIdx.z == 0) {
            const uint32_t* ar = A + (m0 + row) * ldw;
            for (int64_t w = half; w < wtot; w += 2) pc += __popc(__ldg(ar + w));
        }
        pc += __shfl_xor_sync(0xffffffffu, pc, 1);
        if (half == 0) rowpop[row] = pc;
    }

#pragma unroll
    for (int s = 0; s < STAGES - 1; ++s) {
        if (s < nk) {
            uint32_t* st = sm + s * STAGE_WORDS;
            load_slab(st, A, M, m0, ldw, wbeg + s * BKW, wend, tid);
            load_slab(st + BM * LDSW, B, N, n0, ldw, wbeg + s * BKW, wend, tid);
        }
        cp_async_commit();
    }

    uint32_t acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0;

    for (int kt = 0; kt < nk; ++kt) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();
        const int pf = kt + STAGES - 1;
        if (pf < nk) {
            uint32_t* st = sm + (pf % STAGES) * STAGE_WORDS;
            load_slab(st, A, M, m0, ldw, wbeg + (int64_t)pf * BKW, wend, tid);
            load_slab(st + BM * LDSW, B, N, n0, ldw, wbeg + (int64_t)pf * BKW, wend, tid);
        }
        cp_async_commit();
        const uint32_t* sA = sm + (kt % STAGES) * STAGE_WORDS;
        const uint32_t* sB = sA + BM * LDSW;
#pragma unroll 2
        for (int kq = 0; kq < BKW / 4; ++kq) {
            uint4 a[8], b[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
                a[i] = *reinterpret_cast<const uint4*>(sA + (ty + 16 * i) * LDSW + kq * 4);
#pragma unroll
            for (int j = 0; j < 8; ++j)
                b[j] = *reinterpret_cast<const uint4*>(sB + (tx + 16 * j) * LDSW + kq * 4);
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (MODE == 2) {
                        acc[i][j] += __popc(a[i].x ^ b[j].x) + __popc(a[i].y ^ b[j].y) +
                                     __popc(a[i].z ^ b[j].z) + __popc(a[i].w ^ b[j].w);
                    } else {
                        acc[i][j] += __popc(a[i].x & b[j].x) + __popc(a[i].y & b[j].y) +
                                     __popc(a[i].z & b[j].z) + __popc(a[i].w & b[j].w);
                    }
                }
        }
    }
    cp_async_wait<0>();
    __syncthreads();

    const bool first = blockIdx.z == 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t m = m0 + ty + 16 * i;
        if (m >= M) continue;
        int32_t base = 0;
        if (MODE == 1 && first) base = -(int32_t)rowpop[ty + 16 * i];
        if (MODE == 2 && first) base = (int32_t)kbits;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t n = n0 + tx + 16 * j;
            if (n >= N) continue;
            int32_t v;
            if (MODE == 0) v = (int32_t)acc[i][j] + base;
            else if (MODE == 1) v = 2 * (int32_t)acc[i][j] + base;
            else v = base - 2 * (int32_t)acc[i][j];
            if (atomic) atomicAdd(C + m * N + n, v);
            else C[m * N + n] = v;
        }
    }
}

// ---- packing ----------------------------------------------------------------------------
// One thread per output word: reads the word's 32 source elements (16-byte loads when the
// row is 16-byte aligned) and sets bit i for element 32 w + i when it is nonzero
// (positive == 0) or > 0 (positive == 1, the {-1,+1} encoding).
template <typename T>
__device__ __forceinline__ bool bit_of(T v, int positive);
template <> __device__ __forceinline__ bool bit_of<float>(float v, int positive) {
    return positive ? v > 0.f : v != 0.f;
}
template <> __device__ __forceinline__ bool bit_of<__half>(__half v, int positive) {
    const float f = __half2float(v);
    return positive ? f > 0.f : f != 0.f;
}
template <> __device__ __forceinline__ bool bit_of<__nv_bfloat16>(__nv_bfloat16 v, int positive) {
    const float f = __bfloat162float(v);
    return positive ? f > 0.f : f != 0.f;
}
template <> __device__ __forceinline__ bool bit_of<uint8_t>(uint8_t v, int positive) {
    return positive ? (int8_t)v > 0 : v != 0;
}

template <typename T>
__global__ void __launch_bounds__(256) bitpack_kernel(const T* __restrict__ x, int64_t rows,
                                                      int64_t K, int64_t ldw, int positive,
                                                      uint32_t* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = rows * ldw;
    if (gid >= total) return;
    const int64_t r = gid / ldw, w = gid - r * ldw;
    const int64_t k0 = w * 32;
    uint32_t word = 0;
    if (k0 < K) {
        const T* src = x + r * K + k0;
        const int n = (int)((K - k0) < 32 ? (K - k0) : 32);
        constexpr int PER16 = 16 / sizeof(T);
        if (n == 32 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
#pragma unroll
            for (int c = 0; c < 32 / PER16; ++c) {
                const uint4 q = __ldcs(reinterpret_cast<const uint4*>(src) + c);
                const T* e = reinterpret_cast<const T*>(&q);
#pragma unroll
                for (int i = 0; i < PER16; ++i)
                    word |= (bit_of<T>(e[i], positive) ? 1u : 0u) << (c * PER16 + i);
            }
        } else {
            for (int i = 0; i < n; ++i) word |= (bit_of<T>(src[i], positive) ? 1u : 0u) << i;
        }
    }
    out[gid] = word;
}

// Peak of the binary GEMM's inner operation on this GPU, for its roofline: every thread
// runs `iters` rounds of 64 independent word-ops -- acc += popc(a & b), the AND, POPC and
// add of bgemm_kernel's inner product -- on register operands.  The AND and the popcount
// are volatile asm, so the compiler can neither hoist the loop-invariant products out of
// the loop nor drop them.  The sum is written only if it equals a value it never takes.
constexpr int POPC_PEAK_THREADS = 256;

__global__ void __launch_bounds__(POPC_PEAK_THREADS) popc_peak_kernel(int iters, uint32_t* sink) {
    uint32_t a[8], b[8], acc[8][8];
    const uint32_t s = blockIdx.x * 7919u + threadIdx.x * 104729u + 12345u;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        a[i] = s * (2u * i + 1u) + 0x9E3779B9u * i;
        b[i] = (~s) * (2u * i + 3u) ^ (0x85EBCA6Bu * i);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0u;
    }
    for (int it = 0; it < iters; ++it) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint32_t t;
                asm volatile("and.b32 %0, %1, %2;\n\tpopc.b32 %0, %0;" : "=r"(t) : "r"(a[i]), "r"(b[j]));
                acc[i][j] += t;
            }
    }
    uint32_t r = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) r += acc[i][j] * (uint32_t)(i * 8 + j + 1);
    if (r == 0x9E3779B9u) sink[threadIdx.x] = r;
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_bitpack(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t ldw,
                            int positive, uint32_t* out, snnb_stream_t stream) {
    if (const int inj = snnb::take_injected_status()) return inj;
    if (rows < 0 || K < 0 || ldw < (K + 31) / 32) return SNNB_ERR_ARG;
    if (rows == 0 || ldw == 0) return SNNB_OK;
    if (!out || (K > 0 && !x)) return SNNB_ERR_ARG;
    const int64_t total = rows * ldw;
    const int64_t blocks = (total + 255) / 256;
    if (blocks > 0x7fffffffll) return SNNB_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (x_dtype) {
        case SNNB_F32: return launch_k(bitpack_kernel<float>, dim3((unsigned)blocks), dim3(256), 0, s, static_cast<const float*>(x), rows, K, ldw, positive, out);
        case SNNB_F16: return launch_k(bitpack_kernel<__half>, dim3((unsigned)blocks), dim3(256), 0, s, static_cast<const __half*>(x), rows, K, ldw, positive, out);
        case SNNB_BF16: return launch_k(bitpack_kernel<__nv_bfloat16>, dim3((unsigned)blocks), dim3(256), 0, s, static_cast<const __nv_bfloat16*>(x), rows, K, ldw, positive, out);
        case SNNB_U8: return launch_k(bitpack_kernel<uint8_t>, dim3((unsigned)blocks), dim3(256), 0, s, static_cast<const uint8_t*>(x), rows, K, ldw, positive, out);
        default: return SNNB_ERR_ARG;
    }
}

extern "C" int snnb_bgemm(const uint32_t* A, const uint32_t* B, int32_t* C, int64_t M, int64_t N,
                          int64_t K, int64_t ldw, int mode, int splits, snnb_stream_t stream) {
    if (const int inj = snnb::take_injected_status()) return inj;
    if (M < 0 || N < 0 || K < 0 || mode < 0 || mode > 2) return SNNB_ERR_ARG;
    if (M == 0 || N == 0) return SNNB_OK;
    if (!A || !B || !C) return SNNB_ERR_ARG;
    const int64_t wtot = (K + 31) / 32;
    if (ldw < wtot || (ldw % 4) != 0 || !aligned16(A) || !aligned16(B)) return SNNB_ERR_ARG;
    if (K > 0x7fffffffll || M * N > ((int64_t)1 << 40)) return SNNB_ERR_ARG;
    const int64_t gx = (N + BN - 1) / BN, gy = (M + BM - 1) / BM;
    if (gx > 0x7fffffffll || gy > 65535) return SNNB_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int64_t kslabs = (wtot + BKW - 1) / BKW;
    if (splits <= 0) {
        // split the k range until the grid covers two waves of 148 SMs (1 CTA / SM)
        splits = 1;
        while (gx * gy * splits < 2 * 148 && splits * 2 <= kslabs && splits < 16) splits *= 2;
    }
    if (splits > kslabs && kslabs > 0) splits = (int)kslabs;
    if (splits < 1) splits = 1;
    const int64_t wps = ((wtot + splits - 1) / splits + BKW - 1) / BKW * BKW;
    const int atomic = splits > 1;
    if (atomic) {
        cudaError_t e = cudaMemsetAsync(C, 0, (size_t)(M * N) * sizeof(int32_t), s);
        if (e != cudaSuccess) return record_cuda_error(e);
    }
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)splits);
    switch (mode) {
        case 0:
            cudaFuncSetAttribute(bgemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
            return launch_k(bgemm_kernel<0>, grid, dim3(THREADS), SMEM_BYTES, s, A, B, C, M, N, ldw, K, wps, atomic);
        case 1:
            cudaFuncSetAttribute(bgemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
            return launch_k(bgemm_kernel<1>, grid, dim3(THREADS), SMEM_BYTES, s, A, B, C, M, N, ldw, K, wps, atomic);
        default:
            cudaFuncSetAttribute(bgemm_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
            return launch_k(bgemm_kernel<2>, grid, dim3(THREADS), SMEM_BYTES, s, A, B, C, M, N, ldw, K, wps, atomic);
    }
    return launch_status();
}

extern "C" int snnb_popc_peak(int64_t blocks, int iters, void* sink, snnb_stream_t stream) {
    if (const int inj = snnb::take_injected_status()) return inj;
    if (blocks <= 0 || blocks > 0x7fffffff || iters <= 0 || !sink) return SNNB_ERR_ARG;
    return snnb::launch_k(snnb::popc_peak_kernel, dim3((unsigned)blocks),
                          dim3(snnb::POPC_PEAK_THREADS), 0, static_cast<cudaStream_t>(stream),
                          iters, static_cast<uint32_t*>(sink));
}
