// Packed spikes between layers: the T-folded fused conv + LIF kernel reading its input as
// packed spikes (conv_lif_tm_kernel with PATCH > 0) and / or writing packed spikes (PKO), the
// unpacking kernel, and the column-group-pool instantiations of the dense 2x2 form (CPOOL):
// the epilogue options that only these launches use are compiled into their own kernels.
//
// Packed layout: NHWC spikes with 32 channels per uint32 word, channel c of a pixel in bit
// c % 32 of word c / 32 (LSB first; the order snnb_bitpack writes for rows of C channels):
// [T*B][H][W][C/32] words, 1/16 of the bf16 layout's bytes.  The conv kernel stages each
// tile's packed input patch (its pixels and 1-pixel halo at every step) in shared memory
// once and expands every k-slab's A operand from it into the swizzled bf16 tile the
// tensor core reads, so no activation bytes cross L2 per k-slab; the weights still arrive
// by TMA.  The products and their accumulation order are those of the bf16-input kernel,
// so the spikes are identical to it.
#include "conv_tm.cuh"

namespace snnb {
namespace {

constexpr int PATCH_BYTES = 32 * 1024;

template <typename K>
int launch_pk_kernel(K k, int dyn, int threads, const CUtensorMap& ta, const CUtensorMap& tb,
                     const ConvParams& p, cudaStream_t s) {
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (e != cudaSuccess) return record_cuda_error(e);
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, k, threads, dyn);
    if (e != cudaSuccess) return record_cuda_error(e);
    if (occ < 1) return SNNB_ERR_UNSUPPORTED;
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t cap = (int64_t)sms * occ;
    const int grid = (int)(p.num_tiles < cap ? p.num_tiles : cap);
    return launch_k(k, dim3(grid), dim3(threads), dyn, s, ta, tb, p);
}

// packed input (four producer warps expanding the staged patch), output packed or bf16
template <int BN, int STAGES, int TS, bool PKO>
int launch_pk(const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
              cudaStream_t s) {
    constexpr int NP = 4;
    constexpr int dyn = SmemTM<BN, STAGES, TS, 1, 1, PATCH_BYTES>::DYN;
    constexpr int threads = THREADS + 32 * (NP - 1) + 128;
    return p.hard
        ? launch_pk_kernel(conv_lif_tm_kernel<BN, STAGES, TS, true, NP, 1, 1, false, 1, PATCH_BYTES, PKO>,
                           dyn, threads, ta, tb, p, s)
        : launch_pk_kernel(conv_lif_tm_kernel<BN, STAGES, TS, false, NP, 1, 1, false, 1, PATCH_BYTES, PKO>,
                           dyn, threads, ta, tb, p, s);
}

// bf16 input by TMA (the stage depths and producer warps of the plain T-folded kernel),
// packed output
template <int BN, int STAGES, int TS>
int launch_po(const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
              cudaStream_t s) {
    constexpr int NP = BN == 256 ? 2 : (BN == 64 ? 4 : 3);
    constexpr int dyn = SmemTM<BN, STAGES, TS, 1>::DYN;
    constexpr int threads = THREADS + 32 * (NP - 1) + 128;
    return p.hard
        ? launch_pk_kernel(conv_lif_tm_kernel<BN, STAGES, TS, true, NP, 1, 1, false, 1, 0, true>,
                           dyn, threads, ta, tb, p, s)
        : launch_pk_kernel(conv_lif_tm_kernel<BN, STAGES, TS, false, NP, 1, 1, false, 1, 0, true>,
                           dyn, threads, ta, tb, p, s);
}

// the dense form of a pooled 2x2-image layer: bf16 in and out, column-group pool
template <int BN, int STAGES, int TS>
int launch_cp(const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
              cudaStream_t s) {
    constexpr int NP = BN == 256 ? 2 : (BN == 64 ? 4 : 3);
    constexpr int dyn = SmemTM<BN, STAGES, TS, 1>::DYN;
    constexpr int threads = THREADS + 32 * (NP - 1) + 128;
    return p.hard
        ? launch_pk_kernel(conv_lif_tm_kernel<BN, STAGES, TS, true, NP, 1, 1, false, 1, 0, false, true>,
                           dyn, threads, ta, tb, p, s)
        : launch_pk_kernel(conv_lif_tm_kernel<BN, STAGES, TS, false, NP, 1, 1, false, 1, 0, false, true>,
                           dyn, threads, ta, tb, p, s);
}

template <int TS>
int launch_cp_ts(int BN, const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
                 cudaStream_t s) {
    switch (BN) {
        case 256: return launch_cp<256, 4, TS>(ta, tb, p, s);
        case 128: return launch_cp<128, 7, TS>(ta, tb, p, s);
        case 64: return launch_cp<64, 9, TS>(ta, tb, p, s);
        default: return launch_cp<32, 10, TS>(ta, tb, p, s);
    }
}

template <int TS>
int launch_pk_ts(int BN, int x_packed, int out_packed, const CUtensorMap& ta,
                 const CUtensorMap& tb, const ConvParams& p, cudaStream_t s) {
    if (!x_packed) {
        switch (BN) {
            case 256: return launch_po<256, 4, TS>(ta, tb, p, s);
            case 128: return launch_po<128, 7, TS>(ta, tb, p, s);
            case 64: return launch_po<64, 9, TS>(ta, tb, p, s);
            default: return launch_po<32, 10, TS>(ta, tb, p, s);
        }
    }
    switch (BN) {
        case 256: return out_packed ? launch_pk<256, 3, TS, true>(ta, tb, p, s)
                                    : launch_pk<256, 3, TS, false>(ta, tb, p, s);
        case 128: return out_packed ? launch_pk<128, 6, TS, true>(ta, tb, p, s)
                                    : launch_pk<128, 6, TS, false>(ta, tb, p, s);
        case 64: return out_packed ? launch_pk<64, 8, TS, true>(ta, tb, p, s)
                                   : launch_pk<64, 8, TS, false>(ta, tb, p, s);
        default: return SNNB_ERR_UNSUPPORTED;
    }
}

// thread = one packed word -> 32 bf16 {0, 1} (four 16-byte stores)
__global__ void __launch_bounds__(256) unpack_spikes_kernel(const uint32_t* __restrict__ words,
                                                            int64_t nwords,
                                                            __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nwords) return;
    const uint32_t w = __ldg(words + i);
    uint4* dst = reinterpret_cast<uint4*>(out + i * 32);
#pragma unroll
    for (int k = 0; k < 4; ++k) dst[k] = spikes_to_bf16x8((w >> (8 * k)) & 0xffu);
}

}  // namespace

int packed_patch_limit() { return PATCH_BYTES; }

int launch_tm_cpool(int TS, int BN, const CUtensorMap& ta, const CUtensorMap& tb,
                    const ConvParams& p, cudaStream_t s) {
    switch (TS) {
        case 2: return launch_cp_ts<2>(BN, ta, tb, p, s);
        case 4: return launch_cp_ts<4>(BN, ta, tb, p, s);
        case 8: return launch_cp_ts<8>(BN, ta, tb, p, s);
        default: return SNNB_ERR_UNSUPPORTED;
    }
}

int launch_tm_packed(int TS, int BN, int x_packed, int out_packed, const CUtensorMap& ta,
                     const CUtensorMap& tb, const ConvParams& p, cudaStream_t s) {
    switch (TS) {
        case 2: return launch_pk_ts<2>(BN, x_packed, out_packed, ta, tb, p, s);
        case 4: return launch_pk_ts<4>(BN, x_packed, out_packed, ta, tb, p, s);
        case 8: return launch_pk_ts<8>(BN, x_packed, out_packed, ta, tb, p, s);
        default: return SNNB_ERR_UNSUPPORTED;
    }
}

}  // namespace snnb

using namespace snnb;

extern "C" int snnb_unpack_spikes(const void* words, int64_t rows, int64_t C, void* out,
                                  snnb_stream_t stream) {
    if (const int inj = snnb::take_injected_status()) return inj;
    if (!words || !out || rows < 0 || C <= 0 || C % 32 != 0) return SNNB_ERR_ARG;
    if (!aligned16(out) || (reinterpret_cast<uintptr_t>(words) & 3u)) return SNNB_ERR_ARG;
    const int64_t nwords = rows * (C / 32);
    if (nwords == 0) return SNNB_OK;
    const int64_t blocks = (nwords + 255) / 256;
    if (blocks > 0x7fffffff) return SNNB_ERR_ARG;
    return launch_k(unpack_spikes_kernel, dim3((unsigned)blocks), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const uint32_t*>(words),
                    nwords, static_cast<__nv_bfloat16*>(out));
}
