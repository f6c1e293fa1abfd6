// Strided and k x k convs on the T-folded fused conv + LIF kernel (conv_lif_tm_kernel with
// GEN): the convs of a spiking ResNet that are not 3x3 / stride 1 -- the 3x3 / stride 2
// first conv of a downsampling block, 1x1 convs (the downsample branch among them) and the
// 7x7 / stride 2 stem.  The activation boxes traverse the input with the conv's stride
// (the tensor map's element strides, encoded by run_tc_layer), so a tile's operand lands in
// shared memory exactly as for a stride-1 conv; only the producers' tap coordinates differ.
// These instantiations live in their own translation unit so they compile beside the
// stride-1 ones, which keep the plain coordinate arithmetic.
#include "conv_tm.cuh"

namespace snnb {
namespace {

template <typename K>
int launch_gen_kernel(K k, int dyn, int threads, const CUtensorMap& ta, const CUtensorMap& tb,
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
    // persistent: one work item per (tile, split), at most the resident CTAs
    const int64_t cap = (int64_t)sms * occ;
    const int64_t items = (int64_t)p.num_tiles * (p.splits > 1 ? p.splits : 1);
    const int grid = (int)(items < cap ? items : cap);
    return launch_k(k, dim3(grid), dim3(threads), dyn, s, ta, tb, p);
}

template <int BN, int STAGES, int TS>
int launch_gen(const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
               cudaStream_t s) {
    constexpr int dyn = SmemTM<BN, STAGES, TS, 1>::DYN;
    constexpr int NP = BN == 256 ? 2 : (BN == 64 ? 4 : 3);
    constexpr int threads = THREADS + 32 * (NP - 1) + 128;
    if (p.res)
        return p.hard
            ? launch_gen_kernel(conv_lif_tm_kernel<BN, STAGES, TS, true, NP, 1, 1, true, 1, 0, false, false, true>,
                                dyn, threads, ta, tb, p, s)
            : launch_gen_kernel(conv_lif_tm_kernel<BN, STAGES, TS, false, NP, 1, 1, true, 1, 0, false, false, true>,
                                dyn, threads, ta, tb, p, s);
    return p.hard
        ? launch_gen_kernel(conv_lif_tm_kernel<BN, STAGES, TS, true, NP, 1, 1, false, 1, 0, false, false, true>,
                            dyn, threads, ta, tb, p, s)
        : launch_gen_kernel(conv_lif_tm_kernel<BN, STAGES, TS, false, NP, 1, 1, false, 1, 0, false, false, true>,
                            dyn, threads, ta, tb, p, s);
}

template <int TS>
int launch_gen_ts(int BN, const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
                  cudaStream_t s) {
    switch (BN) {       // the ring depths of the stride-1 forms (conv_lif.cu: launch_tm_bn)
        case 256: return launch_gen<256, 4, TS>(ta, tb, p, s);
        case 128: return launch_gen<128, 7, TS>(ta, tb, p, s);
        case 64: return launch_gen<64, 9, TS>(ta, tb, p, s);
        default: return launch_gen<32, 10, TS>(ta, tb, p, s);
    }
}

}  // namespace

int launch_tm_general(int TS, int BN, const CUtensorMap& ta, const CUtensorMap& tb,
                      const ConvParams& p, cudaStream_t s) {
    switch (TS) {
        case 2: return launch_gen_ts<2>(BN, ta, tb, p, s);
        case 4: return launch_gen_ts<4>(BN, ta, tb, p, s);
        case 8: return launch_gen_ts<8>(BN, ta, tb, p, s);
        default: return SNNB_ERR_UNSUPPORTED;
    }
}

}  // namespace snnb
