// Cluster split-K form of the T-folded fused conv + LIF kernel (conv_lif_tm_kernel, SK > 1).
//
// For layers with few output pixels (VGG16's 2x2 and 4x4 layers at batch 64) a grid of
// 128-row tiles leaves most SMs idle unless the K range is split.  Here the SK splits of a
// tile run as one thread-block cluster: each CTA accumulates its k-slab range in TMEM,
// stages the float32 partial sums in its drained operand ring, and after a cluster barrier
// finishes 1/SK of the tile's channels -- it adds the SK partial sums of its slices in
// split order from the CTAs' shared memory (ld.shared::cluster), then runs bias, residual,
// LIF, pooling and the spike stores exactly as the single-CTA epilogue does.  The split
// boundaries and the summation order are those of the two-launch split-K form
// (conv_lif.cu: partial sums in global memory + splitsum_lif_kernel), so the results are
// bit-identical to it, with no partial-sum round trip through L2 and no second launch.
#include "conv_tm.cuh"

namespace snnb {
namespace {

template <int BN, int STAGES, int TS, int SK>
int launch_ck(const CUtensorMap& ta, const CUtensorMap& tb, const ConvParams& p,
              cudaStream_t s) {
    constexpr int dyn = SmemTM<BN, STAGES, TS, 1>::DYN;
    constexpr int NP = BN == 256 ? 2 : (BN == 64 ? 4 : 3);
    constexpr int threads = THREADS + 32 * (NP - 1) + 128;
    void (*k)(const CUtensorMap, const CUtensorMap, const ConvParams) =
        p.hard ? (p.res ? conv_lif_tm_kernel<BN, STAGES, TS, true, NP, 1, 1, true, SK>
                        : conv_lif_tm_kernel<BN, STAGES, TS, true, NP, 1, 1, false, SK>)
               : (p.res ? conv_lif_tm_kernel<BN, STAGES, TS, false, NP, 1, 1, true, SK>
                        : conv_lif_tm_kernel<BN, STAGES, TS, false, NP, 1, 1, false, SK>);
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn);
    if (e != cudaSuccess) return record_cuda_error(e);
    // SK CTAs of ~227 KB each must fit in one GPC at once
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)SK);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = dyn;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = SK;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, k, &cfg);
    if (e != cudaSuccess) return record_cuda_error(e);
    if (clusters < 1) return SNNB_ERR_UNSUPPORTED;
    // one cluster per tile (the staged partial sums alias the operand ring, so a cluster
    // never takes a second tile)
    return launch_kc(k, dim3((unsigned)(p.num_tiles * SK)), dim3(threads), dyn, s,
                     (unsigned)SK, ta, tb, p);
}

template <int TS>
int launch_ck_ts(int BN, int SK, const CUtensorMap& ta, const CUtensorMap& tb,
                 const ConvParams& p, cudaStream_t s) {
    if (BN == 128 && SK == 2) return launch_ck<128, 7, TS, 2>(ta, tb, p, s);
    if (BN == 128 && SK == 4) return launch_ck<128, 7, TS, 4>(ta, tb, p, s);
    if (BN == 256 && SK == 2) return launch_ck<256, 4, TS, 2>(ta, tb, p, s);
    if (BN == 256 && SK == 4) return launch_ck<256, 4, TS, 4>(ta, tb, p, s);
    if (BN == 256 && SK == 8) return launch_ck<256, 4, TS, 8>(ta, tb, p, s);
    return SNNB_ERR_UNSUPPORTED;
}

}  // namespace

int launch_tm_cluster(int TS, int BN, int SK, const CUtensorMap& ta, const CUtensorMap& tb,
                      const ConvParams& p, cudaStream_t s) {
    if ((int64_t)p.num_tiles * SK > 0x7fffffff) return SNNB_ERR_ARG;
    switch (TS) {
        case 2: return launch_ck_ts<2>(BN, SK, ta, tb, p, s);
        case 4: return launch_ck_ts<4>(BN, SK, ta, tb, p, s);
        case 8: return launch_ck_ts<8>(BN, SK, ta, tb, p, s);
        default: return SNNB_ERR_UNSUPPORTED;
    }
}

}  // namespace snnb
