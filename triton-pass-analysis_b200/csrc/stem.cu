// Data movement around a spiking ResNet's stem (snn_compiler/zoo/resnet.py:128-131: 7x7 /
// stride 2 conv + BN + neuron on the image, then nn.MaxPool2d(3, stride=2, padding=1)).
//
// Window gather (snnb_window_gather_nhwc): with 3 image channels a 7x7 conv would give each
// tap's 64-wide k-slab 3 useful channels, so the window is gathered into the channel
// dimension first and the conv runs as a 1x1 conv with K = 147 on the tensor-core kernel.
// The pixel's K columns are ordered (dy, dx, c) and zero padded to Kp.  The staged kernel
// below takes the windows from shared memory; where its window does not fit, one thread per
// (output pixel, 8 columns) gathers from global memory with 2-byte loads.
//
// Max-pool (snnb_maxpool_nhwc): k x k with stride and padding on NHWC bf16 frames, applied
// per frame.  Memory-bound: one thread per (output pixel, 8 channels) reads the window's
// 16-byte chunks and writes one; padding positions are skipped (max over the in-image
// window, as torch's -inf padding gives).  On {0, 1} spikes the max is the OR of the window.
#include "common.cuh"

namespace snnb {
namespace {

__global__ void __launch_bounds__(256) window_gather_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t frames, int H, int W, int C, int k, int stride,
    int pad, int Ho, int Wo, int Kp, __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    // thread = (output pixel, group of 8 columns): adjacent threads store adjacent 16 bytes
    const int KG = Kp / 8;
    const int64_t total = frames * Ho * Wo * KG;
    const int K = k * k * C;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int grp = (int)(i % KG);
        const int64_t pix = i / KG;
        const int wo = (int)(pix % Wo);
        const int64_t r = pix / Wo;
        const int ho = (int)(r % Ho);
        const int64_t f = r / Ho;
        const __nv_bfloat16* src = x + f * H * W * C;
        const int h0 = ho * stride - pad, w0 = wo * stride - pad;
        // column j = (dy * k + dx) * C + c
        int j = grp * 8;
        int c = j % C, t = j / C;
        int dx = t % k, dy = t / k;
        uint32_t v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e, ++j) {
            v[e] = 0;
            if (j < K) {
                const int h = h0 + dy, w = w0 + dx;
                if (h >= 0 && h < H && w >= 0 && w < W)
                    v[e] = __bfloat16_as_ushort(src[((int64_t)h * W + w) * C + c]);
                if (++c == C) {
                    c = 0;
                    if (++dx == k) { dx = 0; ++dy; }
                }
            }
        }
        uint4 q;
        q.x = v[0] | (v[1] << 16);
        q.y = v[2] | (v[3] << 16);
        q.z = v[4] | (v[5] << 16);
        q.w = v[6] | (v[7] << 16);
        reinterpret_cast<uint4*>(out)[i] = q;
    }
}

// Staged form: CTA = (frame, output row, 64 output columns).  The k input rows x the
// (63 * stride + k) input columns the 64 windows span are loaded once into shared memory
// (coalesced: consecutive threads, consecutive values of a row; zeros outside the image),
// then the threads build the pixels' 16-byte column groups from shared memory and the CTA
// stores its 64 pixels' Kp columns as one contiguous run.  Run-time divisions stay out of
// the loops (an earlier form with four per staged value was issue-bound at ~1 ms for the
// ResNet stem at batch 64).
constexpr int GATHER_WB = 64;                 // output columns per CTA
constexpr int GATHER_SMEM = 16 * 1024;        // largest staged window (bytes)

__global__ void __launch_bounds__(128) window_gather_staged_kernel(
    const __nv_bfloat16* __restrict__ x, int H, int W, int C, int k, int stride, int pad,
    int Ho, int Wo, int Kp, __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    __shared__ uint16_t win[GATHER_SMEM / 2];
    const int nwb = (Wo + GATHER_WB - 1) / GATHER_WB;
    const int wb = (int)(blockIdx.x % nwb);
    const int ho = (int)((blockIdx.x / nwb) % Ho);
    const int64_t f = (int64_t)blockIdx.x / nwb / Ho;
    const int wo0 = wb * GATHER_WB;
    const int cols = (GATHER_WB - 1) * stride + k;          // input columns of the 32 windows
    const int rowv = cols * C;                                // values per staged row
    const int h0 = ho * stride - pad, w0 = wo0 * stride - pad;
    const __nv_bfloat16* src = x + f * H * W * C;
    // a staged row is one contiguous run of the image row (columns w0 .. w0 + cols - 1);
    // the columns outside the image are the values q < qlo or q >= qhi (no division)
    const int qlo = w0 < 0 ? -w0 * C : 0, qhi = (W - w0) * C;
    for (int r = 0; r < k; ++r) {
        const int h = h0 + r;
        const bool hin = h >= 0 && h < H;
        const int64_t rb = ((int64_t)(hin ? h : 0) * W + w0) * C;   // value q at rb + q
        for (int q = threadIdx.x; q < rowv; q += blockDim.x)
            win[r * rowv + q] = (hin && q >= qlo && q < qhi) ? __bfloat16_as_ushort(src[rb + q])
                                                              : (uint16_t)0;
    }
    // thread = one column group g (8 columns) for pixels lane, lane + lanes, ...: the 8
    // columns' offsets in the staged window are computed once (the run-time divisions by C
    // and k stay out of the pixel loop); consecutive threads store consecutive 16 bytes
    const int KG = Kp / 8, K = k * k * C;
    const int lanes = blockDim.x / KG;                        // >= 1 (host: KG <= blockDim)
    const int g = threadIdx.x % KG, lane = threadIdx.x / KG;
    int off[8];
    {
        int j = g * 8, c = j % C, t = j / C, dx = t % k, dy = t / k;   // one division set
#pragma unroll
        for (int e = 0; e < 8; ++e, ++j) {
            off[e] = j < K ? dy * rowv + dx * C + c : -1;
            if (++c == C) {
                c = 0;
                if (++dx == k) { dx = 0; ++dy; }
            }
        }
    }
    __syncthreads();
    const int npix = Wo - wo0 < GATHER_WB ? Wo - wo0 : GATHER_WB;
    uint4* dst = reinterpret_cast<uint4*>(out + (((f * Ho + ho) * Wo) + wo0) * Kp);
    if (lane >= lanes) return;
    for (int p = lane; p < npix; p += lanes) {
        const int base = p * stride * C;
        uint32_t v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = off[e] >= 0 ? win[base + off[e]] : 0u;
        uint4 q;
        q.x = v[0] | (v[1] << 16);
        q.y = v[2] | (v[3] << 16);
        q.z = v[4] | (v[5] << 16);
        q.w = v[6] | (v[7] << 16);
        dst[p * KG + g] = q;
    }
}

__global__ void __launch_bounds__(256) maxpool_nhwc_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t frames, int H, int W, int C, int k, int stride,
    int pad, int Ho, int Wo, __nv_bfloat16* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    const int C8 = C / 8;
    const int64_t total = frames * Ho * Wo * C8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int c8 = (int)(i % C8);
        int64_t r = i / C8;
        const int wo = (int)(r % Wo);
        r /= Wo;
        const int ho = (int)(r % Ho);
        const int64_t f = r / Ho;
        const int h0 = ho * stride - pad, w0 = wo * stride - pad;
        __nv_bfloat162 m[4];
        bool first = true;
        for (int dy = 0; dy < k; ++dy) {
            const int h = h0 + dy;
            if (h < 0 || h >= H) continue;
            for (int dx = 0; dx < k; ++dx) {
                const int w = w0 + dx;
                if (w < 0 || w >= W) continue;
                const uint4 q = __ldg(reinterpret_cast<const uint4*>(
                    x + ((f * H + h) * W + w) * C) + c8);
                const __nv_bfloat162* v = reinterpret_cast<const __nv_bfloat162*>(&q);
#pragma unroll
                for (int j = 0; j < 4; ++j) m[j] = first ? v[j] : __hmax2(m[j], v[j]);
                first = false;
            }
        }
        uint4 o;
        __nv_bfloat162* ov = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) ov[j] = m[j];
        reinterpret_cast<uint4*>(out + ((f * Ho + ho) * Wo + wo) * C)[c8] = o;
    }
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_maxpool_nhwc(const void* x, int64_t frames, int64_t H, int64_t W, int64_t C,
                                 int k, int stride, int pad, void* out, snnb_stream_t stream) {
    if (const int inj = take_injected_status()) return inj;
    if (!x || !out || frames < 0 || H <= 0 || W <= 0 || C <= 0 || C % 8) return SNNB_ERR_ARG;
    // (pad < k: every window touches the image)
    if (k < 1 || k > 8 || stride < 1 || stride > 8 || pad < 0 || pad >= k) return SNNB_ERR_ARG;
    if (H > 0x7fffffff || W > 0x7fffffff || C > 0x7fffffff || !aligned16(x) || !aligned16(out))
        return SNNB_ERR_ARG;
    if (H + 2 * pad < k || W + 2 * pad < k) return SNNB_ERR_ARG;
    const int64_t Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
    if (frames > ((int64_t)1 << 40) / (Ho * Wo * C)) return SNNB_ERR_ARG;
    const int64_t total = frames * Ho * Wo * (C / 8);
    if (total == 0) return SNNB_OK;
    const int64_t blocks = (total + 255) / 256;
    const int grid = (int)(blocks < 148 * 32 ? blocks : 148 * 32);
    return launch_k(maxpool_nhwc_kernel, dim3(grid), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x),
                    frames, (int)H, (int)W, (int)C, k, stride, pad, (int)Ho, (int)Wo,
                    static_cast<__nv_bfloat16*>(out));
}

extern "C" int snnb_window_gather_nhwc(const void* x, int64_t frames, int64_t H, int64_t W,
                                       int64_t C, int k, int stride, int pad, int64_t Kp,
                                       void* out, snnb_stream_t stream) {
    if (const int inj = take_injected_status()) return inj;
    if (!x || !out || frames < 0 || H <= 0 || W <= 0 || C <= 0) return SNNB_ERR_ARG;
    if (k < 1 || k > 11 || stride < 1 || stride > 8 || pad < 0 || pad >= k) return SNNB_ERR_ARG;
    if (H > 0x7fffffff || W > 0x7fffffff || C > 4096 || Kp % 8 || Kp < (int64_t)k * k * C ||
        Kp > 0x7fffffff || !aligned16(out))
        return SNNB_ERR_ARG;
    if (H + 2 * pad < k || W + 2 * pad < k) return SNNB_ERR_ARG;
    const int64_t Ho = (H + 2 * pad - k) / stride + 1, Wo = (W + 2 * pad - k) / stride + 1;
    if (frames > ((int64_t)1 << 40) / (Ho * Wo * Kp)) return SNNB_ERR_ARG;
    const int64_t total = frames * Ho * Wo * (Kp / 8);
    if (total == 0) return SNNB_OK;
    const int64_t staged = (int64_t)k * ((GATHER_WB - 1) * stride + k) * C * 2;
    const int64_t ctas = frames * Ho * ((Wo + GATHER_WB - 1) / GATHER_WB);
    if (staged <= GATHER_SMEM && Kp / 8 <= 128 && ctas <= 0x7fffffff)
        return launch_k(window_gather_staged_kernel, dim3((unsigned)ctas), dim3(128), 0,
                        static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x),
                        (int)H, (int)W, (int)C, k, stride, pad, (int)Ho, (int)Wo, (int)Kp,
                        static_cast<__nv_bfloat16*>(out));
    const int64_t blocks = (total + 255) / 256;
    const int grid = (int)(blocks < 148 * 32 ? blocks : 148 * 32);
    return launch_k(window_gather_kernel, dim3(grid), dim3(256), 0,
                    static_cast<cudaStream_t>(stream), static_cast<const __nv_bfloat16*>(x),
                    frames, (int)H, (int)W, (int)C, k, stride, pad, (int)Ho, (int)Wo, (int)Kp,
                    static_cast<__nv_bfloat16*>(out));
}
