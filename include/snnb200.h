/*
 * snnb200.h -- C ABI of libsnnb200.so, the sm_100a (B200) kernels behind the
 * snn_compiler.kernels / snn_compiler.nn API.
 *
 * Every entry point
 *   - takes plain device pointers, element counts and a CUDA stream
 *     (snnb_stream_t is a cudaStream_t; NULL means the legacy default stream),
 *   - launches asynchronously on that stream and never synchronises it (except
 *     snnb_read_device_status, which must read the status word back),
 *   - allocates nothing: the caller owns every input, output and workspace,
 *     and passes workspace explicitly where a kernel needs scratch memory.  The
 *     one exception is snnb_conv3x3_lif_static_scratch, whose scratch is a fixed
 *     16 MiB array inside the library (held on every GPU that loads it),
 *   - returns an int status (SNNB_OK or a negative SNNB_ERR_*), never aborts and
 *     never throws across the boundary.
 * Shapes follow the reference's flattening: a multi-step tensor [T, B, ...] is
 * [T, N] with N = numel of one step, in memory order.
 */
#ifndef SNNB200_H
#define SNNB200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* snnb_stream_t;

/* status codes */
#define SNNB_OK                 0
#define SNNB_ERR_ARG           -1   /* bad pointer / size / alignment / combination */
#define SNNB_ERR_UNSUPPORTED   -2   /* valid request this build does not implement */
#define SNNB_ERR_CUDA          -3   /* a CUDA runtime call or launch failed */
#define SNNB_ERR_TIMEOUT       -4   /* a bounded device-side wait gave up */
#define SNNB_ERR_DEVICE        -5   /* a device-side check recorded an error */

/* element types */
#define SNNB_F32   0
#define SNNB_F16   1
#define SNNB_BF16  2
#define SNNB_U8    3

/* threshold modes, snn_compiler/kernels/neurons.py:66-68 */
#define SNNB_THR_SCALAR       0
#define SNNB_THR_PER_CHANNEL  1
#define SNNB_THR_PER_NEURON   2

/* ABI revision of this header; bumped on any signature change. */
int snnb_abi_version(void);

/* Human-readable text of a status code (static storage). */
const char* snnb_status_string(int status);

/* Text of the last CUDA error seen by this library on the calling thread. */
const char* snnb_last_cuda_error(void);

/*
 * K2 -- multi-step IF / LIF / PLIF neuron over x [T, N].
 *
 * Replaces the Triton kernels and Python entry points
 *   if_lif                      snn_compiler/kernels/neurons.py:311-376 (_if_lif_kernel :85-138)
 *   fused_bias_if_lif           snn_compiler/kernels/fused.py:117-226   (_bias_if_lif_kernel :50-114)
 *   fused_bias_if_lif_rate      snn_compiler/kernels/fused.py:303-382   (kernel :242-300)
 *   fused_bias_if_lif_stateful  snn_compiler/kernels/fused.py:444-507   (kernel :398-441)
 * in one launch.  Per element n and step t, every operation rounded to float32
 * in this order (no FMA contraction):
 *   in = x[t,n] (+ bias[c]) (+ residual[t,n]);  v = decay*v + input_scale*in;
 *   s = v >= thr;  soft: v -= s*thr;  hard: v = s ? v_reset : v
 * with c = n % C (channel_last) or (n / HW) % C.
 *
 * x, residual   : [T, N] of x_dtype (F32 / F16 / BF16); residual may be NULL.
 * bias          : [C] float32 or NULL.
 * plif_w        : NULL, or a device float32 scalar w; then input_scale = k and
 *                 decay = 1 - k with k = sigmoid(w) (evaluated in double and
 *                 rounded to float32), overriding the two float arguments -- PLIF in
 *                 the reference's charge form; snnb_neuron_plif has SpikingJelly's.
 * thr           : [C] (per channel) or [N] (per neuron) float32 for those modes.
 * v_init        : [N] float32 initial potential, or NULL for zeros.
 * outputs (any subset, NULL = not written):
 *   spikes        [T, N] of spikes_dtype (F32 / F16 / BF16 / U8), values 0 or 1
 *   spikes_packed [T, ceil(N/32)] uint32: bit i of word w of step t = s[t, 32w+i]
 *   count         [N] float32 = sum over t of s  (rate-coded output)
 *   v_out         [N] float32 potential after the last step
 * Vectorised 16-byte loads are used when N is a multiple of 8 and every
 * pointer is 16-byte aligned; otherwise a scalar path runs.
 */
int snnb_neuron_multistep(
    const void* x, int x_dtype, int64_t T, int64_t N,
    const float* bias, const void* residual, int64_t C, int64_t HW, int channel_last,
    float decay, float input_scale, const float* plif_w,
    int hard_reset, float v_reset,
    int thr_mode, float thr_scalar, const float* thr,
    const float* v_init,
    void* spikes, int spikes_dtype,
    uint32_t* spikes_packed, float* count, float* v_out,
    snnb_stream_t stream);

/*
 * K2 -- SpikingJelly ParametricLIFNode (PLIF) over x [T, N] (no snn_compiler counterpart:
 * PLIF lives in SpikingJelly, which the reference drives through
 * examples/snn_triton_pipeline/.../_common/sj_compat.py:39-44).  k is a device float32
 * scalar, SpikingJelly's w.sigmoid() (the caller evaluates it, as SpikingJelly does with
 * torch on the module's device).  Per element, every operation rounded to float32 in
 * SpikingJelly's order:
 *   decay_input:                          v = v + (x - (v - v_reset)) * k
 *   not decay_input, v_reset 0 or soft:   v = v * (1 - k) + x
 *   not decay_input, v_reset != 0:        v = v - (v - v_reset) * k + x
 *   s = v >= v_threshold;  hard: v = s ? v_reset : v;  soft: v = s ? v - v_threshold : v
 * (soft reset is SpikingJelly's v_reset = None: the charge uses 0 for v_reset).  v starts at
 * v_init, or 0 when v_init is NULL (SpikingJelly starts a hard-reset neuron at v_reset: pass
 * v_init filled with it).  Outputs as snnb_neuron_multistep.
 */
int snnb_neuron_plif(const void* x, int x_dtype, int64_t T, int64_t N, const float* k,
                     int decay_input, int hard_reset, float v_reset, float v_threshold,
                     const float* v_init, void* spikes, int spikes_dtype,
                     uint32_t* spikes_packed, float* count, float* v_out,
                     snnb_stream_t stream);

/* two-state / nonlinear neuron models of snnb_neuron_cuba_eif */
#define SNNB_MODEL_CUBA  0
#define SNNB_MODEL_EIF   1

/*
 * K2, second form -- multi-step CubaLIF or exponential IF over x [T, N] -> spikes of
 * x's dtype.
 *
 * Replaces the Triton kernels and Python entry points
 *   cuba_lif   snn_compiler/kernels/neurons.py:379-418 (_cuba_lif_kernel :143-194)
 *   eif        snn_compiler/kernels/neurons.py:421-457 (_eif_kernel :200-261)
 * following their eager restatements naive_cuba_lif / naive_eif (:505-557): per element n
 * and step t, each operation rounded to float32 in this order (no FMA contraction):
 *   CUBA:  i = a*i + input_scale*x;  v = b*v + i
 *   EIF :  e = exp(min((v - v_rh) / delta_T, 16));  v = (a*v + delta_T*e) + input_scale*x
 *   s = v >= thr;  soft: v -= s*thr;  hard: v = s ? v_reset : v
 * (a = alpha, b = beta for CUBA; a = decay for EIF; i and v start at 0).  exp is CUDA's
 * expf, which may differ from a CPU exp in the last bit.  thr modes and the channel index
 * (c = n % C when channel_last, else (n / HW) % C) as for snnb_neuron_multistep.
 */
int snnb_neuron_cuba_eif(
    const void* x, int x_dtype, int64_t T, int64_t N, int64_t C, int64_t HW, int channel_last,
    int model, float a, float b, float input_scale, float delta_T, float v_rh,
    int hard_reset, float v_reset, int thr_mode, float thr_scalar, const float* thr,
    void* spikes, snnb_stream_t stream);

/*
 * K4 -- bit packing of {0,1} or {-1,+1} rows into 32-bit words.
 *
 * Replaces _pack_N_kernel / _pack_N (snn_compiler/kernels/attention.py:195-242) and
 * the torch bit-pack bitpack_N (snn_compiler/explore/attention/phase6b_bitpack.py:35-46):
 * element k of row r goes to bit (k % 32) of word out[r * ldw + k / 32] (LSB first);
 * words from ceil(K/32) to ldw-1 are written as zero.
 * x        : [rows, K] of SNNB_F32 / F16 / BF16 / U8, row-major.
 * positive : 0 -> bit = (x != 0)  ({0,1} spikes);  1 -> bit = (x > 0)  ({-1,+1} signs).
 * ldw      : words per packed row, >= ceil(K/32) (use a multiple of 4 for snnb_bgemm).
 */
int snnb_bitpack(const void* x, int x_dtype, int64_t rows, int64_t K, int64_t ldw,
                 int positive, uint32_t* out, snnb_stream_t stream);

/*
 * K4 -- binary GEMM over packed rows with AND / XOR + popcount.
 *
 * Replaces _ktv_popcount_kernel (snn_compiler/kernels/attention.py:217-233) and
 * spike_ktv_popcount (attention.py:245-258), generalised:
 *   mode 0: C[m,n] = sum_k A[m,k] B[n,k]                 A, B in {0,1}
 *   mode 1: C[m,n] = sum_k A[m,k] (2 Bbit[n,k] - 1)      A in {0,1}, B in {-1,+1}
 *   mode 2: C[m,n] = sum_k (2 Abit - 1)(2 Bbit - 1)      A, B in {-1,+1} (XNOR form)
 * A [M, ldw], B [N, ldw] packed as by snnb_bitpack (16-byte aligned, ldw % 4 == 0,
 * zero padding words); C [M, N] int32 row-major, exact.
 * splits: number of k-range splits (0 = choose to fill the GPU); with more than
 * one split C is zeroed with cudaMemsetAsync and partial sums are added atomically.
 */
int snnb_bgemm(const uint32_t* A, const uint32_t* B, int32_t* C, int64_t M, int64_t N,
               int64_t K, int64_t ldw, int mode, int splits, snnb_stream_t stream);

/*
 * Measurement helper (no reference counterpart): the binary GEMM's inner operation at this
 * GPU's peak -- `blocks` CTAs of 256 threads, each thread `iters` rounds of 64 independent
 * word-ops acc += popc(a & b) on registers, i.e. blocks * 256 * iters * 64 word-ops per
 * launch; time it to get the roofline denominator of snnb_bgemm.  sink: >= 1 KB of device
 * memory (written only in a case that does not occur).
 */
int snnb_popc_peak(int64_t blocks, int iters, void* sink, snnb_stream_t stream);

/*
 * K1 -- fused conv3x3 (stride 1, pad 1) + folded-BN bias + multi-step LIF (+ 2x2 max-pool)
 * on the tcgen05 tensor cores (bf16 x bf16 -> f32 in TMEM, operands fed by TMA).
 *
 * Replaces, per layer, F.conv2d + _bias_if_lif_kernel + nn.MaxPool2d of
 *   FusedConvBNNeuron.forward   snn_compiler/nn/modules.py:347-357 (_conv_bn :324-345)
 *   fused_bias_if_lif           snn_compiler/kernels/fused.py:117-226
 *   VGGSNN pool                 snn_compiler/zoo/vgg.py:56, :100-104 (pool='max')
 * x    : bf16 spikes / activations NHWC [T*B, H, W, Cin] (frame t*B + b), Cin % 8 == 0
 *        (channels are consumed in 64-wide slabs; a partial last slab reads zeros)
 * w    : bf16 folded weights [Cout, 3, 3, Cin] (K-major), Cout % 32 == 0
 * bias : f32 [Cout] folded bias b' (added inside the neuron, fused.py:106-108)
 * out  : bf16 spikes NHWC [T*B, Ho, Wo, Cout], Ho = H/2 and Wo = W/2 when pool != 0
 * The neuron is v = decay*v + input_scale*(conv + b'); s = v >= v_threshold; reset.
 * variant : 0 = choose; 1 = the CTA walks the T steps of a 128-pixel block with two
 *           TMEM accumulators; 2 = T folded into the 128 accumulator rows (128/T pixels
 *           per CTA, T in {2, 4, 8}) for layers too small to fill the GPU otherwise;
 *           3 = as 1 on bands of 128/W whole image rows (W in {8, 16, 32, 64}), each
 *           64-channel slab loaded once per column tap with its halo rows and reused by
 *           the three row taps, the channel block's weights resident in shared memory
 *           (9 * ceil(Cin/64) * block_n <= 864; SNNB_ERR_UNSUPPORTED otherwise);
 *           4 = as 2 with two 128-row tiles per CTA sharing every weight stage (block_n <= 128);
 *           5 = as 2 on CTA pairs (clusters of 2, M = 256 tcgen05 MMAs with cta_group::2):
 *           each CTA stages its own 128-row tile and half of the block_n weight rows
 *           (block_n 64 / 128 / 256);
 *           6 = as 2 with the K range split across a thread-block cluster of `splits`
 *           CTAs (2 or 4 with block_n 128; 2, 4 or 8 with block_n 256; default block_n
 *           128, 256 for 8) that add their partial sums through distributed shared
 *           memory in the order of the two-launch split-K form (bit-identical to it), each
 *           CTA running the neuron on block_n / splits channels: one launch, no workspace;
 *           7 = as 3 with ONE band copy per stage (W in {8, 16, 32}): each tap row's three
 *           column taps run as one MMA of N = 3 * block_n into three accumulators that the
 *           epilogue adds shifted by one column (9 * ceil(Cin/64) * block_n <= 1280).
 * block_n : output channels per CTA (per CTA pair for variant 5), 0 = choose, or 32 / 64 /
 *           128 (dividing Cout), or 256 with variants 2 and 5; 32 / 64 with variants 3
 *           and 7.
 * splits  : 1, or 2..8 k-range splits for small layers (variant 2): each split's float32
 *           partial sums go to `workspace` (caller-owned, >= snnb_split_workspace_bytes,
 *           16-byte aligned) and a second kernel adds them in a fixed order, adds the bias
 *           and runs the neuron (+ pool).  workspace may be NULL when splits == 1.
 * Pixel blocks: W must divide the block's pixel count or be a multiple of it, likewise
 * H for the rows per block; pooling needs even H and W.
 */
int snnb_conv3x3_lif(const void* x, int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin,
                     const void* w, const float* bias, int64_t Cout,
                     float decay, float input_scale, float v_threshold, float v_reset,
                     int hard_reset, int pool, int variant, int block_n, int splits,
                     void* workspace, int64_t workspace_bytes, void* out,
                     snnb_stream_t stream);

/*
 * K1 with a residual input (ResNet / SEW-ResNet blocks): as snnb_conv3x3_lif without
 * pooling, the neuron's input being (conv + bias) + residual.
 *
 * Replaces FusedConvBNAddNeuron.forward (snn_compiler/nn/modules.py:415-443: conv + BN, then
 * fused_bias_if_lif with residual, fused.py:97-108).
 * residual       : NHWC [T*B, H, W, Cout] (the output's layout) of residual_dtype
 *                  (SNNB_BF16 or SNNB_F32), 16-byte aligned.
 * variant        : 0, 1 (block_n <= 64), 2 (any splits) or 6; 3, 4 and 5 return
 *                  SNNB_ERR_UNSUPPORTED.
 */
int snnb_conv3x3_lif_res(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                         int64_t Cin, const void* w, const float* bias, int64_t Cout,
                         float decay, float input_scale, float v_threshold, float v_reset,
                         int hard_reset, const void* residual, int residual_dtype, int variant,
                         int block_n, int splits, void* workspace, int64_t workspace_bytes,
                         void* out, snnb_stream_t stream);

/*
 * K1 for the other convs of a spiking ResNet: k x k / padding k / 2 with k in {1, 3, 5, 7}
 * (3x3, pointwise and the 7x7 stem), stride 1 or 2, on spike (or any bf16) input, + bias ->
 * multi-step neuron, optionally with the
 * residual input of snnb_conv3x3_lif_res.  Replaces FusedConvBNNeuron.forward and
 * FusedConvBNAddNeuron.forward for these geometries (snn_compiler/nn/modules.py:324-357,
 * :415-443: F.conv2d with stride, then fused_bias_if_lif), i.e. the strided first conv of a
 * downsampling BasicBlock (snn_compiler/zoo/resnet.py:30-117), 1x1 convs and the stem
 * (zoo/resnet.py:120-131; its float32 image as split bf16 terms).  The activation
 * boxes traverse the input with the conv's stride (TMA traversal stride), so the strided
 * conv is the same implicit GEMM as the stride-1 one with no gather.
 * x        : bf16 NHWC [T*B, H, W, Cin] (H, W: the INPUT's sizes), Cin % 8 == 0
 * w        : bf16 [Cout, ksize, ksize, Cin], Cout % 32 == 0
 * out      : bf16 spikes NHWC [T*B, Ho, Wo, Cout], Ho = (H - 1) / stride + 1 (same for W)
 * residual : nullptr, or NHWC [T*B, Ho, Wo, Cout] of residual_dtype (SNNB_BF16 / SNNB_F32)
 * variant / block_n / splits / workspace: as snnb_conv3x3_lif_res; with stride 2 or k > 3
 * (general tap coordinates) variants 0, 1 and 2 only -- 3 to 7 return SNNB_ERR_UNSUPPORTED;
 * snnb_split_workspace_bytes takes the OUTPUT sizes.
 */
int snnb_conv_lif_strided(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                          int64_t Cin, const void* w, const float* bias, int64_t Cout, int ksize,
                          int stride, float decay, float input_scale, float v_threshold,
                          float v_reset, int hard_reset, const void* residual, int residual_dtype,
                          int variant, int block_n, int splits, void* workspace,
                          int64_t workspace_bytes, void* out, snnb_stream_t stream);

/*
 * Window gather for a k x k conv on an image of few channels (no kernel of its own in the
 * reference, whose stem runs F.conv2d: snn_compiler/zoo/resnet.py:128-130 -> nn/modules.py:
 * 324-357): x bf16 NHWC [frames, H, W, C] -> out bf16 [frames, Ho, Wo, Kp], column
 * (dy * k + dx) * C + c = x[stride * ho + dy - pad, stride * wo + dx - pad, c] (zero outside
 * the image), columns k*k*C .. Kp-1 zero; Ho = (H + 2 pad - k) / stride + 1.  The conv is then
 * a 1x1 conv (snnb_conv_lif_strided with ksize 1) against w [Cout, k, k, C] viewed as
 * [Cout, 1, 1, k*k*C] (zero padded to Kp).  Kp % 8 == 0, out 16-byte aligned, C <= 4096.
 */
int snnb_window_gather_nhwc(const void* x, int64_t frames, int64_t H, int64_t W, int64_t C,
                            int k, int stride, int pad, int64_t Kp, void* out,
                            snnb_stream_t stream);

/*
 * k x k max-pool (stride, padding; each window clipped to the image, as torch's -inf padding
 * gives) on bf16 NHWC frames [frames, H, W, C] -> [frames, Ho, Wo, C], Ho = (H + 2 pad - k) /
 * stride + 1 (W likewise).  Replaces the spiking ResNet stem's nn.MaxPool2d(3, stride=2,
 * padding=1) (snn_compiler/zoo/resnet.py:131) applied per frame; on {0, 1} spikes it is the
 * OR of the window.  C % 8 == 0; x and out 16-byte aligned; 1 <= k, stride <= 8; 0 <= pad < k.
 */
int snnb_maxpool_nhwc(const void* x, int64_t frames, int64_t H, int64_t W, int64_t C, int k,
                      int stride, int pad, void* out, snnb_stream_t stream);

/*
 * A conv with a float32 result and no neuron: out = conv(x, w) + bias, k x k / padding
 * k / 2 (k in {1, 3, 5, 7}), stride 1 or 2.  Replaces the downsample branch of a spiking ResNet block,
 * nn.Sequential(Conv2d 1x1 stride 2, BatchNorm2d) with BN folded into w and bias
 * (snn_compiler/zoo/resnet.py:139-142, applied in BasicBlockSNN.forward :96-117), whose
 * result is the float32 residual input of the block's second conv (snnb_conv3x3_lif_res).
 * x: bf16 NHWC [T*B, H, W, Cin] (input sizes), Cin % 8 == 0; w: bf16 [Cout, ksize, ksize,
 * Cin], Cout % 32 == 0; out: f32 NHWC [T*B, Ho, Wo, Cout] as snnb_conv_lif_strided;
 * T in {2, 4, 8} (the T-folded kernel).
 */
int snnb_conv_f32(const void* x, int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cin,
                  const void* w, const float* bias, int64_t Cout, int ksize, int stride,
                  float* out, snnb_stream_t stream);

/*
 * K1, linear variant: spikes [T*B, K] bf16 @ w [N, K] bf16 + bias -> multi-step LIF ->
 * bf16 spikes [T*B, N].  Replaces FusedLinearNeuron.forward
 * (snn_compiler/nn/modules.py:241-255: F.linear + fused_bias_if_lif).  K % 8 == 0,
 * N % 32 == 0; variant / block_n as for snnb_conv3x3_lif.
 */
int snnb_linear_lif(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                    const float* bias, int64_t N, float decay, float input_scale,
                    float v_threshold, float v_reset, int hard_reset, int variant, int block_n,
                    int splits, void* workspace, int64_t workspace_bytes, void* out,
                    snnb_stream_t stream);

/*
 * K1 on images of at most 2 x 2 pixels (no counterpart in the reference, which runs these
 * layers through snnb_conv3x3_lif's path: F.conv2d + fused_bias_if_lif,
 * snn_compiler/nn/modules.py:324-357): there every output pixel's 3x3 window covers the
 * whole image, so the conv is one dense GEMM per image, K = H*W*Cin -> N = H*W*Cout, and
 * the zero-padding taps (5 of 9 at 2x2) leave the tensor-core work.  Same neuron and
 * result as snnb_conv3x3_lif up to float32 summation order.
 * x      : bf16 spikes NHWC [T*B, H, W, Cin], H and W in {1, 2}
 * wd     : bf16 [H*W*Cout, H*W*Cin]: row (p, co), column (q, ci) holds
 *          w[co, qh - ph + 1, qw - pw + 1, ci] (pixels p, q row-major, NHWC columns); with
 *          pool != 0 the rows are ordered (co, p) instead (pixel fastest)
 * bias_d : f32 [H*W*Cout], b'[co] for row (p, co) (or (co, p) with pool)
 * pool   : 2x2 max-pool (H == W == 2): out [T*B, 1, 1, Cout]; else out [T*B, H, W, Cout]
 * variant / block_n / splits / workspace: as snnb_linear_lif for an N = H*W*Cout layer;
 * with pool: variant 0 or 2, splits == 1.
 */
int snnb_conv3x3_lif_dense(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                           int64_t Cin, const void* wd, const float* bias_d, int64_t Cout,
                           float decay, float input_scale, float v_threshold, float v_reset,
                           int hard_reset, int pool, int variant, int block_n, int splits,
                           void* workspace, int64_t workspace_bytes, void* out,
                           snnb_stream_t stream);

/*
 * K1 with packed spikes between layers (no counterpart in the reference, whose layers pass
 * float / bf16 spike tensors): snnb_conv3x3_lif on the T-folded kernel (T in {2, 4, 8}) with
 * its input and / or output as packed spikes -- NHWC with 32 channels per uint32 word,
 * channel c in bit c % 32 of word c / 32 (LSB first, as snnb_bitpack packs rows of C
 * channels), 1/16 of the bf16 bytes.  With x_packed the kernel stages each tile's packed
 * input patch (pixels plus 1-pixel halo, every step) in shared memory once and expands every
 * k-slab's A operand from it into bf16 in shared memory; the spikes are identical to
 * snnb_conv3x3_lif's.
 * x        : packed words [T*B, H, W, Cin/32] (x_packed, Cin % 64 == 0, 4-byte aligned),
 *            or bf16 spikes [T*B, H, W, Cin]
 * out      : packed words [T*B, Ho, Wo, Cout/32] (out_packed) or bf16 [T*B, Ho, Wo, Cout]
 * block_n  : 0 = choose, 64 / 128 / 256 (32 also without x_packed)
 * Returns SNNB_ERR_UNSUPPORTED when a tile's packed patch exceeds the kernel's 32 KB.
 */
int snnb_conv3x3_lif_packed(const void* x, int x_packed, int64_t T, int64_t B, int64_t H,
                            int64_t W, int64_t Cin, const void* w, const float* bias,
                            int64_t Cout, float decay, float input_scale, float v_threshold,
                            float v_reset, int hard_reset, int pool, int out_packed, int block_n,
                            void* out, snnb_stream_t stream);

/* Packed spikes [rows, C/32] uint32 (C % 32 == 0) -> bf16 {0,1} [rows, C] (16-byte aligned). */
int snnb_unpack_spikes(const void* words, int64_t rows, int64_t C, void* out,
                       snnb_stream_t stream);

/* Workspace bytes snnb_conv3x3_lif / snnb_linear_lif (H = W = 1) need for `splits`; 0 when
 * splits <= 1, negative when a size is negative or the byte count overflows int64. */
int64_t snnb_split_workspace_bytes(int64_t T, int64_t B, int64_t H, int64_t W, int64_t Cout,
                                   int splits);

/*
 * snnb_conv3x3_lif for callers that cannot allocate (no counterpart in the reference):
 * the same fused conv + bias + LIF (+ pool), with the split-K partial sums kept in a fixed
 * scratch array inside the library (16 MiB, held on every GPU that loads the library until
 * the process exits) instead of a caller workspace.  Meant for plugin or runtime hosts that
 * offer no scratch buffer and forbid cudaMalloc / cudaFree (which may also synchronise the
 * device) once they are running.  The call itself allocates nothing.
 *   - Requests whose partial sums exceed 16 MiB (snnb_split_workspace_bytes) return
 *     SNNB_ERR_ARG.
 *   - The first call on a device looks up the array's device address with that device
 *     current; make that first call before any stream capture.
 *   - Every call on a device shares the one array, and its contents persist between calls
 *     (nothing in it needs to start at zero).  Calls whose kernels overlap on the GPU --
 *     different streams, or concurrent host threads -- race on it: serialise them.
 * Arguments as snnb_conv3x3_lif, with variant chosen (split-K when splits > 1).
 */
int snnb_conv3x3_lif_static_scratch(const void* x, int64_t T, int64_t B, int64_t H, int64_t W,
                                    int64_t Cin, const void* w, const float* bias, int64_t Cout,
                                    float decay, float input_scale, float v_threshold,
                                    float v_reset, int hard_reset, int pool, int block_n,
                                    int splits, void* out, snnb_stream_t stream);

/*
 * Classifier head: out[b, n] = mean over t of (x[t*B+b] @ w[n]^T + bias[n]), f32.
 * Replaces the last nn.Linear of VGGSNN (snn_compiler/zoo/vgg.py:84, :111-114) and the
 * caller's mean over T (examples/vgg16_snn/vgg16_test.py:243).  K % 8 == 0, N <= 64;
 * a few dot products per sample, computed on the CUDA cores.
 */
int snnb_linear_mean(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                     const float* bias, int64_t N, float* out, snnb_stream_t stream);

/*
 * Classifier head without the mean: out[t*B + b, n] = x[t*B+b] @ w[n]^T + bias[n], f32
 * [T*B, N] -- the per-step logits VGGSNN.forward returns (snn_compiler/zoo/vgg.py:111-115).
 * K % 8 == 0, N <= 64.
 */
int snnb_linear_out(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                    const float* bias, int64_t N, float* out, snnb_stream_t stream);

/*
 * First (real-valued input) layer of a spiking CNN: float32 direct conv3x3 (pad 1)
 * + bias + multi-step LIF (+ 2x2 max-pool) -> bf16 spikes NHWC [T*B, Ho, Wo, Cout].
 * Replaces the first FusedConvBNNeuron of VGGSNN, whose input is the float image
 * (snn_compiler/zoo/vgg.py:88-94).  x: f32 NCHW [Ti, B, Cin, H, W]; Ti = T, or Ti = 1
 * when the same image drives every step (direct encoding: the conv runs once).
 * w: f32 [Cout, Cin, 3, 3]; Cout % 8 == 0.
 */
int snnb_first_conv_lif(const float* x, int64_t Ti, int64_t T, int64_t B, int64_t Cin,
                        int64_t H, int64_t W, const float* w, const float* bias, int64_t Cout,
                        float decay, float input_scale, float v_threshold, float v_reset,
                        int hard_reset, int pool, void* out, snnb_stream_t stream);

/*
 * Linear layer with a float32 result and no neuron: out[t*B+b, n] = x[t*B+b] @ w[n]^T +
 * bias[n] for spike (or any bf16) rows x [T*B, K] and bf16 w [N, K]; out f32 [T*B, N].
 * Replaces the projection Conv1d 1x1 (+ folded BN) that ends the spiking self-attention
 * block (snn_compiler/nn/attention.py:154-160).  T in {2, 4, 8}, K % 8 == 0, N % 32 == 0.
 */
int snnb_linear_f32(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                    const float* bias, int64_t N, float* out, snnb_stream_t stream);

/*
 * K3 -- spiking self-attention core: kv = K^T V (bit-packed AND + popcount), then
 * a = Q kv and a multi-step neuron on a * scale, v kept across t in registers.
 * Replaces spike_ktv / spike_ktv_popcount (snn_compiler/kernels/attention.py:177-258),
 * spike_av_lif (attention.py:107-137) and their use in FusedSpikeAttention.forward
 * (snn_compiler/nn/attention.py:149-150).  q, k, v: bf16 {0,1} with element (t, b, h, n, i)
 * at base + t*st + b*sb + h*sh + n*sn + i (a fused [T, B, N, 3D] projection output or
 * separate [T, B, H, N, d] tensors).  d <= 32, N <= 256, N*d <= 8192 (d % 4 == 0) or
 * N*d <= 2048.
 * kv_in  : optional f32 [T, B, H, d, d]; when given, K and V are not read.
 * kv_out : optional f32 [T, B, H, d, d] (K^T V as float).
 * out    : bf16 spikes at out + t*ot + b*ob + h*oh + n*on + j, or NULL (kv only).
 * Neuron: v = decay*v + input_scale*(a*scale); s = v >= v_threshold; reset.
 */
int snnb_spike_attention_core(const void* q, const void* k, const void* v, int64_t st,
                              int64_t sb, int64_t sh, int64_t sn, const float* kv_in,
                              float* kv_out, void* out, int64_t ot, int64_t ob, int64_t oh,
                              int64_t on, int64_t T, int64_t B, int64_t H, int64_t N, int64_t d,
                              float decay, float input_scale, float scale, float v_threshold,
                              float v_reset, int hard_reset, snnb_stream_t stream);

/*
 * Linear + bias + multi-step LIF in the transposed form, for layers with few rows (the
 * classifier FusedLinearNeuron, modules.py:241-255, and the dense form of 3x3 layers on 2x2
 * images; reference: F.linear + fused_bias_if_lif).  x [T, B, K] bf16, w [N, K] bf16
 * (N % 128 == 0, K % 8 == 0), bias [N] f32 -> spikes [T, B, N] bf16, or with pool4 the OR
 * of 4 consecutive features [T, B, N / 4].  D^T = W X^T on tcgen05: 128 features x the
 * T * (256 / T) rows of a column tile per CTA; splits in {1, 2, 4, 8} split K over a
 * cluster whose float32 partial sums go to `workspace`
 * (>= snnb_linear_t_workspace_bytes, 16-byte aligned) and are added in split order.
 * T in {1, 2, 4, 8}.
 */
int snnb_linear_lif_t(const void* x, int64_t T, int64_t B, int64_t K, const void* w,
                      const float* bias, int64_t N, float decay, float input_scale,
                      float v_threshold, float v_reset, int hard_reset, int pool4, int splits,
                      void* workspace, int64_t workspace_bytes, void* out,
                      snnb_stream_t stream);

/* Workspace bytes of snnb_linear_lif_t (0 when splits <= 1, negative when invalid). */
int64_t snnb_linear_t_workspace_bytes(int64_t T, int64_t B, int64_t N, int splits);

/*
 * Image (first) layer on the tensor cores: replaces the first FusedConvBNNeuron of VGGSNN
 * (snn_compiler/zoo/vgg.py:88-94 -> nn/modules.py:347-357, F.conv2d in float32 +
 * fused_bias_if_lif) for direct encoding -- x [B, Cin, H, W] float32 NCHW, the same image at
 * every one of the T steps, so the conv runs once per pixel and the neuron T times from it.
 * The conv is float32-accurate: image and weights as three bf16 terms each, six products
 * summed by tcgen05 MMAs into float32 (see snnb_split_bf16_terms).  w_split [Cout, KP] bf16
 * is the folded weight's terms, groups [hi, mid, lo, hi, mid, hi] of the 9 * Cin values in
 * torch's (ci, ky, kx) order, each group G = 9 * Cin + (Cin & 1) entries wide (one zero after
 * the values when 9 * Cin is odd), zero-padded to KP = snnb_first_conv_tc_weight_k(Cin).
 * out [T, B, H, W, Cout] bf16 spikes (no pooling), 32-byte aligned.  Cin 1..4,
 * Cout 32 / 64 / 128.
 */
int snnb_first_conv_lif_tc(const float* x, int64_t T, int64_t B, int64_t Cin, int64_t H,
                           int64_t W, const void* w_split, const float* bias, int64_t Cout,
                           float decay, float input_scale, float v_threshold, float v_reset,
                           int hard_reset, void* out, snnb_stream_t stream);

/* KP of snnb_first_conv_lif_tc's w_split for Cin input channels (-1 if Cin is not 1..4). */
int64_t snnb_first_conv_tc_weight_k(int64_t Cin);

/*
 * float32 operands for the bf16 tensor-core kernels (no kernel of its own in the reference:
 * it keeps the reference's float32 F.conv2d / F.linear on real-valued inputs float32-exact,
 * snn_compiler/nn/modules.py:194-206, 241-255, 324-345).  x [rows, C] float32 -> out
 * [rows, 6 * Cp] bf16: each value a as three bf16 terms hi = rn(a), mid = rn(a - hi),
 * lo = rn(a - hi - mid), written as six channel groups [hi, hi, hi, mid, mid, lo] of Cp
 * channels (channels C .. Cp-1 of each group zero).  Against weights split the same way and
 * grouped [hi, mid, lo, hi, mid, hi], one bf16 conv / GEMM over the 6 * Cp channels sums the
 * six larger term products, each exact in float32 (the three dropped ones stay below 2^-23
 * of the product).  Cp >= C, Cp % 4 == 0 (so 6 * Cp % 8 == 0); x 16-byte aligned when
 * C % 4 == 0, out 8-byte aligned.
 */
int snnb_split_bf16_terms(const float* x, int64_t rows, int64_t C, int64_t Cp, void* out,
                          snnb_stream_t stream);

/*
 * Reads and clears the device status word that kernels with bounded waits write
 * (SNNB_ERR_TIMEOUT after a wait gave up).  Synchronises `stream`.
 */
int snnb_read_device_status(snnb_stream_t stream, int* status_out);

/*
 * Spin limit, in SM clock cycles, of the tensor-core kernels' progress waits (a stage's
 * copies, an accumulator, a free ring slot) on the current device; 0 restores the default
 * of 4e9 cycles (~2 s at 1.9 GHz), other values must be >= 1000.  A wait that runs out
 * sets SNNB_ERR_TIMEOUT in the device status word and the launch stops early, leaving its
 * output incomplete.  The waits that drain copies or MMAs already issued after such a
 * failure keep the default, so no CTA exits with copies in flight.  A wait's clock starts
 * when the wait does, which with programmatic dependent launch can be before the previous
 * kernel on the stream has finished: keep the limit well above the longest kernel.
 * No counterpart in the reference (its Triton kernels have no waits); it exists so that a
 * host can bound how long a failed launch holds the GPU, and so the tests can make a wait
 * run out.
 */
int snnb_set_wait_limit(int64_t cycles);

/*
 * Test hooks (no counterpart in the reference), for exercising the failure paths without
 * faulting a GPU:
 *   snnb_debug_inject_status(status, count): the next `count` entry-point calls (any entry
 *     that launches work) return `status` (a negative SNNB_ERR_*) without launching.
 *   snnb_debug_inject_stall(count): in the next `count` launches of the T-sequential conv
 *     kernel (snnb_conv3x3_lif variant 1), the producer warp of CTA 0 withholds every
 *     stage; that CTA's MMA warp then waits until the wait limit runs out and the launch
 *     reports SNNB_ERR_TIMEOUT (CTA 0's output is left unspecified).
 * Both are process-wide; count 0 cancels.
 */
int snnb_debug_inject_status(int status, int count);
int snnb_debug_inject_stall(int count);

#ifdef __cplusplus
}
#endif

#endif /* SNNB200_H */
