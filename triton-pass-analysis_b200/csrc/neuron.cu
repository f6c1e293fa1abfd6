// K2 -- multi-step IF / LIF / PLIF neuron (HBM-bound streaming kernel).
//
// Replaces the reference's Triton kernels _if_lif_kernel (snn_compiler/kernels/
// neurons.py:85-138), _bias_if_lif_kernel (fused.py:50-114), the rate-coded
// variant (fused.py:242-300) and the stateful variant (fused.py:398-441) with one
// kernel whose outputs are selected by non-null pointers.
//
// Design (B200): each thread owns 8 consecutive neurons of one time step row and
// walks the T axis with the membrane potential, threshold and bias in registers.
// The loads of four steps are issued before any of them is used (64-128 bytes in
// flight per thread), rows are read with 16-byte streaming loads (ld.global.cs)
// and spikes leave with 16-byte streaming stores, so the only DRAM traffic is one
// read of x (and residual) and one write of each requested output.  Packed spikes
// are built from 8-bit per-thread nibbles OR-ed across the 4 lanes that share a
// 32-bit word.  Grid: one thread per 8 neurons, 256-thread CTAs.
#include "common.cuh"

namespace snnb {

int* device_status_ptr();

namespace {

struct NeuronParams {
    const void* x;
    const void* residual;
    const float* bias;
    const float* thr;
    const float* v_init;
    const float* plif_w;
    const float* plif_k;       // charge modes 1-3: device scalar k (SpikingJelly's w.sigmoid())
    void* spikes;
    uint32_t* packed;
    float* count;
    float* v_out;
    int64_t T, N, C, HW, words;
    float df, sc, v_reset, thr_scalar;
    int hard, thr_mode, channel_last;
    int charge_mode;
    int* status;               // debug build: where a failed index check is recorded
};

__device__ __forceinline__ int64_t channel_of(int64_t n, const NeuronParams& p) {
    if (p.N <= 0xffffffffll) {
        const uint32_t u = (uint32_t)n;
        return p.channel_last ? (int64_t)(u % (uint32_t)p.C)
                              : (int64_t)((u / (uint32_t)p.HW) % (uint32_t)p.C);
    }
    return p.channel_last ? n % p.C : (n / p.HW) % p.C;
}

// Charge modes.  0: the reference's v = decay*v + input_scale*in (neurons.py:129-132,
// fused.py:106-110).  1-3: SpikingJelly ParametricLIFNode.neuronal_charge, term by term in
// its order, with k = sigmoid(w) computed by the caller:
//   1  decay_input:                     v = v + (in - (v - v_reset)) * k
//   2  not decay_input, v_reset 0/None: v = v * (1 - k) + in
//   3  not decay_input, v_reset != 0:   v = v - (v - v_reset) * k + in
// (for v_reset == 0, mode 1 is SpikingJelly's v + (in - v) * k exactly: v - 0 == v).
template <int CM>
__device__ __forceinline__ float charge_cm(float v, float df, float sc, float in, float k,
                                           float om, float vr) {
    if constexpr (CM == 0) {
        return charge(v, df, sc, in);
    } else if constexpr (CM == 1) {
        return __fadd_rn(v, __fmul_rn(__fsub_rn(in, __fsub_rn(v, vr)), k));
    } else if constexpr (CM == 2) {
        return __fadd_rn(__fmul_rn(v, om), in);
    } else {
        return __fadd_rn(__fsub_rn(v, __fmul_rn(__fsub_rn(v, vr), k)), in);
    }
}

__device__ __forceinline__ void neuron_coeffs(const NeuronParams& p, float& df, float& sc) {
    df = p.df;
    sc = p.sc;
    if (p.plif_w) {
        const double w = (double)__ldg(p.plif_w);
        const float k = (float)(1.0 / (1.0 + exp(-w)));
        sc = k;
        df = __fsub_rn(1.0f, k);
    }
}

// ---- 8-wide streaming loads / stores ------------------------------------------------
__device__ __forceinline__ void load8(const float* ptr, float (&o)[8]) {
    const float4 a = __ldcs(reinterpret_cast<const float4*>(ptr));
    const float4 b = __ldcs(reinterpret_cast<const float4*>(ptr) + 1);
    o[0] = a.x; o[1] = a.y; o[2] = a.z; o[3] = a.w;
    o[4] = b.x; o[5] = b.y; o[6] = b.z; o[7] = b.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* ptr, float (&o)[8]) {
    const uint4 r = __ldcs(reinterpret_cast<const uint4*>(ptr));
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        o[2 * i] = __uint_as_float(w[i] << 16);
        o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ void load8(const __half* ptr, float (&o)[8]) {
    const uint4 r = __ldcs(reinterpret_cast<const uint4*>(ptr));
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        const float2 f = __half22float2(h);
        o[2 * i] = f.x;
        o[2 * i + 1] = f.y;
    }
}

__device__ __forceinline__ void store8(float* ptr, uint32_t bits) {
    float4 a, b;
    a.x = (bits & 1u) ? 1.f : 0.f;   a.y = (bits & 2u) ? 1.f : 0.f;
    a.z = (bits & 4u) ? 1.f : 0.f;   a.w = (bits & 8u) ? 1.f : 0.f;
    b.x = (bits & 16u) ? 1.f : 0.f;  b.y = (bits & 32u) ? 1.f : 0.f;
    b.z = (bits & 64u) ? 1.f : 0.f;  b.w = (bits & 128u) ? 1.f : 0.f;
    __stcs(reinterpret_cast<float4*>(ptr), a);
    __stcs(reinterpret_cast<float4*>(ptr) + 1, b);
}
__device__ __forceinline__ uint32_t two16(uint32_t bits, int i, uint32_t one) {
    return (((bits >> (2 * i)) & 1u) ? one : 0u) | (((bits >> (2 * i + 1)) & 1u) ? (one << 16) : 0u);
}
__device__ __forceinline__ void store8(__nv_bfloat16* ptr, uint32_t bits) {
    uint4 r;
    r.x = two16(bits, 0, 0x3F80u); r.y = two16(bits, 1, 0x3F80u);
    r.z = two16(bits, 2, 0x3F80u); r.w = two16(bits, 3, 0x3F80u);
    __stcs(reinterpret_cast<uint4*>(ptr), r);
}
__device__ __forceinline__ void store8(__half* ptr, uint32_t bits) {
    uint4 r;
    r.x = two16(bits, 0, 0x3C00u); r.y = two16(bits, 1, 0x3C00u);
    r.z = two16(bits, 2, 0x3C00u); r.w = two16(bits, 3, 0x3C00u);
    __stcs(reinterpret_cast<uint4*>(ptr), r);
}
__device__ __forceinline__ void store8(uint8_t* ptr, uint32_t bits) {
    // spread 8 bits into 8 bytes of 0x00 / 0x01
    uint32_t lo = (bits & 0xfu), hi = (bits >> 4) & 0xfu;
    lo = (lo | (lo << 7) | (lo << 14) | (lo << 21)) & 0x01010101u;
    hi = (hi | (hi << 7) | (hi << 14) | (hi << 21)) & 0x01010101u;
    __stcs(reinterpret_cast<uint2*>(ptr), make_uint2(lo, hi));
}

constexpr int VEC = 8;     // neurons per thread
constexpr int TU = 4;      // time steps whose loads are in flight together
constexpr int THREADS = 256;

template <typename TX, typename TS, int CM>
__global__ void __launch_bounds__(THREADS) neuron_vec8_kernel(NeuronParams p) {
    pdl_wait();
    pdl_trigger();
    const int64_t g = (int64_t)blockIdx.x * THREADS + threadIdx.x;
    const int64_t n0 = g * VEC;
    const bool active = n0 < p.N;          // N % VEC == 0: a vector is all in or all out
    const int lane = threadIdx.x & 31;
    float df, sc;
    neuron_coeffs(p, df, sc);
    const float pk = CM ? __ldg(p.plif_k) : 0.0f;
    const float om = CM == 2 ? __fsub_rn(1.0f, pk) : 0.0f;

    float v[VEC], th[VEC], bb[VEC], cnt[VEC];
    const bool need_c = (p.bias != nullptr) || (p.thr_mode == SNNB_THR_PER_CHANNEL);
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
        const int64_t n = n0 + k;
        const int64_t c = (active && need_c) ? channel_of(n, p) : 0;
        v[k] = (active && p.v_init) ? __ldg(p.v_init + n) : 0.0f;
        th[k] = p.thr_mode == SNNB_THR_SCALAR ? p.thr_scalar
              : (!active ? 0.0f
                 : (p.thr_mode == SNNB_THR_PER_CHANNEL ? __ldg(p.thr + c) : __ldg(p.thr + n)));
        bb[k] = (active && p.bias) ? __ldg(p.bias + c) : 0.0f;
        cnt[k] = 0.0f;
    }
    const TX* x = static_cast<const TX*>(p.x);
    const TX* res = static_cast<const TX*>(p.residual);
    TS* sp = static_cast<TS*>(p.spikes);
    const bool has_bias = p.bias != nullptr;

    for (int64_t t0 = 0; t0 < p.T; t0 += TU) {
        float xr[TU][VEC];
        float rr[TU][VEC];
#pragma unroll
        for (int u = 0; u < TU; ++u) {
            const bool ok = active && (t0 + u < p.T) &&
                            SNNB_IN_BOUNDS((t0 + u) * p.N + n0 + VEC - 1, p.T * p.N, p.status);
            if (ok) {
                load8(x + (t0 + u) * p.N + n0, xr[u]);
            } else {
#pragma unroll
                for (int k = 0; k < VEC; ++k) xr[u][k] = 0.0f;
            }
            if (ok && res) {
                load8(res + (t0 + u) * p.N + n0, rr[u]);
            } else {
#pragma unroll
                for (int k = 0; k < VEC; ++k) rr[u][k] = 0.0f;
            }
        }
#pragma unroll
        for (int u = 0; u < TU; ++u) {
            const int64_t t = t0 + u;
            if (t >= p.T) break;
            uint32_t bits = 0;
#pragma unroll
            for (int k = 0; k < VEC; ++k) {
                float in = xr[u][k];
                if (has_bias) in = __fadd_rn(in, bb[k]);
                if (res) in = __fadd_rn(in, rr[u][k]);
                float vv = charge_cm<CM>(v[k], df, sc, in, pk, om, p.v_reset);
                const bool s = vv >= th[k];
                if (p.hard) {
                    vv = s ? p.v_reset : vv;
                } else {
                    vv = s ? __fsub_rn(vv, th[k]) : vv;
                }
                v[k] = vv;
                cnt[k] = __fadd_rn(cnt[k], s ? 1.0f : 0.0f);
                bits |= (s ? 1u : 0u) << k;
            }
            if (!active) bits = 0;
            if (sp && active && SNNB_IN_BOUNDS(t * p.N + n0 + VEC - 1, p.T * p.N, p.status))
                store8(sp + t * p.N + n0, bits);
            if (p.packed) {
                uint32_t w = bits << (8 * (lane & 3));
                w |= __shfl_xor_sync(0xffffffffu, w, 1);
                w |= __shfl_xor_sync(0xffffffffu, w, 2);
                if ((lane & 3) == 0 && active &&
                    SNNB_IN_BOUNDS(t * p.words + (n0 >> 5), p.T * p.words, p.status))
                    __stcs(p.packed + t * p.words + (n0 >> 5), w);
            }
        }
    }
    if (active && SNNB_IN_BOUNDS(n0 + VEC - 1, p.N, p.status)) {
#pragma unroll
        for (int k = 0; k < VEC; ++k) {
            if (p.count) p.count[n0 + k] = cnt[k];
            if (p.v_out) p.v_out[n0 + k] = v[k];
        }
    }
}

// Scalar path for ragged N or unaligned pointers: one neuron per thread; a warp
// covers 32 consecutive neurons, so one ballot is one packed word.
template <typename TX, typename TS, int CM>
__global__ void __launch_bounds__(THREADS) neuron_scalar_kernel(NeuronParams p) {
    pdl_wait();
    pdl_trigger();
    const int64_t n = (int64_t)blockIdx.x * THREADS + threadIdx.x;
    const bool active = n < p.N;
    const int lane = threadIdx.x & 31;
    float df, sc;
    neuron_coeffs(p, df, sc);
    const float pk = CM ? __ldg(p.plif_k) : 0.0f;
    const float om = CM == 2 ? __fsub_rn(1.0f, pk) : 0.0f;
    const bool need_c = (p.bias != nullptr) || (p.thr_mode == SNNB_THR_PER_CHANNEL);
    const int64_t c = (active && need_c) ? channel_of(n, p) : 0;
    float v = (active && p.v_init) ? p.v_init[n] : 0.0f;
    const float th = p.thr_mode == SNNB_THR_SCALAR ? p.thr_scalar
                   : (!active ? 0.0f : (p.thr_mode == SNNB_THR_PER_CHANNEL ? p.thr[c] : p.thr[n]));
    const float bb = (active && p.bias) ? p.bias[c] : 0.0f;
    float cnt = 0.0f;
    const TX* x = static_cast<const TX*>(p.x);
    const TX* res = static_cast<const TX*>(p.residual);
    TS* sp = static_cast<TS*>(p.spikes);
    for (int64_t t = 0; t < p.T; ++t) {
        bool s = false;
        if (active && SNNB_IN_BOUNDS(t * p.N + n, p.T * p.N, p.status)) {
            float in = to_f32(x[t * p.N + n]);
            if (p.bias) in = __fadd_rn(in, bb);
            if (res) in = __fadd_rn(in, to_f32(res[t * p.N + n]));
            float vv = charge_cm<CM>(v, df, sc, in, pk, om, p.v_reset);
            s = vv >= th;
            if (p.hard) vv = s ? p.v_reset : vv;
            else vv = s ? __fsub_rn(vv, th) : vv;
            v = vv;
            cnt = __fadd_rn(cnt, s ? 1.0f : 0.0f);
            if (sp) sp[t * p.N + n] = spike_value<TS>(s);
        }
        if (p.packed) {
            const uint32_t w = __ballot_sync(0xffffffffu, s);
            if (lane == 0 && active &&
                SNNB_IN_BOUNDS(t * p.words + (n >> 5), p.T * p.words, p.status))
                p.packed[t * p.words + (n >> 5)] = w;
        }
    }
    if (active) {
        if (p.count) p.count[n] = cnt;
        if (p.v_out) p.v_out[n] = v;
    }
}

template <typename TX, typename TS, int CM>
int launch_cm(const NeuronParams& p, bool vec, cudaStream_t s) {
    if (vec) {
        const int64_t threads = (p.N + VEC - 1) / VEC;
        const int64_t blocks = (threads + THREADS - 1) / THREADS;
        return launch_k(neuron_vec8_kernel<TX, TS, CM>, dim3((unsigned)blocks), dim3(THREADS), 0,
                        s, p);
    }
    const int64_t blocks = (p.N + THREADS - 1) / THREADS;
    return launch_k(neuron_scalar_kernel<TX, TS, CM>, dim3((unsigned)blocks), dim3(THREADS), 0,
                    s, p);
}

template <typename TX, typename TS>
int launch_typed(const NeuronParams& p, bool vec, cudaStream_t s) {
    switch (p.charge_mode) {
        case 1: return launch_cm<TX, TS, 1>(p, vec, s);
        case 2: return launch_cm<TX, TS, 2>(p, vec, s);
        case 3: return launch_cm<TX, TS, 3>(p, vec, s);
        default: return launch_cm<TX, TS, 0>(p, vec, s);
    }
}

template <typename TX>
int launch_x(const NeuronParams& p, int spikes_dtype, bool vec, cudaStream_t s) {
    switch (spikes_dtype) {
        case SNNB_F32: return launch_typed<TX, float>(p, vec, s);
        case SNNB_F16: return launch_typed<TX, __half>(p, vec, s);
        case SNNB_BF16: return launch_typed<TX, __nv_bfloat16>(p, vec, s);
        case SNNB_U8: return launch_typed<TX, uint8_t>(p, vec, s);
        default: return SNNB_ERR_ARG;
    }
}

// ---- CubaLIF / EIF ---------------------------------------------------------------------
// Same streaming structure as neuron_vec8_kernel (8 neurons per thread, 16-byte loads and
// stores), with two state registers per neuron for CubaLIF and the exponential term for EIF.
struct Neuron2Params {
    const void* x;
    const float* thr;
    void* spikes;
    int64_t T, N, C, HW;
    float a, b, sc, delta_T, v_rh, v_reset, thr_scalar;
    int thr_mode, channel_last;
};

__device__ __forceinline__ int64_t channel_of2(int64_t n, const Neuron2Params& p) {
    return p.channel_last ? n % p.C : (n / p.HW) % p.C;
}

// One step of neuron n: returns the spike; i (CubaLIF synaptic current) and v updated.
template <int MODEL, bool HARD>
__device__ __forceinline__ bool step2(float& v, float& i, float x, float th, const Neuron2Params& p) {
    if (MODEL == SNNB_MODEL_CUBA) {
        i = __fadd_rn(__fmul_rn(p.a, i), __fmul_rn(p.sc, x));
        v = __fadd_rn(__fmul_rn(p.b, v), i);
    } else {
        const float z = fminf(__fdiv_rn(__fsub_rn(v, p.v_rh), p.delta_T), 16.0f);
        const float e = expf(z);
        v = __fadd_rn(__fadd_rn(__fmul_rn(p.a, v), __fmul_rn(p.delta_T, e)), __fmul_rn(p.sc, x));
    }
    const bool s = v >= th;
    v = reset_v<HARD>(v, s, th, p.v_reset);
    return s;
}

__device__ __forceinline__ float thr_of(int64_t n, const Neuron2Params& p) {
    if (p.thr_mode == SNNB_THR_SCALAR) return p.thr_scalar;
    return p.thr_mode == SNNB_THR_PER_CHANNEL ? __ldg(p.thr + channel_of2(n, p)) : __ldg(p.thr + n);
}

template <typename TX, int MODEL, bool HARD>
__global__ void __launch_bounds__(THREADS) neuron2_vec8_kernel(Neuron2Params p) {
    pdl_wait();
    pdl_trigger();
    const int64_t n0 = ((int64_t)blockIdx.x * THREADS + threadIdx.x) * VEC;
    if (n0 >= p.N) return;                 // N % VEC == 0: a vector is all in or all out
    float v[VEC], cur[VEC], th[VEC];
#pragma unroll
    for (int k = 0; k < VEC; ++k) {
        v[k] = 0.0f;
        cur[k] = 0.0f;
        th[k] = thr_of(n0 + k, p);
    }
    const TX* x = static_cast<const TX*>(p.x);
    TX* sp = static_cast<TX*>(p.spikes);
    float xc[VEC], xn[VEC];
    load8(x + n0, xc);
    for (int64_t t = 0; t < p.T; ++t) {
        if (t + 1 < p.T) load8(x + (t + 1) * p.N + n0, xn);   // next step in flight
        uint32_t bits = 0;
#pragma unroll
        for (int k = 0; k < VEC; ++k)
            bits |= (step2<MODEL, HARD>(v[k], cur[k], xc[k], th[k], p) ? 1u : 0u) << k;
        store8(sp + t * p.N + n0, bits);
#pragma unroll
        for (int k = 0; k < VEC; ++k) xc[k] = xn[k];
    }
}

template <typename TX, int MODEL, bool HARD>
__global__ void __launch_bounds__(THREADS) neuron2_scalar_kernel(Neuron2Params p) {
    pdl_wait();
    pdl_trigger();
    const int64_t n = (int64_t)blockIdx.x * THREADS + threadIdx.x;
    if (n >= p.N) return;
    const float th = thr_of(n, p);
    float v = 0.0f, cur = 0.0f;
    const TX* x = static_cast<const TX*>(p.x);
    TX* sp = static_cast<TX*>(p.spikes);
    for (int64_t t = 0; t < p.T; ++t) {
        const bool s = step2<MODEL, HARD>(v, cur, to_f32(x[t * p.N + n]), th, p);
        sp[t * p.N + n] = spike_value<TX>(s);
    }
}

template <typename TX, int MODEL, bool HARD>
int launch_neuron2_m(const Neuron2Params& p, bool vec, cudaStream_t s) {
    if (vec) {
        const int64_t blocks = ((p.N + VEC - 1) / VEC + THREADS - 1) / THREADS;
        return launch_k(neuron2_vec8_kernel<TX, MODEL, HARD>, dim3((unsigned)blocks),
                        dim3(THREADS), 0, s, p);
    }
    const int64_t blocks = (p.N + THREADS - 1) / THREADS;
    return launch_k(neuron2_scalar_kernel<TX, MODEL, HARD>, dim3((unsigned)blocks),
                    dim3(THREADS), 0, s, p);
}

template <typename TX>
int launch_neuron2(const Neuron2Params& p, int model, bool hard, bool vec, cudaStream_t s) {
    if (model == SNNB_MODEL_CUBA)
        return hard ? launch_neuron2_m<TX, SNNB_MODEL_CUBA, true>(p, vec, s)
                    : launch_neuron2_m<TX, SNNB_MODEL_CUBA, false>(p, vec, s);
    return hard ? launch_neuron2_m<TX, SNNB_MODEL_EIF, true>(p, vec, s)
                : launch_neuron2_m<TX, SNNB_MODEL_EIF, false>(p, vec, s);
}

}  // namespace
}  // namespace snnb

using namespace snnb;

extern "C" int snnb_neuron_cuba_eif(
    const void* x, int x_dtype, int64_t T, int64_t N, int64_t C, int64_t HW, int channel_last,
    int model, float a, float b, float input_scale, float delta_T, float v_rh,
    int hard_reset, float v_reset, int thr_mode, float thr_scalar, const float* thr,
    void* spikes, snnb_stream_t stream)
{
    if (const int inj = snnb::take_injected_status()) return inj;
    if (T < 0 || N < 0) return SNNB_ERR_ARG;
    if (x_dtype != SNNB_F32 && x_dtype != SNNB_F16 && x_dtype != SNNB_BF16) return SNNB_ERR_ARG;
    if (model != SNNB_MODEL_CUBA && model != SNNB_MODEL_EIF) return SNNB_ERR_ARG;
    if (thr_mode != SNNB_THR_SCALAR && thr_mode != SNNB_THR_PER_CHANNEL &&
        thr_mode != SNNB_THR_PER_NEURON) return SNNB_ERR_ARG;
    if (thr_mode != SNNB_THR_SCALAR && thr == nullptr) return SNNB_ERR_ARG;
    if (thr_mode == SNNB_THR_PER_CHANNEL && (C <= 0 || (!channel_last && HW <= 0)))
        return SNNB_ERR_ARG;
    if (N == 0 || T == 0) return SNNB_OK;
    if (x == nullptr || spikes == nullptr) return SNNB_ERR_ARG;
    if (T > (int64_t)1 << 40 || N > (int64_t)1 << 40) return SNNB_ERR_ARG;
    if ((N + 255) / 256 > 0x7fffffffll) return SNNB_ERR_ARG;
    Neuron2Params p;
    p.x = x; p.thr = thr; p.spikes = spikes;
    p.T = T; p.N = N; p.C = C > 0 ? C : 1; p.HW = HW > 0 ? HW : 1;
    p.a = a; p.b = b; p.sc = input_scale; p.delta_T = delta_T; p.v_rh = v_rh;
    p.v_reset = v_reset; p.thr_scalar = thr_scalar;
    p.thr_mode = thr_mode; p.channel_last = channel_last ? 1 : 0;
    const bool vec = (N % VEC == 0) && aligned16(x) && aligned16(spikes);
    const bool hard = hard_reset != 0;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (x_dtype) {
        case SNNB_F32: return launch_neuron2<float>(p, model, hard, vec, s);
        case SNNB_F16: return launch_neuron2<__half>(p, model, hard, vec, s);
        default: return launch_neuron2<__nv_bfloat16>(p, model, hard, vec, s);
    }
}

extern "C" int snnb_neuron_multistep(
    const void* x, int x_dtype, int64_t T, int64_t N,
    const float* bias, const void* residual, int64_t C, int64_t HW, int channel_last,
    float decay, float input_scale, const float* plif_w,
    int hard_reset, float v_reset,
    int thr_mode, float thr_scalar, const float* thr,
    const float* v_init,
    void* spikes, int spikes_dtype,
    uint32_t* spikes_packed, float* count, float* v_out,
    snnb_stream_t stream)
{
    if (const int inj = snnb::take_injected_status()) return inj;
    if (T < 0 || N < 0) return SNNB_ERR_ARG;
    if (x_dtype != SNNB_F32 && x_dtype != SNNB_F16 && x_dtype != SNNB_BF16) return SNNB_ERR_ARG;
    if (spikes && (spikes_dtype < SNNB_F32 || spikes_dtype > SNNB_U8)) return SNNB_ERR_ARG;
    if (thr_mode != SNNB_THR_SCALAR && thr_mode != SNNB_THR_PER_CHANNEL &&
        thr_mode != SNNB_THR_PER_NEURON) return SNNB_ERR_ARG;
    if (thr_mode != SNNB_THR_SCALAR && thr == nullptr) return SNNB_ERR_ARG;
    const bool need_c = bias != nullptr || thr_mode == SNNB_THR_PER_CHANNEL;
    if (need_c && (C <= 0 || (!channel_last && HW <= 0))) return SNNB_ERR_ARG;
    if (N == 0) return SNNB_OK;
    if (T > 0 && x == nullptr) return SNNB_ERR_ARG;
    if (T > (int64_t)1 << 40 || N > (int64_t)1 << 40) return SNNB_ERR_ARG;
    if ((N + 255) / 256 > 0x7fffffffll) return SNNB_ERR_ARG;

    NeuronParams p = {};
    p.x = x; p.residual = residual; p.bias = bias; p.thr = thr; p.v_init = v_init;
    p.plif_w = plif_w; p.spikes = spikes; p.packed = spikes_packed; p.count = count;
    p.v_out = v_out;
    p.T = T; p.N = N; p.C = C > 0 ? C : 1; p.HW = HW > 0 ? HW : 1; p.words = (N + 31) / 32;
    p.df = decay; p.sc = input_scale; p.v_reset = v_reset; p.thr_scalar = thr_scalar;
    p.hard = hard_reset ? 1 : 0; p.thr_mode = thr_mode; p.channel_last = channel_last ? 1 : 0;
#ifdef SNNB_CHECK_BOUNDS
    p.status = device_status_ptr();
#endif

    const bool vec = (N % VEC == 0) && aligned16(x) && (!residual || aligned16(residual)) &&
                     (!spikes || aligned16(spikes));
    const int sd = spikes ? spikes_dtype : SNNB_U8;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (x_dtype) {
        case SNNB_F32: return launch_x<float>(p, sd, vec, s);
        case SNNB_F16: return launch_x<__half>(p, sd, vec, s);
        default: return launch_x<__nv_bfloat16>(p, sd, vec, s);
    }
}

extern "C" int snnb_neuron_plif(
    const void* x, int x_dtype, int64_t T, int64_t N, const float* k, int decay_input,
    int hard_reset, float v_reset, float v_threshold, const float* v_init,
    void* spikes, int spikes_dtype, uint32_t* spikes_packed, float* count, float* v_out,
    snnb_stream_t stream)
{
    if (const int inj = snnb::take_injected_status()) return inj;
    if (T < 0 || N < 0 || !k) return SNNB_ERR_ARG;
    if (x_dtype != SNNB_F32 && x_dtype != SNNB_F16 && x_dtype != SNNB_BF16) return SNNB_ERR_ARG;
    if (spikes && (spikes_dtype < SNNB_F32 || spikes_dtype > SNNB_U8)) return SNNB_ERR_ARG;
    if (N == 0) return SNNB_OK;
    if (T > 0 && x == nullptr) return SNNB_ERR_ARG;
    if (T > (int64_t)1 << 40 || N > (int64_t)1 << 40) return SNNB_ERR_ARG;
    if ((N + 255) / 256 > 0x7fffffffll) return SNNB_ERR_ARG;
    NeuronParams p = {};
    p.x = x; p.v_init = v_init; p.plif_k = k;
    p.spikes = spikes; p.packed = spikes_packed; p.count = count; p.v_out = v_out;
    p.T = T; p.N = N; p.C = 1; p.HW = 1; p.words = (N + 31) / 32;
    // SpikingJelly's soft reset (v_reset None) charges as v_reset == 0
    const float vr = hard_reset ? v_reset : 0.0f;
    p.v_reset = vr; p.thr_scalar = v_threshold;
    p.hard = hard_reset ? 1 : 0; p.thr_mode = SNNB_THR_SCALAR;
    p.charge_mode = decay_input ? 1 : (vr == 0.0f ? 2 : 3);
#ifdef SNNB_CHECK_BOUNDS
    p.status = device_status_ptr();
#endif
    const bool vec = (N % VEC == 0) && aligned16(x) && (!spikes || aligned16(spikes));
    const int sd = spikes ? spikes_dtype : SNNB_U8;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (x_dtype) {
        case SNNB_F32: return launch_x<float>(p, sd, vec, s);
        case SNNB_F16: return launch_x<__half>(p, sd, vec, s);
        default: return launch_x<__nv_bfloat16>(p, sd, vec, s);
    }
}
