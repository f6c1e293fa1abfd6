/*
 * CPU oracle for the multi-step IF/LIF/PLIF neuron (TEST INFRASTRUCTURE ONLY).
 *
 * This is the checker the CUDA kernels are compared against, and the timed
 * CPU baseline.  It is never part of the product path: only tests/, the smoke
 * check and bench.py's CPU legs load it.
 *
 * It restates, in plain C with float32 arithmetic and no FMA contraction
 * (built with -ffp-contract=off), the reference's pure-torch loop
 *   snn_compiler/kernels/neurons.py:467-502   (naive_if_lif)
 * extended with the per-channel bias / residual input of
 *   snn_compiler/kernels/fused.py:99-114      (_bias_if_lif_kernel T-loop)
 * the spike-count output of
 *   snn_compiler/kernels/fused.py:287-300     (_bias_if_lif_rate_kernel)
 * the per-step charged potential (before the threshold test, for checking
 * that a spike flip sits at the threshold), and the v_init / v_final state I/O of
 *   snn_compiler/kernels/fused.py:419-441     (_bias_if_lif_stateful_kernel).
 *
 * Per element n and step t (every operation rounded to float32 in this order,
 * exactly as torch-CPU eager executes naive_if_lif):
 *   in  = x[t,n]  (+ bias[c(n)])  (+ residual[t,n])
 *   v   = (df * v) + (sc * in)
 *   s   = (v >= thr(n))
 *   soft: v = v - s * thr(n)          hard: v = s ? v_reset : v
 * with c(n) = n % C (channels-last) or (n / HW) % C (NCHW), fused.py:82-85.
 */
#include <stdint.h>
#include <stddef.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

enum { THR_SCALAR = 0, THR_PER_CHANNEL = 1, THR_PER_NEURON = 2 };

static inline int64_t chan_of(int64_t n, int64_t C, int64_t HW, int channel_last) {
    return channel_last ? (n % C) : ((n / HW) % C);
}

/* Returns 0 on success, -1 on a bad argument. */
int oracle_lif(const float* x, int64_t T, int64_t N,
               const float* bias, const float* residual,
               int64_t C, int64_t HW, int channel_last,
               float df, float sc, int hard_reset, float v_reset,
               int thr_mode, float thr_scalar, const float* thr,
               const float* v_init,
               float* spikes, float* count, float* v_out, float* v_pre,
               int nthreads)
{
    if (T < 0 || N < 0 || (thr_mode != THR_SCALAR && thr == NULL)) return -1;
    if ((bias || thr_mode == THR_PER_CHANNEL) && (C <= 0 || HW <= 0)) return -1;
    const int64_t BLK = 2048;
    const int64_t nblk = (N + BLK - 1) / BLK;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
#endif
    for (int64_t b = 0; b < nblk; ++b) {
        float v[2048], th[2048], bb[2048], cnt[2048];
        const int64_t n0 = b * BLK;
        const int64_t m = (N - n0) < BLK ? (N - n0) : BLK;
        for (int64_t i = 0; i < m; ++i) {
            const int64_t n = n0 + i;
            int64_t c = (bias || thr_mode == THR_PER_CHANNEL) ? chan_of(n, C, HW, channel_last) : 0;
            v[i] = v_init ? v_init[n] : 0.0f;
            th[i] = thr_mode == THR_SCALAR ? thr_scalar
                  : (thr_mode == THR_PER_CHANNEL ? thr[c] : thr[n]);
            bb[i] = bias ? bias[c] : 0.0f;
            cnt[i] = 0.0f;
        }
        for (int64_t t = 0; t < T; ++t) {
            const float* xt = x + t * N + n0;
            const float* rt = residual ? residual + t * N + n0 : NULL;
            float* st = spikes ? spikes + t * N + n0 : NULL;
            float* pt = v_pre ? v_pre + t * N + n0 : NULL;
            for (int64_t i = 0; i < m; ++i) {
                float in = xt[i];
                if (bias) in = in + bb[i];
                if (rt) in = in + rt[i];
                float a = df * v[i];
                float d = sc * in;
                float vv = a + d;
                if (pt) pt[i] = vv;
                float s = (vv >= th[i]) ? 1.0f : 0.0f;
                if (hard_reset) {
                    vv = (s > 0.0f) ? v_reset : vv;
                } else {
                    float sub = s * th[i];
                    vv = vv - sub;
                }
                v[i] = vv;
                if (st) st[i] = s;
                cnt[i] = cnt[i] + s;
            }
        }
        for (int64_t i = 0; i < m; ++i) {
            if (count) count[n0 + i] = cnt[i];
            if (v_out) v_out[n0 + i] = v[i];
        }
    }
    return 0;
}

/* Number of OpenMP threads this build would use (1 without OpenMP). */
int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
