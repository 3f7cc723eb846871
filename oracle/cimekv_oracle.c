/*
 * cimekv_oracle.c — CPU restatement of the reference Flash-EKV LUT path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker for the CUDA library
 * (tests, smoke check, the CPU baseline leg of bench.py); nothing in the
 * operator calls it.
 *
 * It restates, in plain C with the same fp32 operation order per lookup:
 *   - the index rule and Triton lerp of _lut_lookup
 *       src/isa/kernels/transformer_ffn/ekv_lut_triton.py:26-34
 *   - the forward kernel (sum over k of (L(x-wp) - L(x-wn)) / (1 + x/V_sat),
 *     clamped to [out_min, out_max])
 *       ekv_lut_triton.py:37-62
 *   - the shared-memory CUDA backward: lut_pair_shared / lut_lookup_shared
 *     (fmaf lerp) and the dX / dWpos / dWneg sums
 *       src/isa/kernels/transformer_ffn/cuda/ekv_cuda.cu:59-87,193-252,296-341
 * Tables are the reference's bf16 tables (delta_lut.py:12-35) widened to fp32.
 *
 * Per-cell lookups are fp32 exactly as in the reference; the sums over k, o
 * and m are accumulated in fp64 so the oracle is the exactly-summed value the
 * fp32 GPU reductions (reference and ours) approximate.  Each output also gets
 * a magnitude (sum of |term|) for scale-aware tolerances.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp, no -ffast-math, no FMA contraction
 * beyond the explicit fmaf calls: -ffp-contract=off).
 */
#include <math.h>
#include <stdint.h>
#include <stddef.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

int oracle_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* f = clamp((dV - dmin) * scale, 0, T-1) in fp32; i0 = trunc(f); a = f - i0
 * (ekv_lut_triton.py:27-31; ekv_cuda.cu:29-32 with __float2int_rz). */
static inline void lut_coord(float dv, float dmin, float scale, int T, int* i0, int* i1, float* a) {
    float s = dv - dmin;
    float f = s * scale;
    f = fminf(fmaxf(f, 0.0f), (float)(T - 1));
    int i = (int)f; /* C truncates toward zero */
    *i0 = i;
    *i1 = i + 1 < T - 1 ? i + 1 : T - 1;
    *a = f - (float)i;
}

void oracle_lut_index(const float* delta, int n, int T, float dmin, float scale, int32_t* index, float* alpha) {
    for (int i = 0; i < n; ++i) {
        int i0, i1;
        float a;
        lut_coord(delta[i], dmin, scale, T, &i0, &i1, &a);
        index[i] = i0;
        alpha[i] = a;
    }
}

/* Triton _lut_lookup lerp: q0 * (1 - a) + q1 * a (ekv_lut_triton.py:34). */
static inline float lookup_triton(const float* table, float dv, float dmin, float scale, int T) {
    int i0, i1;
    float a;
    lut_coord(dv, dmin, scale, T, &i0, &i1, &a);
    float w0 = 1.0f - a;
    float t0 = table[i0] * w0;
    float t1 = table[i1] * a;
    return t0 + t1;
}

/* CUDA lut_lookup_shared lerp: fmaf(a, q1 - q0, q0) (ekv_cuda.cu:59-70). */
static inline float lookup_fma(const float* table, float dv, float dmin, float scale, int T) {
    int i0, i1;
    float a;
    lut_coord(dv, dmin, scale, T, &i0, &i1, &a);
    return fmaf(a, table[i1] - table[i0], table[i0]);
}

/*
 * out[m,o]  = clamp(sum_k (Lp - Ln) / (1 + x/v_sat), out_min, out_max)
 * mag[m,o]  = sum_k |(Lp - Ln) / (1 + x/v_sat)|            (may be NULL)
 */
void oracle_forward(const float* x, const float* wp, const float* wn, const float* table_i, int M, int K, int O,
                    int T, float dmin, float scale, float v_sat, float out_min, float out_max, float* out,
                    float* mag, int nthreads) {
    set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (long mo = 0; mo < (long)M * O; ++mo) {
        const long m = mo / O, o = mo % O;
        const float* xr = x + m * K;
        const float* pr = wp + o * K;
        const float* nr = wn + o * K;
        double acc = 0.0, am = 0.0;
        for (int k = 0; k < K; ++k) {
            const float xv = xr[k];
            const float bp = lookup_triton(table_i, xv - pr[k], dmin, scale, T);
            const float bn = lookup_triton(table_i, xv - nr[k], dmin, scale, T);
            float denom = 1.0f + xv / v_sat;
            const float term = (bp - bn) / denom;
            acc += term;
            am += fabs(term);
        }
        float v = (float)acc;
        v = fminf(fmaxf(v, out_min), out_max);
        out[mo] = v;
        if (mag) mag[mo] = (float)am;
    }
}

/*
 * grad_x[m,k]    = sum_o g[m,o] * ((dp - dn) * inv_d - (bp - bn) * dterm)
 * grad_wpos[o,k] = sum_m g[m,o] * (-dp * inv_d)
 * grad_wneg[o,k] = sum_m g[m,o] * ( dn * inv_d)
 * inv_d = 1/(1 + x/v_sat), dterm = 1/(v_sat * d * d)   (ekv_cuda.cu:224-251, 320-340)
 * Any output pointer may be NULL; mag_* receive sums of |term| (may be NULL).
 */
void oracle_backward(const float* x, const float* wp, const float* wn, const float* g, const float* table_i,
                     const float* table_dd, int M, int K, int O, int T, float dmin, float scale, float v_sat,
                     float* grad_x, float* grad_wp, float* grad_wn, float* mag_x, float* mag_wp, float* mag_wn,
                     int nthreads) {
    set_threads(nthreads);
    if (grad_x) {
#pragma omp parallel for schedule(static)
        for (long mk = 0; mk < (long)M * K; ++mk) {
            const long m = mk / K, k = mk % K;
            const float xv = x[mk];
            float d = 1.0f + xv / v_sat;
            const float inv_d = 1.0f / d;
            float vd = v_sat * d;
            float vdd = vd * d;
            const float dterm = 1.0f / vdd;
            double acc = 0.0, am = 0.0;
            for (int o = 0; o < O; ++o) {
                const float dvp = xv - wp[(long)o * K + k];
                const float dvn = xv - wn[(long)o * K + k];
                const float pb = lookup_fma(table_i, dvp, dmin, scale, T);
                const float pd = lookup_fma(table_dd, dvp, dmin, scale, T);
                const float nb = lookup_fma(table_i, dvn, dmin, scale, T);
                const float nd = lookup_fma(table_dd, dvn, dmin, scale, T);
                float t1 = (pd - nd) * inv_d;
                float t2 = (pb - nb) * dterm;
                const float deriv = t1 - t2;
                const float term = g[m * O + o] * deriv;
                acc += term;
                am += fabs(term);
            }
            grad_x[mk] = (float)acc;
            if (mag_x) mag_x[mk] = (float)am;
        }
    }
    if (grad_wp || grad_wn) {
#pragma omp parallel for schedule(static)
        for (long ok = 0; ok < (long)O * K; ++ok) {
            const long o = ok / K, k = ok % K;
            const float wpv = wp[ok], wnv = wn[ok];
            double ap = 0.0, an = 0.0, mp = 0.0, mn = 0.0;
            for (int m = 0; m < M; ++m) {
                const float xv = x[(long)m * K + k];
                const float gv = g[(long)m * O + o];
                float d = 1.0f + xv / v_sat;
                const float inv_d = 1.0f / d;
                const float pd = lookup_fma(table_dd, xv - wpv, dmin, scale, T);
                const float nd = lookup_fma(table_dd, xv - wnv, dmin, scale, T);
                float tp = -pd * inv_d;
                float tn = nd * inv_d;
                const float vp = gv * tp, vn = gv * tn;
                ap += vp;
                an += vn;
                mp += fabs(vp);
                mn += fabs(vn);
            }
            if (grad_wp) grad_wp[ok] = (float)ap;
            if (grad_wn) grad_wn[ok] = (float)an;
            if (mag_wp) mag_wp[ok] = (float)mp;
            if (mag_wn) mag_wn[ok] = (float)mn;
        }
    }
}

/* ------------------------------------------------------------------------
 * Exact-formula path (cfg ekv_approx != "lut"), in fp64.
 * Follows the reference's CPU formulation, src/isa/device_models/
 * flash_transistor.py:27-82 (ekv_current, ekv_current_grad_v,
 * ekv_current_grad_vth; torch softplus with threshold 20), which its exact
 * Triton kernels (src/isa/kernels/transformer_ffn/ekv_triton.py:23-150)
 * evaluate in fp32.  Magnitudes sum |I_pos| + |I_neg| per term, because the two
 * branches are evaluated independently and their fp32 errors do not cancel.
 * ------------------------------------------------------------------------ */
static inline double sp_exact(double u) { return u > 20.0 ? u : log1p(exp(u)); }
static inline double sig_exact(double u) { return 1.0 / (1.0 + exp(-u)); }

/* I_S (sp1^2 - sp2^2) and its derivative in dV (without the 1/(1+V/V_sat) factor). */
static inline void ekv_exact(double dv, double inv, double vd, double is, double* I, double* dI) {
    const double u1 = dv * inv, u2 = (dv - vd) * inv;
    const double s1 = sp_exact(u1), s2 = sp_exact(u2);
    *I = is * (s1 * s1 - s2 * s2);
    if (dI) *dI = is * 2.0 * inv * (s1 * sig_exact(u1) - s2 * sig_exact(u2));
}

void oracle_exact_forward(const float* x, const float* wp, const float* wn, int M, int K, int O, double inv,
                          double vd, double is, double v_sat, float* out, float* mag, int nthreads) {
    set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (long mo = 0; mo < (long)M * O; ++mo) {
        const long m = mo / O, o = mo % O;
        double acc = 0.0, am = 0.0;
        for (int k = 0; k < K; ++k) {
            const double xv = x[m * K + k];
            double ip, in_;
            ekv_exact(xv - (double)wp[o * K + k], inv, vd, is, &ip, NULL);
            ekv_exact(xv - (double)wn[o * K + k], inv, vd, is, &in_, NULL);
            const double d = 1.0 + xv / v_sat;
            acc += (ip - in_) / d;
            am += (fabs(ip) + fabs(in_)) / fabs(d);
        }
        out[mo] = (float)acc;
        if (mag) mag[mo] = (float)am;
    }
}

void oracle_exact_backward(const float* x, const float* wp, const float* wn, const float* g, int M, int K, int O,
                           double inv, double vd, double is, double v_sat, float* grad_x, float* grad_wp,
                           float* grad_wn, float* mag_x, float* mag_wp, float* mag_wn, int nthreads) {
    set_threads(nthreads);
    if (grad_x) {
#pragma omp parallel for schedule(static)
        for (long mk = 0; mk < (long)M * K; ++mk) {
            const long m = mk / K, k = mk % K;
            const double xv = x[mk];
            const double d = 1.0 + xv / v_sat;
            double acc = 0.0, am = 0.0;
            for (int o = 0; o < O; ++o) {
                double ip, dip, in_, din;
                ekv_exact(xv - (double)wp[(long)o * K + k], inv, vd, is, &ip, &dip);
                ekv_exact(xv - (double)wn[(long)o * K + k], inv, vd, is, &in_, &din);
                const double gv = g[m * O + o];
                acc += gv * ((dip - din) / d - (ip - in_) / (v_sat * d * d));
                am += fabs(gv) * ((fabs(dip) + fabs(din)) / fabs(d) + (fabs(ip) + fabs(in_)) / (v_sat * d * d));
            }
            grad_x[mk] = (float)acc;
            if (mag_x) mag_x[mk] = (float)am;
        }
    }
    if (grad_wp || grad_wn) {
#pragma omp parallel for schedule(static)
        for (long ok = 0; ok < (long)O * K; ++ok) {
            const long o = ok / K, k = ok % K;
            double ap = 0.0, an = 0.0, mp = 0.0, mn = 0.0;
            for (int m = 0; m < M; ++m) {
                const double xv = x[(long)m * K + k];
                const double gv = g[(long)m * O + o];
                const double d = 1.0 + xv / v_sat;
                double ip, dip, in_, din;
                ekv_exact(xv - (double)wp[ok], inv, vd, is, &ip, &dip);
                ekv_exact(xv - (double)wn[ok], inv, vd, is, &in_, &din);
                ap += gv * (-dip / d);
                an += gv * (din / d);
                mp += fabs(gv * dip / d);
                mn += fabs(gv * din / d);
            }
            if (grad_wp) grad_wp[ok] = (float)ap;
            if (grad_wn) grad_wn[ok] = (float)an;
            if (mag_wp) mag_wp[ok] = (float)mp;
            if (mag_wn) mag_wn[ok] = (float)mn;
        }
    }
}
