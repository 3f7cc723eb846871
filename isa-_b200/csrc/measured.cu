// measured.cu — measured-codebook CIM forward (DeploymentAwareCIMLinear,
// "measured" mode) and its input gradient, sm_100a.
//
// Each crossbar device o,k is assigned one of S measured I-V curves for the
// positive and one for the negative branch (pos_idx / neg_idx, int16 [O,K]).
// A curve is piecewise linear over a strictly increasing gate-voltage grid
// vg[G]: on segment j (vg[j] <= v < vg[j+1]) I_s(v) = a[s][j] v + b[s][j].
//   out[m,o] = clamp(r_tia * sum_k (x (a_p - a_n) + (b_p - b_n)), lo, hi)
// with x = clamp(x[m,k], lookup_min, lookup_max) and j = searchsorted(vg, x,
// right) - 1 clamped to [0, G-2]  (reference: measured_deployment/operator.py
// measured_forward, :163-206; its active-segment masked GEMMs compute the same
// per-cell term x*(slope_p - slope_n) + (icpt_p - icpt_n)).
//
// The segment depends only on (m,k), so it is found once per staged element
// (binary search over vg in shared memory) and shared by all outputs; the
// per-cell work is two gathers of {a, b} from a shared-memory coefficient
// table and two FMAs.

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "cimekv.h"

// Shared with cimekv.cu: records the message cimekv_last_error() returns.
void cimekv_internal_set_error(const char* msg);

namespace {

int fail(int code, const char* msg) {
    cimekv_internal_set_error(msg);
    return code;
}

constexpr int kThreads = 256;
constexpr int kMT = 64;   // tokens per tile
constexpr int kOT = 64;   // outputs per tile
constexpr int kKC = 16;   // inputs per staged chunk
constexpr int kLD = 68;   // padded row stride of the k-major tiles
constexpr int kMaxCoef = 16384;  // S * (G - 1) coefficient pairs held in shared memory (128 KiB)

struct MeasParams {
    const float* x;
    const int16_t* pos;
    const int16_t* neg;
    const float* vg;
    const float2* coef;  // [S][G-1] {slope, intercept}
    const float* r_tia;
    float* idiff;        // optional pre-TIA sum
    float* out;
    int M, K, O, S, G;
    float lookup_min, lookup_max, lo, hi;
};

// Segment j with vg[j] <= v < vg[j+1] (right-bisect minus one), clamped to
// [0, G-2]; vg is in shared memory.
__device__ __forceinline__ int segment_of(const float* vg, int G, float v) {
    int lo = 0, hi = G;  // first index with vg[idx] > v lies in [lo, hi]
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (vg[mid] <= v) lo = mid + 1;
        else hi = mid;
    }
    int j = lo - 1;
    j = j < 0 ? 0 : j;
    return j > G - 2 ? G - 2 : j;
}

__device__ __forceinline__ float clamp_nan(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }

__global__ void __launch_bounds__(kThreads) measured_fwd_kernel(MeasParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int nseg = p.G - 1;
    // Coefficients transposed to [segment][state]: a warp reads one segment for
    // its lanes' (random) states, i.e. adjacent words instead of a fixed stride.
    float2* coef = reinterpret_cast<float2*>(smem);                  // [G-1][S]
    float* vg = reinterpret_cast<float*>(coef + p.S * nseg);         // [G] (+pad)
    float* xs = vg + ((p.G + 3) & ~3);                                // [KC][LD] clamped x
    int* js = reinterpret_cast<int*>(xs + kKC * kLD);                 // [KC][LD] segment * S
    int* ps = js + kKC * kLD;                                         // [KC][LD] pos state
    int* ns = ps + kKC * kLD;                                         // [KC][LD] neg state
    for (int i = threadIdx.x; i < p.S * nseg; i += blockDim.x) {
        const int st = i / nseg, sg = i - st * nseg;
        coef[sg * p.S + st] = p.coef[i];
    }
    for (int i = threadIdx.x; i < p.G; i += blockDim.x) vg[i] = p.vg[i];
    __syncthreads();
    const float r = __ldg(p.r_tia);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_o = (p.O + kOT - 1) / kOT;
    const int ntiles = ((p.M + kMT - 1) / kMT) * tiles_o;
    for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const int m0 = (tile / tiles_o) * kMT, o0 = (tile % tiles_o) * kOT;
        float acc[8][2];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = 0.0f;
        for (int k0 = 0; k0 < p.K; k0 += kKC) {
            __syncthreads();
            for (int e = threadIdx.x; e < kMT * kKC; e += blockDim.x) {
                const int row = e >> 4, kk = e & 15, k = k0 + kk;
                const int m = m0 + row, o = o0 + row;
                const bool kin = k < p.K;
                float xv = (kin && m < p.M) ? __ldg(p.x + (int64_t)m * p.K + k) : p.lookup_min;
                xv = fminf(fmaxf(xv, p.lookup_min), p.lookup_max);  // torch clamp on a finite range
                // (padded k beyond K is staged but never summed: the loop below stops at kc)
                xs[kk * kLD + row] = xv;
                js[kk * kLD + row] = segment_of(vg, p.G, xv) * p.S;
                const bool oin = kin && o < p.O;
                ps[kk * kLD + row] = oin ? (int)p.pos[(int64_t)o * p.K + k] : 0;
                ns[kk * kLD + row] = oin ? (int)p.neg[(int64_t)o * p.K + k] : 0;
            }
            __syncthreads();
            const int kc = p.K - k0 < kKC ? p.K - k0 : kKC;
            for (int kk = 0; kk < kc; ++kk) {
                int pi[2], ni[2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    pi[j] = ps[kk * kLD + lane + 32 * j];
                    ni[j] = ns[kk * kLD + lane + 32 * j];
                }
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float xv = xs[kk * kLD + warp * 8 + i];
                    const int seg = js[kk * kLD + warp * 8 + i];
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const float2 cp = coef[pi[j] + seg], cn = coef[ni[j] + seg];
                        acc[i][j] += fmaf(xv, cp.x - cn.x, cp.y - cn.y);
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int m = m0 + warp * 8 + i;
            if (m >= p.M) continue;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int o = o0 + lane + 32 * j;
                if (o >= p.O) continue;
                if (p.idiff) p.idiff[(int64_t)m * p.O + o] = acc[i][j];
                p.out[(int64_t)m * p.O + o] = clamp_nan(__fmul_rn(acc[i][j], r), p.lo, p.hi);
            }
        }
    }
}

// grad_x[m,k] = [lookup_min <= x <= lookup_max] * sum_o g'[m,o] (a_p - a_n)[seg(x)]
// with g' = g * r_tia * [lo <= idiff * r_tia <= hi] (the autograd of the
// reference's clamp(x), masked GEMMs, * r_tia and clamp).  One thread per
// (m,k); the warp shares m, so g' is a broadcast read.
__global__ void __launch_bounds__(kThreads) measured_dx_kernel(MeasParams p, const float* __restrict__ g,
                                                                float* __restrict__ gx) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int nseg = p.G - 1;
    float2* coef = reinterpret_cast<float2*>(smem);  // [G-1][S]
    float* vg = reinterpret_cast<float*>(coef + p.S * nseg);
    for (int i = threadIdx.x; i < p.S * nseg; i += blockDim.x) {
        const int st = i / nseg, sg = i - st * nseg;
        coef[sg * p.S + st] = p.coef[i];
    }
    for (int i = threadIdx.x; i < p.G; i += blockDim.x) vg[i] = p.vg[i];
    __syncthreads();
    const float r = __ldg(p.r_tia);
    const int64_t n = (int64_t)p.M * p.K;
    for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t m = e / p.K;
        const int k = (int)(e - m * p.K);
        const float xr = p.x[e];
        if (!(xr >= p.lookup_min && xr <= p.lookup_max)) {  // clamp passes no gradient
            gx[e] = 0.0f;
            continue;
        }
        const int seg = segment_of(vg, p.G, xr) * p.S;
        float acc = 0.0f;
        for (int o = 0; o < p.O; ++o) {
            const float id = p.idiff[m * p.O + o];
            const float v = __fmul_rn(id, r);
            if (!(v >= p.lo && v <= p.hi)) continue;
            const float gm = __fmul_rn(g[m * p.O + o], r);
            const int64_t w = (int64_t)o * p.K + k;
            acc = fmaf(gm, coef[seg + (int)p.pos[w]].x - coef[seg + (int)p.neg[w]].x, acc);
        }
        gx[e] = acc;
    }
}

int check_args(const MeasParams& p) {
    if (p.M < 0 || p.K < 0 || p.O < 0) return fail(CIMEKV_EINVAL_SHAPE, "negative size");
    if (p.S < 1 || p.G < 2) return fail(CIMEKV_EINVAL_SHAPE, "need >= 1 state and >= 2 grid points");
    if ((int64_t)p.S * (p.G - 1) > kMaxCoef)
        return fail(CIMEKV_ELUT_TOO_LARGE, "states*(grid points-1) exceeds 16384 coefficient pairs");
    if (!p.vg || !p.coef || !p.r_tia || (p.M * (int64_t)p.O > 0 && !p.out) ||
        ((int64_t)p.M * p.K * p.O > 0 && (!p.x || !p.pos || !p.neg)))
        return fail(CIMEKV_EINVAL_SHAPE, "null pointer");
    return CIMEKV_OK;
}

size_t smem_bytes(const MeasParams& p, bool fwd) {
    size_t b = (size_t)p.S * (p.G - 1) * sizeof(float2) + (size_t)((p.G + 3) & ~3) * 4;
    if (fwd) b += (size_t)4 * kKC * kLD * 4;
    return b;
}

int launch_setup(const MeasParams& p, bool fwd, size_t* smem, int* sms) {
    int dev;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(CIMEKV_ECUDA, "cudaGetDevice failed");
    int optin = 0;
    cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    *smem = smem_bytes(p, fwd);
    if (*smem > (size_t)optin) return fail(CIMEKV_ELUT_TOO_LARGE, "codebook does not fit shared memory");
    cudaError_t e = fwd ? cudaFuncSetAttribute(measured_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin)
                        : cudaFuncSetAttribute(measured_dx_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
    if (e != cudaSuccess) return fail(CIMEKV_ECUDA, cudaGetErrorString(e));
    return CIMEKV_OK;
}

MeasParams make_params(const float* x, const int16_t* pos, const int16_t* neg, const float* vg, const float* coef,
                       int M, int K, int O, int S, int G, float lookup_min, float lookup_max, const float* r_tia,
                       float out_min, float out_max, float* idiff, float* out) {
    MeasParams p;
    p.x = x;
    p.pos = pos;
    p.neg = neg;
    p.vg = vg;
    p.coef = reinterpret_cast<const float2*>(coef);
    p.r_tia = r_tia;
    p.idiff = idiff;
    p.out = out;
    p.M = M;
    p.K = K;
    p.O = O;
    p.S = S;
    p.G = G;
    p.lookup_min = lookup_min;
    p.lookup_max = lookup_max;
    p.lo = out_min;
    p.hi = out_max;
    return p;
}

}  // namespace

extern "C" int cimekv_measured_forward(const float* x, const int16_t* pos_idx, const int16_t* neg_idx,
                                       const float* vg, const float* coef, int M, int K, int O, int S, int G,
                                       float lookup_min, float lookup_max, const float* r_tia, float out_min,
                                       float out_max, float* idiff, float* out, void* stream) {
    cimekv_internal_set_error("");
    MeasParams p = make_params(x, pos_idx, neg_idx, vg, coef, M, K, O, S, G, lookup_min, lookup_max, r_tia,
                               out_min, out_max, idiff, out);
    int rc = check_args(p);
    if (rc || M == 0 || O == 0) return rc;
    size_t smem;
    int sms;
    if ((rc = launch_setup(p, true, &smem, &sms))) return rc;
    const long tiles = (long)((M + kMT - 1) / kMT) * ((O + kOT - 1) / kOT);
    long grid = (long)sms * 2;
    if (grid > tiles) grid = tiles;
    measured_fwd_kernel<<<(unsigned)grid, kThreads, smem, (cudaStream_t)stream>>>(p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CIMEKV_OK : fail(CIMEKV_ECUDA, cudaGetErrorString(e));
}

extern "C" int cimekv_measured_backward_x(const float* x, const int16_t* pos_idx, const int16_t* neg_idx,
                                          const float* vg, const float* coef, int M, int K, int O, int S, int G,
                                          float lookup_min, float lookup_max, const float* r_tia, float out_min,
                                          float out_max, const float* idiff, const float* grad_out,
                                          float* grad_x, void* stream) {
    cimekv_internal_set_error("");
    MeasParams p = make_params(x, pos_idx, neg_idx, vg, coef, M, K, O, S, G, lookup_min, lookup_max, r_tia,
                               out_min, out_max, const_cast<float*>(idiff), grad_x);
    int rc = check_args(p);
    if (rc || M == 0 || K == 0) return rc;
    if (O > 0 && (!idiff || !grad_out)) return fail(CIMEKV_EINVAL_SHAPE, "null pointer");
    size_t smem;
    int sms;
    if ((rc = launch_setup(p, false, &smem, &sms))) return rc;
    const int64_t n = (int64_t)M * K;
    long grid = (long)((n + kThreads - 1) / kThreads);
    if (grid > (long)sms * 8) grid = (long)sms * 8;
    measured_dx_kernel<<<(unsigned)grid, kThreads, smem, (cudaStream_t)stream>>>(p, grad_out, grad_x);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CIMEKV_OK : fail(CIMEKV_ECUDA, cudaGetErrorString(e));
}
