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
// per-cell work is four conflict-free 32-bit gathers (slope and intercept of
// both branches) from shared-memory tables and an FMA.

#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

#include "cimekv.h"

// Shared with cimekv.cu: records the message cimekv_last_error() returns.
void cimekv_internal_set_error(const char* msg);
// Shared with cimekv.cu: clears the message, fails on a CUDA error left pending by earlier work.
int cimekv_internal_begin_call();
// Shared with cimekv.cu: fails when a CUDA error from earlier work is pending.
int cimekv_internal_no_pending_error();

namespace {

int fail(int code, const char* msg) {
    cimekv_internal_set_error(msg);
    return code;
}

#ifndef CIMEKV_MEAS_FWD_CTAS
#define CIMEKV_MEAS_FWD_CTAS 4  // resident forward CTAs per SM (persistent grid)
#endif

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

// The codebook in shared memory: slopes and intercepts as two tables laid out
// [segment][state], the intercepts at a compile-time byte offset kIcOff from
// the slopes (one address serves both loads).  A warp's lanes (outputs) read
// one segment at their states, i.e. at most S <= 32 adjacent words of one
// table: conflict-free.
template <int kIcOff>
__device__ __forceinline__ void stage_codebook(const MeasParams& p, float* sl, float* vg, bool with_icpt) {
    const int nseg = p.G - 1;
    for (int i = threadIdx.x; i < p.S * nseg; i += blockDim.x) {
        const int st = i / nseg, sg = i - st * nseg;
        const float2 c = p.coef[i];
        sl[sg * p.S + st] = c.x;
        if (with_icpt) sl[kIcOff / 4 + sg * p.S + st] = c.y;
    }
    for (int i = threadIdx.x; i < p.G; i += blockDim.x) vg[i] = p.vg[i];
}

__device__ __forceinline__ float lds_f32(uint32_t addr) {
    float v;
    asm("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
    return v;
}
template <int kOff>
__device__ __forceinline__ float lds_f32_off(uint32_t addr) {
    float v;
    asm("ld.shared.f32 %0, [%1+%2];" : "=f"(v) : "r"(addr), "n"(kOff));
    return v;
}

// Byte size of the slope + intercept region of the forward (kIcOff each).
constexpr int kIcOffSmall = 4096;   // S*(G-1) <= 1024
constexpr int kIcOffLarge = 65536;  // S*(G-1) <= 16384

template <int kIcOff>
__global__ void __launch_bounds__(kThreads) measured_fwd_kernel(MeasParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    float* sl = reinterpret_cast<float*>(smem);                       // [G-1][S] slopes; intercepts at +kIcOff
    float* vg = reinterpret_cast<float*>(smem + 2 * kIcOff);           // [G] (+pad)
    float* xs = vg + ((p.G + 3) & ~3);                                // [KC][LD] clamped x
    int* js = reinterpret_cast<int*>(xs + kKC * kLD);                 // [KC][LD] byte offset of the segment row
    uint32_t* ps = reinterpret_cast<uint32_t*>(js + kKC * kLD);       // [KC][LD] 4 pos | 4 neg << 16
    stage_codebook<kIcOff>(p, sl, vg, true);
    __syncthreads();
    const uint32_t sl_base = static_cast<uint32_t>(__cvta_generic_to_shared(sl));
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
                js[kk * kLD + row] = (int)sl_base + segment_of(vg, p.G, xv) * p.S * 4;
                const bool oin = kin && o < p.O;
                const uint32_t sp = oin ? (uint32_t)p.pos[(int64_t)o * p.K + k] * 4u : 0u;
                const uint32_t sn = oin ? (uint32_t)p.neg[(int64_t)o * p.K + k] * 4u : 0u;
                ps[kk * kLD + row] = sp | (sn << 16);
            }
            __syncthreads();
            const int kc = p.K - k0 < kKC ? p.K - k0 : kKC;
#pragma unroll 2
            for (int kk = 0; kk < kc; ++kk) {
                int pi[2], ni[2];
#pragma unroll
                for (int j = 0; j < 2; ++j) {
                    const uint32_t v = ps[kk * kLD + lane + 32 * j];
                    pi[j] = (int)(v & 0xFFFFu);
                    ni[j] = (int)(v >> 16);
                }
                const float4 xa = *reinterpret_cast<const float4*>(xs + kk * kLD + warp * 8);
                const float4 xb = *reinterpret_cast<const float4*>(xs + kk * kLD + warp * 8 + 4);
                const int4 ja = *reinterpret_cast<const int4*>(js + kk * kLD + warp * 8);
                const int4 jb = *reinterpret_cast<const int4*>(js + kk * kLD + warp * 8 + 4);
                const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
                const int seg[8] = {ja.x, ja.y, ja.z, ja.w, jb.x, jb.y, jb.z, jb.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
#pragma unroll
                    for (int j = 0; j < 2; ++j) {
                        const uint32_t ap = (uint32_t)(seg[i] + pi[j]), an = (uint32_t)(seg[i] + ni[j]);
                        const float da = lds_f32(ap) - lds_f32(an);
                        const float db = lds_f32_off<kIcOff>(ap) - lds_f32_off<kIcOff>(an);
                        acc[i][j] += fmaf(xv[i], da, db);
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
// reference's clamp(x), masked GEMMs, * r_tia and clamp).
//
// Tiled like the forward: CTA = kDxKT inputs x one token split; per 64-token
// tile, warp w owns tokens [8w, 8w+8) and lane l walks outputs o = 32c + l, so
// the slope gathers of a warp hit one segment row at the lanes' states
// (conflict-free).  g' is formed once per (token, output) per CTA from
// loads prefetched a chunk ahead; the assignment of the CTA's inputs
// ([O][kDxKT] pos/neg) is staged once.  dX of a thread's 8 tokens x 4 inputs
// sums in registers over its outputs, then one 32-lane transpose-reduce per
// tile.
constexpr int kDxKT = 4;
constexpr int kDxMinBlocks = 3;

__global__ void __launch_bounds__(kThreads, kDxMinBlocks)
    measured_dx_kernel(MeasParams p, const float* __restrict__ g, float* __restrict__ gx, int nsplit) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int ncoef = p.S * (p.G - 1);
    const int opad = (p.O + 31) / 32 * 32;
    float* sl = reinterpret_cast<float*>(smem);                       // [G-1][S] slopes
    float* vg = sl + ((ncoef + 3) & ~3);                               // [G] (+pad to 16 bytes)
    int* seg_s = reinterpret_cast<int*>(vg + ((p.G + 3) & ~3));        // [4 inputs][64 tokens] row address
    int* ok_s = seg_s + kMT * kDxKT;                                   // [4 inputs][64 tokens] x inside the range
    int4* st_s = reinterpret_cast<int4*>(ok_s + kMT * kDxKT);          // [opad] {4p | 4n << 16} per input
    stage_codebook<0>(p, sl, vg, false);
    const uint32_t sl_base = static_cast<uint32_t>(__cvta_generic_to_shared(sl));
    const int k0 = blockIdx.x * kDxKT;
    for (int o = threadIdx.x; o < opad; o += blockDim.x) {
        int v[kDxKT];
#pragma unroll
        for (int kk = 0; kk < kDxKT; ++kk) {
            const int k = k0 + kk;
            const bool in = o < p.O && k < p.K;
            const int ps = in ? (int)p.pos[(int64_t)o * p.K + k] : 0;
            const int ns = in ? (int)p.neg[(int64_t)o * p.K + k] : 0;
            v[kk] = (int)((uint32_t)(ps * 4) | ((uint32_t)(ns * 4) << 16));
        }
        st_s[o] = make_int4(v[0], v[1], v[2], v[3]);
    }
    const float r = __ldg(p.r_tia);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (p.M + kMT - 1) / kMT;
    const int tile_lo = (int)((int64_t)blockIdx.y * tiles_m / nsplit);
    const int tile_hi = (int)((int64_t)(blockIdx.y + 1) * tiles_m / nsplit);
    const int nchunks = opad / 32;
    for (int tile = tile_lo; tile < tile_hi; ++tile) {
        const int m0 = tile * kMT;
        __syncthreads();  // codebook/assignment staged; previous tile's readers of seg_s done
        {
            const int t = threadIdx.x >> 2, kk = threadIdx.x & 3;
            const int m = m0 + t, k = k0 + kk;
            int sg = 0, ok = 0;
            if (m < p.M && k < p.K) {
                const float xr = __ldg(p.x + (int64_t)m * p.K + k);
                if (xr >= p.lookup_min && xr <= p.lookup_max) {
                    sg = segment_of(vg, p.G, xr) * p.S * 4;
                    ok = 1;
                }
            }
            seg_s[kk * kMT + t] = (int)sl_base + sg;
            ok_s[kk * kMT + t] = ok;
        }
        __syncthreads();
        // Upstream gradient and I_diff of this warp's 8 tokens at output
        // 32c + lane, prefetched one chunk ahead (both loads in flight at once).
        float nid[8], ng[8];
        const bool rows_full = m0 + kMT <= p.M;
        auto load = [&](int c) {
            const int o = c * 32 + lane;
            const int64_t e0 = (int64_t)(m0 + warp * 8) * p.O + o;
            if (rows_full && (c + 1) * 32 <= p.O) {  // interior chunk: no bounds tests
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    nid[i] = __ldg(p.idiff + e0 + (int64_t)i * p.O);
                    ng[i] = __ldg(g + e0 + (int64_t)i * p.O);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const bool in = o < p.O && m0 + warp * 8 + i < p.M;
                    nid[i] = in ? __ldg(p.idiff + e0 + (int64_t)i * p.O) : 0.0f;
                    ng[i] = in ? __ldg(g + e0 + (int64_t)i * p.O) : 0.0f;
                }
            }
        };
        float dx[8 * kDxKT];
#pragma unroll
        for (int i = 0; i < 8 * kDxKT; ++i) dx[i] = 0.0f;
        if (nchunks > 0) load(0);
        for (int c = 0; c < nchunks; ++c) {
            float gm[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float v = __fmul_rn(nid[i], r);
                gm[i] = (v >= p.lo && v <= p.hi) ? __fmul_rn(ng[i], r) : 0.0f;
            }
            if (c + 1 < nchunks) load(c + 1);
            const int4 st = st_s[c * 32 + lane];
            const int sv[kDxKT] = {st.x, st.y, st.z, st.w};
#pragma unroll
            for (int kk = 0; kk < kDxKT; ++kk) {
                const int pb = sv[kk] & 0xFFFF, nb = (int)((uint32_t)sv[kk] >> 16);
                const int4 sa = reinterpret_cast<const int4*>(seg_s + kk * kMT + warp * 8)[0];
                const int4 sb = reinterpret_cast<const int4*>(seg_s + kk * kMT + warp * 8)[1];
                const int sg[8] = {sa.x, sa.y, sa.z, sa.w, sb.x, sb.y, sb.z, sb.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float da = lds_f32((uint32_t)(sg[i] + pb)) - lds_f32((uint32_t)(sg[i] + nb));
                    dx[i * kDxKT + kk] = fmaf(gm[i], da, dx[i * kDxKT + kk]);
                }
            }
        }
        // 32-lane transpose-reduce: afterwards lane l holds the sum of element
        // l = (token l/4, input l%4).
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) {
            const bool upper = (lane & s) != 0;
#pragma unroll
            for (int j = 0; j < s; ++j) {
                const float send = upper ? dx[j] : dx[j + s];
                const float keep = upper ? dx[j + s] : dx[j];
                dx[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
            }
        }
        const int t = warp * 8 + (lane >> 2), kk = lane & 3;
        const int m = m0 + t, k = k0 + kk;
        if (m < p.M && k < p.K) gx[(int64_t)m * p.K + k] = ok_s[kk * kMT + t] ? dx[0] : 0.0f;
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

int fwd_ic_off(const MeasParams& p) { return (int64_t)p.S * (p.G - 1) * 4 <= kIcOffSmall ? kIcOffSmall : kIcOffLarge; }

size_t smem_bytes(const MeasParams& p, bool fwd) {
    const size_t ncoef = (size_t)p.S * (p.G - 1);
    const size_t vgb = (size_t)((p.G + 3) & ~3) * 4;
    if (fwd) return (size_t)2 * fwd_ic_off(p) + vgb + (size_t)3 * kKC * kLD * 4;
    return ((ncoef + 3) & ~(size_t)3) * 4 + vgb + (size_t)2 * kMT * kDxKT * 4 +
           (size_t)(p.O + 31) / 32 * 32 * sizeof(int4);
}

int launch_setup(const MeasParams& p, bool fwd, size_t* smem, int* sms) {
    int dev;
    if (cudaGetDevice(&dev) != cudaSuccess) return fail(CIMEKV_ECUDA, "cudaGetDevice failed");
    int optin = 0;
    cudaDeviceGetAttribute(sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    *smem = smem_bytes(p, fwd);
    if (*smem > (size_t)optin)
        return fail(CIMEKV_ELUT_TOO_LARGE, fwd ? "codebook does not fit shared memory"
                                               : "codebook plus the [O][4] assignment tile does not fit shared memory");
    cudaError_t e = !fwd ? cudaFuncSetAttribute(measured_dx_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, optin)
                    : fwd_ic_off(p) == kIcOffSmall
                        ? cudaFuncSetAttribute(measured_fwd_kernel<kIcOffSmall>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, optin)
                        : cudaFuncSetAttribute(measured_fwd_kernel<kIcOffLarge>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, optin);
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
    if (int rc0 = cimekv_internal_begin_call()) return rc0;
    MeasParams p = make_params(x, pos_idx, neg_idx, vg, coef, M, K, O, S, G, lookup_min, lookup_max, r_tia,
                               out_min, out_max, idiff, out);
    int rc = check_args(p);
    if (rc || M == 0 || O == 0) return rc;
    size_t smem;
    int sms;
    if ((rc = launch_setup(p, true, &smem, &sms))) return rc;
    const long tiles = (long)((M + kMT - 1) / kMT) * ((O + kOT - 1) / kOT);
    long grid = (long)sms * CIMEKV_MEAS_FWD_CTAS;
    if (grid > tiles) grid = tiles;
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    if (fwd_ic_off(p) == kIcOffSmall)
        measured_fwd_kernel<kIcOffSmall><<<(unsigned)grid, kThreads, smem, (cudaStream_t)stream>>>(p);
    else
        measured_fwd_kernel<kIcOffLarge><<<(unsigned)grid, kThreads, smem, (cudaStream_t)stream>>>(p);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CIMEKV_OK : fail(CIMEKV_ECUDA, cudaGetErrorString(e));
}

extern "C" int cimekv_measured_backward_x(const float* x, const int16_t* pos_idx, const int16_t* neg_idx,
                                          const float* vg, const float* coef, int M, int K, int O, int S, int G,
                                          float lookup_min, float lookup_max, const float* r_tia, float out_min,
                                          float out_max, const float* idiff, const float* grad_out,
                                          float* grad_x, void* stream) {
    if (int rc0 = cimekv_internal_begin_call()) return rc0;
    MeasParams p = make_params(x, pos_idx, neg_idx, vg, coef, M, K, O, S, G, lookup_min, lookup_max, r_tia,
                               out_min, out_max, const_cast<float*>(idiff), grad_x);
    int rc = check_args(p);
    if (rc || M == 0 || K == 0) return rc;
    if (O > 0 && (!idiff || !grad_out)) return fail(CIMEKV_EINVAL_SHAPE, "null pointer");
    size_t smem;
    int sms;
    if ((rc = launch_setup(p, false, &smem, &sms))) return rc;
    // grid: one CTA column per group of 4 inputs, the token tiles split into
    // enough rows for about eight waves of resident CTAs
    const int kgroups = (K + kDxKT - 1) / kDxKT;
    const int tiles_m = (M + kMT - 1) / kMT;
    int nsplit = (8 * kDxMinBlocks * sms + kgroups - 1) / kgroups;  // ~8 waves: small tail
    if (nsplit > tiles_m) nsplit = tiles_m;
    if (nsplit < 1) nsplit = 1;
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    measured_dx_kernel<<<dim3((unsigned)kgroups, (unsigned)nsplit), kThreads, smem, (cudaStream_t)stream>>>(
        p, grad_out, grad_x, nsplit);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? CIMEKV_OK : fail(CIMEKV_ECUDA, cudaGetErrorString(e));
}
