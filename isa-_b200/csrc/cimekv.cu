// cimekv.cu — Flash-EKV CIMLinear LUT operator for B200 (sm_100a).
//
// One (token m, input k, output o) "cell" evaluates the EKV branch current of
// both transistors of a differential pair through a 1-D table over
// dV = x[m,k] - vth[o,k] with linear interpolation, divides by the velocity
// saturation term d = 1 + x/V_sat and sums over k (forward) or produces the
// two gradients dX (sum over o) and dVth (sum over m) (backward).
//
// The work is a "non-dense" contraction: every cell needs a data-dependent
// table lookup, so it runs on the FP32/INT CUDA-core pipes with the tables held
// in shared memory; the tensor cores cannot express it.  Design points:
//  * the table index is computed exactly like the reference
//    (f = (fl(x-w) - dmin) * scale, clamp to [0,T-1], i0 = trunc(f),
//    a = f - i0; ekv_lut_triton.py:26-31, ekv_cuda.cu:29-32) but truncation
//    uses the IEEE round-toward-zero add of 2^23, whose result bits hold i0 and
//    double as the shared-memory address (no F2I/I2F conversions);
//  * the clamp is skipped for every tile whose x and Vth ranges provably keep
//    f inside the table (checked with the same monotone fp32 ops per tile);
//  * tables are packed as bf16 pairs (the reference tables are bf16-exact,
//    delta_lut.py:35), so one 32-bit shared load returns both interpolation
//    nodes of I, and one more (same index, fixed offset) both nodes of dI/dV;
//  * two adjacent tokens share every fp32 instruction through sm_100's packed
//    f32x2 arithmetic (bit-identical to two scalar ops);
//  * the backward computes dX and dVth from the same lookups in one pass; dX
//    is reduced in registers over all outputs, dVth over the tile's tokens in
//    shared memory and over token splits by a deterministic second kernel;
//  * the same tiles also run the exact EKV formula instead of the table
//    (cfg ekv_approx != "lut"), and the forward epilogue can apply the TIA
//    stage (* R_TIA, signed clamp).

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <mutex>

#include "cimekv.h"
#include <nvtx3/nvToolsExt.h>

// Compile-time tuning knobs.
#ifndef CIMEKV_FWD_MIN_BLOCKS
#define CIMEKV_FWD_MIN_BLOCKS 3  // resident forward CTAs per SM the register budget is sized for
#endif
#ifndef CIMEKV_DEBUG_BOUNDS
#define CIMEKV_DEBUG_BOUNDS 0  // 1: check every table index against T (debug library variant)
#endif
#ifndef CIMEKV_BWD_MIN_BLOCKS
#define CIMEKV_BWD_MIN_BLOCKS 2  // resident backward CTAs per SM the register budget is sized for
#endif
#ifndef CIMEKV_BWD_DW_FOR_OCCUPANCY
#define CIMEKV_BWD_DW_FOR_OCCUPANCY 1  // trade the shared dVth accumulator for a 2nd resident CTA
#endif
#ifndef CIMEKV_MIXED_BF16
#define CIMEKV_MIXED_BF16 1  // table differences by mixed bf16/fp32 subtract (sm_100)
#endif
#ifndef CIMEKV_FWD_KK_UNROLL
#define CIMEKV_FWD_KK_UNROLL 4
#endif

namespace {

// NVTX range for the duration of one C-ABI call (host side: it brackets the
// launches, which is what a profiler timeline needs to attribute kernels).
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
};

// ---------------------------------------------------------------- errors --

thread_local char g_last_error[512] = "";

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
    va_end(ap);
    return code;
}

}  // namespace

void cimekv_internal_set_error(const char* msg) { snprintf(g_last_error, sizeof(g_last_error), "%s", msg); }

// Start of every entry point: clears the message of the previous call.
int cimekv_internal_begin_call() {
    g_last_error[0] = '\0';
    return CIMEKV_OK;
}

// Called right before an entry point's first launch: refuses to run when a CUDA
// error is already pending from earlier work of the process (a launch by another
// library on this thread), so that the check after this call's own launches
// reports only errors of this library's kernels.
int cimekv_internal_no_pending_error() {
    const cudaError_t e = cudaPeekAtLastError();
    if (e != cudaSuccess) {
        (void)cudaGetLastError();  // consume it: it belongs to earlier work, not to this call
        return set_error(CIMEKV_ECUDA, "CUDA error pending before this call (raised by earlier work, not by "
                         "this library): %s", cudaGetErrorString(e));
    }
    return CIMEKV_OK;
}

namespace {

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return set_error(CIMEKV_ECUDA, "%s: %s", what, cudaGetErrorString(e));
    }
    return CIMEKV_OK;
}

// --------------------------------------------------------- device limits --

constexpr int kMaxDevices = 64;
std::mutex g_dev_mutex;
int g_sm_count[kMaxDevices] = {0};
int g_smem_optin[kMaxDevices] = {0};
bool g_attr_set[kMaxDevices][16] = {};

int current_device(int* dev) {
    cudaError_t e = cudaGetDevice(dev);
    if (e != cudaSuccess) return set_error(CIMEKV_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (*dev < 0 || *dev >= kMaxDevices) return set_error(CIMEKV_ECUDA, "device ordinal %d out of range", *dev);
    return CIMEKV_OK;
}

int device_limits(int dev, int* sms, int* smem_optin) {
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (g_sm_count[dev] == 0) {
        cudaError_t e1 = cudaDeviceGetAttribute(&g_sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
        cudaError_t e2 = cudaDeviceGetAttribute(&g_smem_optin[dev], cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (e1 != cudaSuccess || e2 != cudaSuccess) {
            g_sm_count[dev] = 0;
            return set_error(CIMEKV_ECUDA, "cudaDeviceGetAttribute failed");
        }
    }
    *sms = g_sm_count[dev];
    *smem_optin = g_smem_optin[dev];
    return CIMEKV_OK;
}

template <typename Kernel>
int allow_smem(int dev, int slot, Kernel kernel, int smem_optin) {
    std::lock_guard<std::mutex> lock(g_dev_mutex);
    if (!g_attr_set[dev][slot]) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_optin);
        if (e != cudaSuccess) {
            return set_error(CIMEKV_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
        }
        g_attr_set[dev][slot] = true;
    }
    return CIMEKV_OK;
}

// ------------------------------------------------------ table + indexing --

__device__ unsigned int g_debug_oob_count = 0;  // table-index violations seen by debug builds

constexpr float kTwo23 = 8388608.0f;       // 2^23
constexpr uint32_t kTwo23Bits = 0x4B000000u;  // bit pattern of 2^23

// Packed table layout in global memory (each part padded to 16 bytes):
//   uint32 lut_i[T]:  lo16 = bf16(I[j]),  hi16 = bf16(I[j+1])
//   uint32 lut_d[T]:  lo16 = bf16(dI[j]), hi16 = bf16(dI[j+1])
// with j+1 clamped to T-1, so entry T-1 interpolates to its own value for any a.
__host__ __device__ inline size_t fwd_table_bytes(int T) { return ((size_t)T * 4 + 15) & ~(size_t)15; }


// Low bf16 of a pair word as fp32 (a byte permute, which issues on the ALU
// pipe and leaves the FMA pipe to the interpolation arithmetic).
__device__ __forceinline__ float bf16_lo(uint32_t w) {
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, 0x1044;" : "=r"(r) : "r"(w));
    return __uint_as_float(r);
}
#if !CIMEKV_MIXED_BF16
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
#endif

// hi(w) - lo in one sm_100 mixed-precision subtract (bf16 minus fp32, rounded
// to fp32): the same value as bf16_hi(w) - lo, since bf16 -> fp32 is exact.
__device__ __forceinline__ float bf16_hi_minus(uint32_t w, float lo) {
#if CIMEKV_MIXED_BF16
    float d;
    asm("{ .reg .b16 l, h; mov.b32 {l, h}, %1; sub.rn.f32.bf16 %0, h, %2; }" : "=f"(d) : "r"(w), "f"(lo));
    return d;
#else
    return __fsub_rn(bf16_hi(w), lo);
#endif
}

// Table coordinate of one lookup: f = (fl(x - w) - dmin) * scale, each step
// rounded to fp32 (never contracted), optionally clamped to [0, T-1].
template <bool kClamp>
__device__ __forceinline__ float lut_coord(float x, float w, float dmin, float scale, float fmax_) {
    const float d = __fsub_rn(x, w);
    float f = __fmul_rn(__fsub_rn(d, dmin), scale);
    if (kClamp) f = fminf(fmaxf(f, 0.0f), fmax_);
    return f;
}

// For 0 <= f < 2^23: t = f + 2^23 rounded toward zero is 2^23 + trunc(f), so
// its bit pattern is kTwo23Bits + i0; a = f - i0 is exact.
__device__ __forceinline__ void lut_split(float f, uint32_t& bits, float& a) {
    const float t = __fadd_rz(f, kTwo23);
    bits = __float_as_uint(t);
    a = __fsub_rn(f, __fsub_rn(t, kTwo23));
}

__device__ __forceinline__ uint32_t smem_u32addr(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// ---- packed fp32x2 arithmetic (sm_100: two fp32 ops per lane per issue) ----
// The kernels pair two adjacent TOKENS (same output, input and branch), so
// every pair op is the reference's scalar op applied twice with the same IEEE
// rounding; only the issue count halves.
typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 pk2(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void unpk2(f32x2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 add2_rz(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("add.rz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
    f32x2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
    f32x2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// Constants of the index math, broadcast into both halves of a pair.
struct LutConsts {
    f32x2 dmin2, scale2, two23;
    float fmax_;
    uint32_t tab_base;
    int T;  // table entries (bounds checks of debug builds)
    // exact-formula mode: log2(e)/(2 n U_T), V_D log2(e)/(2 n U_T)
    float inv, vd;
};

// ---- exact EKV branch current (no table) ----
// I(dV)      = I_S (sp(u1)^2 - sp(u2)^2),  u1 = dV/(2nU_T), u2 = (dV - V_D)/(2nU_T)
// dI/d(dV)   = I_S 2/(2nU_T) (sp(u1) sig(u1) - sp(u2) sig(u2))
// sp = softplus, sig = logistic (the reference's _softplus/_sigmoid,
// ekv_triton.py:23-31; torch softplus on the CPU path).
//
// The kernels work in base-2 units: u' = u log2(e) (so e^-|u| = 2^-|u'|, one
// SFU op) and sp' = sp log2(e) = max(u', 0) + log2(e) log1p(t); the factors
// ln2^2 (for I) and ln2 (for dI/dV) ride on the staged per-(token, input)
// weights with I_S.  log1p(t) = 2 atanh(z), z = t / (2 + t) <= 1/3, with
// atanh(z)/z a degree-4 polynomial in z^2 fitted for minimum maximum relative
// error (iteratively reweighted least squares; 4e-9 in exact arithmetic),
// its coefficients scaled by 2 log2(e).  This keeps full relative accuracy deep
// in subthreshold (where log(1 + e^u) in fp32 rounds to 0).  The same t gives
// the logistic: sig(u) = 1/(1+t) for u >= 0, t/(1+t) otherwise.
__device__ __forceinline__ float exp2_approx(float v) {  // PTX ex2.approx.ftz.f32
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
    return r;
}

__device__ __forceinline__ void softplus_sigmoid(float u, float& sp, float* sig) {
    const float t = exp2_approx(-fabsf(u));
    const float z = __fdividef(t, 2.0f + t);
    const float z2 = z * z;
    float p = 0.4065274f;
    p = fmaf(p, z2, 0.40338615f);
    p = fmaf(p, z2, 0.5774374f);
    p = fmaf(p, z2, 0.96179163f);
    p = fmaf(p, z2, 2.88539004f);
    sp = fmaf(z, p, fmaxf(u, 0.0f));
    if (sig != nullptr) {
        const float r = __fdividef(1.0f, 1.0f + t);
        *sig = u >= 0.0f ? r : t * r;
    }
}

// c.inv = log2(e)/(2nU_T), c.vd = V_D log2(e)/(2nU_T).
__device__ __forceinline__ void ekv_exact1(float dv, const LutConsts& c, float& base, float* deriv) {
    const float u1 = __fmul_rn(dv, c.inv);
    const float u2 = __fsub_rn(u1, c.vd);
    float sp1, sp2, s1, s2;
    softplus_sigmoid(u1, sp1, deriv ? &s1 : nullptr);
    softplus_sigmoid(u2, sp2, deriv ? &s2 : nullptr);
    // I/(I_S ln2^2) and (dI/dV)/(2 I_S ln2/(2nU_T)): the constant factors are
    // folded into the per-(token, input) weights the kernels stage.
    base = sp1 * sp1 - sp2 * sp2;
    if (deriv != nullptr) *deriv = sp1 * s1 - sp2 * s2;
}

__device__ __forceinline__ f32x2 exact_fwd2(f32x2 xx, f32x2 ww, const LutConsts& c) {
    float d0, d1, b0, b1;
    unpk2(sub2(xx, ww), d0, d1);
    ekv_exact1(d0, c, b0, nullptr);
    ekv_exact1(d1, c, b1, nullptr);
    return pk2(b0, b1);
}

__device__ __forceinline__ void exact_bwd2(f32x2 xx, f32x2 ww, const LutConsts& c, f32x2& base, f32x2& deriv) {
    float d0, d1, b0, b1, g0, g1;
    unpk2(sub2(xx, ww), d0, d1);
    ekv_exact1(d0, c, b0, &g0);
    ekv_exact1(d1, c, b1, &g1);
    base = pk2(b0, b1);
    deriv = pk2(g0, g1);
}

#if CIMEKV_DEBUG_BOUNDS
// Debug builds: a table index outside [0, T) is counted and redirected to entry
// 0 instead of reading outside the staged table.
__device__ __forceinline__ void debug_check_index(uint32_t& bits, int T) {
    if (bits - kTwo23Bits >= (uint32_t)T) {
        atomicAdd(&g_debug_oob_count, 1u);
        bits = kTwo23Bits;
    }
}
#endif

// Interpolation of two pair words {v[j], v[j+1]} at fractions a (two tokens):
// v[j] + a (v[j+1] - v[j]) per half.
__device__ __forceinline__ f32x2 lerp_pair2(f32x2 a, uint32_t e0, uint32_t e1) {
    const float l0 = bf16_lo(e0), l1 = bf16_lo(e1);
#if CIMEKV_MIXED_BF16
    return fma2(a, pk2(bf16_hi_minus(e0, l0), bf16_hi_minus(e1, l1)), pk2(l0, l1));
#else
    const f32x2 q0 = pk2(l0, l1);
    return fma2(a, sub2(pk2(bf16_hi(e0), bf16_hi(e1)), q0), q0);
#endif
}

// Table coordinate of two lookups (two tokens against one threshold):
// returns the bit patterns of t = f + 2^23 (rz) per half and a = f - trunc(f).
template <bool kClamp>
__device__ __forceinline__ f32x2 lut_coord2(f32x2 xx, f32x2 ww, const LutConsts& c, uint32_t& b0, uint32_t& b1) {
    f32x2 f = mul2(sub2(sub2(xx, ww), c.dmin2), c.scale2);
    if (kClamp) {
        float f0, f1;
        unpk2(f, f0, f1);
        f = pk2(fminf(fmaxf(f0, 0.0f), c.fmax_), fminf(fmaxf(f1, 0.0f), c.fmax_));
    }
    const f32x2 t = add2_rz(f, c.two23);
    float t0, t1;
    unpk2(t, t0, t1);
    b0 = __float_as_uint(t0);
    b1 = __float_as_uint(t1);
#if CIMEKV_DEBUG_BOUNDS
    debug_check_index(b0, c.T);
    debug_check_index(b1, c.T);
#endif
    return sub2(f, sub2(t, c.two23));
}

// Forward lookup pair: interpolated I at two tokens.
template <bool kClamp>
__device__ __forceinline__ f32x2 lut_fwd2(f32x2 xx, f32x2 ww, const LutConsts& c) {
    uint32_t b0, b1;
    const f32x2 a = lut_coord2<kClamp>(xx, ww, c, b0, b1);
    const uint32_t e0 = lds32(c.tab_base + (b0 << 2));
    const uint32_t e1 = lds32(c.tab_base + (b1 << 2));
    return lerp_pair2(a, e0, e1);
}

// fp32 tile-range test: true when every cell of a tile whose x lie in
// [xmin, xmax] and thresholds in [wmin, wmax] has 0 <= f < T, i.e. the clamp is
// a no-op.  Valid because fp32 subtraction and multiplication by a positive
// constant are monotone under round-to-nearest.
__device__ __forceinline__ bool tile_in_table(float xmin, float xmax, float wmin, float wmax,
                                              bool has_nan, float dmin, float scale, int T) {
    const float flo = lut_coord<false>(xmin, wmax, dmin, scale, 0.0f);
    const float fhi = lut_coord<false>(xmax, wmin, dmin, scale, 0.0f);
    return !has_nan && flo >= 0.0f && fhi < static_cast<float>(T);
}

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, s));
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, s));
    return v;
}

// Block-wide min/max of (a_min, a_max, b_min, b_max) and OR of a NaN flag.
// `red` holds >= 8 float4 + 8 ints after it.  Contains __syncthreads().
__device__ __forceinline__ void block_range4(float4 v, bool nan, float4* red, int* red_nan,
                                             float4& out, bool& out_nan) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    v.x = warp_min(v.x);
    v.y = warp_max(v.y);
    v.z = warp_min(v.z);
    v.w = warp_max(v.w);
    const bool any_nan = __any_sync(0xffffffffu, nan);
    if (lane == 0) {
        red[warp] = v;
        red_nan[warp] = any_nan ? 1 : 0;
    }
    __syncthreads();
    float4 r = red[0];
    int n = red_nan[0];
    for (int w = 1; w < nwarps; ++w) {
        const float4 q = red[w];
        r.x = fminf(r.x, q.x);
        r.y = fmaxf(r.y, q.y);
        r.z = fminf(r.z, q.z);
        r.w = fmaxf(r.w, q.w);
        n |= red_nan[w];
    }
    out = r;
    out_nan = n != 0;
}

// -------------------------------------------------------------- packing --

__global__ void lut_pack_kernel(const uint16_t* __restrict__ ti, const uint16_t* __restrict__ td, int T,
                                uint32_t* __restrict__ lut_i, uint32_t* __restrict__ lut_d, int words) {
    for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < words; j += gridDim.x * blockDim.x) {
        if (j < T) {
            const int j1 = j + 1 < T ? j + 1 : T - 1;
            lut_i[j] = (uint32_t)ti[j] | ((uint32_t)ti[j1] << 16);
            lut_d[j] = (uint32_t)td[j] | ((uint32_t)td[j1] << 16);
        } else {
            lut_i[j] = 0u;  // alignment padding, never indexed
            lut_d[j] = 0u;
        }
    }
}

__global__ void lut_index_kernel(const float* __restrict__ delta, int n, int T, float dmin, float scale,
                                 int32_t* __restrict__ index, float* __restrict__ alpha) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    // dV is handed in directly: same coordinate as lut_coord with x = dV, w = 0
    // (fl(dV - 0) = dV).
    const float f = lut_coord<true>(delta[i], 0.0f, dmin, scale, static_cast<float>(T - 1));
    uint32_t bits;
    float a;
    lut_split(f, bits, a);
    index[i] = static_cast<int32_t>(bits - kTwo23Bits);
    alpha[i] = a;
}

// -------------------------------------------------------------- forward --
//
// CTA tile: 64 tokens x 64 outputs, 256 threads.  Warp w owns tokens
// [8w, 8w+8) of the tile; lane l owns outputs l and l+32.  The k dimension is
// streamed in chunks of 16 through shared memory (x and 1/d transposed to
// k-major so a warp reads its 8 tokens with two broadcast 128-bit loads), with
// the next chunk prefetched into registers while the current one computes.
// Persistent grid: each CTA stages the table once and walks a strided list of
// tiles.

constexpr int kFwdKkUnroll = CIMEKV_FWD_KK_UNROLL;
constexpr int kFwdThreads = 256;
constexpr int kFwdMT = 64;
constexpr int kFwdOT = 64;
#ifndef CIMEKV_FWD_KC
#define CIMEKV_FWD_KC 16  // k-chunk staged per barrier
#endif
constexpr int kFwdKC = CIMEKV_FWD_KC;
constexpr int kFwdLD = 68;  // padded row stride (floats) of the k-major tiles
constexpr int kFwdStageFloats = 4 * kFwdKC * kFwdLD;
constexpr int kFwdPerThread = kFwdMT * kFwdKC / kFwdThreads;  // 4 elements of each tile

struct FwdParams {
    const float* x;
    const float* wp;
    const float* wn;
    const uint32_t* lut;
    float* out;               // I_diff, clamped to [out_min, out_max]
    const float* r_tia;       // device scalar R_TIA (used when tia_out != nullptr)
    float* tia_out;           // optional clamp(I_diff * R_TIA, tia_lo, tia_hi)
    int M, K, O, T;
    float dmin, scale, vsat, out_min, out_max, tia_lo, tia_hi;
    float inv, vd, i_s, di_s;  // exact-formula mode
    int ksplit;  // 1, or 2: each tile's k range in two halves, raw sums added into a zeroed out
};

// torch.clamp semantics (NaN passes through).
__device__ __forceinline__ float clamp_keep_nan(float v, float lo, float hi) {
    return v < lo ? lo : (v > hi ? hi : v);
}

template <bool kClamp, bool kExact>
__device__ __forceinline__ void fwd_chunk(const float* __restrict__ xs, const float* __restrict__ is,
                                          const float* __restrict__ ps, const float* __restrict__ ns,
                                          const LutConsts& c, f32x2 (&acc)[4][2]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#ifndef CIMEKV_FWD_KK_UNROLL_EXACT
#define CIMEKV_FWD_KK_UNROLL_EXACT 1
#endif
    constexpr int kUnroll = kExact ? CIMEKV_FWD_KK_UNROLL_EXACT : kFwdKkUnroll;  // the exact-formula cell is long: less unrolling
#pragma unroll kUnroll
    for (int kk = 0; kk < kFwdKC; ++kk) {
        const float4 xa = *reinterpret_cast<const float4*>(xs + kk * kFwdLD + warp * 8);
        const float4 xb = *reinterpret_cast<const float4*>(xs + kk * kFwdLD + warp * 8 + 4);
        const float4 ia = *reinterpret_cast<const float4*>(is + kk * kFwdLD + warp * 8);
        const float4 ib = *reinterpret_cast<const float4*>(is + kk * kFwdLD + warp * 8 + 4);
        const f32x2 xx[4] = {pk2(xa.x, xa.y), pk2(xa.z, xa.w), pk2(xb.x, xb.y), pk2(xb.z, xb.w)};
        const f32x2 iv[4] = {pk2(ia.x, ia.y), pk2(ia.z, ia.w), pk2(ib.x, ib.y), pk2(ib.z, ib.w)};
        f32x2 wp[2], wn[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float p = ps[kk * kFwdLD + lane + 32 * j], n = ns[kk * kFwdLD + lane + 32 * j];
            wp[j] = pk2(p, p);
            wn[j] = pk2(n, n);
        }
#pragma unroll
        for (int ip = 0; ip < 4; ++ip) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const f32x2 vp = kExact ? exact_fwd2(xx[ip], wp[j], c) : lut_fwd2<kClamp>(xx[ip], wp[j], c);
                const f32x2 vn = kExact ? exact_fwd2(xx[ip], wn[j], c) : lut_fwd2<kClamp>(xx[ip], wn[j], c);
                acc[ip][j] = fma2(sub2(vp, vn), iv[ip], acc[ip][j]);
            }
        }
    }
}

template <bool kExact>
__global__ void __launch_bounds__(kFwdThreads, CIMEKV_FWD_MIN_BLOCKS) fwd_kernel(FwdParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int T = p.T;
    uint32_t* tab = reinterpret_cast<uint32_t*>(smem);
    float* stage = reinterpret_cast<float*>(smem + fwd_table_bytes(T));
    float* xs = stage;
    float* is = stage + kFwdKC * kFwdLD;
    float* ps = stage + 2 * kFwdKC * kFwdLD;
    float* ns = stage + 3 * kFwdKC * kFwdLD;
    float4* red = reinterpret_cast<float4*>(stage + kFwdStageFloats);
    int* red_nan = reinterpret_cast<int*>(red + 8);

    {   // stage the table once per CTA
        const uint4* src = reinterpret_cast<const uint4*>(p.lut);
        uint4* dst = reinterpret_cast<uint4*>(tab);
        const int n16 = static_cast<int>(fwd_table_bytes(T) / 16);
        for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
    }
    // Biased shared address: tab_base + (bits << 2) = &tab[bits - kTwo23Bits].
    LutConsts lc;
    lc.tab_base = smem_u32addr(tab) - (kTwo23Bits << 2);
    lc.fmax_ = static_cast<float>(T - 1);
    lc.T = T;
    lc.dmin2 = pk2(p.dmin, p.dmin);
    lc.scale2 = pk2(p.scale, p.scale);
    lc.two23 = pk2(kTwo23, kTwo23);
    lc.inv = p.inv;
    lc.vd = p.vd;
    const float r_tia = p.tia_out != nullptr ? __ldg(p.r_tia) : 0.0f;
    const float inv_vsat = 1.0f / p.vsat;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tiles_m = (p.M + kFwdMT - 1) / kFwdMT;
    const int tiles_o = (p.O + kFwdOT - 1) / kFwdOT;
    const int ntiles = tiles_m * tiles_o;
    const int nchunks = (p.K + kFwdKC - 1) / kFwdKC;

    // Work item = (tile, part of the k range); with ksplit == 2 the two halves of
    // a tile add their raw sums into the zeroed output (two adds onto 0.0f give
    // a + b in either order: deterministic) and fwd_split_epilogue_kernel clamps.
    const int nitems = ntiles * p.ksplit;
    for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
        const int tile = item % ntiles, part = item / ntiles;
        const int c_lo = (int)((int64_t)part * nchunks / p.ksplit);
        const int c_hi = (int)((int64_t)(part + 1) * nchunks / p.ksplit);
        const int m0 = (tile / tiles_o) * kFwdMT;
        const int o0 = (tile % tiles_o) * kFwdOT;
        f32x2 acc[4][2];  // [token pair][output]
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = pk2(0.0f, 0.0f);

        // Register prefetch of one chunk: element e = tid + 256 r of a 64x16 tile
        // is (row e>>4, col e&15); rows are tokens for x, outputs for w.
        float rx[kFwdPerThread], rp[kFwdPerThread], rn[kFwdPerThread];
        auto load_chunk = [&](int k0) {
#pragma unroll
            for (int r = 0; r < kFwdPerThread; ++r) {
                const int e = threadIdx.x + kFwdThreads * r;
                const int row = e / kFwdKC, k = k0 + (e % kFwdKC);
                const bool kin = k < p.K;
                const int gm = m0 + row, go = o0 + row;
                rx[r] = (kin && gm < p.M) ? __ldg(p.x + (int64_t)gm * p.K + k) : 0.0f;
                rp[r] = (kin && go < p.O) ? __ldg(p.wp + (int64_t)go * p.K + k) : 0.0f;
                rn[r] = (kin && go < p.O) ? __ldg(p.wn + (int64_t)go * p.K + k) : 0.0f;
            }
        };
        if (c_hi > c_lo) load_chunk(c_lo * kFwdKC);
        for (int c = c_lo; c < c_hi; ++c) {
            __syncthreads();  // previous chunk's readers are done with the stage
            float4 rng = make_float4(INFINITY, -INFINITY, INFINITY, -INFINITY);
            bool nan = false;
#pragma unroll
            for (int r = 0; r < kFwdPerThread; ++r) {
                const int e = threadIdx.x + kFwdThreads * r;
                const int row = e / kFwdKC, kk = e % kFwdKC;
                const int k = c * kFwdKC + kk;
                const bool valid = k < p.K && m0 + row < p.M;
                const float xv = rx[r];
                xs[kk * kFwdLD + row] = xv;
                // 1/(1 + x/V_sat) to within 2 ulp (the reference divides; the difference is far
                // below the fp32 summation error of the K-term sum)
                // (exact mode: times I_S, the factor the cell evaluation leaves out)
                is[kk * kFwdLD + row] = valid ? __fdividef(kExact ? p.i_s : 1.0f, fmaf(xv, inv_vsat, 1.0f)) : 0.0f;
                ps[kk * kFwdLD + row] = rp[r];
                ns[kk * kFwdLD + row] = rn[r];
                rng.x = fminf(rng.x, xv);
                rng.y = fmaxf(rng.y, xv);
                rng.z = fminf(rng.z, fminf(rp[r], rn[r]));
                rng.w = fmaxf(rng.w, fmaxf(rp[r], rn[r]));
                nan |= (xv != xv) | (rp[r] != rp[r]) | (rn[r] != rn[r]);
            }
            float4 tr;
            bool tnan;
            block_range4(rng, nan, red, red_nan, tr, tnan);  // includes the barrier
            if (c + 1 < c_hi) load_chunk((c + 1) * kFwdKC);
            if (kExact) {
                fwd_chunk<false, true>(xs, is, ps, ns, lc, acc);
            } else if (tile_in_table(tr.x, tr.y, tr.z, tr.w, tnan, p.dmin, p.scale, T)) {
                fwd_chunk<false, false>(xs, is, ps, ns, lc, acc);
            } else {
                fwd_chunk<true, false>(xs, is, ps, ns, lc, acc);
            }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int m = m0 + warp * 8 + i;
            if (m >= p.M) continue;
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int o = o0 + lane + 32 * j;
                float v0, v1;
                unpk2(acc[i >> 1][j], v0, v1);
                if (o < p.O && p.ksplit > 1) {
                    atomicAdd(p.out + (int64_t)m * p.O + o, (i & 1) ? v1 : v0);
                } else if (o < p.O) {
                    const float id = fminf(fmaxf((i & 1) ? v1 : v0, p.out_min), p.out_max);
                    p.out[(int64_t)m * p.O + o] = id;
                    if (p.tia_out != nullptr)  // fused TIA: the reference's `I_diff * r_tia` then clamp
                        p.tia_out[(int64_t)m * p.O + o] = clamp_keep_nan(__fmul_rn(id, r_tia), p.tia_lo, p.tia_hi);
                }
            }
        }
    }
}

// Epilogue of a k-split forward: the clamp of I_diff and the fused TIA output,
// the same operations as the forward's own epilogue.
__global__ void fwd_split_epilogue_kernel(float* __restrict__ out, float* __restrict__ tia_out,
                                          const float* __restrict__ r_tia, int64_t n, float out_min,
                                          float out_max, float tia_lo, float tia_hi) {
    const float r = tia_out != nullptr ? __ldg(r_tia) : 0.0f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float id = fminf(fmaxf(out[i], out_min), out_max);
        out[i] = id;
        if (tia_out != nullptr) tia_out[i] = clamp_keep_nan(__fmul_rn(id, r), tia_lo, tia_hi);
    }
}

size_t fwd_smem_bytes(int T) {
    return fwd_table_bytes(T) + (size_t)kFwdStageFloats * 4 + 8 * sizeof(float4) + 8 * sizeof(int);
}

// ------------------------------------------------------------- backward --
//
// CTA = 4 inputs (k0..k0+3) x one token split; 256 threads.  For each 64-token
// tile of the split, warp w owns tokens [8w, 8w+8) (4 adjacent pairs) and lane
// l walks outputs o = 32c + l.  Per thread and chunk c: 8 tokens x 4 inputs =
// 32 cells.
//   * the chunk's thresholds (32 outputs x 4 inputs x 2 branches) are staged
//     once per CTA in a double-buffered shared tile, prefetched a chunk ahead;
//   * the table is two 32-bit pair tables (I and dI/dV), the second at the
//     compile-time offset kStride words, so one index feeds both loads;
//   * dX[m,k] accumulates in registers over all o of the lane, then one
//     32-lane transpose-reduce per tile leaves lane l holding dX of
//     (token l/4, input l%4);
//   * dVth partials (sum over the thread's 8 tokens) are summed over the 8
//     warps through shared memory into a per-CTA accumulator dW[2][O][4]
//     that lives for the whole split; at the end it goes to the workspace
//     slice of this split, and bwd_reduce_kernel sums the splits in a fixed
//     order (deterministic).

constexpr int kBwdThreads = 256;
constexpr int kBwdMT = 64;
constexpr int kBwdKT = 4;
constexpr int kBwdTok = 8;  // tokens per thread
// Row stride (floats) of the staged chunk thresholds [32 outputs][8 slots]: 12
// puts the 128-bit reads of 8 consecutive lanes on 32 distinct banks.
constexpr int kWsLd = 12;
// Where thread t's threshold fetch (output t/8, slot t%8) lands in a buffer.
__device__ __forceinline__ int ws_slot() { return (threadIdx.x >> 3) * kWsLd + (threadIdx.x & 7); }

struct BwdParams {
    const float* x;
    const float* wp;
    const float* wn;
    const float* g;
    const uint32_t* lut_i;   // [T] {I[j], I[j+1]}
    const uint32_t* lut_d;   // [T] {dI[j], dI[j+1]}
    float* grad_x;
    float* part;  // [nsplit][2][O][K]
    int M, K, O, T;
    int tiles_m, nsplit;
    float dmin, scale, vsat;
    float inv, vd, i_s, di_s;  // exact-formula mode (kStride == 0)
    int dw_global;  // 1: accumulate dVth directly in this CTA's workspace slice (shared memory too small)
};

// Table stride (words) of the backward: the smallest supported size >= T.
int bwd_stride(int T) { return T <= 4096 ? 4096 : (T <= 8192 ? 8192 : 16384); }

size_t bwd_smem_bytes_stride(int stride, int O, bool dw_global = false) {
    const int opad = (O + 31) / 32 * 32;
    return (size_t)8 * stride                        // I and dI/dV pair tables (none in exact mode)
           + (dw_global ? 0 : (size_t)2 * opad * kBwdKT * 4)  // dW accumulator
           + (size_t)3 * kBwdMT * kBwdKT * 4         // x, 1/d, -1/(vsat d^2): k-major [4][64]
           + (size_t)2 * 32 * kWsLd * 4              // double-buffered chunk thresholds
           + (size_t)2 * 8 * 8 * 32 * 4              // double-buffered cross-warp dW exchange
           + 8 * sizeof(float4) + 8 * sizeof(int);   // range reduction
}

template <int kOff>
__device__ __forceinline__ uint32_t lds32_off(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.b32 %0, [%1+%2];" : "=r"(v) : "r"(addr), "n"(kOff));
    return v;
}

// Backward lookup pair: interpolated (I, dI/dV) at two tokens.
template <bool kClamp, int kStride>
__device__ __forceinline__ void lut_bwd2(f32x2 xx, f32x2 ww, const LutConsts& c, f32x2& base, f32x2& deriv) {
    uint32_t b0, b1;
    const f32x2 a = lut_coord2<kClamp>(xx, ww, c, b0, b1);
    const uint32_t a0 = c.tab_base + (b0 << 2), a1 = c.tab_base + (b1 << 2);
    const uint32_t i0 = lds32(a0), i1 = lds32(a1);
    const uint32_t d0 = lds32_off<4 * kStride>(a0), d1 = lds32_off<4 * kStride>(a1);
    base = lerp_pair2(a, i0, i1);
    deriv = lerp_pair2(a, d0, d1);
}

// One chunk of 32 outputs for this thread's 8 tokens (4 pairs) x 4 inputs.
// Xk/Ik/Nk: k-major [4][64] tiles of x, 1/d and -1/(v_sat d^2); ws: this
// chunk's thresholds [32 outputs][p k0..3, n k0..3].
template <bool kClamp, int kStride>
__device__ __forceinline__ void bwd_chunk(const float* __restrict__ Xk, const float* __restrict__ Ik,
                                          const float* __restrict__ Nk, const float* __restrict__ ws,
                                          const float (&g)[kBwdTok], const LutConsts& c,
                                          f32x2 (&dx)[4][kBwdKT], f32x2 (&ap)[kBwdKT], f32x2 (&an)[kBwdKT]) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const f32x2 G[4] = {pk2(g[0], g[1]), pk2(g[2], g[3]), pk2(g[4], g[5]), pk2(g[6], g[7])};
    const float4 wp4 = *reinterpret_cast<const float4*>(ws + lane * kWsLd);
    const float4 wn4 = *reinterpret_cast<const float4*>(ws + lane * kWsLd + 4);
    const float wp[4] = {wp4.x, wp4.y, wp4.z, wp4.w};
    const float wn[4] = {wn4.x, wn4.y, wn4.z, wn4.w};
#pragma unroll
    for (int kk = 0; kk < kBwdKT; ++kk) {
        const float* xr = Xk + kk * kBwdMT + warp * kBwdTok;
        const float* ir = Ik + kk * kBwdMT + warp * kBwdTok;
        const float* nr = Nk + kk * kBwdMT + warp * kBwdTok;
        const float4 xa = *reinterpret_cast<const float4*>(xr), xb = *reinterpret_cast<const float4*>(xr + 4);
        const float4 ia = *reinterpret_cast<const float4*>(ir), ib = *reinterpret_cast<const float4*>(ir + 4);
        const float4 na = *reinterpret_cast<const float4*>(nr), nb4 = *reinterpret_cast<const float4*>(nr + 4);
        const f32x2 X[4] = {pk2(xa.x, xa.y), pk2(xa.z, xa.w), pk2(xb.x, xb.y), pk2(xb.z, xb.w)};
        const f32x2 IV[4] = {pk2(ia.x, ia.y), pk2(ia.z, ia.w), pk2(ib.x, ib.y), pk2(ib.z, ib.w)};
        const f32x2 NT[4] = {pk2(na.x, na.y), pk2(na.z, na.w), pk2(nb4.x, nb4.y), pk2(nb4.z, nb4.w)};
        const f32x2 WP = pk2(wp[kk], wp[kk]), WN = pk2(wn[kk], wn[kk]);
#pragma unroll
        for (int ip = 0; ip < 4; ++ip) {
            f32x2 pb, pd, nb, nd;
            if (kStride == 0) {  // exact formula
                exact_bwd2(X[ip], WP, c, pb, pd);
                exact_bwd2(X[ip], WN, c, nb, nd);
            } else {
                lut_bwd2<kClamp, kStride>(X[ip], WP, c, pb, pd);
                lut_bwd2<kClamp, kStride>(X[ip], WN, c, nb, nd);
            }
            // d(I_diff/d)/dx = (dp - dn)/d - (bp - bn)/(v_sat d^2)
            const f32x2 e = fma2(sub2(pb, nb), NT[ip], mul2(sub2(pd, nd), IV[ip]));
            dx[ip][kk] = fma2(G[ip], e, dx[ip][kk]);
            const f32x2 gi = mul2(G[ip], IV[ip]);
            ap[kk] = fma2(gi, pd, ap[kk]);
            an[kk] = fma2(gi, nd, an[kk]);
        }
    }
}

template <int kStride>
__global__ void __launch_bounds__(kBwdThreads, CIMEKV_BWD_MIN_BLOCKS) bwd_kernel(BwdParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int T = p.T;
    const int opad = (p.O + 31) / 32 * 32;
    uint32_t* tab = reinterpret_cast<uint32_t*>(smem);                // [kStride] I pairs, [kStride] dI pairs
    float* dWs = reinterpret_cast<float*>(smem + 8 * kStride);       // [2][opad][4] unless dw_global
    float* Xk = dWs + (p.dw_global ? 0 : 2 * opad * kBwdKT);  // [4][64] x
    float* Ik = Xk + kBwdKT * kBwdMT;      // [4][64] 1/d
    float* Nk = Ik + kBwdKT * kBwdMT;      // [4][64] -1/(v_sat d^2)
    float* wsm = Nk + kBwdKT * kBwdMT;     // [2][32 outputs][kWsLd]
    float* xch = wsm + 2 * 32 * kWsLd;     // [2][8 warps][8 vals][32 lanes]
    float4* red = reinterpret_cast<float4*>(xch + 2 * 8 * 8 * 32);
    int* red_nan = reinterpret_cast<int*>(red + 8);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int k0 = blockIdx.x * kBwdKT;
    const int split = blockIdx.y;
    const int tile_lo = (int)((int64_t)split * p.tiles_m / p.nsplit);
    const int tile_hi = (int)((int64_t)(split + 1) * p.tiles_m / p.nsplit);
    const int nchunks = (p.O + 31) / 32;

    // Threshold staging: thread t fetches (output t/8 of the chunk, slot t%8),
    // slot = branch*4 + input.
    const int w_o = threadIdx.x >> 3, w_slot = threadIdx.x & 7;
    const int w_k = k0 + (w_slot & 3);
    const float* w_src = (w_slot < 4) ? p.wp : p.wn;
    auto fetch_w = [&](int c) -> float {
        const int o = c * 32 + w_o;
        return (o < p.O && w_k < p.K) ? __ldg(w_src + (int64_t)o * p.K + w_k) : 0.0f;
    };

    {
        for (int i = threadIdx.x; i < T; i += blockDim.x) {
            tab[i] = p.lut_i[i];
            tab[kStride + i] = p.lut_d[i];
        }
        if (!p.dw_global) {
            for (int i = threadIdx.x; i < 2 * opad * kBwdKT; i += blockDim.x) dWs[i] = 0.0f;
        } else if (p.part != nullptr) {  // this CTA's slice of the workspace is its accumulator
            for (int e = threadIdx.x; e < 2 * p.O * kBwdKT; e += blockDim.x) {
                const int br = e / (p.O * kBwdKT), rem = e - br * p.O * kBwdKT;
                const int o = rem >> 2, kk = rem & 3;
                if (k0 + kk < p.K) p.part[(((int64_t)split * 2 + br) * p.O + o) * p.K + k0 + kk] = 0.0f;
            }
        }
        if (nchunks > 0) wsm[ws_slot()] = fetch_w(0);  // chunk 0 into buffer 0
    }
    LutConsts lc;
    lc.tab_base = smem_u32addr(tab) - (kTwo23Bits << 2);
    lc.fmax_ = static_cast<float>(T - 1);
    lc.T = T;
    lc.dmin2 = pk2(p.dmin, p.dmin);
    lc.scale2 = pk2(p.scale, p.scale);
    lc.two23 = pk2(kTwo23, kTwo23);
    lc.inv = p.inv;
    lc.vd = p.vd;

    // Threshold range of this CTA's inputs over all outputs (pads count as 0).
    float4 wr;
    bool wnan;
    {
        float4 v = make_float4(INFINITY, -INFINITY, INFINITY, -INFINITY);
        bool nan = false;
        for (int e = threadIdx.x; e < opad * kBwdKT; e += blockDim.x) {
            const int o = e >> 2, k = k0 + (e & 3);
            const bool valid = o < p.O && k < p.K;
            const float a = valid ? __ldg(p.wp + (int64_t)o * p.K + k) : 0.0f;
            const float b = valid ? __ldg(p.wn + (int64_t)o * p.K + k) : 0.0f;
            v.z = fminf(v.z, fminf(a, b));
            v.w = fmaxf(v.w, fmaxf(a, b));
            nan |= (a != a) | (b != b);
        }
        block_range4(v, nan, red, red_nan, wr, wnan);  // barrier: table, dWs, wsm[0] visible
    }

    int buf = 0;  // parity of the chunk-sized double buffers (thresholds, exchange)
    for (int tile = tile_lo; tile < tile_hi; ++tile) {
        const int m0 = tile * kBwdMT;
        __syncthreads();  // previous tile's readers of Xk/Ik/Nk and red are done
        float xval;
        {
            const int t = threadIdx.x >> 2, kk = threadIdx.x & 3;
            const int m = m0 + t, k = k0 + kk;
            const bool valid = m < p.M && k < p.K;
            xval = valid ? __ldg(p.x + (int64_t)m * p.K + k) : 0.0f;
            const float d = __fadd_rn(1.0f, __fdiv_rn(xval, p.vsat));
            Xk[kk * kBwdMT + t] = xval;
            // exact mode (kStride == 0): times the constant factors of dI/dV and I
            // that the cell evaluation leaves out
            const float fi = kStride == 0 ? p.di_s : 1.0f, fn = kStride == 0 ? p.i_s : 1.0f;
            Ik[kk * kBwdMT + t] = valid ? __fdiv_rn(fi, d) : 0.0f;
            Nk[kk * kBwdMT + t] = valid ? -__fdiv_rn(fn, __fmul_rn(__fmul_rn(p.vsat, d), d)) : 0.0f;
        }
        float4 xr;
        bool xnan;
        block_range4(make_float4(xval, xval, INFINITY, -INFINITY), xval != xval, red, red_nan, xr, xnan);
        const bool fast = kStride == 0 || tile_in_table(xr.x, xr.y, wr.z, wr.w, xnan || wnan, p.dmin, p.scale, T);

        f32x2 dx2[4][kBwdKT];  // [token pair][input]
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int kk = 0; kk < kBwdKT; ++kk) dx2[i][kk] = pk2(0.0f, 0.0f);

        // Register prefetch of g (8 tokens of this warp, output of this lane).
        float gn[kBwdTok];
        auto load_g = [&](int c) {
            if (m0 + kBwdMT <= p.M && (c + 1) * 32 <= p.O) {
                // interior chunk: no bounds tests, one base pointer
                const float* src = p.g + (int64_t)(m0 + warp * kBwdTok) * p.O + c * 32 + lane;
#pragma unroll
                for (int i = 0; i < kBwdTok; ++i) gn[i] = __ldg(src + (int64_t)i * p.O);
            } else {
                const int o = c * 32 + lane;
                const bool oin = o < p.O;
#pragma unroll
                for (int i = 0; i < kBwdTok; ++i) {
                    const int m = m0 + warp * kBwdTok + i;
                    gn[i] = (oin && m < p.M) ? __ldg(p.g + (int64_t)m * p.O + o) : 0.0f;
                }
            }
        };
        if (nchunks > 0) load_g(0);
        for (int c = 0; c < nchunks; ++c) {
            float g[kBwdTok];
#pragma unroll
            for (int i = 0; i < kBwdTok; ++i) g[i] = gn[i];
            if (c + 1 < nchunks) load_g(c + 1);
            // next chunk's thresholds (wrapping to chunk 0 for the next tile)
            const float wnext = fetch_w(c + 1 < nchunks ? c + 1 : 0);
            const float* ws = wsm + buf * (32 * kWsLd);
            f32x2 ap2[kBwdKT], an2[kBwdKT];
#pragma unroll
            for (int kk = 0; kk < kBwdKT; ++kk) ap2[kk] = an2[kk] = pk2(0.0f, 0.0f);
            if (fast) {
                bwd_chunk<false, kStride>(Xk, Ik, Nk, ws, g, lc, dx2, ap2, an2);
            } else {
                bwd_chunk<true, kStride>(Xk, Ik, Nk, ws, g, lc, dx2, ap2, an2);
            }
            wsm[(buf ^ 1) * (32 * kWsLd) + ws_slot()] = wnext;
            // Cross-warp sum of the dVth partials, accumulated into dWs.
            float* xb = xch + buf * (8 * 8 * 32);
#pragma unroll
            for (int kk = 0; kk < kBwdKT; ++kk) {
                float a0, a1, b0, b1;
                unpk2(ap2[kk], a0, a1);
                unpk2(an2[kk], b0, b1);
                xb[(warp * 8 + kk) * 32 + lane] = a0 + a1;
                xb[(warp * 8 + 4 + kk) * 32 + lane] = b0 + b1;
            }
            __syncthreads();
            {
                const int v = threadIdx.x >> 5;  // value slot 0..7 (p k0..3, n k0..3)
                float s = 0.0f;
#pragma unroll
                for (int w = 0; w < 8; ++w) s += xb[(w * 8 + v) * 32 + lane];
                const int o = c * 32 + lane;
                if (!p.dw_global) {
                    dWs[((v >> 2) * opad + o) * kBwdKT + (v & 3)] += s;
                } else if (p.part != nullptr && o < p.O && k0 + (v & 3) < p.K) {
                    // only this thread ever touches this element of the CTA's slice
                    p.part[(((int64_t)split * 2 + (v >> 2)) * p.O + o) * p.K + k0 + (v & 3)] += s;
                }
            }
            buf ^= 1;
        }
        float dx[kBwdTok * kBwdKT];  // element (token i, input kk) at i * 4 + kk
#pragma unroll
        for (int ip = 0; ip < 4; ++ip)
#pragma unroll
            for (int kk = 0; kk < kBwdKT; ++kk)
                unpk2(dx2[ip][kk], dx[(2 * ip) * kBwdKT + kk], dx[(2 * ip + 1) * kBwdKT + kk]);
        // 32-lane transpose-reduce of dx: afterwards lane l holds the full sum
        // of element l = (token l/4, input l%4).
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
        if (p.grad_x != nullptr) {
            const int m = m0 + warp * kBwdTok + (lane >> 2), k = k0 + (lane & 3);
            if (m < p.M && k < p.K) p.grad_x[(int64_t)m * p.K + k] = dx[0];
        }
    }
    __syncthreads();
    if (p.part != nullptr && !p.dw_global) {
        for (int e = threadIdx.x; e < 2 * p.O * kBwdKT; e += blockDim.x) {
            const int br = e / (p.O * kBwdKT);
            const int rem = e - br * p.O * kBwdKT;
            const int o = rem >> 2, kk = rem & 3;
            if (k0 + kk < p.K) {
                p.part[(((int64_t)split * 2 + br) * p.O + o) * p.K + k0 + kk] = dWs[(br * opad + o) * kBwdKT + kk];
            }
        }
    }
}

// grad_wpos = -sum_s part[s][0], grad_wneg = +sum_s part[s][1], fixed order.
__global__ void bwd_reduce_kernel(const float* __restrict__ part, int nsplit, int64_t n,
                                  float* __restrict__ gwp, float* __restrict__ gwn) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float sp = 0.0f, sn = 0.0f;
        for (int s = 0; s < nsplit; ++s) {
            sp += part[((int64_t)s * 2 + 0) * n + i];
            sn += part[((int64_t)s * 2 + 1) * n + i];
        }
        gwp[i] = -sp;
        gwn[i] = sn;
    }
}

__global__ void fill_zero_kernel(float* __restrict__ p, int64_t n) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        p[i] = 0.0f;
}

// ---------------------------------------------------------- TIA stage --
//
// Backward of out = clamp(I_diff * R_TIA, lo, hi) (reference cim.py:192-193,
// differentiated by autograd there): grad_I_diff = [lo <= I_diff*R <= hi] * g * R
// and dL/dR = sum [..] * g * I_diff.  One pass over [M,O]; the sum goes through
// fixed per-block partials and a one-block reduction (deterministic).

constexpr int kTiaBlocks = 592;

__global__ void __launch_bounds__(256) tia_bwd_kernel(const float* __restrict__ g, const float* __restrict__ idiff,
                                                      const float* __restrict__ r_ptr, int64_t n, float lo, float hi,
                                                      float* __restrict__ g_idiff, float* __restrict__ partial) {
    const float r = __ldg(r_ptr);
    float acc = 0.0f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float id = idiff[i], gv = g[i];
        const float v = __fmul_rn(id, r);
        const bool pass = (v >= lo) && (v <= hi);
        const float gm = pass ? gv : 0.0f;
        g_idiff[i] = __fmul_rn(gm, r);
        acc = fmaf(gm, id, acc);
    }
    __shared__ float red[8];
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
        partial[blockIdx.x] = t;
    }
}

__global__ void sum_partials_kernel(const float* __restrict__ partial, int n, float* __restrict__ out) {
    __shared__ float red[256];
    float t = 0.0f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) t += partial[i];
    red[threadIdx.x] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
        float u = 0.0f;
        for (int i = 0; i < (int)blockDim.x; ++i) u += red[i];
        out[0] = u;
    }
}

#include "bwd_cluster.cuh"

// Token splits of the backward: enough CTAs to fill the GPU in whole waves.
struct BwdPlan {
    int kblocks, tiles_m, nsplit;
    size_t smem, workspace;
    int dw_global;
};

// stride: table stride of the kernel instance (0 = exact formula, no table);
// negative selects the LUT stride for T.
int plan_backward(int M, int K, int O, int T, BwdPlan* plan, int stride = -1) {
    int dev, sms, optin;
    int rc = current_device(&dev);
    if (rc) return rc;
    if ((rc = device_limits(dev, &sms, &optin))) return rc;
    plan->kblocks = (K + kBwdKT - 1) / kBwdKT;
    plan->tiles_m = (M + kBwdMT - 1) / kBwdMT;
    const int st = stride < 0 ? bwd_stride(T) : stride;
    plan->smem = bwd_smem_bytes_stride(st, O);
    plan->dw_global = 0;
    const size_t per_sm_smem = 228 * 1024;
    const size_t smem_global = bwd_smem_bytes_stride(st, O, true);
    if (plan->smem > (size_t)optin ||  // large tables with many outputs, or
        (CIMEKV_BWD_DW_FOR_OCCUPANCY && 2 * (plan->smem + 1024) > per_sm_smem &&
         2 * (smem_global + 1024) <= per_sm_smem)) {  // a second resident CTA per SM
        plan->smem = smem_global;  // dVth accumulator in the workspace
        plan->dw_global = 1;
    }
    if (plan->smem > (size_t)optin) {
        return set_error(CIMEKV_ELUT_TOO_LARGE,
                         "backward needs %zu B of shared memory (LUT size %d, out_features %d); device allows %d",
                         plan->smem, T, O, optin);
    }
    // Resident CTAs per SM: 2 by registers, fewer if shared memory is short.
    const size_t per_sm = 228 * 1024;
    int resident = (int)(per_sm / (plan->smem + 1024));
    if (resident > CIMEKV_BWD_MIN_BLOCKS) resident = CIMEKV_BWD_MIN_BLOCKS;
    if (resident < 1) resident = 1;
    const int slots = sms * resident;
    int best = 1;
    double best_cost = 1e30;
    const int max_split = plan->tiles_m < 64 ? (plan->tiles_m > 0 ? plan->tiles_m : 1) : 64;
    for (int s = 1; s <= max_split; ++s) {
        const long total = (long)plan->kblocks * s;
        const long waves = (total + slots - 1) / slots;
        // time ~ waves * (tiles per split); small penalty per split for the
        // workspace traffic of the reduction.
        const double tiles_per_split = (double)((plan->tiles_m + s - 1) / s);
        const double cost = (double)waves * tiles_per_split * (double)O + 4.0 * s * (double)O / 64.0;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = s;
        }
    }
    plan->nsplit = best;
    plan->workspace = (size_t)best * 2 * (size_t)O * (size_t)K * sizeof(float);
    return CIMEKV_OK;
}

// Plan of the clustered backward (bwd_cluster.cuh).  *ok = false when it does
// not apply; the caller then runs bwd_kernel.  It applies from
// cluster_min_outputs(T) up to kCluMaxOutputs outputs, when tables + g tile fit
// shared memory.  Measured on B200 at 32k tokens against the unclustered
// kernel: 384 outputs T=4096 28.0-28.6 vs 29.2 ms, 384 outputs T=8192 28.3-29.0
// vs 32.7 ms, 256 outputs T=8192 14.0-14.2 vs 14.8 ms (two columns per warp),
// 768..3072 outputs 3-14 % faster; smaller layers are not measured and keep
// the unclustered kernel.
struct Bwd2Plan {
    int kt, wpk, cpw, ncl, opad, tm, kgroups, tiles_m, nsplit, items, grid, sort_n, band;
    size_t smem, co_off, cr_off, part_off, workspace;
};

size_t align256(size_t n) { return (n + 255) & ~(size_t)255; }

// CIMEKV_BWD_CLUSTER=0 in the environment selects the unclustered kernel.
bool cluster_enabled() {
    static const bool on = [] {
        const char* e = getenv("CIMEKV_BWD_CLUSTER");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Smallest layer (outputs) the clustered kernel takes: kCluMinOutputs for
// tables up to 4096 entries, kCluMinOutputsLargeT above (wider threshold
// windows, more conflicts for the unclustered kernel).  CIMEKV_BWD_CLUSTER_MIN=<n>
// in the environment overrides both (experiments).
int cluster_min_outputs(int T) {
    static const int v = [] {
        const char* e = getenv("CIMEKV_BWD_CLUSTER_MIN");
        return e ? atoi(e) : -1;
    }();
    if (v >= 0) return v;
    return T > 4096 ? kCluMinOutputsLargeT : kCluMinOutputs;
}

int plan_backward2(int M, int K, int O, int T, Bwd2Plan* pl, bool* ok) {
    *ok = false;
    if (!cluster_enabled() || O < cluster_min_outputs(T) || O > kCluMaxOutputs || M <= 0 || K <= 0) return CIMEKV_OK;
    int dev, sms, optin;
    int rc = current_device(&dev);
    if (rc || (rc = device_limits(dev, &sms, &optin))) return rc;
    const int stride = bwd_stride(T);
    pl->ncl = (O + 31) / 32;
    pl->opad = pl->ncl * 32;
    int kmax = 1;
    while (kmax < K && kmax < kB2MaxKT) kmax <<= 1;
    // Largest column group whose clusters fit kB2UMax per warp: kt <= 16 columns
    // share the 16 warps (wpk warps per column); kt = 32 gives each warp two
    // whole columns (layers of up to 12 clusters, i.e. 384 outputs).
    for (pl->kt = kmax; pl->kt >= 1; pl->kt >>= 1) {
        if (pl->kt > kB2Warps) {
            pl->cpw = pl->kt / kB2Warps;
            pl->wpk = 1;
        } else {
            if (kB2Warps % pl->kt) continue;
            pl->cpw = 1;
            pl->wpk = kB2Warps / pl->kt;
        }
        if ((pl->ncl + pl->wpk - 1) / pl->wpk * pl->cpw <= kB2UMax) break;
    }
    if (pl->kt < 1) return CIMEKV_OK;
    pl->tm = 8;
    pl->smem = bwd2_smem_bytes(stride, 8, pl->opad, pl->kt, pl->cpw);
    if (pl->smem > (size_t)optin) {
        pl->tm = 4;
        pl->smem = bwd2_smem_bytes(stride, 4, pl->opad, pl->kt, pl->cpw);
    }
    if (pl->smem > (size_t)optin) return CIMEKV_OK;
    pl->kgroups = (K + pl->kt - 1) / pl->kt;
    pl->tiles_m = (M + pl->tm - 1) / pl->tm;
    // Token splits: whole waves of work items over the SMs; a small charge per
    // split for the workspace the reduction writes and reads.
    int best = 1;
    double best_cost = 1e300;
    const int max_split = pl->tiles_m < 512 ? pl->tiles_m : 512;
    for (int sp = 1; sp <= max_split; ++sp) {
        const long items = (long)pl->kgroups * sp;
        const long waves = (items + sms - 1) / sms;
        const double cost = (double)waves * (double)((pl->tiles_m + sp - 1) / sp) + 0.002 * sp * pl->tiles_m;
        if (cost < best_cost - 1e-9) {
            best_cost = cost;
            best = sp;
        }
    }
    pl->nsplit = best;
    pl->items = pl->kgroups * best;
    pl->grid = pl->items < sms ? pl->items : sms;
    pl->sort_n = 32;
    while (pl->sort_n < O) pl->sort_n <<= 1;
    int nb = (int)std::lround(std::sqrt((double)pl->ncl));
    if (nb < 1) nb = 1;
    pl->band = (pl->ncl + nb - 1) / nb * 32;
    pl->co_off = align256((size_t)K * pl->opad * sizeof(float2));
    pl->cr_off = pl->co_off + align256((size_t)K * pl->opad * sizeof(int));
    pl->part_off = pl->cr_off + align256((size_t)K * sizeof(float4));
    pl->workspace = pl->part_off + (size_t)best * 2 * (size_t)O * (size_t)K * sizeof(float);
    *ok = true;
    return CIMEKV_OK;
}

template <int kStride>
int launch_backward2_stride(const Bwd2Plan& pl, int dev, int optin, const float* x, const float* wpos,
                            const float* wneg, const float* grad_out, const void* lut, int M, int K, int O, int T,
                            float dmin, float scale, float vsat, float* grad_x, bool want_w, void* workspace,
                            cudaStream_t s) {
    const int slot = 8 + 2 * (kStride == 4096 ? 0 : (kStride == 8192 ? 1 : 2)) + (pl.tm == 4 ? 1 : 0);
    int rc = pl.tm == 8 ? allow_smem(dev, slot, bwd2_kernel<kStride, 8>, optin)
                        : allow_smem(dev, slot, bwd2_kernel<kStride, 4>, optin);
    if (rc) return rc;
    unsigned char* ws = static_cast<unsigned char*>(workspace);
    Bwd2Params p;
    p.x = x;
    p.g = grad_out;
    p.cw = reinterpret_cast<const float2*>(ws);
    p.co = reinterpret_cast<const int*>(ws + pl.co_off);
    p.crange = reinterpret_cast<const float4*>(ws + pl.cr_off);
    p.lut_i = static_cast<const uint32_t*>(lut);
    p.lut_d = p.lut_i + fwd_table_bytes(T) / 4;
    p.grad_x = grad_x;
    p.part = want_w ? reinterpret_cast<float*>(ws + pl.part_off) : nullptr;
    p.M = M;
    p.K = K;
    p.O = O;
    p.opad = pl.opad;
    p.T = T;
    p.kt = pl.kt;
    p.wpk = pl.wpk;
    p.cpw = pl.cpw;
    p.ncl = pl.ncl;
    p.kgroups = pl.kgroups;
    p.tiles_m = pl.tiles_m;
    p.nsplit = pl.nsplit;
    p.items = pl.items;
    p.dmin = dmin;
    p.scale = scale;
    p.vsat = vsat;
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    cluster_kernel<<<K, 512, (size_t)pl.sort_n * sizeof(unsigned long long), s>>>(
        wpos, wneg, K, O, pl.sort_n, pl.band, reinterpret_cast<float2*>(ws), reinterpret_cast<int*>(ws + pl.co_off),
        reinterpret_cast<float4*>(ws + pl.cr_off));
    if ((rc = check_launch("cluster_kernel"))) return rc;
    if (pl.tm == 8) bwd2_kernel<kStride, 8><<<pl.grid, kB2Threads, pl.smem, s>>>(p);
    else bwd2_kernel<kStride, 4><<<pl.grid, kB2Threads, pl.smem, s>>>(p);
    return check_launch("bwd2_kernel");
}

// Clustered backward plus the split reduction; `workspace` laid out as pl says.
int launch_backward2(const Bwd2Plan& pl, const float* x, const float* wpos, const float* wneg,
                     const float* grad_out, const void* lut, int M, int K, int O, int T, float dmin, float scale,
                     float vsat, float* grad_x, float* grad_wpos, float* grad_wneg, void* workspace,
                     cudaStream_t s) {
    int dev, sms, optin, rc;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = device_limits(dev, &sms, &optin))) return rc;
    const bool want_w = grad_wpos != nullptr;
    const int st = bwd_stride(T);
    if (st == 4096)
        rc = launch_backward2_stride<4096>(pl, dev, optin, x, wpos, wneg, grad_out, lut, M, K, O, T, dmin, scale,
                                           vsat, grad_x, want_w, workspace, s);
    else if (st == 8192)
        rc = launch_backward2_stride<8192>(pl, dev, optin, x, wpos, wneg, grad_out, lut, M, K, O, T, dmin, scale,
                                           vsat, grad_x, want_w, workspace, s);
    else
        rc = launch_backward2_stride<16384>(pl, dev, optin, x, wpos, wneg, grad_out, lut, M, K, O, T, dmin, scale,
                                            vsat, grad_x, want_w, workspace, s);
    if (rc || !want_w) return rc;
    const int64_t n = (int64_t)O * K;
    int blocks = (int)((n + 255) / 256);
    if (blocks > sms * 8) blocks = sms * 8;
    bwd_reduce_kernel<<<blocks, 256, 0, s>>>(
        reinterpret_cast<const float*>(static_cast<unsigned char*>(workspace) + pl.part_off), pl.nsplit, n,
        grad_wpos, grad_wneg);
    return check_launch("bwd_reduce_kernel");
}

int check_lut_size(int T) {
    if (T < 2 || T > CIMEKV_MAX_LUT_SIZE) {
        return set_error(CIMEKV_ELUT_TOO_LARGE, "LUT size %d outside [2, %d]", T, CIMEKV_MAX_LUT_SIZE);
    }
    return CIMEKV_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

// ================================================================ C ABI ==

extern "C" {

int cimekv_abi_version(void) { return 1; }

const char* cimekv_last_error(void) { return g_last_error; }

size_t cimekv_lut_bytes(int table_size) {
    if (table_size < 2 || table_size > CIMEKV_MAX_LUT_SIZE) return 0;
    return 2 * fwd_table_bytes(table_size);
}

int cimekv_lut_pack(const uint16_t* table_i, const uint16_t* table_ddelta, int table_size, void* lut,
                    void* stream) {
    NvtxRange nvtx_range("cimekv_lut_pack");
    int rc = cimekv_internal_begin_call();
    if (rc || (rc = check_lut_size(table_size))) return rc;
    if (rc) return rc;
    if (!table_i || !table_ddelta || !lut) return set_error(CIMEKV_EINVAL_SHAPE, "null pointer");
    if (!aligned16(lut)) return set_error(CIMEKV_EINVAL_SHAPE, "lut must be 16-byte aligned");
    const int words = (int)(fwd_table_bytes(table_size) / 4);
    uint32_t* lut_i = static_cast<uint32_t*>(lut);
    uint32_t* lut_d = lut_i + words;
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    lut_pack_kernel<<<(words + 255) / 256, 256, 0, (cudaStream_t)stream>>>(table_i, table_ddelta, table_size,
                                                                            lut_i, lut_d, words);
    return check_launch("lut_pack_kernel");
}

struct ExactArgs {
    float inv, vd, i_s, di_s;
};

// Constants of the base-2 cell evaluation (see softplus_sigmoid).
ExactArgs exact_args(float inv_2nut, float v_d, float i_s) {
    const double log2e = 1.4426950408889634, ln2 = 0.6931471805599453;
    ExactArgs e;
    e.inv = (float)((double)inv_2nut * log2e);
    e.vd = (float)((double)v_d * (double)inv_2nut * log2e);
    e.i_s = (float)((double)i_s * ln2 * ln2);
    e.di_s = (float)(2.0 * (double)inv_2nut * (double)i_s * ln2);
    return e;
}

// ex == nullptr: LUT path; otherwise the exact EKV formula (no table).
static int launch_forward(const float* x, const float* wpos, const float* wneg, const void* lut, int M, int K,
                          int O, int table_size, float delta_min, float delta_scale, float v_sat, float out_min,
                          float out_max, float* out, const float* r_tia, float tia_lo, float tia_hi, float* tia_out,
                          void* stream, const ExactArgs* ex = nullptr) {
    int rc = cimekv_internal_begin_call();
    if (rc || (rc = ex ? CIMEKV_OK : check_lut_size(table_size))) return rc;
    if (rc) return rc;
    if (M < 0 || K < 0 || O < 0) return set_error(CIMEKV_EINVAL_SHAPE, "negative size M=%d K=%d O=%d", M, K, O);
    if (M == 0 || O == 0) return CIMEKV_OK;
    if ((!lut && !ex) || !out || (K > 0 && (!x || !wpos || !wneg)) || (tia_out && !r_tia))
        return set_error(CIMEKV_EINVAL_SHAPE, "null pointer");
    if (!ex && !aligned16(lut)) return set_error(CIMEKV_EINVAL_SHAPE, "lut must be 16-byte aligned");
    if (!ex && !(delta_scale > 0.0f)) return set_error(CIMEKV_EINVAL_SHAPE, "delta_scale must be > 0");
    if (ex) table_size = 0;
    int dev, sms, optin;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = device_limits(dev, &sms, &optin))) return rc;
    const size_t smem = fwd_smem_bytes(table_size);
    if (smem > (size_t)optin) return set_error(CIMEKV_ELUT_TOO_LARGE, "forward needs %zu B shared memory", smem);
    if ((rc = ex ? allow_smem(dev, 4, fwd_kernel<true>, optin) : allow_smem(dev, 0, fwd_kernel<false>, optin)))
        return rc;
    FwdParams p;
    p.x = x;
    p.wp = wpos;
    p.wn = wneg;
    p.lut = static_cast<const uint32_t*>(lut);
    p.out = out;
    p.M = M;
    p.K = K;
    p.O = O;
    p.T = table_size;
    p.dmin = delta_min;
    p.scale = delta_scale;
    p.vsat = v_sat;
    p.out_min = out_min;
    p.out_max = out_max;
    p.r_tia = r_tia;
    p.tia_out = tia_out;
    p.tia_lo = tia_lo;
    p.tia_hi = tia_hi;
    p.inv = ex ? ex->inv : 0.0f;
    p.vd = ex ? ex->vd : 0.0f;
    p.i_s = ex ? ex->i_s : 0.0f;
    p.di_s = ex ? ex->di_s : 0.0f;
    const long ntiles = (long)((M + kFwdMT - 1) / kFwdMT) * ((O + kFwdOT - 1) / kFwdOT);
    int resident = (int)((228 * 1024) / (smem + 1024));
    if (resident > CIMEKV_FWD_MIN_BLOCKS) resident = CIMEKV_FWD_MIN_BLOCKS;
    if (resident < 1) resident = 1;
    const long slots = (long)sms * resident;
    // Split each tile's k range in two when the tiles fill the resident CTAs
    // badly (few tiles: small per-GPU batches), e.g. 594 tiles on 444 slots run
    // 2 waves at 67 % occupancy, 1188 half-tiles 3 waves at 89 %.
    const int nchunks = (K + kFwdKC - 1) / kFwdKC;
    const double eff1 = (double)ntiles / ((double)((ntiles + slots - 1) / slots) * slots);
    const double eff2 = (double)(2 * ntiles) / ((double)((2 * ntiles + slots - 1) / slots) * slots);
    p.ksplit = (nchunks >= 2 && eff2 > eff1 + 0.05) ? 2 : 1;
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    if (p.ksplit > 1) {
        cudaError_t e = cudaMemsetAsync(out, 0, (size_t)M * O * sizeof(float), (cudaStream_t)stream);
        if (e != cudaSuccess) return set_error(CIMEKV_ECUDA, "cudaMemsetAsync: %s", cudaGetErrorString(e));
    }
    long grid = slots;
    if (grid > ntiles * p.ksplit) grid = ntiles * p.ksplit;
    if (ex) fwd_kernel<true><<<(unsigned)grid, kFwdThreads, smem, (cudaStream_t)stream>>>(p);
    else fwd_kernel<false><<<(unsigned)grid, kFwdThreads, smem, (cudaStream_t)stream>>>(p);
    if ((rc = check_launch("fwd_kernel"))) return rc;
    if (p.ksplit > 1) {
        fwd_split_epilogue_kernel<<<(unsigned)(sms * 4), 256, 0, (cudaStream_t)stream>>>(
            out, tia_out, r_tia, (int64_t)M * O, out_min, out_max, tia_lo, tia_hi);
        return check_launch("fwd_split_epilogue_kernel");
    }
    return CIMEKV_OK;
}

int cimekv_forward(const float* x, const float* wpos, const float* wneg, const void* lut, int M, int K, int O,
                   int table_size, float delta_min, float delta_scale, float v_sat, float out_min, float out_max,
                   float* out, void* stream) {
    NvtxRange nvtx_range("cimekv_forward");
    return launch_forward(x, wpos, wneg, lut, M, K, O, table_size, delta_min, delta_scale, v_sat, out_min, out_max,
                          out, nullptr, 0.0f, 0.0f, nullptr, stream);
}

int cimekv_forward_tia(const float* x, const float* wpos, const float* wneg, const void* lut, int M, int K, int O,
                       int table_size, float delta_min, float delta_scale, float v_sat, float idiff_min,
                       float idiff_max, const float* r_tia, float out_min, float out_max, float* idiff, float* out,
                       void* stream) {
    NvtxRange nvtx_range("cimekv_forward_tia");
    if (!out || !r_tia) {
        g_last_error[0] = '\0';
        return set_error(CIMEKV_EINVAL_SHAPE, "null pointer");
    }
    return launch_forward(x, wpos, wneg, lut, M, K, O, table_size, delta_min, delta_scale, v_sat, idiff_min,
                          idiff_max, idiff, r_tia, out_min, out_max, out, stream);
}

size_t cimekv_tia_workspace_bytes(long long n) {
    (void)n;
    return (size_t)kTiaBlocks * sizeof(float);
}

int cimekv_tia_backward(const float* grad_out, const float* idiff, const float* r_tia, long long n, float out_min,
                        float out_max, float* grad_idiff, float* grad_r_tia, void* workspace, size_t workspace_bytes,
                        void* stream) {
    NvtxRange nvtx_range("cimekv_tia_backward");
    if (int rc0 = cimekv_internal_begin_call()) return rc0;
    if (n < 0) return set_error(CIMEKV_EINVAL_SHAPE, "negative n");
    if (!r_tia || !grad_r_tia || (n > 0 && (!grad_out || !idiff || !grad_idiff)))
        return set_error(CIMEKV_EINVAL_SHAPE, "null pointer");
    if (!workspace || workspace_bytes < (size_t)kTiaBlocks * sizeof(float))
        return set_error(CIMEKV_EWORKSPACE, "TIA backward workspace needs %zu B", (size_t)kTiaBlocks * sizeof(float));
    cudaStream_t s = (cudaStream_t)stream;
    float* partial = static_cast<float*>(workspace);
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    tia_bwd_kernel<<<kTiaBlocks, 256, 0, s>>>(grad_out, idiff, r_tia, (int64_t)n, out_min, out_max, grad_idiff,
                                              partial);
    int rc = check_launch("tia_bwd_kernel");
    if (rc) return rc;
    sum_partials_kernel<<<1, 256, 0, s>>>(partial, kTiaBlocks, grad_r_tia);
    return check_launch("sum_partials_kernel");
}

size_t cimekv_backward_workspace_bytes(int M, int K, int O, int table_size) {
    if (M <= 0 || K <= 0 || O <= 0 || check_lut_size(table_size)) return 0;
    Bwd2Plan plan2;
    bool ok2 = false;
    if (plan_backward2(M, K, O, table_size, &plan2, &ok2)) return 0;
    if (ok2) return plan2.workspace;
    BwdPlan plan;
    if (plan_backward(M, K, O, table_size, &plan)) return 0;
    return plan.workspace;
}

int cimekv_backward(const float* x, const float* wpos, const float* wneg, const float* grad_out, const void* lut,
                    int M, int K, int O, int table_size, float delta_min, float delta_scale, float v_sat,
                    float* grad_x, float* grad_wpos, float* grad_wneg, void* workspace, size_t workspace_bytes,
                    void* stream) {
    NvtxRange nvtx_range("cimekv_backward");
    int rc = cimekv_internal_begin_call();
    if (rc || (rc = check_lut_size(table_size))) return rc;
    if (M < 0 || K < 0 || O < 0) return set_error(CIMEKV_EINVAL_SHAPE, "negative size M=%d K=%d O=%d", M, K, O);
    if ((grad_wpos == nullptr) != (grad_wneg == nullptr))
        return set_error(CIMEKV_EINVAL_SHAPE, "grad_wpos and grad_wneg must both be given or both be NULL");
    const bool want_w = grad_wpos != nullptr;
    cudaStream_t s = (cudaStream_t)stream;
    if (K == 0) return CIMEKV_OK;
    if (M == 0 || O == 0) {
        // Empty sums: gradients are zero.
        if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
        if (want_w && O > 0) {
            fill_zero_kernel<<<64, 256, 0, s>>>(grad_wpos, (int64_t)O * K);
            fill_zero_kernel<<<64, 256, 0, s>>>(grad_wneg, (int64_t)O * K);
        }
        if (grad_x && M > 0) fill_zero_kernel<<<64, 256, 0, s>>>(grad_x, (int64_t)M * K);
        return check_launch("fill_zero_kernel");
    }
    if (!grad_x && !want_w) return CIMEKV_OK;
    if (!x || !wpos || !wneg || !grad_out || !lut) return set_error(CIMEKV_EINVAL_SHAPE, "null pointer");
    if (!aligned16(lut)) return set_error(CIMEKV_EINVAL_SHAPE, "lut must be 16-byte aligned");
    if (!(delta_scale > 0.0f)) return set_error(CIMEKV_EINVAL_SHAPE, "delta_scale must be > 0");
    Bwd2Plan plan2;
    bool ok2 = false;
    if ((rc = plan_backward2(M, K, O, table_size, &plan2, &ok2))) return rc;
    if (ok2 && want_w && (!workspace || workspace_bytes < plan2.workspace))
        return set_error(CIMEKV_EWORKSPACE, "backward workspace needs %zu B, got %zu B", plan2.workspace,
                         workspace_bytes);
    if (ok2 && workspace && workspace_bytes >= plan2.workspace) {
        // Clustered kernel (a dX-only call without a workspace takes bwd_kernel).
        if (!aligned16(workspace)) return set_error(CIMEKV_EINVAL_SHAPE, "workspace must be 16-byte aligned");
        return launch_backward2(plan2, x, wpos, wneg, grad_out, lut, M, K, O, table_size, delta_min, delta_scale,
                                v_sat, grad_x, grad_wpos, grad_wneg, workspace, s);
    }
    BwdPlan plan;
    if ((rc = plan_backward(M, K, O, table_size, &plan))) return rc;
    if (want_w) {
        if (!workspace || workspace_bytes < plan.workspace)
            return set_error(CIMEKV_EWORKSPACE, "backward workspace needs %zu B, got %zu B", plan.workspace,
                             workspace_bytes);
        if (!aligned16(workspace)) return set_error(CIMEKV_EINVAL_SHAPE, "workspace must be 16-byte aligned");
    }
    int dev, sms, optin;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = device_limits(dev, &sms, &optin))) return rc;
    const int stride = bwd_stride(table_size);
    const int slot = stride == 4096 ? 1 : (stride == 8192 ? 2 : 3);
    if (stride == 4096) rc = allow_smem(dev, slot, bwd_kernel<4096>, optin);
    else if (stride == 8192) rc = allow_smem(dev, slot, bwd_kernel<8192>, optin);
    else rc = allow_smem(dev, slot, bwd_kernel<16384>, optin);
    if (rc) return rc;
    BwdParams p;
    p.x = x;
    p.wp = wpos;
    p.wn = wneg;
    p.g = grad_out;
    p.lut_i = static_cast<const uint32_t*>(lut);
    p.lut_d = p.lut_i + fwd_table_bytes(table_size) / 4;
    p.grad_x = grad_x;
    p.part = want_w ? static_cast<float*>(workspace) : nullptr;
    p.M = M;
    p.K = K;
    p.O = O;
    p.T = table_size;
    p.tiles_m = plan.tiles_m;
    p.nsplit = plan.nsplit;
    p.dw_global = plan.dw_global;
    p.dmin = delta_min;
    p.scale = delta_scale;
    p.vsat = v_sat;
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    dim3 grid(plan.kblocks, plan.nsplit);
    if (stride == 4096) bwd_kernel<4096><<<grid, kBwdThreads, plan.smem, s>>>(p);
    else if (stride == 8192) bwd_kernel<8192><<<grid, kBwdThreads, plan.smem, s>>>(p);
    else bwd_kernel<16384><<<grid, kBwdThreads, plan.smem, s>>>(p);
    if ((rc = check_launch("bwd_kernel"))) return rc;
    if (want_w) {
        const int64_t n = (int64_t)O * K;
        int blocks = (int)((n + 255) / 256);
        if (blocks > sms * 8) blocks = sms * 8;
        bwd_reduce_kernel<<<blocks, 256, 0, s>>>(p.part, plan.nsplit, n, grad_wpos, grad_wneg);
        if ((rc = check_launch("bwd_reduce_kernel"))) return rc;
    }
    return CIMEKV_OK;
}

int cimekv_lut_index(const float* delta, int n, int table_size, float delta_min, float delta_scale, int32_t* index,
                     float* alpha, void* stream) {
    int rc = cimekv_internal_begin_call();
    if (rc || (rc = check_lut_size(table_size))) return rc;
    if (n < 0) return set_error(CIMEKV_EINVAL_SHAPE, "negative n");
    if (n == 0) return CIMEKV_OK;
    if (!delta || !index || !alpha) return set_error(CIMEKV_EINVAL_SHAPE, "null pointer");
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    lut_index_kernel<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(delta, n, table_size, delta_min,
                                                                         delta_scale, index, alpha);
    return check_launch("lut_index_kernel");
}

}  // extern "C"

// ----------------------------------------------- allocation-free backward --
//
// Scratch for callers that cannot allocate device memory themselves (see
// cimekv_backward_noalloc in cimekv.h).  It lives in the library's own static
// device memory: every GPU that loads the library holds these
// CIMEKV_NOALLOC_SCRATCH_BYTES until the process exits.  Host code must not use
// the symbol's name as a pointer; the device address is looked up once per
// device with cudaGetSymbolAddress.

static __device__ __align__(256) float g_noalloc_scratch[CIMEKV_NOALLOC_SCRATCH_BYTES / sizeof(float)];

namespace {

std::mutex g_noalloc_mutex;
float* g_noalloc_ptr[kMaxDevices] = {};

// Device address of the scratch array on device `dev` (which must be current).
int noalloc_scratch(int dev, float** out) {
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    if (g_noalloc_ptr[dev] == nullptr) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr) {
            return set_error(CIMEKV_ECUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        }
        g_noalloc_ptr[dev] = static_cast<float*>(ptr);
    }
    *out = g_noalloc_ptr[dev];
    return CIMEKV_OK;
}

}  // namespace

extern "C" int cimekv_backward_noalloc(const float* x, const float* wpos, const float* wneg,
                                       const float* grad_out, const void* lut, int M, int K, int O,
                                       int table_size, float delta_min, float delta_scale, float v_sat,
                                       float* grad_x, float* grad_wpos, float* grad_wneg, void* stream) {
    NvtxRange nvtx_range("cimekv_backward_noalloc");
    int rc = cimekv_internal_begin_call();
    if (rc || (rc = check_lut_size(table_size))) return rc;
    if (M < 0 || K < 0 || O < 0) return set_error(CIMEKV_EINVAL_SHAPE, "negative size M=%d K=%d O=%d", M, K, O);
    if ((grad_wpos == nullptr) != (grad_wneg == nullptr))
        return set_error(CIMEKV_EINVAL_SHAPE, "grad_wpos and grad_wneg must both be given or both be NULL");
    const bool want_w = grad_wpos != nullptr;
    // One token split needs 2*O*K floats of scratch; refuse what cannot fit.
    const size_t per_split = (size_t)2 * (size_t)O * (size_t)K * sizeof(float);
    if (want_w && per_split > CIMEKV_NOALLOC_SCRATCH_BYTES) {
        return set_error(CIMEKV_EWORKSPACE,
                         "cimekv_backward_noalloc: out_features*in_features = %lld needs %zu B of scratch per "
                         "token split, above the library's fixed %zu B (at most %zu threshold pairs)",
                         (long long)O * K, per_split, (size_t)CIMEKV_NOALLOC_SCRATCH_BYTES,
                         (size_t)CIMEKV_NOALLOC_SCRATCH_BYTES / (2 * sizeof(float)));
    }
    cudaStream_t s = (cudaStream_t)stream;
    if (K == 0) return CIMEKV_OK;
    if (M == 0 || O == 0) {
        if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
        if (want_w && O > 0) {
            fill_zero_kernel<<<64, 256, 0, s>>>(grad_wpos, (int64_t)O * K);
            fill_zero_kernel<<<64, 256, 0, s>>>(grad_wneg, (int64_t)O * K);
        }
        if (grad_x && M > 0) fill_zero_kernel<<<64, 256, 0, s>>>(grad_x, (int64_t)M * K);
        return check_launch("fill_zero_kernel");
    }
    if (!grad_x && !want_w) return CIMEKV_OK;
    if (!x || !wpos || !wneg || !grad_out || !lut) return set_error(CIMEKV_EINVAL_SHAPE, "null pointer");
    if (!aligned16(lut)) return set_error(CIMEKV_EINVAL_SHAPE, "lut must be 16-byte aligned");
    if (!(delta_scale > 0.0f)) return set_error(CIMEKV_EINVAL_SHAPE, "delta_scale must be > 0");
    BwdPlan plan;
    if ((rc = plan_backward(M, K, O, table_size, &plan))) return rc;
    // Fewer token splits when the planned ones do not fit the fixed scratch.
    const int max_split = (int)(CIMEKV_NOALLOC_SCRATCH_BYTES / per_split);
    if (plan.nsplit > max_split) plan.nsplit = max_split;
    int dev, sms, optin;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = device_limits(dev, &sms, &optin))) return rc;
    float* scratch = nullptr;
    {
        // Clustered kernel when its column clusters and at least one token
        // split fit the scratch (the same kernel, and so the same grad_x bits,
        // as cimekv_backward); fewer splits than planned when needed.
        Bwd2Plan plan2;
        bool ok2 = false;
        if ((rc = plan_backward2(M, K, O, table_size, &plan2, &ok2))) return rc;
        const size_t per_split2 = (size_t)2 * O * K * sizeof(float);
        if (ok2 && plan2.part_off + per_split2 <= CIMEKV_NOALLOC_SCRATCH_BYTES) {
            const int fit = (int)((CIMEKV_NOALLOC_SCRATCH_BYTES - plan2.part_off) / per_split2);
            if (plan2.nsplit > fit) {
                plan2.nsplit = fit;
                plan2.items = plan2.kgroups * fit;
                plan2.grid = plan2.items < sms ? plan2.items : sms;
            }
            if ((rc = noalloc_scratch(dev, &scratch))) return rc;
            return launch_backward2(plan2, x, wpos, wneg, grad_out, lut, M, K, O, table_size, delta_min,
                                    delta_scale, v_sat, grad_x, grad_wpos, grad_wneg, scratch, s);
        }
    }
    if (want_w && (rc = noalloc_scratch(dev, &scratch))) return rc;
    const int stride = bwd_stride(table_size);
    const int slot = stride == 4096 ? 1 : (stride == 8192 ? 2 : 3);
    if (stride == 4096) rc = allow_smem(dev, slot, bwd_kernel<4096>, optin);
    else if (stride == 8192) rc = allow_smem(dev, slot, bwd_kernel<8192>, optin);
    else rc = allow_smem(dev, slot, bwd_kernel<16384>, optin);
    if (rc) return rc;
    BwdParams p;
    p.x = x;
    p.wp = wpos;
    p.wn = wneg;
    p.g = grad_out;
    p.lut_i = static_cast<const uint32_t*>(lut);
    p.lut_d = p.lut_i + fwd_table_bytes(table_size) / 4;
    p.grad_x = grad_x;
    // Every split slice of the scratch is fully overwritten by the kernel before
    // the reduction reads it, so nothing left from an earlier call is used.
    p.part = want_w ? scratch : nullptr;
    p.M = M;
    p.K = K;
    p.O = O;
    p.T = table_size;
    p.tiles_m = plan.tiles_m;
    p.nsplit = plan.nsplit;
    p.dw_global = plan.dw_global;
    p.dmin = delta_min;
    p.scale = delta_scale;
    p.vsat = v_sat;
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    dim3 grid(plan.kblocks, plan.nsplit);
    if (stride == 4096) bwd_kernel<4096><<<grid, kBwdThreads, plan.smem, s>>>(p);
    else if (stride == 8192) bwd_kernel<8192><<<grid, kBwdThreads, plan.smem, s>>>(p);
    else bwd_kernel<16384><<<grid, kBwdThreads, plan.smem, s>>>(p);
    if ((rc = check_launch("bwd_kernel"))) return rc;
    if (want_w) {
        const int64_t n = (int64_t)O * K;
        int blocks = (int)((n + 255) / 256);
        if (blocks > sms * 8) blocks = sms * 8;
        bwd_reduce_kernel<<<blocks, 256, 0, s>>>(p.part, plan.nsplit, n, grad_wpos, grad_wneg);
        if ((rc = check_launch("bwd_reduce_kernel"))) return rc;
    }
    return CIMEKV_OK;
}

// ==================================================== exact-formula path ==

extern "C" int cimekv_exact_forward(const float* x, const float* wpos, const float* wneg, int M, int K, int O,
                                    float inv_2nut, float v_d, float i_s, float v_sat, float* out, void* stream) {
    NvtxRange nvtx_range("cimekv_exact_forward");
    const ExactArgs ex = exact_args(inv_2nut, v_d, i_s);
    return launch_forward(x, wpos, wneg, nullptr, M, K, O, 0, 0.0f, 1.0f, v_sat, -INFINITY, INFINITY, out, nullptr,
                          0.0f, 0.0f, nullptr, stream, &ex);
}

extern "C" size_t cimekv_exact_backward_workspace_bytes(int M, int K, int O) {
    if (M <= 0 || K <= 0 || O <= 0) return 0;
    BwdPlan plan;
    if (plan_backward(M, K, O, 0, &plan, 0)) return 0;
    return plan.workspace;
}

extern "C" int cimekv_exact_backward(const float* x, const float* wpos, const float* wneg, const float* grad_out,
                                     int M, int K, int O, float inv_2nut, float v_d, float i_s, float v_sat,
                                     float* grad_x, float* grad_wpos, float* grad_wneg, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    NvtxRange nvtx_range("cimekv_exact_backward");
    if (int rc0 = cimekv_internal_begin_call()) return rc0;
    if (M < 0 || K < 0 || O < 0) return set_error(CIMEKV_EINVAL_SHAPE, "negative size M=%d K=%d O=%d", M, K, O);
    if ((grad_wpos == nullptr) != (grad_wneg == nullptr))
        return set_error(CIMEKV_EINVAL_SHAPE, "grad_wpos and grad_wneg must both be given or both be NULL");
    const bool want_w = grad_wpos != nullptr;
    cudaStream_t s = (cudaStream_t)stream;
    if (K == 0) return CIMEKV_OK;
    if (M == 0 || O == 0) {
        if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
        if (want_w && O > 0) {
            fill_zero_kernel<<<64, 256, 0, s>>>(grad_wpos, (int64_t)O * K);
            fill_zero_kernel<<<64, 256, 0, s>>>(grad_wneg, (int64_t)O * K);
        }
        if (grad_x && M > 0) fill_zero_kernel<<<64, 256, 0, s>>>(grad_x, (int64_t)M * K);
        return check_launch("fill_zero_kernel");
    }
    if (!grad_x && !want_w) return CIMEKV_OK;
    if (!x || !wpos || !wneg || !grad_out) return set_error(CIMEKV_EINVAL_SHAPE, "null pointer");
    BwdPlan plan;
    int rc;
    if ((rc = plan_backward(M, K, O, 0, &plan, 0))) return rc;
    if (want_w) {
        if (!workspace || workspace_bytes < plan.workspace)
            return set_error(CIMEKV_EWORKSPACE, "backward workspace needs %zu B, got %zu B", plan.workspace,
                             workspace_bytes);
        if (!aligned16(workspace)) return set_error(CIMEKV_EINVAL_SHAPE, "workspace must be 16-byte aligned");
    }
    int dev, sms, optin;
    if ((rc = current_device(&dev))) return rc;
    if ((rc = device_limits(dev, &sms, &optin))) return rc;
    if ((rc = allow_smem(dev, 5, bwd_kernel<0>, optin))) return rc;
    const ExactArgs ex = exact_args(inv_2nut, v_d, i_s);
    BwdParams p;
    p.x = x;
    p.wp = wpos;
    p.wn = wneg;
    p.g = grad_out;
    p.lut_i = nullptr;
    p.lut_d = nullptr;
    p.grad_x = grad_x;
    p.part = want_w ? static_cast<float*>(workspace) : nullptr;
    p.M = M;
    p.K = K;
    p.O = O;
    p.T = 0;
    p.tiles_m = plan.tiles_m;
    p.nsplit = plan.nsplit;
    p.dw_global = plan.dw_global;
    p.dmin = 0.0f;
    p.scale = 1.0f;
    p.vsat = v_sat;
    p.inv = ex.inv;
    p.vd = ex.vd;
    p.i_s = ex.i_s;
    p.di_s = ex.di_s;
    if (int rc_p = cimekv_internal_no_pending_error()) return rc_p;
    dim3 grid(plan.kblocks, plan.nsplit);
    bwd_kernel<0><<<grid, kBwdThreads, plan.smem, s>>>(p);
    if ((rc = check_launch("bwd_kernel<exact>"))) return rc;
    if (want_w) {
        const int64_t n = (int64_t)O * K;
        int blocks = (int)((n + 255) / 256);
        if (blocks > sms * 8) blocks = sms * 8;
        bwd_reduce_kernel<<<blocks, 256, 0, s>>>(p.part, plan.nsplit, n, grad_wpos, grad_wneg);
        if ((rc = check_launch("bwd_reduce_kernel"))) return rc;
    }
    return CIMEKV_OK;
}

// ======================================================== debug support ==

extern "C" unsigned int cimekv_debug_oob_count(int reset) {
    unsigned int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_debug_oob_count, sizeof(v)) != cudaSuccess) return 0xFFFFFFFFu;
    if (reset) {
        const unsigned int zero = 0;
        cudaMemcpyToSymbol(g_debug_oob_count, &zero, sizeof(zero));
    }
    return v;
}

extern "C" int cimekv_debug_build(void) { return CIMEKV_DEBUG_BOUNDS; }
