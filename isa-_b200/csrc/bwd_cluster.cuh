// bwd_cluster.cuh — clustered LUT backward (included by cimekv.cu inside its
// anonymous namespace; uses its table, index and packed-fp32 helpers).
//
// Why: in the LUT backward a warp request gathers 32 table words for 32
// outputs of one (token, input) cell row.  Their entries differ only through
// the thresholds Vth[o,k] (x is common), and with outputs in their natural
// order the words fall at random inside the ~67-entry (T=4096) window that the
// threshold spread spans: ~2.7 shared-memory wavefronts per request, which
// made the data pipe the bound.  Any 32 entries inside one 32-word window sit
// in distinct banks, so this path regroups the outputs of every input column
// into clusters of 32 with close thresholds in BOTH branches:
//   1. sort the column's outputs by Vth_pos; cut the order into ~sqrt(n/32)
//      bands whose sizes are multiples of 32;
//   2. sort each band by Vth_neg; cluster c = positions [32c, 32c+32).
// A cluster then spans a few table entries per branch (about one wavefront
// per request).  The permutation is per column, so the upstream gradient of a
// lane (g[m, o] for its output o) changes with the column: the token tile's
// g rows are staged in shared memory by async copies, and each lane gathers
// its own entries.
//
// Work split: a persistent CTA (512 threads, one per SM) walks work items =
// (group of kt input columns, token split).  Warp w serves column kk = w / wpk
// and clusters cb, cb + wpk, ... (cb = w % wpk); for layers with few outputs
// (kt > 16) it serves whole columns w, w + 16, ... (cpw of them), so that every
// warp has enough clusters per tile to amortise the tile's barrier and staging.  Its
// dVth partial sums live in shared memory ([warp][cluster][lane], updated once
// per cluster and tile, which keeps registers free for overlapping the
// lookups) across all tiles of the item and go to the split's workspace slice
// once at the end (reduced in a fixed order by bwd_reduce_kernel).  The
// thresholds and output index of the next cluster are fetched while the
// current one runs; the table is staged as interleaved {I pair, dI pair}
// words, so one 64-bit shared load serves a lookup.  Per kTM-token tile a warp
// sums its dX partials over lanes by a butterfly; the warps of one column add theirs in a fixed order
// after the next tile's barrier.  The cell arithmetic, index rule and
// interpolation are those of the unclustered kernel (lut_bwd2).

constexpr int kCluMaxOutputs = 4096;  // outputs one column sort handles (o fits 13 key bits)
constexpr int kCluMinOutputs = 256;        // T <= 4096: smallest layer measured faster than the unclustered kernel
constexpr int kCluMinOutputsLargeT = 256;  // T > 4096
constexpr int kB2Threads = 512;
constexpr int kB2Warps = kB2Threads / 32;
constexpr int kB2UMax = 24;  // clusters per warp (dVth sums in shared memory, [warp][cluster][lane])
constexpr int kB2MaxKT = 32;  // input columns per work item (two per warp for layers of <= 12 clusters)

// Unsigned key with the order of the fp32 values (negatives reversed).
__device__ __forceinline__ uint32_t float_order_bits(float v) {
    const uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// In-place ascending bitonic sort of n (a power of two) keys in shared memory.
__device__ void bitonic_sort_u64(unsigned long long* key, int n) {
    for (int size = 2; size <= n; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < (n >> 1); i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool asc = (lo & size) == 0;
                const unsigned long long a = key[lo], b = key[hi];
                if ((a > b) == asc) {
                    key[lo] = b;
                    key[hi] = a;
                }
            }
            __syncthreads();
        }
    }
}

// One CTA per input column k: cluster order of the column's outputs.
//   cw[k][j] = {Vth_pos, Vth_neg} and co[k][j] = output of position j
//   (j < opad; positions >= O are pads: thresholds 0, output O, whose staged
//   upstream-gradient column is zero);
//   crange[k] = {min, max over both branches (pads count as 0), NaN seen, 0}.
// Keys: pass 1 = (order(Vth_pos) << 32) | o; pass 2 = (band << 45) |
// (order(Vth_neg) << 13) | o, o < 8192.  Deterministic for any input.
__global__ void __launch_bounds__(512) cluster_kernel(const float* __restrict__ wp, const float* __restrict__ wn,
                                                      int K, int O, int n, int band, float2* __restrict__ cw,
                                                      int* __restrict__ co, float4* __restrict__ crange) {
    extern __shared__ unsigned long long ckey[];
    __shared__ float2 red[16];
    __shared__ int red_nan[16];
    const int k = blockIdx.x;
    const int opad = (O + 31) & ~31;
    float lo = INFINITY, hi = -INFINITY;
    bool nan = false;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        if (i < O) {
            const float a = __ldg(wp + (int64_t)i * K + k);
            const float b = __ldg(wn + (int64_t)i * K + k);
            lo = fminf(lo, fminf(a, b));
            hi = fmaxf(hi, fmaxf(a, b));
            nan |= (a != a) | (b != b);
            ckey[i] = ((unsigned long long)float_order_bits(a) << 32) | (unsigned)i;
        } else {
            ckey[i] = ~0ull;
        }
    }
    if (opad > O) {
        lo = fminf(lo, 0.0f);
        hi = fmaxf(hi, 0.0f);
    }
    {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        lo = warp_min(lo);
        hi = warp_max(hi);
        const bool any = __any_sync(0xffffffffu, nan);
        if (lane == 0) {
            red[warp] = make_float2(lo, hi);
            red_nan[warp] = any;
        }
    }
    __syncthreads();
    bitonic_sort_u64(ckey, n);
    for (int i = threadIdx.x; i < O; i += blockDim.x) {
        const int o = (int)(ckey[i] & 0xffffffffu);
        const float b = __ldg(wn + (int64_t)o * K + k);
        ckey[i] = ((unsigned long long)(i / band) << 45) | ((unsigned long long)float_order_bits(b) << 13) |
                  (unsigned)o;
    }
    __syncthreads();
    bitonic_sort_u64(ckey, n);
    for (int j = threadIdx.x; j < opad; j += blockDim.x) {
        float2 w = make_float2(0.0f, 0.0f);
        int o = O;
        if (j < O) {
            o = (int)(ckey[j] & 0x1fffu);
            w = make_float2(__ldg(wp + (int64_t)o * K + k), __ldg(wn + (int64_t)o * K + k));
        }
        cw[(int64_t)k * opad + j] = w;
        co[(int64_t)k * opad + j] = o;
    }
    if (threadIdx.x == 0) {
        float2 r = red[0];
        int nn = red_nan[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
            r.x = fminf(r.x, red[w].x);
            r.y = fmaxf(r.y, red[w].y);
            nn |= red_nan[w];
        }
        crange[k] = make_float4(r.x, r.y, nn ? 1.0f : 0.0f, 0.0f);
    }
}

struct Bwd2Params {
    const float* x;
    const float* g;
    const float2* cw;      // [K][opad] cluster-ordered thresholds
    const int* co;         // [K][opad] cluster-ordered outputs
    const float4* crange;  // [K]
    const uint32_t* lut_i;
    const uint32_t* lut_d;
    float* grad_x;
    float* part;  // [nsplit][2][O][K]
    int M, K, O, opad, T;
    int kt, wpk, cpw, ncl, kgroups, tiles_m, nsplit, items;  // cpw > 1 only with wpk == 1
    float dmin, scale, vsat;
};

__host__ __device__ inline size_t bwd2_smem_bytes(int stride, int tm, int opad, int kt, int cpw) {
    return (size_t)8 * stride                       // I and dI/dV pair tables
           + (size_t)2 * tm * opad * 4              // double-buffered g tile [tm/2][opad][2]
           + (size_t)2 * 3 * kt * tm * 4            // x, 1/d, -1/(v_sat d^2) per (column, token)
           + (size_t)2 * kB2Warps * cpw * tm * 4    // per-(warp, column slot) dX sums
           + (size_t)2 * kB2Warps * sizeof(float4)   // x range per staging warp
           + (size_t)kB2Warps * kB2UMax * 32 * sizeof(float2);  // dVth sums per (warp, cluster, lane)
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

__device__ __forceinline__ f32x2 lds64(uint32_t addr) {
    f32x2 v;
    asm volatile("ld.shared.b64 %0, [%1];" : "=l"(v) : "r"(addr));
    return v;
}

// Backward lookup pair from the interleaved table {I pair word, dI pair word}
// (8 bytes per entry; tab_base is pre-offset by -(2^23 bits) * 8).
template <bool kClamp>
__device__ __forceinline__ void lut_bwd2_il(f32x2 xx, f32x2 ww, const LutConsts& c, f32x2& base, f32x2& deriv) {
    uint32_t b0, b1;
    const f32x2 a = lut_coord2<kClamp>(xx, ww, c, b0, b1);
    uint32_t i0, d0, i1, d1;
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(i0), "=r"(d0) : "r"(c.tab_base + (b0 << 3)));
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(i1), "=r"(d1) : "r"(c.tab_base + (b1 << 3)));
    base = lerp_pair2(a, i0, i1);
    deriv = lerp_pair2(a, d0, d1);
}

// Stage token tile `tile`'s g rows into buffer b as token pairs
// [tm/2][opad][2] (async copies; rows past M are zero).
template <int kTM>
__device__ __forceinline__ void b2_stage_g(const Bwd2Params& p, int tile, int b, float* gb) {
    const int m0 = tile * kTM;
    float* dst = gb + (size_t)b * kTM * p.opad;
    const uint32_t dst_s = smem_u32addr(dst);
#pragma unroll
    for (int r = 0; r < kTM; ++r) {
        const int m = m0 + r;
        const uint32_t row = dst_s + (uint32_t)(((r >> 1) * p.opad * 2 + (r & 1)) * 4);
        if (m < p.M) {
            const float* src = p.g + (int64_t)m * p.O;
            for (int o = threadIdx.x; o < p.O; o += kB2Threads) cp_async4(row + (uint32_t)o * 8u, src + o);
        } else {
            float* drow = dst + (r >> 1) * p.opad * 2 + (r & 1);
            for (int o = threadIdx.x; o < p.O; o += kB2Threads) drow[2 * o] = 0.0f;
        }
    }
    cp_async_commit();
}

// x of (token tt, column kk) of tile `tile` for thread t = kk * kTM + tt < kt * kTM
// (0 outside the matrix).  Issued a tile ahead of its use, so the load latency
// overlaps the current tile's cells.
template <int kTM>
__device__ __forceinline__ float b2_load_x(const Bwd2Params& p, int tile, int k0) {
    const int t = threadIdx.x;
    if (t >= p.kt * kTM) return 0.0f;
    const int kk = t / kTM, tt = t % kTM;
    const int m = tile * kTM + tt, k = k0 + kk;
    return (m < p.M && k < p.K) ? __ldg(p.x + (int64_t)m * p.K + k) : 0.0f;
}

// x, 1/d and -1/(v_sat d^2) of tile `tile` into buffer b, with the x range per
// staging warp (whole warps of threads < kt * kTM rounded up to 32).
template <int kTM>
__device__ __forceinline__ void b2_store_x(const Bwd2Params& p, float xv, int tile, int b, int k0, float* xb,
                                           float4* rng) {
    const int nx = p.kt * kTM;
    if (threadIdx.x >= ((nx + 31) & ~31)) return;
    const int t = threadIdx.x;
    if (t < nx) {
        const int kk = t / kTM, tt = t % kTM;
        const bool valid = tile * kTM + tt < p.M && k0 + kk < p.K;
        const float d = __fadd_rn(1.0f, __fdiv_rn(xv, p.vsat));
        float* xs = xb + (size_t)b * 3 * nx;
        xs[kk * kTM + tt] = xv;
        xs[nx + kk * kTM + tt] = valid ? __fdiv_rn(1.0f, d) : 0.0f;
        xs[2 * nx + kk * kTM + tt] = valid ? -__fdiv_rn(1.0f, __fmul_rn(__fmul_rn(p.vsat, d), d)) : 0.0f;
    }
    const float lo = warp_min(xv), hi = warp_max(xv);
    const bool nan = __any_sync(0xffffffffu, xv != xv);
    if ((threadIdx.x & 31) == 0) rng[b * kB2Warps + (threadIdx.x >> 5)] = make_float4(lo, hi, nan ? 1.0f : 0.0f, 0.0f);
}

// dX of tile `tile`: sum of the column's warps in a fixed order.
template <int kTM>
__device__ __forceinline__ void b2_finish_dx(const Bwd2Params& p, int tile, int b, int k0, const float* dxr) {
    const int t = threadIdx.x;
    if (p.grad_x == nullptr || t >= p.kt * kTM) return;
    const int kk = t / kTM, tt = t % kTM;
    const int m = tile * kTM + tt, k = k0 + kk;
    if (m >= p.M || k >= p.K) return;
    float s = 0.0f;
    if (p.cpw == 1) {
        for (int c = 0; c < p.wpk; ++c) s += dxr[(b * kB2Warps + kk * p.wpk + c) * kTM + tt];
    } else {  // one warp per column: warp kk % kB2Warps, slot kk / kB2Warps
        s = dxr[((b * kB2Warps + kk % kB2Warps) * p.cpw + kk / kB2Warps) * kTM + tt];
    }
    p.grad_x[(int64_t)m * p.K + k] = s;
}

// One warp, one tile: all cells (tile tokens x 32 lanes of each of the warp's
// clusters) of column k.  gt: this buffer's g tile (shared address);
// xs: this buffer's staged per-token values.
template <bool kClamp, int kStride, int kTM>
__device__ __forceinline__ void b2_compute(const Bwd2Params& p, const LutConsts& c, int k, int kk, int cb,
                                           uint32_t gt, const float* xs, float2* accw, float* dxr_w) {
    constexpr int kP = kTM / 2;
    const int lane = threadIdx.x & 31;
    f32x2 X[kP], IV[kP], NT[kP];
#pragma unroll
    for (int q = 0; q < kP / 2; ++q) {
        const float4 a = *reinterpret_cast<const float4*>(xs + kk * kTM + 4 * q);
        const float4 i = *reinterpret_cast<const float4*>(xs + p.kt * kTM + kk * kTM + 4 * q);
        const float4 n = *reinterpret_cast<const float4*>(xs + 2 * p.kt * kTM + kk * kTM + 4 * q);
        X[2 * q] = pk2(a.x, a.y);
        X[2 * q + 1] = pk2(a.z, a.w);
        IV[2 * q] = pk2(i.x, i.y);
        IV[2 * q + 1] = pk2(i.z, i.w);
        NT[2 * q] = pk2(n.x, n.y);
        NT[2 * q + 1] = pk2(n.z, n.w);
    }
    f32x2 dx[kP];
#pragma unroll
    for (int ip = 0; ip < kP; ++ip) dx[ip] = pk2(0.0f, 0.0f);
    const float2* cwk = p.cw + (int64_t)k * p.opad;
    const int* cok = p.co + (int64_t)k * p.opad;
    const uint32_t pair_stride = (uint32_t)p.opad * 8u;
    // Clusters of this warp: cb, cb + wpk, ...; their thresholds and outputs are
    // fetched one cluster ahead so the loads overlap the previous cluster's cells.
    const int nun = cb < p.ncl ? (p.ncl - cb + p.wpk - 1) / p.wpk : 0;
    float2 w_next = make_float2(0.0f, 0.0f);
    int o_next = 0;
    if (nun > 0) {
        w_next = __ldg(cwk + cb * 32 + lane);
        o_next = __ldg(cok + cb * 32 + lane);
    }
#pragma unroll 3
    for (int s = 0; s < nun; ++s) {
        {
            f32x2 ua = pk2(0.0f, 0.0f), un = pk2(0.0f, 0.0f);
            const float2 w = w_next;
            const int o = o_next;
            if (s + 1 < nun) {
                const int jn = (cb + (s + 1) * p.wpk) * 32 + lane;
                w_next = __ldg(cwk + jn);
                o_next = __ldg(cok + jn);
            }
            const f32x2 WP = pk2(w.x, w.x), WN = pk2(w.y, w.y);
            const uint32_t ga = gt + (uint32_t)o * 8u;
#pragma unroll
            for (int ip = 0; ip < kP; ++ip) {
                const f32x2 G = lds64(ga + ip * pair_stride);
                f32x2 pb, pd, nb, nd;
                lut_bwd2_il<kClamp>(X[ip], WP, c, pb, pd);
                lut_bwd2_il<kClamp>(X[ip], WN, c, nb, nd);
                // d(I_diff/d)/dx = (dp - dn)/d - (bp - bn)/(v_sat d^2)
                const f32x2 e = fma2(sub2(pb, nb), NT[ip], mul2(sub2(pd, nd), IV[ip]));
                dx[ip] = fma2(G, e, dx[ip]);
                const f32x2 gi = mul2(G, IV[ip]);
                ua = fma2(gi, pd, ua);
                un = fma2(gi, nd, un);
            }
            {
                float a0, a1, b0, b1;
                unpk2(ua, a0, a1);
                unpk2(un, b0, b1);
                float2 v = accw[s * 32 + lane];
                v.x += a0 + a1;
                v.y += b0 + b1;
                accw[s * 32 + lane] = v;
            }
        }
    }
    // Butterfly over the 32 lanes: afterwards lane l holds the full sum of
    // token (l >> (5 - log2 kTM)) & (kTM - 1).
    float v[kTM];
#pragma unroll
    for (int ip = 0; ip < kP; ++ip) unpk2(dx[ip], v[2 * ip], v[2 * ip + 1]);
    int n = kTM;
#pragma unroll
    for (int s = 16; s >= 1; s >>= 1) {
        if (n > 1) {
            const int h = n >> 1;
            const bool upper = (lane & s) != 0;
#pragma unroll
            for (int j = 0; j < h; ++j) {
                const float send = upper ? v[j] : v[j + h];
                const float keep = upper ? v[j + h] : v[j];
                v[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
            }
            n = h;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], s);
        }
    }
    constexpr int kLog = kTM == 16 ? 4 : (kTM == 8 ? 3 : (kTM == 4 ? 2 : 1));
    if ((lane & ((1 << (5 - kLog)) - 1)) == 0) dxr_w[(lane >> (5 - kLog)) & (kTM - 1)] = v[0];
}

template <int kStride, int kTM>
__global__ void __launch_bounds__(kB2Threads, 1) bwd2_kernel(Bwd2Params p) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint32_t* tab = reinterpret_cast<uint32_t*>(smem);                  // [kStride] I, [kStride] dI/dV
    float* gb = reinterpret_cast<float*>(smem + 8 * kStride);          // [2][kTM/2][opad][2]
    float* xb = gb + (size_t)2 * kTM * p.opad;                          // [2][3][kt][kTM]
    float* dxr = xb + 2 * 3 * p.kt * kTM;                               // [2][kB2Warps][cpw][kTM]
    float4* rng = reinterpret_cast<float4*>(dxr + 2 * kB2Warps * p.cpw * kTM);  // [2][kB2Warps]
    const int warp = threadIdx.x >> 5;
    float2* accw = reinterpret_cast<float2*>(rng + 2 * kB2Warps) + warp * kB2UMax * 32;  // this warp's dVth sums

    for (int i = threadIdx.x; i < p.T; i += kB2Threads) reinterpret_cast<uint2*>(tab)[i] = make_uint2(p.lut_i[i], p.lut_d[i]);
    // Pad outputs [O, opad) of both g buffers: zero once, never overwritten.
    for (int e = threadIdx.x; e < kTM * (p.opad - p.O); e += kB2Threads) {
        const int r = e / (p.opad - p.O), o = p.O + e % (p.opad - p.O);
        gb[((r >> 1) * p.opad + o) * 2 + (r & 1)] = 0.0f;
        gb[(size_t)kTM * p.opad + ((r >> 1) * p.opad + o) * 2 + (r & 1)] = 0.0f;
    }
    LutConsts lc;
    lc.tab_base = smem_u32addr(tab) - (kTwo23Bits << 3);
    lc.fmax_ = static_cast<float>(p.T - 1);
    lc.T = p.T;
    lc.dmin2 = pk2(p.dmin, p.dmin);
    lc.scale2 = pk2(p.scale, p.scale);
    lc.two23 = pk2(kTwo23, kTwo23);
    lc.inv = 0.0f;
    lc.vd = 0.0f;

    const int kk_w = warp / p.wpk, cb = warp - kk_w * p.wpk;  // column slot 0; slot cs adds cs * kB2Warps
    const int slot_units = (p.ncl + p.wpk - 1) / p.wpk;        // accumulator slots per column slot
    const int nslots = (p.kt * kTM + 31) >> 5;
    const uint32_t gb_s = smem_u32addr(gb);
    int buf = 0;
    for (int item = blockIdx.x; item < p.items; item += gridDim.x) {
        const int kg = item % p.kgroups, split = item / p.kgroups;
        const int k0 = kg * p.kt;
        const int tlo = (int)((int64_t)split * p.tiles_m / p.nsplit);
        const int thi = (int)((int64_t)(split + 1) * p.tiles_m / p.nsplit);
        float wmin = INFINITY, wmax = -INFINITY;
        bool wnan = false;
        for (int kk = 0; kk < p.kt && k0 + kk < p.K; ++kk) {
            const float4 r = __ldg(p.crange + k0 + kk);
            wmin = fminf(wmin, r.x);
            wmax = fmaxf(wmax, r.y);
            wnan |= r.z != 0.0f;
        }
        for (int s = 0; s < kB2UMax; ++s) accw[s * 32 + (threadIdx.x & 31)] = make_float2(0.0f, 0.0f);

        float xnext = 0.0f;  // x of the tile after the next one to stage
        if (tlo < thi) {
            b2_stage_g<kTM>(p, tlo, buf, gb);
            b2_store_x<kTM>(p, b2_load_x<kTM>(p, tlo, k0), tlo, buf, k0, xb, rng);
            if (tlo + 1 < thi) xnext = b2_load_x<kTM>(p, tlo + 1, k0);
        }
        for (int tile = tlo; tile < thi; ++tile) {
            cp_async_wait_all();
            __syncthreads();  // tile's g and x landed; buffer buf^1 and its dX slots are free
            if (tile > tlo) b2_finish_dx<kTM>(p, tile - 1, buf ^ 1, k0, dxr);
            if (tile + 1 < thi) {
                b2_stage_g<kTM>(p, tile + 1, buf ^ 1, gb);
                b2_store_x<kTM>(p, xnext, tile + 1, buf ^ 1, k0, xb, rng);
                if (tile + 2 < thi) xnext = b2_load_x<kTM>(p, tile + 2, k0);
            }
            float4 xr = rng[buf * kB2Warps];
            for (int s = 1; s < nslots; ++s) {
                const float4 q = rng[buf * kB2Warps + s];
                xr.x = fminf(xr.x, q.x);
                xr.y = fmaxf(xr.y, q.y);
                xr.z = fmaxf(xr.z, q.z);
            }
            const bool fast = tile_in_table(xr.x, xr.y, wmin, wmax, wnan || xr.z != 0.0f, p.dmin, p.scale, p.T);
            const uint32_t gt = gb_s + (uint32_t)(buf * kTM * p.opad * 4);
            const float* xs = xb + (size_t)buf * 3 * p.kt * kTM;
            if (p.cpw == 1) {  // straight-line path (a runtime slot loop here measured 6 % slower at 4-token tiles)
                const int k = k0 + kk_w;
                if (k < p.K) {
                    float* dxr_w = dxr + (buf * kB2Warps + warp) * kTM;
                    if (fast) {
                        b2_compute<false, kStride, kTM>(p, lc, k, kk_w, cb, gt, xs, accw, dxr_w);
                    } else {
                        b2_compute<true, kStride, kTM>(p, lc, k, kk_w, cb, gt, xs, accw, dxr_w);
                    }
                }
            } else {
                for (int cs = 0; cs < p.cpw; ++cs) {
                    const int kk = kk_w + cs * kB2Warps, k = k0 + kk;
                    if (k >= p.K) break;
                    float* dxr_w = dxr + ((buf * kB2Warps + warp) * p.cpw + cs) * kTM;
                    float2* acc_cs = accw + cs * slot_units * 32;
                    if (fast) {
                        b2_compute<false, kStride, kTM>(p, lc, k, kk, cb, gt, xs, acc_cs, dxr_w);
                    } else {
                        b2_compute<true, kStride, kTM>(p, lc, k, kk, cb, gt, xs, acc_cs, dxr_w);
                    }
                }
            }
            buf ^= 1;
        }
        __syncthreads();  // last tile's dX slots complete
        if (tlo < thi) b2_finish_dx<kTM>(p, thi - 1, buf ^ 1, k0, dxr);
        for (int cs = 0; p.part != nullptr && cs < p.cpw; ++cs) {
            const int k = k0 + kk_w + cs * kB2Warps;
            if (k >= p.K) break;
            const int lane = threadIdx.x & 31;
            for (int s = 0; s < slot_units; ++s) {
                const int cl = cb + s * p.wpk;
                if (cl < p.ncl) {
                    const int o = __ldg(p.co + (int64_t)k * p.opad + cl * 32 + lane);
                    if (o < p.O) {
                        const float2 v = accw[(cs * slot_units + s) * 32 + lane];
                        p.part[(((int64_t)split * 2 + 0) * p.O + o) * p.K + k] = v.x;
                        p.part[(((int64_t)split * 2 + 1) * p.O + o) * p.K + k] = v.y;
                    }
                }
            }
        }
    }
    cp_async_wait_all();
}
