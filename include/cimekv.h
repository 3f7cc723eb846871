/*
 * cimekv.h — C ABI of the B200 (sm_100a) Flash-EKV CIMLinear LUT operator.
 *
 * Plain pointers and sizes only; every tensor argument is a DEVICE pointer to
 * contiguous row-major fp32 data (bf16 bit patterns as uint16 for the raw
 * tables) on the device that is current when the call is made.  `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  Calls are
 * asynchronous with respect to the host and return a status code; the text of
 * the last error on the calling thread is available from cimekv_last_error().
 * The library allocates no device memory: outputs and the backward workspace
 * are owned by the caller.
 *
 * Shapes follow the reference operator: x[M,K] (tokens x in_features),
 * wpos/wneg[O,K] (threshold voltages, out_features x in_features),
 * out/grad_out[M,O].
 */
#ifndef CIMEKV_H
#define CIMEKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    CIMEKV_OK = 0,
    CIMEKV_EINVAL_SHAPE = 1,    /* bad sizes, null or misaligned pointers  */
    CIMEKV_ELUT_TOO_LARGE = 2,  /* table or tile does not fit shared memory */
    CIMEKV_ECUDA = 3,           /* a CUDA runtime call or launch failed     */
    CIMEKV_EWORKSPACE = 4       /* backward workspace too small             */
};

/* Largest LUT_DELTA_SIZE the kernels accept. */
#define CIMEKV_MAX_LUT_SIZE 16384

/* Version of the ABI (bumped on any signature or layout change). */
int cimekv_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* cimekv_last_error(void);

/* Bytes of the packed device table for a LUT of `table_size` entries. */
size_t cimekv_lut_bytes(int table_size);

/*
 * Pack the two bf16 tables (table_i = I(dV), table_ddelta = dI/ddV, each
 * `table_size` entries, the layout returned by the reference builder
 * get_ekv_lut_tables, src/isa/approximations/delta_lut.py:41-63) into the
 * layout the kernels stage in shared memory.  `lut` receives
 * cimekv_lut_bytes(table_size) bytes and must be 16-byte aligned.
 */
int cimekv_lut_pack(const uint16_t* table_i, const uint16_t* table_ddelta,
                    int table_size, void* lut, void* stream);

/*
 * Forward: out[m,o] = clamp(sum_k (L(x[m,k]-wpos[o,k]) - L(x[m,k]-wneg[o,k]))
 *                           / (1 + x[m,k]/v_sat), out_min, out_max)
 * with L the linear interpolation of table_i at
 *   f = clamp((dV - delta_min) * delta_scale, 0, T-1).
 * Replaces the reference Triton _forward_kernel launched by
 * LUTTritonEKVMatmulFn.forward (src/isa/kernels/transformer_ffn/
 * ekv_lut_triton.py:37-62,151-157); delta_scale = float((T-1)/(dmax-dmin)).
 * For launches with few output tiles the kernel splits the k range in two and
 * uses `out` as its accumulator (zeroed on `stream` first), so `out` must not
 * alias an input.  The same holds for the other forward entry points.
 */
int cimekv_forward(const float* x, const float* wpos, const float* wneg,
                   const void* lut, int M, int K, int O, int table_size,
                   float delta_min, float delta_scale, float v_sat,
                   float out_min, float out_max, float* out, void* stream);

/*
 * Forward with the TIA stage fused into the epilogue: besides
 * idiff = clamp(I_diff, idiff_min, idiff_max) (as cimekv_forward, may be NULL
 * when not needed) it writes out = clamp(idiff * (*r_tia), out_min, out_max),
 * the reference's `idiff * r_tia` then `clamp` done by torch in
 * CIMLinear.forward (src/isa/operators/cim.py:192-193).  r_tia is a DEVICE
 * pointer to one float, so a learnable gain needs no host synchronisation.
 */
int cimekv_forward_tia(const float* x, const float* wpos, const float* wneg,
                       const void* lut, int M, int K, int O, int table_size,
                       float delta_min, float delta_scale, float v_sat,
                       float idiff_min, float idiff_max, const float* r_tia,
                       float out_min, float out_max, float* idiff, float* out,
                       void* stream);

/* Workspace bytes of cimekv_tia_backward (a fixed, small number). */
size_t cimekv_tia_workspace_bytes(long long n);

/*
 * Backward of the TIA stage, one pass over n = M*O elements: with
 * v = idiff * r_tia, grad_idiff = [out_min <= v <= out_max] * grad_out * r_tia
 * and *grad_r_tia = sum [..] * grad_out * idiff (device scalar, deterministic
 * order).  Replaces the autograd of `idiff * r_tia` and `clamp` in the
 * reference's CIMLinear.forward (cim.py:192-193).
 */
int cimekv_tia_backward(const float* grad_out, const float* idiff, const float* r_tia,
                        long long n, float out_min, float out_max,
                        float* grad_idiff, float* grad_r_tia,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * Workspace bytes cimekv_backward needs for these sizes on the current device.
 */
size_t cimekv_backward_workspace_bytes(int M, int K, int O, int table_size);

/*
 * Fused backward, one pass over the (m,o,k) cells:
 *   grad_x[m,k]    = sum_o g[m,o] * ((dp-dn)/d - (bp-bn)/(v_sat d^2))
 *   grad_wpos[o,k] = sum_m g[m,o] * (-dp/d)
 *   grad_wneg[o,k] = sum_m g[m,o] * ( dn/d)
 * with d = 1 + x/v_sat, b* / d* the interpolated table_i / table_ddelta at
 * dV = x - w*.  Replaces the reference's two CUDA kernels
 * ekv_grad_x_shared_kernel and ekv_grad_w_shared_kernel
 * (src/isa/kernels/transformer_ffn/cuda/ekv_cuda.cu:193-341, host wrappers
 * :433-574, bound as grad_x_shared / grad_w_shared in cuda/binding.cpp:56-62).
 * grad_x may be NULL (no input gradient); grad_wpos and grad_wneg may both be
 * NULL (no threshold gradient).  The result is deterministic.
 * workspace: at least cimekv_backward_workspace_bytes(M, K, O, table_size)
 * bytes, 16-byte aligned.  It holds the per-token-split threshold partials
 * and, for layers of 256 to 4096 outputs, per input column the outputs
 * regrouped into clusters of close thresholds (so the table gathers of a warp
 * hit distinct shared-memory banks).
 * A call with grad_wpos == grad_wneg == NULL may pass workspace = NULL; it then
 * runs the unclustered kernel, whose grad_x differs from the clustered one in
 * fp32 summation order only.  Give the workspace to get the same bits as a
 * full call.
 */
int cimekv_backward(const float* x, const float* wpos, const float* wneg,
                    const float* grad_out, const void* lut,
                    int M, int K, int O, int table_size,
                    float delta_min, float delta_scale, float v_sat,
                    float* grad_x, float* grad_wpos, float* grad_wneg,
                    void* workspace, size_t workspace_bytes, void* stream);

/*
 * Exact-formula path (cfg ekv_approx != "lut"): the same forward and fused
 * backward with the EKV branch current evaluated per cell instead of looked up,
 *   I(dV) = I_S (sp(u1)^2 - sp(u2)^2),  u1 = dV*inv_2nut, u2 = (dV - V_D)*inv_2nut,
 *   sp(u) = u for u > 20, log(1 + e^u) otherwise,
 * out[m,o] = sum_k (I(x-wpos) - I(x-wneg)) / (1 + x/v_sat), unclamped.
 * Replaces the reference's exact Triton kernels _forward_kernel, _grad_x_kernel
 * and _grad_w_kernel (src/isa/kernels/transformer_ffn/ekv_triton.py:69-150),
 * reached through triton_ekv_matmul (ekv_triton.py:211-214, cim.py:186).
 */
int cimekv_exact_forward(const float* x, const float* wpos, const float* wneg,
                         int M, int K, int O, float inv_2nut, float v_d, float i_s,
                         float v_sat, float* out, void* stream);
size_t cimekv_exact_backward_workspace_bytes(int M, int K, int O);
int cimekv_exact_backward(const float* x, const float* wpos, const float* wneg,
                          const float* grad_out, int M, int K, int O,
                          float inv_2nut, float v_d, float i_s, float v_sat,
                          float* grad_x, float* grad_wpos, float* grad_wneg,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * Measured-codebook forward (DeploymentAwareCIMLinear "measured" mode,
 * src/isa/measured_deployment/operator.py:163-206; its fused Triton kernel
 * measured_deployment/kernels/measured_lut_triton.py:24-...).  Each device
 * (o,k) uses measured curve pos_idx[o,k] / neg_idx[o,k] (int16, S states); a
 * curve is piecewise linear over the strictly increasing grid vg[G], with
 * coef[s][j] = {slope, intercept} on segment j.  With x clamped to
 * [lookup_min, lookup_max] and j = searchsorted(vg, x, right) - 1:
 *   idiff[m,o] = sum_k x (a_p - a_n) + (b_p - b_n)       (may be NULL)
 *   out[m,o]   = clamp(idiff * (*r_tia), out_min, out_max)
 * S*(G-1) <= 16384.  r_tia is a device scalar.
 */
int cimekv_measured_forward(const float* x, const int16_t* pos_idx, const int16_t* neg_idx,
                            const float* vg, const float* coef, int M, int K, int O, int S, int G,
                            float lookup_min, float lookup_max, const float* r_tia,
                            float out_min, float out_max, float* idiff, float* out, void* stream);

/*
 * Input gradient of cimekv_measured_forward (the curves are fixed buffers, so
 * there is no threshold gradient; r_tia is detached as in the reference):
 *   grad_x[m,k] = [lookup_min <= x <= lookup_max]
 *                 * sum_o g[m,o] r [out_min <= idiff r <= out_max] (a_p - a_n)[j(x)]
 * The slopes (4 S (G-1) bytes) and the assignment of 4 inputs (16 O bytes)
 * are held in shared memory: CIMEKV_ELUT_TOO_LARGE when they exceed it
 * (O up to about 10000 with the largest codebook).
 */
int cimekv_measured_backward_x(const float* x, const int16_t* pos_idx, const int16_t* neg_idx,
                               const float* vg, const float* coef, int M, int K, int O, int S, int G,
                               float lookup_min, float lookup_max, const float* r_tia,
                               float out_min, float out_max, const float* idiff,
                               const float* grad_out, float* grad_x, void* stream);

/*
 * Index selection of one lookup, for parity tests: for each dV in delta[n],
 * writes the table entry i0 the kernels use and the interpolation weight a,
 * computed by the same device code as the forward and backward
 * (reference rule: ekv_lut_triton.py:26-31, ekv_cuda.cu:29-32).
 */
int cimekv_lut_index(const float* delta, int n, int table_size,
                     float delta_min, float delta_scale,
                     int32_t* index, float* alpha, void* stream);

/* Fixed device scratch of cimekv_backward_noalloc (32 MiB per GPU). */
#define CIMEKV_NOALLOC_SCRATCH_BYTES ((size_t)32 << 20)

/*
 * Allocation-free variant of cimekv_backward; it has no counterpart in the
 * reference.  Same arguments and results as cimekv_backward, minus the
 * workspace: the per-column output clusters and the token-split dVth partials
 * go to a scratch array compiled into this library (CIMEKV_NOALLOC_SCRATCH_BYTES of static device memory, held by
 * every GPU that loads the library until the process exits).  It is for callers
 * that cannot call cudaMalloc or an allocator around this operator — e.g. code
 * running under a memory pool it does not own, a host runtime with no device
 * allocator bound, or a plugin that must not grow the process's footprint per
 * call.  It allocates nothing and calls no allocating routine.
 *   - The first call on a device looks up the scratch's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.  The address is kept for the life of the
 *     process, so do not use the library across a cudaDeviceReset of that
 *     device (the reset ends the context the address belongs to).
 *   - Fails with CIMEKV_EWORKSPACE when 2*out_features*in_features*4 bytes
 *     exceed the scratch (out*in > 4,194,304); larger token counts only lower
 *     the number of token splits, never the result's correctness.
 *   - All calls share the one scratch: calls that may run at the same time on
 *     the GPU (different streams, different threads without ordering) race and
 *     give wrong dVth.  Calls ordered on one stream are safe.  Each call
 *     overwrites every scratch element it reads, so nothing needs clearing.
 *   - Results are identical to cimekv_backward's up to the order of the
 *     deterministic split reduction (which may use fewer splits).  Layers whose
 *     clusters (12*out*in bytes plus 16 per input) and one split do not fit
 *     the scratch together (out*in above ~1.6 M) run the unclustered kernel;
 *     their grad_x then differs from cimekv_backward's in fp32 summation order.
 */
int cimekv_backward_noalloc(const float* x, const float* wpos, const float* wneg,
                            const float* grad_out, const void* lut,
                            int M, int K, int O, int table_size,
                            float delta_min, float delta_scale, float v_sat,
                            float* grad_x, float* grad_wpos, float* grad_wneg, void* stream);

/*
 * Debug support, no counterpart in the reference.  cimekv_debug_build()
 * returns 1 for the library variant built with CIMEKV_DEBUG_BOUNDS=1
 * (libcimekv_debug.so), whose kernels check every table index against the
 * table size and count violations instead of reading out of bounds;
 * cimekv_debug_oob_count(reset) returns that count (synchronising with the
 * device; 0 in release builds) and optionally clears it.
 */
int cimekv_debug_build(void);
unsigned int cimekv_debug_oob_count(int reset);

/*
 * Measurement utility with no counterpart in the reference: launches `blocks`
 * CTAs of 256 threads that each issue iters*128 independent FFMAs, and
 * reports the lane-ops issued in *lane_ops.  Timed with events by the caller,
 * it gives the FP32 CUDA-core peak that the operator's roofline is quoted
 * against.  `sink` is a device float that is (almost) never written.
 */
int cimekv_fp32_probe(float* sink, int iters, int blocks, long long* lane_ops, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CIMEKV_H */
