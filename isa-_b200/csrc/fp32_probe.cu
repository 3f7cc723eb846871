// fp32_probe.cu — FFMA throughput probe: the measured denominator of the
// FP32 CUDA-core roofline the LUT kernels are reported against.
//
// Every thread runs 8 independent FFMA chains (enough ILP to issue one FFMA
// per cycle per scheduler); one FFMA is counted as one lane-op, the unit in
// which the operator's algorithmic work is counted.

#include <cuda_runtime.h>

#include "cimekv.h"

namespace {

__global__ void __launch_bounds__(256) ffma_probe_kernel(float* out, int iters, float a, float b) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = threadIdx.x * 1e-3f + j;
    for (int i = 0; i < iters; ++i) {
#pragma unroll
        for (int r = 0; r < 16; ++r) {
#pragma unroll
            for (int j = 0; j < 8; ++j) v[j] = fmaf(v[j], a, b);
        }
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += v[j];
    if (s == 12345.678f) out[0] = s;  // keeps the chains live
}

}  // namespace

extern "C" int cimekv_fp32_probe(float* sink, int iters, int blocks, long long* lane_ops, void* stream) {
    if (!sink || iters <= 0 || blocks <= 0 || !lane_ops) return CIMEKV_EINVAL_SHAPE;
    ffma_probe_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(sink, iters, 0.999999f, 1e-7f);
    *lane_ops = (long long)blocks * 256 * iters * 16 * 8;
    return cudaGetLastError() == cudaSuccess ? CIMEKV_OK : CIMEKV_ECUDA;
}
