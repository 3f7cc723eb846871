from isa_b200.kernels.transformer_ffn.ekv_lut import (  # noqa: F401
    LUTCudaEKVMatmulFn,
    LUTCudaEKVTIAFn,
    cuda_lut_ekv_matmul,
    cuda_lut_ekv_matmul_tia,
    triton_lut_ekv_matmul,
)
