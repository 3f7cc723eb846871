from isa_b200.kernels.transformer_ffn.ekv_lut import (  # noqa: F401
    LUTCudaEKVMatmulFn,
    cuda_lut_ekv_matmul,
    triton_lut_ekv_matmul,
)
