"""B200-native (sm_100a) Flash-EKV CIMLinear operator.

A drop-in for the LUT hot path of ISA's compute-in-memory FFN: the
``CIMLinear`` module (``isa.operators.cim``), its backend entry
``triton_lut_ekv_matmul`` and the LUT builder, backed by hand-written CUDA
kernels behind the C ABI declared in ``include/cimekv.h``.
"""

from isa_b200.device_models.config import (  # noqa: F401
    FLASH_TRANSISTOR_EKV_CONFIG,
    FLASH_TRANSISTOR_PARAMETERS,
    make_flash_transistor_ekv_config,
)

__all__ = [
    "FLASH_TRANSISTOR_EKV_CONFIG",
    "FLASH_TRANSISTOR_PARAMETERS",
    "make_flash_transistor_ekv_config",
]
