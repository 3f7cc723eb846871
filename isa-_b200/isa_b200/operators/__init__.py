from isa_b200.operators.cim import (  # noqa: F401
    CIMLinear,
    HybridFFN,
    PhysicalFFN,
    VoltageMapping,
    clamp_signed,
)
