"""GPT-2 language models built on the CIM operator (reference ``src/isa/language``)."""

from isa_b200.language.models import (  # noqa: F401
    GPT2Block,
    GPT2Model,
    GPT2PhysicalFFN,
    HybridFFN,
    ModelConfig,
    StandardFFN,
    SIZE_PRESETS,
    create_model,
)
