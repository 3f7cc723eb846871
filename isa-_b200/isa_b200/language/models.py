"""GPT-2 models whose FFN is the CIM operator: the callers of the hot path on the
language side.

Drop-in for ``src/isa/language/models.py`` and ``language/config.py`` of the
reference at the level of module names, constructor arguments and state-dict
keys, so a reference checkpoint loads unchanged:

* ``HybridFFN`` (``models.py:48-63``): VoltageMapping -> ``cim1`` (CIMLinear,
  up projection) -> ``fc2`` (digital nn.Linear) -> per-channel ADC affine ->
  dropout.  This is the GPT-side hybrid block; the operator-level
  ``isa_b200.operators.cim.HybridFFN`` (fc1/fc2, no affine) is a different
  module, as in the reference.
* ``GPT2PhysicalFFN`` (``models.py:66-74``): ``cim_ffn`` = the operator-level
  PhysicalFFN (VoltageMapping -> CIMLinear -> CIMLinear -> ADC affine), then
  dropout.
* ``GPT2Block`` / ``GPT2Model`` (``models.py:81-177``): pre-LayerNorm blocks,
  causal scaled-dot-product attention over the weights of an
  ``nn.MultiheadAttention`` (used as the parameter container, keys
  ``attn.in_proj_weight`` / ``attn.out_proj.*``), token + position embeddings,
  tied LM head.

The CIM layers run on this package's sm_100a kernels; everything else is
plain PyTorch.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from isa_b200.device_models.config import make_flash_transistor_ekv_config
from isa_b200.operators.cim import CIMLinear, PhysicalFFN, VoltageMapping

# The language experiments pin the table size to 4096 (reference config.py:13;
# EKV_LUT_SIZE in the environment still overrides it).
PHYSICAL_CONFIG = make_flash_transistor_ekv_config(default_lut_size=4096)

# Model size presets (reference config.py:16-38): embed dim, FFN dim, heads, depth.
SIZE_PRESETS: Dict[str, Dict] = {
    "tiny": dict(embed_dim=192, ffn_dim=768, num_heads=3, depth=12, dropout=0.0),
    "mid": dict(embed_dim=384, ffn_dim=1536, num_heads=6, depth=12, dropout=0.0),
    "small": dict(embed_dim=768, ffn_dim=3072, num_heads=12, depth=12, dropout=0.0),
}


@dataclass
class ModelConfig:
    """Architecture of a GPT-2 model (field names of the reference ModelConfig)."""

    size: str = "tiny"
    model_type: str = "standard"  # "standard" | "hybrid" | "physical"
    vocab_size: int = 50257
    max_seq_len: int = 128
    embed_dim: int = 192
    ffn_dim: int = 768
    num_heads: int = 3
    depth: int = 12
    dropout: float = 0.0
    voltage_max: float = 4.0
    affine_scope: str = "final"
    output_chunk_size: int = 16

    @classmethod
    def from_preset(cls, size: str, model_type: str, **kwargs) -> "ModelConfig":
        return cls(size=size, model_type=model_type, **SIZE_PRESETS[size], **kwargs)


class StandardFFN(nn.Module):
    """Digital FFN (Linear -> GELU -> Linear), the baseline the CIM variants replace."""

    def __init__(self, embed_dim: int, ffn_dim: int, dropout: float = 0.0):
        super().__init__()
        self.fc1 = nn.Linear(embed_dim, ffn_dim)
        self.fc2 = nn.Linear(ffn_dim, embed_dim)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc2(self.dropout(F.gelu(self.fc1(x))))


class HybridFFN(nn.Module):
    """CIM up projection, digital down projection, ADC affine."""

    def __init__(self, embed_dim: int, ffn_dim: int, voltage_max: float = 4.0, dropout: float = 0.0):
        super().__init__()
        self.input_mapping = VoltageMapping(voltage_max=voltage_max)
        self.cim1 = CIMLinear(embed_dim, ffn_dim)
        self.fc2 = nn.Linear(ffn_dim, embed_dim)
        self.adc_affine_scale = nn.Parameter(torch.ones(embed_dim))
        self.adc_affine_shift = nn.Parameter(torch.zeros(embed_dim))
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.fc2(self.cim1(self.input_mapping(x)))
        return self.dropout(h * self.adc_affine_scale + self.adc_affine_shift)


class GPT2PhysicalFFN(nn.Module):
    """Both projections on the CIM operator (the operator-level PhysicalFFN)."""

    def __init__(self, embed_dim: int, ffn_dim: int, voltage_max: float = 4.0, dropout: float = 0.0,
                 physical_config: Optional[Dict] = None):
        super().__init__()
        self.cim_ffn = PhysicalFFN(embed_dim, ffn_dim, physical_config or PHYSICAL_CONFIG, voltage_max)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.dropout(self.cim_ffn(x))


class GPT2Block(nn.Module):
    """Pre-LayerNorm transformer block: causal attention, then the FFN variant."""

    def __init__(self, embed_dim: int, ffn_dim: int, num_heads: int, model_type: str, voltage_max: float = 4.0,
                 dropout: float = 0.0, physical_config: Optional[Dict] = None):
        super().__init__()
        if embed_dim % num_heads:
            raise ValueError(f"embed_dim={embed_dim} must be divisible by num_heads={num_heads}")
        self.num_heads = num_heads
        self.head_dim = embed_dim // num_heads
        self.ln1 = nn.LayerNorm(embed_dim)
        # parameter container only (in_proj_weight/bias, out_proj); the forward
        # calls scaled_dot_product_attention on these weights directly
        self.attn = nn.MultiheadAttention(embed_dim, num_heads, dropout=dropout, batch_first=True)
        self.ln2 = nn.LayerNorm(embed_dim)
        if model_type == "standard":
            self.ffn = StandardFFN(embed_dim, ffn_dim, dropout)
        elif model_type == "hybrid":
            self.ffn = HybridFFN(embed_dim, ffn_dim, voltage_max, dropout)
        elif model_type == "physical":
            self.ffn = GPT2PhysicalFFN(embed_dim, ffn_dim, voltage_max, dropout, physical_config)
        else:
            raise ValueError(f"Unknown model_type: {model_type}")

    def attention(self, x: torch.Tensor) -> torch.Tensor:
        b, t, d = x.shape
        qkv = F.linear(self.ln1(x), self.attn.in_proj_weight, self.attn.in_proj_bias)
        q, k, v = (h.transpose(1, 2) for h in qkv.view(b, t, 3, self.num_heads, self.head_dim).unbind(2))
        p = float(self.attn.dropout) if self.training else 0.0
        y = F.scaled_dot_product_attention(q, k, v, dropout_p=p, is_causal=True)
        return F.linear(y.transpose(1, 2).reshape(b, t, d), self.attn.out_proj.weight, self.attn.out_proj.bias)

    def forward(self, x: torch.Tensor, need_intermediate: bool = False):
        x = x + self.attention(x)
        ffn_out = self.ffn(self.ln2(x))
        out = x + ffn_out
        if need_intermediate:
            return out, {"ffn_output": ffn_out, "block_output": out}
        return out


class GPT2Model(nn.Module):
    """GPT-2 with the FFN variant of ``cfg.model_type`` in every block."""

    def __init__(self, cfg: ModelConfig, physical_config: Optional[Dict] = None):
        super().__init__()
        self.cfg = cfg
        self.token_embedding = nn.Embedding(cfg.vocab_size, cfg.embed_dim)
        self.pos_embedding = nn.Embedding(cfg.max_seq_len, cfg.embed_dim)
        self.drop = nn.Dropout(cfg.dropout)
        self.blocks = nn.ModuleList(
            GPT2Block(cfg.embed_dim, cfg.ffn_dim, cfg.num_heads, cfg.model_type, cfg.voltage_max, cfg.dropout,
                      physical_config)
            for _ in range(cfg.depth))
        self.ln_f = nn.LayerNorm(cfg.embed_dim)
        self.lm_head = nn.Linear(cfg.embed_dim, cfg.vocab_size, bias=False)
        self.lm_head.weight = self.token_embedding.weight
        self.register_buffer("pos_ids", torch.arange(cfg.max_seq_len).unsqueeze(0), persistent=False)

    def forward(self, input_ids: torch.Tensor, need_intermediate: bool = False):
        b, t = input_ids.shape
        x = self.drop(self.token_embedding(input_ids) + self.pos_embedding(self.pos_ids[:, :t].expand(b, -1)))
        inter: List[Dict[str, torch.Tensor]] = []
        for blk in self.blocks:
            if need_intermediate:
                x, info = blk(x, need_intermediate=True)
                inter.append(info)
            else:
                x = blk(x)
        logits = self.lm_head(self.ln_f(x))
        return (logits, inter) if need_intermediate else logits

    def cim_layers(self) -> List[CIMLinear]:
        return [m for m in self.modules() if isinstance(m, CIMLinear)]

    def configure_optimizer_groups(self, weight_decay: float, lr: float, ffn_only: bool = False):
        """AdamW groups: thresholds, TIA gains, embeddings / LM head and 1-D
        parameters take no weight decay (reference models.py:179-201)."""
        decay, no_decay = [], []
        for name, p in self.named_parameters():
            if not p.requires_grad or (ffn_only and ".ffn." not in name):
                continue
            exempt = name.startswith(("lm_head", "token_embedding")) or "vth_" in name or "r_tia" in name
            (no_decay if exempt or p.dim() < 2 else decay).append(p)
        return [{"params": decay, "weight_decay": weight_decay, "lr": lr},
                {"params": no_decay, "weight_decay": 0.0, "lr": lr}]


def create_model(cfg: ModelConfig, physical_config: Optional[Dict] = None) -> GPT2Model:
    return GPT2Model(cfg, physical_config)
