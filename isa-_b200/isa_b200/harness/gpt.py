"""Physical GPT-2 training step — a caller of the CIM operator, for measurement.

Mirrors the shape of the reference's language model (``src/isa/language/
models.py:81-177``, preset ``small``: d=768, FFN 3072, 12 heads, 12 blocks,
vocab 50257, tied LM head): pre-LayerNorm blocks with causal scaled-dot-product
attention and a Physical FFN (VoltageMapping -> CIMLinear -> CIMLinear -> ADC
affine, ``cim.py:217-247``) in every block.  The training step follows the LM
phase of ``language/train.py:717-764``: bf16 autocast, cross-entropy,
backward, gradient clipping at 1.0, AdamW (lr 3e-4, betas (0.9, 0.999), no
weight decay on thresholds / TIA), then ``clamp_vth`` on every CIM layer.
Weights are random-init and inputs are synthetic token ids.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from isa_b200.device_models.config import make_flash_transistor_ekv_config
from isa_b200.operators.cim import CIMLinear, PhysicalFFN


@dataclass
class GPTConfig:
    vocab_size: int = 50257
    max_seq_len: int = 1024
    embed_dim: int = 768
    ffn_dim: int = 3072
    num_heads: int = 12
    depth: int = 12
    lut_size: int = 4096  # language configs pin EKV_LUT_SIZE=4096


class Block(nn.Module):
    def __init__(self, cfg: GPTConfig, cim_cfg: dict):
        super().__init__()
        self.heads = cfg.num_heads
        self.ln1 = nn.LayerNorm(cfg.embed_dim)
        self.qkv = nn.Linear(cfg.embed_dim, 3 * cfg.embed_dim)
        self.proj = nn.Linear(cfg.embed_dim, cfg.embed_dim)
        self.ln2 = nn.LayerNorm(cfg.embed_dim)
        self.ffn = PhysicalFFN(cfg.embed_dim, cfg.ffn_dim, cim_cfg)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, t, d = x.shape
        q, k, v = self.qkv(self.ln1(x)).view(b, t, 3, self.heads, d // self.heads).unbind(2)
        att = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                             is_causal=True)
        x = x + self.proj(att.transpose(1, 2).reshape(b, t, d))
        return x + self.ffn(self.ln2(x))


class PhysicalGPT(nn.Module):
    def __init__(self, cfg: GPTConfig):
        super().__init__()
        cim_cfg = make_flash_transistor_ekv_config(default_lut_size=cfg.lut_size)
        cim_cfg["LUT_DELTA_SIZE"] = cfg.lut_size
        self.cfg = cfg
        self.tok = nn.Embedding(cfg.vocab_size, cfg.embed_dim)
        self.pos = nn.Embedding(cfg.max_seq_len, cfg.embed_dim)
        self.blocks = nn.ModuleList(Block(cfg, cim_cfg) for _ in range(cfg.depth))
        self.ln_f = nn.LayerNorm(cfg.embed_dim)
        self.head = nn.Linear(cfg.embed_dim, cfg.vocab_size, bias=False)
        self.head.weight = self.tok.weight

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        pos = torch.arange(ids.shape[1], device=ids.device)
        x = self.tok(ids) + self.pos(pos)
        for blk in self.blocks:
            x = blk(x)
        return self.head(self.ln_f(x))

    def cim_layers(self):
        return [m for m in self.modules() if isinstance(m, CIMLinear)]

    def optimizer(self, lr: float = 3e-4) -> torch.optim.Optimizer:
        decay, no_decay = [], []
        for name, p in self.named_parameters():
            if p.dim() >= 2 and "vth_" not in name and not name.startswith(("tok", "head")):
                decay.append(p)
            else:
                no_decay.append(p)
        return torch.optim.AdamW([{"params": decay, "weight_decay": 0.0}, {"params": no_decay, "weight_decay": 0.0}],
                                 lr=lr, betas=(0.9, 0.999))


def train_step(model: nn.Module, opt: torch.optim.Optimizer, ids: torch.Tensor, cim_layers) -> torch.Tensor:
    """One LM-phase step; returns the (device) loss."""
    opt.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        logits = model(ids[:, :-1])
        loss = F.cross_entropy(logits.float().reshape(-1, logits.shape[-1]), ids[:, 1:].reshape(-1))
    loss.backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    opt.step()
    for m in cim_layers:
        m.clamp_vth()
    return loss.detach()
