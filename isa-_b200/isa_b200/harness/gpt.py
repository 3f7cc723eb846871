"""Physical GPT-2 training step — a caller of the CIM operator, for measurement.

The model is ``isa_b200.language.GPT2Model`` at the reference's ``small``
preset (d=768, FFN 3072, 12 heads, 12 blocks, vocab 50257, tied LM head;
``src/isa/language/config.py:31-37``) with ``model_type="physical"``: a Physical
FFN (VoltageMapping -> CIMLinear -> CIMLinear -> ADC affine) in every block,
its state-dict keys those of the reference GPT2Model.  The training step follows
the LM phase of ``language/train.py:717-764``: bf16 autocast, cross-entropy,
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
from isa_b200.language.models import GPT2Model, ModelConfig


@dataclass
class GPTConfig:
    vocab_size: int = 50257
    max_seq_len: int = 1024
    size: str = "small"
    lut_size: int = 4096  # language configs pin EKV_LUT_SIZE=4096


class PhysicalGPT(GPT2Model):
    def __init__(self, cfg: GPTConfig):
        cim_cfg = make_flash_transistor_ekv_config(default_lut_size=cfg.lut_size)
        cim_cfg["LUT_DELTA_SIZE"] = cfg.lut_size
        super().__init__(ModelConfig.from_preset(cfg.size, "physical", vocab_size=cfg.vocab_size,
                                                 max_seq_len=cfg.max_seq_len), cim_cfg)

    def optimizer(self, lr: float = 3e-4) -> torch.optim.Optimizer:
        return torch.optim.AdamW(self.configure_optimizer_groups(0.0, lr), lr=lr, betas=(0.9, 0.999))


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
