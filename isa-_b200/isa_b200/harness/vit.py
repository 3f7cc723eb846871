"""Physical ViT training step — a caller of the CIM operator, for measurement.

Shape of the reference's vision model (``src/isa/vision/models.py:93-250``,
preset ``small``: d=384, 6 heads, MLP ratio 4, 12 blocks): convolutional patch
embedding, CLS token, learned positions, pre-LayerNorm blocks with a Physical
FFN (two CIMLinear, ``cim.py:217-247``), final LayerNorm and a linear head.
The step follows ``vision/train.py:146-232`` (fp16 autocast with GradScaler,
cross-entropy, clip 1.0, AdamW, ``clamp_vth``), MixUp/CutMix off; random-init weights,
synthetic images and labels.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from isa_b200.device_models.config import make_flash_transistor_ekv_config
from isa_b200.operators.cim import CIMLinear, PhysicalFFN


@dataclass
class ViTConfig:
    img_size: int = 224
    patch_size: int = 16
    num_classes: int = 200
    embed_dim: int = 384
    num_heads: int = 6
    depth: int = 12
    mlp_ratio: float = 4.0
    lut_size: int = 8192  # vision configs pin EKV_LUT_SIZE=8192


class ViTBlock(nn.Module):
    def __init__(self, cfg: ViTConfig, cim_cfg: dict):
        super().__init__()
        d = cfg.embed_dim
        self.heads = cfg.num_heads
        self.norm1 = nn.LayerNorm(d)
        self.qkv = nn.Linear(d, 3 * d)
        self.proj = nn.Linear(d, d)
        self.norm2 = nn.LayerNorm(d)
        self.mlp = PhysicalFFN(d, int(d * cfg.mlp_ratio), cim_cfg)

    def forward(self, x):
        b, t, d = x.shape
        q, k, v = self.qkv(self.norm1(x)).view(b, t, 3, self.heads, d // self.heads).unbind(2)
        a = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
        x = x + self.proj(a.transpose(1, 2).reshape(b, t, d))
        return x + self.mlp(self.norm2(x))


class PhysicalViT(nn.Module):
    def __init__(self, cfg: ViTConfig):
        super().__init__()
        cim_cfg = make_flash_transistor_ekv_config(default_lut_size=cfg.lut_size)
        cim_cfg["LUT_DELTA_SIZE"] = cfg.lut_size
        n = (cfg.img_size // cfg.patch_size) ** 2
        self.patch_embed = nn.Conv2d(3, cfg.embed_dim, cfg.patch_size, cfg.patch_size)
        self.cls_token = nn.Parameter(torch.zeros(1, 1, cfg.embed_dim))
        self.pos_embed = nn.Parameter(torch.zeros(1, n + 1, cfg.embed_dim))
        nn.init.trunc_normal_(self.pos_embed, std=0.02)
        nn.init.trunc_normal_(self.cls_token, std=0.02)
        self.blocks = nn.ModuleList(ViTBlock(cfg, cim_cfg) for _ in range(cfg.depth))
        self.norm = nn.LayerNorm(cfg.embed_dim)
        self.head = nn.Linear(cfg.embed_dim, cfg.num_classes)

    def forward(self, img):
        x = self.patch_embed(img).flatten(2).transpose(1, 2)
        x = torch.cat([self.cls_token.expand(x.shape[0], -1, -1), x], dim=1) + self.pos_embed
        for blk in self.blocks:
            x = blk(x)
        return self.head(self.norm(x)[:, 0])

    def cim_layers(self):
        return [m for m in self.modules() if isinstance(m, CIMLinear)]


def train_step(model, opt, scaler, images, labels, cim_layers):
    """One fp16-autocast step with loss scaling; returns the (device) loss."""
    opt.zero_grad(set_to_none=True)
    with torch.autocast("cuda", dtype=torch.float16):
        loss = F.cross_entropy(model(images).float(), labels)
    scaler.scale(loss).backward()
    scaler.unscale_(opt)
    torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)  # vision/train.py:202-204
    scaler.step(opt)
    scaler.update()
    for m in cim_layers:
        m.clamp_vth()
    return loss.detach()
