"""CIM FFN operators backed by the sm_100a LUT kernels.

Drop-in for ``src/isa/operators/cim.py`` of the reference: the same classes
(``VoltageMapping``, ``CIMLinear``, ``PhysicalFFN``, ``HybridFFN``), constructor
arguments, parameter and buffer names (``vth_pos``, ``vth_neg``,
``r_tia_base``, ``r_tia_log_scale``; ``[out, in]`` fp32) and methods, so
reference state dicts load unchanged.

``CIMLinear.forward`` follows the reference GPU branch (``cim.py:180-199``):
I_diff from the LUT matmul, times the learnable TIA gain, clamped to the signed
output range, with autograd handling the gain and the clamp.  The reference's
CPU branch evaluates the exact EKV formula instead of the LUT and is not part
of this operator: CPU inputs raise.
"""

from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn as nn

from isa_b200.device_models.config import FLASH_TRANSISTOR_EKV_CONFIG as PHYSICAL_CONFIG
from isa_b200.kernels.transformer_ffn.ekv_exact import cuda_ekv_matmul
from isa_b200.kernels.transformer_ffn.ekv_lut import cuda_lut_ekv_matmul, cuda_lut_ekv_matmul_tia


class VoltageMapping(nn.Module):
    """Affine map of digital activations onto the gate-voltage range [0, voltage_max]
    (reference ``cim.py:23-39``)."""

    def __init__(self, voltage_max: float = 4.0):
        super().__init__()
        self.voltage_max = voltage_max
        self.scale = nn.Parameter(torch.tensor(1.0))
        self.shift = nn.Parameter(torch.tensor(0.0))

    @torch.no_grad()
    def set_affine(self, scale: float, shift: float) -> None:
        self.scale.fill_(float(scale))
        self.shift.fill_(float(shift))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        v = torch.clamp(x.float() * self.scale + self.shift, 0.0, self.voltage_max)
        return v.to(dtype=x.dtype)


def clamp_signed(v: torch.Tensor, v_min: float = -4.0, v_max: float = 4.0) -> torch.Tensor:
    return v.clamp(v_min, v_max)


def _uses_lut(cfg: Dict) -> bool:
    """The reference dispatch (cim.py:183-186): 'lut' -> LUT kernels, anything
    else -> exact-formula kernels."""
    return str(cfg.get("ekv_approx", "lut")).lower() == "lut"


class CIMLinear(nn.Module):
    """Crossbar linear layer: EKV differential current summed over inputs, then TIA.

    Same state as the reference ``CIMLinear`` (``cim.py:46-214``).
    """

    def __init__(self, in_features: int, out_features: int, physical_config: Optional[Dict[str, float]] = None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.cfg = dict(physical_config or PHYSICAL_CONFIG)

        self.vth_pos = nn.Parameter(torch.empty(out_features, in_features))
        self.vth_neg = nn.Parameter(torch.empty(out_features, in_features))
        self.register_buffer("r_tia_base", torch.full((1,), float(self.cfg.get("R_TIA", 1e5)), dtype=torch.float32))
        self.r_tia_log_scale = nn.Parameter(torch.zeros(1, dtype=torch.float32))
        self.track_output_stats = False
        self.register_buffer("_stat_total", torch.zeros((), dtype=torch.float64), persistent=False)
        self.register_buffer("_stat_clipped", torch.zeros((), dtype=torch.float64), persistent=False)
        self.register_buffer("_stat_abs_max", torch.zeros((), dtype=torch.float32), persistent=False)
        self.reset_vth(mode="centered_random", eps_k=0.5, symmetric=False)

    # -- TIA gain ---------------------------------------------------------
    @property
    def r_tia(self) -> torch.Tensor:
        lo = float(self.cfg.get("R_TIA_LOG_SCALE_MIN", -2.0))
        hi = float(self.cfg.get("R_TIA_LOG_SCALE_MAX", 2.0))
        return self.r_tia_base * torch.exp(self.r_tia_log_scale.clamp(lo, hi))

    def set_r_tia(self, value: float) -> None:
        with torch.no_grad():
            self.r_tia_base.fill_(float(value))
            self.r_tia_log_scale.zero_()

    # -- output statistics ------------------------------------------------
    def reset_output_stats(self) -> None:
        for buf in (self._stat_total, self._stat_clipped, self._stat_abs_max):
            buf.zero_()

    def set_output_stats_tracking(self, enabled: bool, reset: bool = False) -> None:
        self.track_output_stats = bool(enabled)
        if reset:
            self.reset_output_stats()

    def output_stats(self) -> Dict[str, float]:
        total = float(self._stat_total.item())
        clipped = float(self._stat_clipped.item())
        return {
            "total": total,
            "clipped": clipped,
            "clip_ratio": clipped / max(total, 1.0),
            "preclamp_abs_max": float(self._stat_abs_max.item()),
        }

    # -- threshold voltages -----------------------------------------------
    def reset_vth(
        self,
        center: float | torch.Tensor | None = None,
        eps_k: float = 0.5,
        symmetric: bool = True,
        mode: str = "centered_symmetric",
    ) -> None:
        """Uniform (random modes) or mirrored-Gaussian (symmetric) init around
        ``center`` with half-width ``eps_k * 2 n U_T`` (reference ``cim.py:113-138``)."""
        v_min = float(self.cfg["V_TH_MIN"])
        v_max = float(self.cfg["V_TH_MAX"])
        like = dict(device=self.vth_pos.device, dtype=self.vth_pos.dtype)
        if center is None:
            center_t = torch.tensor(0.5 * (v_min + v_max), **like)
        elif torch.is_tensor(center):
            center_t = center.to(**like)
        else:
            center_t = torch.tensor(float(center), **like)
        center_t = center_t.clamp(v_min, v_max)
        eps = float(eps_k) * 2.0 * float(self.cfg["n"]) * float(self.cfg["U_T"])
        with torch.no_grad():
            if mode in {"random", "centered_random"} or not symmetric:
                self.vth_pos.uniform_(-eps, eps).add_(center_t)
                self.vth_neg.uniform_(-eps, eps).add_(center_t)
            else:
                noise = torch.empty_like(self.vth_pos).normal_(0.0, eps)
                self.vth_pos.copy_(center_t + noise)
                self.vth_neg.copy_(center_t - noise)
            self.clamp_vth()

    def clamp_vth(self) -> None:
        with torch.no_grad():
            self.vth_pos.clamp_(self.cfg["V_TH_MIN"], self.cfg["V_TH_MAX"])
            self.vth_neg.clamp_(self.cfg["V_TH_MIN"], self.cfg["V_TH_MAX"])

    # -- compute ------------------------------------------------------------
    @torch.no_grad()
    def estimate_idiff(self, x: torch.Tensor, max_rows: int = 4096) -> torch.Tensor:
        """I_diff of the first ``max_rows`` rows, without TIA (reference ``cim.py:140-163``)."""
        flat = x.reshape(-1, self.in_features)
        flat = flat[:max_rows].contiguous()
        if _uses_lut(self.cfg):
            return cuda_lut_ekv_matmul(flat, self.vth_pos, self.vth_neg, self.cfg)
        return cuda_ekv_matmul(flat, self.vth_pos, self.vth_neg, self.cfg)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, n, in_f = x.shape
        if in_f != self.in_features:
            raise ValueError(f"expected {self.in_features} input features, got {in_f}")
        r_tia = self.r_tia.to(device=x.device, dtype=torch.float32)
        flat = x.reshape(b * n, in_f)
        if _uses_lut(self.cfg):
            # I_diff, * R_TIA and the signed clamp in one fused kernel (reference:
            # LUT matmul, then `* r_tia` and `clamp` in torch).
            out = cuda_lut_ekv_matmul_tia(flat, self.vth_pos, self.vth_neg, r_tia, self.cfg)
        else:
            v_lo = float(self.cfg.get("V_signed_min", -4.0))
            v_hi = float(self.cfg.get("V_signed_max", 4.0))
            out = (cuda_ekv_matmul(flat, self.vth_pos, self.vth_neg, self.cfg) * r_tia).clamp(v_lo, v_hi)
        out = out.view(b, n, self.out_features)
        if self.track_output_stats:
            with torch.no_grad():
                self._stat_total.add_(out.numel())
                self._stat_abs_max.copy_(torch.maximum(self._stat_abs_max, out.detach().abs().max().float()))
        return out


class PhysicalFFN(nn.Module):
    """VoltageMapping -> CIMLinear -> CIMLinear -> per-channel ADC affine
    (reference ``cim.py:217-247``)."""

    def __init__(self, dim: int, hidden_dim: int, physical_config: Optional[Dict[str, float]] = None,
                 voltage_max: float = 4.0):
        super().__init__()
        self.input_mapping = VoltageMapping(voltage_max=voltage_max)
        self.fc1 = CIMLinear(dim, hidden_dim, physical_config)
        self.fc2 = CIMLinear(hidden_dim, dim, physical_config)
        self.adc_affine_scale = nn.Parameter(torch.ones(dim))
        self.adc_affine_shift = nn.Parameter(torch.zeros(dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h = self.fc2(self.fc1(self.input_mapping(x)))
        return h * self.adc_affine_scale + self.adc_affine_shift

    def clamp_vth(self) -> None:
        self.fc1.clamp_vth()
        self.fc2.clamp_vth()


class HybridFFN(nn.Module):
    """VoltageMapping -> CIMLinear -> digital nn.Linear (reference ``cim.py:250-280``)."""

    def __init__(self, dim: int, hidden_dim: int, physical_config: Optional[Dict[str, float]] = None,
                 voltage_max: float = 4.0):
        super().__init__()
        self.input_mapping = VoltageMapping(voltage_max=voltage_max)
        self.fc1 = CIMLinear(dim, hidden_dim, physical_config)
        self.fc2 = nn.Linear(hidden_dim, dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.fc2(self.fc1(self.input_mapping(x)))

    def clamp_vth(self) -> None:
        self.fc1.clamp_vth()
