"""Bf16 lookup tables of the EKV branch current and its derivative over dV.

The table build restates the reference builder (``src/isa/approximations/
delta_lut.py:12-35``) step for step with the same torch CPU operations, so the
bf16 tables here are bit-identical to the reference's for the same cfg.  That
identity is what lets the kernels match the reference LUT path to fp32
rounding; the steps are therefore kept alike on purpose:

    delta    = linspace(dmin, dmax, T)                       (fp32)
    u1, u2   = delta / (2 n U_T), (delta - V_D) / (2 n U_T)
    base     = I_S (softplus(u1)^2 - softplus(u2)^2)
    ddelta   = I_S * 2/(2 n U_T) * (sp1 sig1 - sp2 sig2),  sig = 1 - exp(-sp)
    both rounded to bf16.

The dV range follows ``delta_lut.py:41-48``: ``LUT_DELTA_MIN`` defaults to
``V_signed_min - V_TH_MAX`` and ``LUT_DELTA_MAX`` to ``V_signed_max - V_TH_MIN``.

On top of the reference API (``get_ekv_lut_tables``) this module provides
``get_packed_lut``: the device-side table layout the sm_100a kernels stage into
shared memory, built on the GPU by ``cimekv_lut_pack`` and cached per
(device, table key).
"""

from __future__ import annotations

from dataclasses import dataclass
from functools import lru_cache
from typing import Any, Dict, Tuple

import numpy as np
import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class LutGeometry:
    """Where the table sits on the dV axis and how a dV maps onto an entry."""

    delta_min: float
    delta_max: float
    size: int

    @property
    def scale(self) -> float:
        """Entries per volt, rounded to fp32 exactly as the reference kernels do
        (``ekv_cuda.cu:371``: double quotient cast to float; Triton folds the same
        quotient as an fp32 constant, ``ekv_lut_triton.py:27``)."""
        return float(np.float32((self.size - 1) / (self.delta_max - self.delta_min)))

    @property
    def delta_min_f32(self) -> float:
        return float(np.float32(self.delta_min))


def lut_geometry(cfg: Dict[str, Any]) -> LutGeometry:
    """dV range and table size from a cfg dict (reference ``delta_lut.py:41-48``)."""
    v_min = float(cfg.get("LUT_V_MIN", cfg.get("V_signed_min", -4.0)))
    v_max = float(cfg.get("LUT_V_MAX", cfg.get("V_signed_max", 4.0)))
    vth_min = float(cfg.get("LUT_VTH_MIN", cfg.get("V_TH_MIN", 0.0)))
    vth_max = float(cfg.get("LUT_VTH_MAX", cfg.get("V_TH_MAX", 5.0)))
    delta_min = float(cfg.get("LUT_DELTA_MIN", v_min - vth_max))
    delta_max = float(cfg.get("LUT_DELTA_MAX", v_max - vth_min))
    size = int(cfg.get("LUT_DELTA_SIZE", 16384))
    if size < 2:
        raise ValueError(f"LUT_DELTA_SIZE must be >= 2, got {size}")
    if not delta_max > delta_min:
        raise ValueError(f"LUT dV range is empty: [{delta_min}, {delta_max}]")
    return LutGeometry(delta_min, delta_max, size)


def _table_key(cfg: Dict[str, Any]) -> Tuple:
    geo = lut_geometry(cfg)
    return (
        float(cfg["n"]),
        float(cfg["V_sat"]),
        float(cfg["I_S"]),
        float(cfg["U_T"]),
        float(cfg["V_D"]),
        geo.delta_min,
        geo.delta_max,
        geo.size,
    )


@lru_cache(maxsize=16)
def _cpu_lut_cached(key: Tuple) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 (base, d/dV) tables on the CPU for one table key."""
    n, _v_sat, i_s, u_t, v_d, delta_min, delta_max, size = key
    delta = torch.linspace(delta_min, delta_max, size, dtype=torch.float32)
    inv_2nut = 1.0 / (2.0 * n * u_t)
    sp1 = F.softplus(delta * inv_2nut)
    sp2 = F.softplus((delta - v_d) * inv_2nut)
    base = i_s * (sp1.square() - sp2.square())
    one = torch.ones_like(sp1)
    sig1 = torch.where(sp1 > 20.0, one, 1.0 - torch.exp(-sp1))
    sig2 = torch.where(sp2 > 20.0, one, 1.0 - torch.exp(-sp2))
    ddelta = i_s * 2.0 * inv_2nut * (sp1 * sig1 - sp2 * sig2)
    return base.contiguous().to(torch.bfloat16), ddelta.contiguous().to(torch.bfloat16)


def build_lut_tables_cpu(cfg: Dict[str, Any]) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 (table_i, table_ddelta) on the CPU for ``cfg``."""
    return _cpu_lut_cached(_table_key(cfg))


_device_tables: dict[Tuple, tuple[torch.Tensor, torch.Tensor]] = {}
_device_packed: dict[Tuple, torch.Tensor] = {}


def get_ekv_lut_tables(cfg: Dict[str, Any], device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """bf16 tables on ``device`` (same API as the reference ``delta_lut.py:41-63``)."""
    key = (str(torch.device(device)), _table_key(cfg))
    if key not in _device_tables:
        _device_tables[key] = tuple(t.to(device=device) for t in build_lut_tables_cpu(cfg))
    return _device_tables[key]


def get_packed_lut(cfg: Dict[str, Any], device: torch.device) -> torch.Tensor:
    """The kernels' packed table for ``cfg`` on CUDA ``device`` (cached).

    Packing runs on the GPU through ``cimekv_lut_pack`` so the layout is defined
    in exactly one place, the CUDA library.
    """
    from isa_b200 import _lib

    device = torch.device(device)
    key = (str(device), _table_key(cfg))
    packed = _device_packed.get(key)
    if packed is None:
        table_i, table_dd = get_ekv_lut_tables(cfg, device)
        size = table_i.numel()
        packed = torch.empty(_lib.lut_bytes(size), dtype=torch.uint8, device=device)
        with torch.cuda.device(device):
            _lib.lut_pack(table_i, table_dd, size, packed, torch.cuda.current_stream(device))
        _device_packed[key] = packed
    return packed
