"""Exact-formula CIM matmul (cfg ``ekv_approx != "lut"``) over the sm_100a kernels.

Drop-in for ``src/isa/kernels/transformer_ffn/ekv_triton.py:153-214``:
``triton_ekv_matmul(x[M,K], wpos[O,K], wneg[O,K], cfg) -> I_diff[M,O]`` with the
EKV current evaluated per cell (no table, no clamp), output in ``x.dtype`` like
the reference, gradients ``(dX, dWpos, dWneg, None)``.  Runs
``cimekv_exact_forward`` / ``cimekv_exact_backward``: the LUT kernels' tiling and
fused backward with the table lookup replaced by the formula.
"""

from __future__ import annotations

from typing import Any, Dict

import torch

from isa_b200 import _lib
from isa_b200.kernels.transformer_ffn.ekv_lut import _as_f32, _check_shapes


def _consts(cfg: Dict[str, Any]):
    inv = 1.0 / (2.0 * float(cfg["n"]) * float(cfg["U_T"]))
    return inv, float(cfg["V_D"]), float(cfg["I_S"]), float(cfg["V_sat"])


class CudaEKVMatmulFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, wpos, wneg, cfg):
        _check_shapes(x, wpos, wneg)
        x32, wp32, wn32 = _as_f32(x), _as_f32(wpos), _as_f32(wneg)
        inv, vd, i_s, v_sat = _consts(cfg)
        out = torch.empty((x32.shape[0], wp32.shape[0]), device=x.device, dtype=torch.float32)
        with torch.cuda.device(x.device):
            _lib.exact_forward(x32, wp32, wn32, inv, vd, i_s, v_sat, out)
        ctx.save_for_backward(x32, wp32, wn32)
        ctx.meta = (inv, vd, i_s, v_sat, x.dtype, wpos.dtype, wneg.dtype)
        return out.to(x.dtype)

    @staticmethod
    def backward(ctx, grad_out):
        x32, wp32, wn32 = ctx.saved_tensors
        inv, vd, i_s, v_sat, x_dt, wp_dt, wn_dt = ctx.meta
        need_x = ctx.needs_input_grad[0]
        need_w = ctx.needs_input_grad[1] or ctx.needs_input_grad[2]
        if not (need_x or need_w):
            return None, None, None, None
        g32 = _as_f32(grad_out)
        m, k = x32.shape
        o = wp32.shape[0]
        gx = torch.empty_like(x32) if need_x else None
        gwp = torch.empty_like(wp32) if need_w else None
        gwn = torch.empty_like(wn32) if need_w else None
        ws = None
        if need_w:
            ws = torch.empty(max(_lib.exact_backward_workspace_bytes(m, k, o), 16), dtype=torch.uint8,
                             device=x32.device)
        with torch.cuda.device(x32.device):
            _lib.exact_backward(x32, wp32, wn32, g32, inv, vd, i_s, v_sat, gx, gwp, gwn, ws)
        return (
            gx.to(x_dt) if gx is not None else None,
            gwp.to(wp_dt) if (gwp is not None and ctx.needs_input_grad[1]) else None,
            gwn.to(wn_dt) if (gwn is not None and ctx.needs_input_grad[2]) else None,
            None,
        )


def cuda_ekv_matmul(x: torch.Tensor, wpos: torch.Tensor, wneg: torch.Tensor, cfg: Dict[str, Any]) -> torch.Tensor:
    """Exact-formula I_diff[M,O] (reference ``ekv_triton.py:211-214``)."""
    return CudaEKVMatmulFn.apply(x, wpos, wneg, cfg)


# The reference's backend entry name.
triton_ekv_matmul = cuda_ekv_matmul
