"""Backend entry of the LUT CIM matmul: autograd Function over the sm_100a kernels.

Drop-in for ``src/isa/kernels/transformer_ffn/ekv_lut_triton.py:131-224``:
``triton_lut_ekv_matmul(x[M,K], wpos[O,K], wneg[O,K], cfg) -> idiff[M,O]`` in
fp32, clamped to ``[V_signed_min, V_signed_max]`` like the reference forward
kernel, with a backward that returns ``(dX, dWpos, dWneg, None)`` cast to the
input dtypes.  The forward runs ``cimekv_forward``; the backward runs the fused
``cimekv_backward`` (dX and dVth from one pass over the cells), which replaces
both the reference's CUDA shared-memory kernels and its Triton fallback, so the
``CUDA_SHARED_BACKWARD`` switch has nothing left to select.
"""

from __future__ import annotations

from typing import Any, Dict

import torch

from isa_b200 import _lib
from isa_b200.approximations.delta_lut import get_packed_lut, lut_geometry


def _as_f32(t: torch.Tensor) -> torch.Tensor:
    return t.to(dtype=torch.float32).contiguous()


def _check_shapes(x: torch.Tensor, wpos: torch.Tensor, wneg: torch.Tensor) -> None:
    if x.dim() != 2 or wpos.dim() != 2 or wneg.dim() != 2:
        raise RuntimeError("expected x[M,K], wpos[O,K], wneg[O,K]")
    if wpos.shape != wneg.shape or wpos.shape[1] != x.shape[1]:
        raise RuntimeError(f"shape mismatch: x {tuple(x.shape)}, wpos {tuple(wpos.shape)}, wneg {tuple(wneg.shape)}")
    for t, name in ((x, "x"), (wpos, "wpos"), (wneg, "wneg")):
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor: the LUT CIM matmul has no CPU implementation")
        if t.device != x.device:
            raise RuntimeError("x, wpos and wneg must be on the same device")


class LUTCudaEKVMatmulFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x: torch.Tensor, wpos: torch.Tensor, wneg: torch.Tensor, cfg: Dict[str, Any]):
        _check_shapes(x, wpos, wneg)
        geo = lut_geometry(cfg)
        lut = get_packed_lut(cfg, x.device)
        x32, wp32, wn32 = _as_f32(x), _as_f32(wpos), _as_f32(wneg)
        m, _ = x32.shape
        o = wp32.shape[0]
        out = torch.empty((m, o), device=x.device, dtype=torch.float32)
        v_sat = float(cfg["V_sat"])
        out_min = float(cfg.get("V_signed_min", -4.0))
        out_max = float(cfg.get("V_signed_max", 4.0))
        with torch.cuda.device(x.device):
            _lib.forward(x32, wp32, wn32, lut, geo.size, geo.delta_min_f32, geo.scale, v_sat,
                         out_min, out_max, out)
        ctx.save_for_backward(x32, wp32, wn32)
        ctx.meta = (geo.size, geo.delta_min_f32, geo.scale, v_sat, x.dtype, wpos.dtype, wneg.dtype)
        ctx.lut = lut
        return out

    @staticmethod
    def backward(ctx, grad_out: torch.Tensor):
        x32, wp32, wn32 = ctx.saved_tensors
        size, dmin, scale, v_sat, x_dtype, wp_dtype, wn_dtype = ctx.meta
        need_x = ctx.needs_input_grad[0]
        need_w = ctx.needs_input_grad[1] or ctx.needs_input_grad[2]
        if not (need_x or need_w):
            return None, None, None, None
        g32 = _as_f32(grad_out)
        m, k = x32.shape
        o = wp32.shape[0]
        grad_x = torch.empty_like(x32) if need_x else None
        grad_wp = torch.empty_like(wp32) if need_w else None
        grad_wn = torch.empty_like(wn32) if need_w else None
        # The workspace holds the per-column output clusters as well as the dVth
        # partials, so it is passed for dX-only calls too (same kernel, same bits).
        ws = _lib.backward_workspace_bytes(m, k, o, size)
        workspace = torch.empty(max(ws, 16), dtype=torch.uint8, device=x32.device)
        with torch.cuda.device(x32.device):
            _lib.backward(x32, wp32, wn32, g32, ctx.lut, size, dmin, scale, v_sat,
                          grad_x, grad_wp, grad_wn, workspace)
        return (
            grad_x.to(x_dtype) if grad_x is not None else None,
            grad_wp.to(wp_dtype) if (grad_wp is not None and ctx.needs_input_grad[1]) else None,
            grad_wn.to(wn_dtype) if (grad_wn is not None and ctx.needs_input_grad[2]) else None,
            None,
        )


class LUTCudaEKVTIAFn(torch.autograd.Function):
    """LUT CIM matmul with the TIA stage fused: returns
    ``clamp(I_diff * r_tia, V_signed_min, V_signed_max)`` — the reference's
    ``triton_lut_ekv_matmul`` followed by ``* r_tia`` and ``clamp`` in
    ``CIMLinear.forward`` (``cim.py:184-193``) — with gradients for x, both
    threshold tensors and ``r_tia``."""

    @staticmethod
    def forward(ctx, x, wpos, wneg, r_tia, cfg):
        _check_shapes(x, wpos, wneg)
        geo = lut_geometry(cfg)
        lut = get_packed_lut(cfg, x.device)
        x32, wp32, wn32 = _as_f32(x), _as_f32(wpos), _as_f32(wneg)
        r32 = r_tia.detach().to(device=x.device, dtype=torch.float32).reshape(1).contiguous()
        m, o = x32.shape[0], wp32.shape[0]
        idiff = torch.empty((m, o), device=x.device, dtype=torch.float32)
        out = torch.empty_like(idiff)
        v_lo = float(cfg.get("V_signed_min", -4.0))
        v_hi = float(cfg.get("V_signed_max", 4.0))
        v_sat = float(cfg["V_sat"])
        with torch.cuda.device(x.device):
            _lib.forward_tia(x32, wp32, wn32, lut, geo.size, geo.delta_min_f32, geo.scale, v_sat, v_lo, v_hi,
                             r32, v_lo, v_hi, idiff, out)
        ctx.save_for_backward(x32, wp32, wn32, idiff, r32)
        ctx.meta = (geo.size, geo.delta_min_f32, geo.scale, v_sat, v_lo, v_hi, x.dtype, wpos.dtype, wneg.dtype,
                    r_tia.dtype, r_tia.shape)
        ctx.lut = lut
        return out

    @staticmethod
    def backward(ctx, grad_out):
        x32, wp32, wn32, idiff, r32 = ctx.saved_tensors
        size, dmin, scale, v_sat, v_lo, v_hi, x_dt, wp_dt, wn_dt, r_dt, r_shape = ctx.meta
        g32 = _as_f32(grad_out)
        g_idiff = torch.empty_like(idiff)
        grad_r = torch.empty(1, device=idiff.device, dtype=torch.float32)
        with torch.cuda.device(idiff.device):
            _lib.tia_backward(g32, idiff, r32, v_lo, v_hi, g_idiff, grad_r)
        need_x = ctx.needs_input_grad[0]
        need_w = ctx.needs_input_grad[1] or ctx.needs_input_grad[2]
        grad_x = grad_wp = grad_wn = None
        if need_x or need_w:
            m, k = x32.shape
            o = wp32.shape[0]
            grad_x = torch.empty_like(x32) if need_x else None
            grad_wp = torch.empty_like(wp32) if need_w else None
            grad_wn = torch.empty_like(wn32) if need_w else None
            ws = torch.empty(max(_lib.backward_workspace_bytes(m, k, o, size), 16), dtype=torch.uint8,
                             device=x32.device)
            with torch.cuda.device(x32.device):
                _lib.backward(x32, wp32, wn32, g_idiff, ctx.lut, size, dmin, scale, v_sat,
                              grad_x, grad_wp, grad_wn, ws)
        return (
            grad_x.to(x_dt) if grad_x is not None else None,
            grad_wp.to(wp_dt) if (grad_wp is not None and ctx.needs_input_grad[1]) else None,
            grad_wn.to(wn_dt) if (grad_wn is not None and ctx.needs_input_grad[2]) else None,
            grad_r.to(r_dt).reshape(r_shape) if ctx.needs_input_grad[3] else None,
            None,
        )


def cuda_lut_ekv_matmul_tia(x: torch.Tensor, wpos: torch.Tensor, wneg: torch.Tensor, r_tia: torch.Tensor,
                            cfg: Dict[str, Any]) -> torch.Tensor:
    """clamp(I_diff * r_tia, V_signed_min, V_signed_max) with the TIA stage fused."""
    return LUTCudaEKVTIAFn.apply(x, wpos, wneg, r_tia, cfg)


def cuda_lut_ekv_matmul(x: torch.Tensor, wpos: torch.Tensor, wneg: torch.Tensor,
                        cfg: Dict[str, Any]) -> torch.Tensor:
    """I_diff[M,O] of the LUT CIM matmul (reference ``ekv_lut_triton.py:221-224``)."""
    return LUTCudaEKVMatmulFn.apply(x, wpos, wneg, cfg)


# The reference's backend entry name, so callers that import it keep working.
triton_lut_ekv_matmul = cuda_lut_ekv_matmul
