"""Measured-codebook deployment of the CIM fc1 layer on sm_100a.

Mirrors ``src/isa/measured_deployment/operator.py:21-249``:
``DeploymentAwareCIMLinear`` is a ``CIMLinear`` whose forward is
``continuous`` (the EKV LUT operator), ``measured`` (every device replaced by
one of S measured, piecewise-linear I-V curves; fixed buffers, gradient to the
input only) or ``ste`` (measured value, continuous gradient).  Parameter names
match ``CIMLinear`` so checkpoints stay compatible; the codebook and
assignment are non-persistent buffers with the reference's names.

The measured forward runs ``cimekv_measured_forward`` (per-cell coefficient
gather, fused ``* r_tia`` and clamp) and its input gradient
``cimekv_measured_backward_x``.  With ``vin_lut_bins > 0`` (binned inputs,
``operator.py:99-110,176-188``) every input is first replaced by the centre of
its bin with the reference's fp32 arithmetic, and the same kernel evaluates the
measured curves there: that is the reference's per-bin difference current
(``currents_at`` at the centre, pos minus neg device) summed over inputs.  As in
the reference, the binned output carries no gradient to the input (the bin
masks are not differentiable).
"""

from __future__ import annotations

from collections.abc import Iterable
from typing import ClassVar

import torch
from torch import nn

from isa_b200 import _lib
from isa_b200.operators.cim import CIMLinear


class _MeasuredFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, layer):
        flat = x.float().reshape(-1, layer.in_features).contiguous()
        m, o = flat.shape[0], layer.out_features
        idiff = torch.empty(m, o, device=x.device, dtype=torch.float32)
        out = torch.empty_like(idiff)
        r = layer.r_tia.detach().float().reshape(1).contiguous()
        lo, hi = float(layer.cfg.get("V_signed_min", -4.0)), float(layer.cfg.get("V_signed_max", 4.0))
        with torch.cuda.device(x.device):
            _lib.measured_forward(flat, layer.pos_idx, layer.neg_idx, layer.measured_vg, layer._coef,
                                  layer.lookup_min, layer.lookup_max, r, lo, hi, idiff, out)
        ctx.save_for_backward(flat, idiff, r)
        ctx.layer = layer
        ctx.meta = (lo, hi, x.shape, x.dtype)
        return out.reshape(*x.shape[:-1], o).to(x.dtype)

    @staticmethod
    def backward(ctx, grad_out):
        flat, idiff, r = ctx.saved_tensors
        layer = ctx.layer
        lo, hi, shape, dtype = ctx.meta
        if not ctx.needs_input_grad[0]:
            return None, None
        g = grad_out.float().reshape(idiff.shape).contiguous()
        gx = torch.empty_like(flat)
        with torch.cuda.device(flat.device):
            _lib.measured_backward_x(flat, layer.pos_idx, layer.neg_idx, layer.measured_vg, layer._coef,
                                     layer.lookup_min, layer.lookup_max, r, lo, hi, idiff, g, gx)
        return gx.reshape(shape).to(dtype), None


class DeploymentAwareCIMLinear(CIMLinear):
    """CIMLinear whose forward can be continuous, measured, or measured+STE."""

    MODES: ClassVar[set[str]] = {"continuous", "measured", "ste"}

    def __init__(self, in_features: int, out_features: int, physical_config=None) -> None:
        super().__init__(in_features, out_features, physical_config)
        self.forward_mode = "continuous"
        self.vin_lut_bins = 0
        self.lookup_min = float(self.cfg.get("V_min", 0.0))
        self.lookup_max = float(self.cfg.get("V_max", 4.0))
        for name in ("measured_vg", "measured_currents", "_coef", "bin_centers", "diff_current"):
            self.register_buffer(name, torch.empty(0), persistent=False)
        self.register_buffer("pos_idx", torch.empty(0, dtype=torch.int16), persistent=False)
        self.register_buffer("neg_idx", torch.empty(0, dtype=torch.int16), persistent=False)

    @classmethod
    def from_cimlinear(cls, original: CIMLinear) -> "DeploymentAwareCIMLinear":
        layer = cls(original.in_features, original.out_features, original.cfg)
        layer.load_state_dict(original.state_dict(), strict=True)
        return layer.to(device=original.vth_pos.device, dtype=original.vth_pos.dtype)

    def set_forward_mode(self, mode: str) -> None:
        if mode not in self.MODES:
            raise ValueError(f"Unsupported deployment-aware forward mode: {mode}")
        self.forward_mode = mode

    @torch.no_grad()
    def configure_codebook(self, vg: torch.Tensor, currents_a: torch.Tensor, vin_lut_bins: int = 0) -> None:
        """S measured curves ``currents_a[S, G]`` on the gate-voltage grid ``vg[G]``;
        ``vin_lut_bins > 0`` bins the inputs (reference ``operator.py:88-110``)."""
        dev = self.vth_pos.device
        vg = vg.detach().to(device=dev, dtype=torch.float32).contiguous()
        cur = currents_a.detach().to(device=dev, dtype=torch.float32).contiguous()
        if vg.ndim != 1 or cur.ndim != 2 or cur.shape[1] != vg.numel():
            raise ValueError("Measured codebook tensors have inconsistent shapes")
        if vg.numel() < 2 or not bool(torch.all(vg[1:] > vg[:-1])):
            raise ValueError("Measured Vg grid must be strictly increasing")
        self.measured_vg = vg
        self.measured_currents = cur
        self.lookup_min = max(float(vg[0]), float(self.cfg.get("V_min", 0.0)))
        self.lookup_max = min(float(vg[-1]), float(self.cfg.get("V_max", 4.0)))
        self.vin_lut_bins = int(vin_lut_bins)
        if self.vin_lut_bins < 0:
            raise ValueError("vin_lut_bins must be non-negative")
        # Per-segment slope and intercept of every curve, computed as in the
        # reference's set_assignment (operator.py:119-123).
        dv = vg[1:] - vg[:-1]
        slopes = (cur[:, 1:] - cur[:, :-1]) / dv.unsqueeze(0)
        intercepts = cur[:, :-1] - slopes * vg[:-1].unsqueeze(0)
        self._coef = torch.stack([slopes, intercepts], dim=-1).contiguous()  # [S][G-1][2]

    @torch.no_grad()
    def set_assignment(self, pos_idx: torch.Tensor, neg_idx: torch.Tensor) -> None:
        if self.measured_vg.numel() == 0:
            raise RuntimeError("configure_codebook must be called before set_assignment")
        expected = (self.out_features, self.in_features)
        if tuple(pos_idx.shape) != expected or tuple(neg_idx.shape) != expected:
            raise ValueError(f"Assignment shape must be {expected}")
        dev = self.vth_pos.device
        pos = pos_idx.to(device=dev, dtype=torch.int16).contiguous()
        neg = neg_idx.to(device=dev, dtype=torch.int16).contiguous()
        if int(pos.min()) < 0 or int(neg.min()) < 0:
            raise ValueError("Assignment contains negative state indices")
        states = int(self.measured_currents.shape[0])
        if int(pos.max()) >= states or int(neg.max()) >= states:
            raise ValueError("Assignment references a state outside the codebook")
        self.pos_idx, self.neg_idx = pos, neg
        if self.vin_lut_bins > 0:
            # Bin centres and the per-bin difference currents, as the reference
            # builds them (operator.py:99-110); the kernel evaluates the same
            # curves at the centres instead of reading diff_current.
            centers = torch.linspace(self.lookup_min, self.lookup_max, self.vin_lut_bins, device=dev,
                                     dtype=torch.float32)
            diff = torch.empty(self.vin_lut_bins, self.out_features, self.in_features, device=dev,
                               dtype=torch.float32)
            pl, nl = pos.long(), neg.long()
            for b in range(self.vin_lut_bins):
                cur = self.currents_at(centers[b])
                diff[b] = cur[pl] - cur[nl]
            self.bin_centers, self.diff_current = centers, diff
        else:
            self.bin_centers = torch.empty(0, device=dev)
            self.diff_current = torch.empty(0, device=dev)

    def _binned_inputs(self, x: torch.Tensor) -> torch.Tensor:
        """Every input replaced by its bin centre, with the reference's fp32 ops
        (clamp, (x - min) * (bins-1)/(max-min), round half to even, clamp)."""
        flat = x.float().clamp(self.lookup_min, self.lookup_max)
        if self.vin_lut_bins == 1:
            ids = torch.zeros_like(flat, dtype=torch.long)
        else:
            scale = (self.vin_lut_bins - 1) / (self.lookup_max - self.lookup_min)
            ids = torch.round((flat - self.lookup_min) * scale).long().clamp(0, self.vin_lut_bins - 1)
        return self.bin_centers[ids]

    def currents_at(self, voltage) -> torch.Tensor:
        """All S curves evaluated at ``voltage`` (reference ``operator.py:147-161``)."""
        if self.measured_vg.numel() == 0:
            raise RuntimeError("Measured codebook has not been configured")
        vg = self.measured_vg
        v = torch.as_tensor(voltage, device=vg.device, dtype=torch.float32).clamp(vg[0], vg[-1])
        upper = torch.searchsorted(vg, v, right=True).clamp(1, vg.numel() - 1)
        lower = upper - 1
        alpha = (v - vg[lower]) / (vg[upper] - vg[lower])
        cur = self.measured_currents
        return cur[:, lower] + alpha * (cur[:, upper] - cur[:, lower])

    def measured_forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.pos_idx.numel() == 0:
            raise RuntimeError("Measured assignment is not initialized")
        if not x.is_cuda:
            raise RuntimeError("measured forward needs a CUDA tensor")
        if self.vin_lut_bins > 0:
            with torch.no_grad():  # bin masks: no gradient to the input (reference behaviour)
                return _MeasuredFn.apply(self._binned_inputs(x.detach()), self).to(x.dtype)
        return _MeasuredFn.apply(x, self)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.forward_mode == "continuous":
            return super().forward(x)
        if self.forward_mode == "measured":
            return self.measured_forward(x)
        with torch.no_grad():
            measured = self.measured_forward(x)
        continuous = super().forward(x)
        return continuous + (measured - continuous).detach()


def replace_physical_fc1(model: nn.Module) -> list[DeploymentAwareCIMLinear]:
    """Swap ``blocks[i].mlp.fc1`` for the deployment-aware layer (reference operator.py:223-233)."""
    layers = []
    for i, block in enumerate(model.blocks):
        original = block.mlp.fc1
        if not isinstance(original, CIMLinear):
            raise TypeError(f"blocks.{i}.mlp.fc1 is not CIMLinear")
        block.mlp.fc1 = DeploymentAwareCIMLinear.from_cimlinear(original)
        layers.append(block.mlp.fc1)
    return layers


def iter_deployment_fc1(model: nn.Module) -> Iterable[tuple[int, DeploymentAwareCIMLinear]]:
    for i, block in enumerate(model.blocks):
        if not isinstance(block.mlp.fc1, DeploymentAwareCIMLinear):
            raise TypeError(f"blocks.{i}.mlp.fc1 is not deployment-aware")
        yield i, block.mlp.fc1


def set_fc1_forward_mode(model: nn.Module, mode: str) -> None:
    for _, layer in iter_deployment_fc1(model):
        layer.set_forward_mode(mode)
