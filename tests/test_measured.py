"""Measured-codebook deployment path: the fp64 oracle pinned to the reference's
own CPU code (golden vectors) and its unit test; the sm_100a kernels against both."""

import numpy as np
import pytest
import torch

from oracle import measured as mref
from tests._util import assert_close_scaled, load_golden

CASES = ["measured_small", "measured_ragged"]


def _args(g):
    return g["vg"], g["currents"], g["pos"], g["neg"], float(g["lookup_min"]), float(g["lookup_max"]), float(g["r_tia"])


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_measured_forward(case):
    g = load_golden(case)
    out, idiff, mag = mref.forward(g["x"], *_args(g))
    assert_close_scaled(out, g["out"], mag * float(g["r_tia"]), what=f"{case} out")
    gx, gmag = mref.backward_x(g["x"], *_args(g), g["grad_out"])
    assert_close_scaled(gx, g["grad_x"], gmag, what=f"{case} grad_x")


def test_oracle_reference_unit_case():
    """The reference's own KAT (tests/test_measured_deployment.py:37-49)."""
    out, _, _ = mref.forward(np.array([[0.25, 0.5]]), [0.0, 1.0, 2.0], [[0.0, 1.0, 2.0], [0.0, 2.0, 4.0]],
                             [[1, 1]], [[0, 0]], 0.0, 4.0, 1.0)
    assert abs(out[0, 0] - 0.75) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("case", CASES)
def test_measured_kernels_match_reference(case):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from isa_b200.operators.measured import DeploymentAwareCIMLinear
    g = load_golden(case)
    m, k = g["x"].shape
    o = g["pos"].shape[0]
    layer = DeploymentAwareCIMLinear(k, o).cuda()
    layer.set_r_tia(float(g["r_tia"]))
    layer.configure_codebook(torch.from_numpy(g["vg"]), torch.from_numpy(g["currents"]))
    layer.set_assignment(torch.from_numpy(g["pos"]), torch.from_numpy(g["neg"]))
    layer.set_forward_mode("measured")
    x = torch.from_numpy(g["x"]).cuda().reshape(1, m, k).requires_grad_(True)
    out = layer(x)
    out.backward(torch.from_numpy(g["grad_out"]).cuda().reshape(1, m, o))
    _, _, mag = mref.forward(g["x"], *_args(g))
    assert_close_scaled(out.detach().cpu().numpy()[0], g["out"], mag * float(g["r_tia"]), what="out vs reference")
    _, gmag = mref.backward_x(g["x"], *_args(g), g["grad_out"])
    assert_close_scaled(x.grad.cpu().numpy()[0], g["grad_x"], gmag, what="grad_x vs reference")
    assert layer.vth_pos.grad is None  # fixed buffers: no threshold gradient


@pytest.mark.gpu
def test_measured_modes_and_unit_case():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from isa_b200.operators.measured import DeploymentAwareCIMLinear
    layer = DeploymentAwareCIMLinear(2, 1).cuda()
    layer.set_r_tia(1.0)
    layer.configure_codebook(torch.tensor([0.0, 1.0, 2.0]), torch.tensor([[0.0, 1.0, 2.0], [0.0, 2.0, 4.0]]))
    layer.set_assignment(torch.tensor([[1, 1]], dtype=torch.int16), torch.tensor([[0, 0]], dtype=torch.int16))
    layer.set_forward_mode("measured")
    out = layer(torch.tensor([[[0.25, 0.50]]], device="cuda"))
    assert torch.allclose(out.cpu(), torch.tensor([[[0.75]]]), atol=1e-6)
    # STE: measured value, continuous (EKV LUT) gradient
    x = torch.rand(1, 5, 2, device="cuda", requires_grad=True)
    layer.set_forward_mode("ste")
    y = layer(x)
    layer.set_forward_mode("measured")
    torch.testing.assert_close(y.detach(), layer(x).detach())
    y.sum().backward()
    assert layer.vth_pos.grad is not None  # gradient came from the continuous path
    with pytest.raises(ValueError):
        layer.configure_codebook(torch.tensor([0.0, 1.0]), torch.tensor([[0.0, 1.0]]), vin_lut_bins=-1)


@pytest.mark.gpu
@pytest.mark.parametrize("shape,states,grid", [((300, 70, 130), 24, 33), ((1025, 37, 96), 5, 4),
                                               ((64, 4, 32), 24, 9), ((129, 130, 1), 7, 17), ((7, 3, 65), 1, 2),
                                               ((200, 40, 70), 24, 65)])  # > 1024 coefficients: large layout
def test_measured_kernels_random_shapes(shape, states, grid):
    """Ragged tiles, inputs outside the lookup range, clamped outputs and small
    codebooks (state tables not a multiple of 4 entries), against the fp64 oracle."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from isa_b200.operators.measured import DeploymentAwareCIMLinear
    m, k, o = shape
    rng = np.random.default_rng(m * 7 + k)
    vg = np.sort(rng.uniform(0.0, 4.0, grid)).astype(np.float32)
    vg[0], vg[-1] = 0.0, 4.0
    currents = np.cumsum(rng.uniform(0.0, 2e-6, (states, grid)), axis=1).astype(np.float32)
    pos = rng.integers(0, states, (o, k)).astype(np.int16)
    neg = rng.integers(0, states, (o, k)).astype(np.int16)
    x = rng.uniform(-0.5, 4.5, (m, k)).astype(np.float32)  # some inputs outside [0, 4]
    layer = DeploymentAwareCIMLinear(k, o).cuda()
    layer.configure_codebook(torch.from_numpy(vg), torch.from_numpy(currents))
    layer.set_assignment(torch.from_numpy(pos), torch.from_numpy(neg))
    layer.set_forward_mode("measured")
    lmin, lmax = layer.lookup_min, layer.lookup_max
    # R_TIA so that roughly a third of the outputs hit the clamp
    _, idiff_ref, _ = mref.forward(x, vg, currents, pos, neg, lmin, lmax, 1.0)
    r = float(4.0 / max(np.quantile(np.abs(idiff_ref), 0.7), 1e-12))
    # keep every |idiff * r| away from the clamp edge, where the fp32 kernel and
    # the fp64 oracle could disagree on the gradient mask
    while np.min(np.abs(np.abs(idiff_ref * r) - 4.0)) < 1e-3:
        r *= 1.0007
    layer.set_r_tia(r)
    g = rng.standard_normal((m, o)).astype(np.float32)
    xd = torch.from_numpy(x).cuda().reshape(1, m, k).requires_grad_(True)
    out = layer(xd)
    out.backward(torch.from_numpy(g).cuda().reshape(1, m, o))
    want, _, mag = mref.forward(x, vg, currents, pos, neg, lmin, lmax, r)
    assert_close_scaled(out.detach().cpu().numpy()[0], want, mag * r, what="measured out")
    gx_want, gmag = mref.backward_x(x, vg, currents, pos, neg, lmin, lmax, r, g)
    assert_close_scaled(xd.grad.cpu().numpy()[0], gx_want, gmag, what="measured grad_x")


BINNED = ["measured_binned", "measured_binned_one", "measured_binned_ragged"]


def _binned_args(g):
    return (*_args(g), int(g["bins"]), g["bin_centers"])


@pytest.mark.parametrize("case", BINNED)
def test_oracle_matches_reference_binned_forward(case):
    """Binned inputs (vin_lut_bins > 0): bin ids bit-exact, output at the suite's tolerance."""
    g = load_golden(case)
    out, _, mag = mref.forward_binned(g["x"], *_binned_args(g))
    assert_close_scaled(out, g["out"], mag * float(g["r_tia"]), what=f"{case} out")


@pytest.mark.gpu
@pytest.mark.parametrize("case", BINNED)
def test_binned_measured_forward_matches_reference(case):
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from isa_b200.operators.measured import DeploymentAwareCIMLinear
    g = load_golden(case)
    m, k = g["x"].shape
    o = g["pos"].shape[0]
    layer = DeploymentAwareCIMLinear(k, o).cuda()
    layer.set_r_tia(float(g["r_tia"]))
    layer.configure_codebook(torch.from_numpy(g["vg"]), torch.from_numpy(g["currents"]), vin_lut_bins=int(g["bins"]))
    layer.set_assignment(torch.from_numpy(g["pos"]), torch.from_numpy(g["neg"]))
    layer.set_forward_mode("measured")
    assert tuple(layer.diff_current.shape) == (int(g["bins"]), o, k)
    x = torch.from_numpy(g["x"]).cuda().reshape(1, m, k).requires_grad_(True)
    out = layer(x)
    assert not out.requires_grad  # bin masks carry no input gradient, as in the reference
    _, _, mag = mref.forward_binned(g["x"], *_binned_args(g))
    assert_close_scaled(out.cpu().numpy()[0], g["out"], mag * float(g["r_tia"]), what=f"{case} out vs reference")
    # STE mode: measured value, continuous gradient
    layer.set_forward_mode("ste")
    out_ste = layer(x)
    assert_close_scaled(out_ste.detach().cpu().numpy()[0], g["out"], mag * float(g["r_tia"]), what="ste value")
    out_ste.sum().backward()
    assert x.grad is not None and bool(torch.isfinite(x.grad).all())
