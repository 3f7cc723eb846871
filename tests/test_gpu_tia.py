"""Fused TIA stage (forward epilogue + one-pass backward) against the
reference's unfused formulation (LUT matmul, then `* r_tia` and `clamp` under
autograd, cim.py:184-193), and the no-grad calibration entry estimate_idiff
(cim.py:140-163)."""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._util import assert_close_scaled

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


@pytest.mark.parametrize("sat,shape", [(0.5, (3, 70, 96, 200)), (0.1, (2, 33, 384, 1536)), (0.0, (1, 64, 40, 24))])
def test_fused_tia_matches_unfused_autograd(sat, shape):
    """sat: target fraction of outputs driven into the +-4 V clamp."""
    from isa_b200.kernels.transformer_ffn.ekv_lut import cuda_lut_ekv_matmul, cuda_lut_ekv_matmul_tia
    from isa_b200.operators.cim import CIMLinear
    b, n, k, o = shape
    torch.manual_seed(1)
    lin = CIMLinear(k, o).cuda()
    x = torch.randn(b * n, k, device="cuda")
    # gain that puts the (1 - sat) quantile of |I_diff| at the clamp (sat=0: tiny gain)
    idiff = lin.estimate_idiff(x, max_rows=b * n).abs().flatten()
    r_value = 4.0 / float(torch.quantile(idiff[:100000], 1.0 - sat)) if sat > 0 else 1e3
    lin.set_r_tia(r_value / 1.3498588)  # times exp(0.3) below
    with torch.no_grad():
        lin.r_tia_log_scale.fill_(0.3)
    g = torch.randn(b * n, o, device="cuda")

    def run(fused):
        xx = x.clone().requires_grad_(True)
        for p in lin.parameters():
            p.grad = None
        r = lin.r_tia
        if fused:
            out = cuda_lut_ekv_matmul_tia(xx, lin.vth_pos, lin.vth_neg, r, lin.cfg)
        else:
            out = (cuda_lut_ekv_matmul(xx, lin.vth_pos, lin.vth_neg, lin.cfg) * r).clamp(-4.0, 4.0)
        out.backward(g)
        return out.detach(), xx.grad, lin.vth_pos.grad.clone(), lin.vth_neg.grad.clone(), \
            lin.r_tia_log_scale.grad.clone()

    f, u = run(True), run(False)
    frac = float((f[0].abs() == 4.0).float().mean())
    assert abs(frac - sat) < 0.05, frac  # the clamp is exercised as intended
    torch.testing.assert_close(f[0], u[0], rtol=0, atol=0)  # same fp32 ops
    torch.testing.assert_close(f[1], u[1], rtol=0, atol=0)  # same masked, scaled gradient into the kernel
    torch.testing.assert_close(f[2], u[2], rtol=0, atol=0)
    torch.testing.assert_close(f[3], u[3], rtol=0, atol=0)
    # dL/dR_TIA: a full sum over M*O in a different order
    torch.testing.assert_close(f[4], u[4], rtol=1e-4, atol=0)


def test_estimate_idiff_matches_oracle():
    from isa_b200.approximations.delta_lut import build_lut_tables_cpu, lut_geometry
    from isa_b200.operators.cim import CIMLinear
    torch.manual_seed(2)
    lin = CIMLinear(64, 96).cuda()
    x = torch.randn(3, 50, 64, device="cuda")
    est = lin.estimate_idiff(x, max_rows=100)
    assert est.shape == (100, 96) and not est.requires_grad
    geo = lut_geometry(lin.cfg)
    ti = build_lut_tables_cpu(lin.cfg)[0].float().numpy()
    ref, mag = oracle.forward(x.reshape(-1, 64)[:100].cpu().numpy(), lin.vth_pos.detach().cpu().numpy(),
                              lin.vth_neg.detach().cpu().numpy(), ti, geo.delta_min_f32, geo.scale,
                              lin.cfg["V_sat"], with_mag=True)
    assert_close_scaled(est.cpu().numpy(), ref, mag, what="estimate_idiff")
