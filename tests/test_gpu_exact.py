"""Exact-formula path (cfg ekv_approx != "lut") on sm_100a against the fp64
oracle of the reference formula and the reference's exact Triton kernels."""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._util import assert_close_scaled, load_golden

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _cfg():
    from isa_b200 import make_flash_transistor_ekv_config
    cfg = make_flash_transistor_ekv_config(4096)
    cfg["ekv_approx"] = "exact"
    return cfg


def _run(x, wp, wn, g, args):
    from isa_b200 import _lib
    xd, pd, nd, gd = (torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda() for a in (x, wp, wn, g))
    m, k = x.shape
    o = wp.shape[0]
    out = torch.empty(m, o, device="cuda")
    _lib.exact_forward(xd, pd, nd, *args, out)
    gx, gwp, gwn = torch.empty_like(xd), torch.empty_like(pd), torch.empty_like(nd)
    ws = torch.empty(max(_lib.exact_backward_workspace_bytes(m, k, o), 16), dtype=torch.uint8, device="cuda")
    _lib.exact_backward(xd, pd, nd, gd, *args, gx, gwp, gwn, ws)
    return [t.cpu().numpy() for t in (out, gx, gwp, gwn)]


def _check(x, wp, wn, g, args, tag):
    out, gx, gwp, gwn = _run(x, wp, wn, g, args)
    ref, mag = oracle.exact_forward(x, wp, wn, *args, with_mag=True)
    assert_close_scaled(out, ref, mag, what=f"{tag} forward")
    (rx, rwp, rwn), (mx, mwp, mwn) = oracle.exact_backward(x, wp, wn, g, *args, with_mag=True)
    assert_close_scaled(gx, rx, mx, what=f"{tag} grad_x")
    assert_close_scaled(gwp, rwp, mwp, what=f"{tag} grad_wpos")
    assert_close_scaled(gwn, rwn, mwn, what=f"{tag} grad_wneg")
    return out, gx, gwp, gwn


@pytest.mark.parametrize("case", ["exact_small", "exact_ragged"])
def test_exact_golden(case):
    gd = load_golden(case)
    args = (1.0 / (2.0 * float(gd["n"]) * float(gd["U_T"])), float(gd["V_D"]), float(gd["I_S"]), float(gd["V_sat"]))
    out, gx, gwp, gwn = _check(gd["x"], gd["wpos"], gd["wneg"], gd["grad_out"], args, case)
    _, mag = oracle.exact_forward(gd["x"], gd["wpos"], gd["wneg"], *args, with_mag=True)
    assert_close_scaled(out, gd["out"], mag, what=f"{case} forward vs reference")


@pytest.mark.parametrize("shape,dist", [((64, 16, 64), "sub"), ((130, 33, 97), "mixed"), ((257, 96, 130), "wide"),
                                        ((1, 1, 1), "mixed")])
def test_exact_random(shape, dist):
    m, k, o = shape
    rng = np.random.default_rng(m + k + o)
    if dist == "sub":  # deep subthreshold: tiny currents, log1p accuracy matters
        x = rng.uniform(0.0, 1.0, (m, k))
    elif dist == "mixed":
        x = rng.uniform(0.0, 4.0, (m, k))
    else:  # far above threshold too: the u > 20 branch
        x = rng.uniform(-4.0, 9.0, (m, k))
    wp = 2.5 + rng.uniform(-0.2, 0.2, (o, k))
    wn = 2.5 + rng.uniform(-0.2, 0.2, (o, k))
    g = rng.standard_normal((m, o))
    from oracle.oracle import exact_consts
    f = np.float32
    _check(x.astype(f), wp.astype(f), wn.astype(f), g.astype(f), exact_consts(_cfg()), f"{shape} {dist}")


def test_exact_module_dispatch():
    from isa_b200.operators.cim import CIMLinear
    torch.manual_seed(3)
    lin = CIMLinear(48, 80, _cfg()).cuda()
    lin.set_r_tia(1e4)
    x = (torch.rand(2, 30, 48, device="cuda") * 4).requires_grad_(True)
    out = lin(x)
    out.sum().backward()
    from oracle.oracle import exact_consts
    args = exact_consts(lin.cfg)
    ref, mag = oracle.exact_forward(x.detach().reshape(60, 48).cpu().numpy(), lin.vth_pos.detach().cpu().numpy(),
                                    lin.vth_neg.detach().cpu().numpy(), *args, with_mag=True)
    want = np.clip(ref * np.float32(1e4), -4, 4).reshape(2, 30, 80)
    assert_close_scaled(out.detach().cpu().numpy(), want, mag.reshape(2, 30, 80) * 1e4, what="module exact forward")
    assert x.grad is not None and torch.isfinite(x.grad).all() and torch.isfinite(lin.vth_pos.grad).all()
