"""Full-size (benchmark shape) checks through size-independent properties, plus
the drop-in nn.Module path."""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._util import assert_close_scaled, bf16_bits_to_f32
from tests.test_gpu_parity import CFG_V_SAT, cfg_tables, pack

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _inputs(m, k, o, seed):
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, device="cuda", generator=gen)
    wp = 2.5 + (torch.rand(o, k, device="cuda", generator=gen) * 2 - 1) * 0.10712
    wn = 2.5 + (torch.rand(o, k, device="cuda", generator=gen) * 2 - 1) * 0.10712
    g = torch.randn(m, o, device="cuda", generator=gen)
    return x, wp, wn, g


def _run(x, wp, wn, g, lut, dmin, scale, size):
    from isa_b200 import _lib
    m, k = x.shape
    o = wp.shape[0]
    out = torch.empty(m, o, device="cuda")
    _lib.forward(x, wp, wn, lut, size, dmin, scale, CFG_V_SAT, -4.0, 4.0, out)
    gx = torch.empty_like(x)
    gwp = torch.empty_like(wp)
    gwn = torch.empty_like(wn)
    ws = torch.empty(_lib.backward_workspace_bytes(m, k, o, size), dtype=torch.uint8, device="cuda")
    _lib.backward(x, wp, wn, g, lut, size, dmin, scale, CFG_V_SAT, gx, gwp, gwn, ws)
    return out, gx, gwp, gwn


# Layer shapes of the benchmark configs, at the token counts one GPU sees:
#   config 3 (GPT-M FFN block, 32x1024 tokens), config 2 (ViT-M block, 128x65),
#   config 4 (GPT-L: 768 <-> 3072, 64x1024 tokens on 1 GPU, 8x1024 per GPU at 8),
#   config 5 (ViT-L: 384 <-> 1536, 256x197 tokens on 1 GPU, 32x197 per GPU at 8).
# The config-4 up projection at 8 GPUs combines the forward's k split (few
# tiles) with the backward's workspace dVth accumulator (O = 3072).
FULL_SHAPES = [
    ((32768, 384, 1536), 4096), ((32768, 1536, 384), 4096), ((8320, 256, 1024), 8192),
    ((65536, 768, 3072), 4096), ((65536, 3072, 768), 4096), ((8192, 768, 3072), 4096), ((8192, 3072, 768), 4096),
    ((50432, 384, 1536), 8192), ((50432, 1536, 384), 8192), ((6304, 384, 1536), 8192), ((6304, 1536, 384), 8192),
]


@pytest.mark.parametrize("shape,size", FULL_SHAPES, ids=[f"{m}x{k}x{o}-T{t}" for (m, k, o), t in FULL_SHAPES])
def test_fullsize_rows_match_oracle_and_dvth_is_additive(shape, size):
    m, k, o = shape
    tib, tdb, dmin, scale, _ = cfg_tables(size)
    lut = pack(tib, tdb)
    x, wp, wn, g = _inputs(m, k, o, seed=m + k)
    out, gx, gwp, gwn = _run(x, wp, wn, g, lut, dmin, scale, size)
    # Row-local outputs (forward row m, dX row m) against the oracle on sampled rows.
    rows = torch.tensor(np.random.default_rng(0).choice(m, 12, replace=False), device="cuda")
    ti, td = bf16_bits_to_f32(tib), bf16_bits_to_f32(tdb)
    xs, gs = x[rows].cpu().numpy(), g[rows].cpu().numpy()
    wpn, wnn = wp.cpu().numpy(), wn.cpu().numpy()
    ref, mag = oracle.forward(xs, wpn, wnn, ti, dmin, scale, CFG_V_SAT, with_mag=True)
    assert_close_scaled(out[rows].cpu().numpy(), ref, mag, what="forward rows")
    (rx, _, _), (mx, _, _) = oracle.backward(xs, wpn, wnn, gs, ti, td, dmin, scale, CFG_V_SAT,
                                             need_w=False, with_mag=True)
    assert_close_scaled(gx[rows].cpu().numpy(), rx, mx, what="grad_x rows")
    # dVth is a sum over tokens: the two token halves add up to the whole.
    h = m // 2
    _, _, p1, n1 = _run(x[:h].contiguous(), wp, wn, g[:h].contiguous(), lut, dmin, scale, size)
    _, _, p2, n2 = _run(x[h:].contiguous(), wp, wn, g[h:].contiguous(), lut, dmin, scale, size)
    # magnitude bound from |g| times the largest derivative entry (per-entry sum of |terms| <= that)
    dmax = float(np.abs(td).max())
    gabs = g.abs().sum(0).unsqueeze(1).expand(o, k).cpu().numpy() * dmax
    assert_close_scaled((p1 + p2).cpu().numpy(), gwp.cpu().numpy(), gabs, rtol=2e-6, what="dWpos additivity")
    assert_close_scaled((n1 + n2).cpu().numpy(), gwn.cpu().numpy(), gabs, rtol=2e-6, what="dWneg additivity")
    # Linearity in the upstream gradient.
    _, gx2, gwp2, _ = _run(x, wp, wn, (2.0 * g).contiguous(), lut, dmin, scale, size)
    # (exact up to subnormal partial sums, where doubling is not exact)
    torch.testing.assert_close(gx2, 2 * gx, rtol=1e-5, atol=1e-30)
    torch.testing.assert_close(gwp2, 2 * gwp, rtol=1e-5, atol=1e-30)
    # A column sample of dVth against the oracle over all tokens.
    cols = np.random.default_rng(1).choice(o, 3, replace=False)
    wsub_p, wsub_n = wpn[cols], wnn[cols]
    gsub = g[:, torch.tensor(cols, device="cuda")].cpu().numpy()
    (_, rwp, rwn), (_, mwp, mwn) = oracle.backward(x.cpu().numpy(), wsub_p, wsub_n, gsub, ti, td, dmin, scale,
                                                   CFG_V_SAT, need_x=False, with_mag=True)
    assert_close_scaled(gwp[cols].cpu().numpy(), rwp, mwp, what="dWpos columns")
    assert_close_scaled(gwn[cols].cpu().numpy(), rwn, mwn, what="dWneg columns")


def test_cimlinear_module_matches_oracle():
    from isa_b200.operators.cim import CIMLinear, PhysicalFFN
    torch.manual_seed(0)
    lin = CIMLinear(96, 160).cuda()
    lin.set_r_tia(3e4)
    x = torch.randn(2, 50, 96, device="cuda", requires_grad=True)
    out = lin(x)
    cfg = lin.cfg
    from isa_b200.approximations.delta_lut import build_lut_tables_cpu, lut_geometry
    geo = lut_geometry(cfg)
    ti, td = (t.float().numpy() for t in build_lut_tables_cpu(cfg))
    xn = x.detach().reshape(100, 96).cpu().numpy()
    wp, wn = lin.vth_pos.detach().cpu().numpy(), lin.vth_neg.detach().cpu().numpy()
    idiff, mag = oracle.forward(xn, wp, wn, ti, geo.delta_min_f32, geo.scale, cfg["V_sat"], with_mag=True)
    want = np.clip(idiff * np.float32(3e4), -4, 4).reshape(2, 50, 160)
    assert_close_scaled(out.detach().cpu().numpy(), want, mag.reshape(2, 50, 160) * 3e4 * 1.0001,
                        what="module forward")
    g = torch.randn_like(out)
    out.backward(g)
    # autograd: clamp mask and TIA gain applied to grad before the LUT backward
    gl = (g * (out.abs() < 4).float() * 3e4).reshape(100, 160).cpu().numpy()
    (rx, rwp, rwn), (mx, mwp, mwn) = oracle.backward(xn, wp, wn, gl, ti, td, geo.delta_min_f32, geo.scale,
                                                     cfg["V_sat"], with_mag=True)
    assert_close_scaled(x.grad.reshape(100, 96).cpu().numpy(), rx, mx, what="module dX")
    assert_close_scaled(lin.vth_pos.grad.cpu().numpy(), rwp, mwp, what="module dVth_pos")
    assert_close_scaled(lin.vth_neg.grad.cpu().numpy(), rwn, mwn, what="module dVth_neg")
    assert lin.r_tia_log_scale.grad is not None
    # Physical FFN end to end runs and produces finite grads under bf16 autocast
    ffn = PhysicalFFN(64, 256).cuda()
    y = torch.randn(4, 33, 64, device="cuda", requires_grad=True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        z = ffn(y)
    z.float().sum().backward()
    for p in ffn.parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all()


def _config1():
    """Benchmark config 1: x[256,192] ~ N(0,1) seed 0, CIMLinear(192,768) init, grad ~ N(0,1) seed 3."""
    from isa_b200.operators.cim import CIMLinear
    torch.manual_seed(0)
    x = torch.randn(256, 192)
    torch.manual_seed(1)
    lin = CIMLinear(192, 768)
    torch.manual_seed(3)
    g = torch.randn(256, 768)
    return x.numpy(), lin, g.numpy()


def test_config1_full_size_against_oracle():
    x, lin, g = _config1()
    wp, wn = lin.vth_pos.detach().numpy(), lin.vth_neg.detach().numpy()
    tib, tdb, dmin, scale, size = cfg_tables(8192)
    lut = pack(tib, tdb)
    xd, pd, nd, gd = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (x, wp, wn, g))
    out, gx, gwp, gwn = _run(xd, pd, nd, gd, lut, dmin, scale, size)
    ti, td = bf16_bits_to_f32(tib), bf16_bits_to_f32(tdb)
    ref, mag = oracle.forward(x, wp, wn, ti, dmin, scale, CFG_V_SAT, with_mag=True)
    assert_close_scaled(out.cpu().numpy(), ref, mag, what="config 1 forward")
    (rx, rwp, rwn), (mx, mwp, mwn) = oracle.backward(x, wp, wn, g, ti, td, dmin, scale, CFG_V_SAT, with_mag=True)
    assert_close_scaled(gx.cpu().numpy(), rx, mx, what="config 1 grad_x")
    assert_close_scaled(gwp.cpu().numpy(), rwp, mwp, what="config 1 grad_wpos")
    assert_close_scaled(gwn.cpu().numpy(), rwn, mwn, what="config 1 grad_wneg")


def test_lut_path_tracks_the_exact_device_model():
    """Physics sanity check: the bf16 LUT path against the exact EKV formula (the
    reference's CPU path, in fp64) at config 1 — agreement to ~1e-2 of the summed
    magnitudes, the gap being the bf16 table quantisation."""
    x, lin, _ = _config1()
    x = np.clip(x + 2.0, 0.0, 4.0).astype(np.float32)  # voltage-mapped input range
    wp, wn = lin.vth_pos.detach().numpy(), lin.vth_neg.detach().numpy()
    tib, tdb, dmin, scale, size = cfg_tables(8192)
    lut = pack(tib, tdb)
    out = torch.empty(256, 768, device="cuda")
    from isa_b200 import _lib
    xd, pd, nd = (torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (x, wp, wn))
    _lib.forward(xd, pd, nd, lut, size, dmin, scale, CFG_V_SAT, -4.0, 4.0, out)
    from oracle.oracle import exact_consts
    from isa_b200 import FLASH_TRANSISTOR_EKV_CONFIG as cfg
    exact, mag = oracle.exact_forward(x, wp, wn, *exact_consts(cfg), with_mag=True)
    assert_close_scaled(out.cpu().numpy(), exact, mag, rtol=2e-2, what="LUT vs exact formula")
