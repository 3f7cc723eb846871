"""The callers of the hot path, against the oracle and against the reference's
own modules on the same GPU.

* PhysicalFFN under bf16 autocast against the oracle composition
  (VoltageMapping -> CIM -> TIA clamp -> CIM -> TIA clamp -> ADC affine), output
  and every parameter gradient: the CIM path stays fp32 under autocast
  (reference cim.py:180-199 casts nothing down), so the bound is the LUT parity
  tolerance, 1e-5 of the summed |terms|.
* PhysicalFFN / HybridFFN (operator level) and GPT2Model with physical and
  hybrid FFNs (language level) against the unmodified reference package in
  baseline/_ref, run on its own GPU path (Triton forward, CUDA shared backward),
  with identical weights: outputs and gradients within rel 2e-2 (norm-wise)
  under bf16 autocast, the tolerance stated for this operator under autocast.
* The reference GPT2Model with only its backend entry patched to this
  operator (``isa.operators.cim.triton_lut_ekv_matmul``, the binding that
  INTEGRATION.md section 2 shows), against the unpatched reference.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._util import assert_close_scaled

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from isa_b200 import build
    build.build_library()


def _reference():
    if not (REF / "isa").is_dir():
        pytest.skip("reference package not installed in baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import isa.operators.cim as ref_cim
    return ref_cim


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.detach().double(), b.detach().double()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


# ------------------------------------------------------- oracle composition --

def _tables(cfg):
    from isa_b200.approximations.delta_lut import build_lut_tables_cpu, lut_geometry
    geo = lut_geometry(cfg)
    ti, td = (t.float().numpy() for t in build_lut_tables_cpu(cfg))
    return ti, td, geo.delta_min_f32, geo.scale, float(cfg["V_sat"])


def _cim_oracle(lin, v, g_out, tabs):
    """One CIMLinear (LUT, TIA gain, signed clamp) forward and backward on the
    CPU oracle: returns (out, mag, dv, dvth_pos, dvth_neg, dlog_scale, mags)."""
    ti, td, dmin, scale, vsat = tabs
    wp = lin.vth_pos.detach().cpu().numpy()
    wn = lin.vth_neg.detach().cpu().numpy()
    r = np.float32(lin.r_tia.detach().cpu().item())
    idiff, mag = oracle.forward(v, wp, wn, ti, dmin, scale, vsat, with_mag=True)
    pre = (idiff * r).astype(np.float32)
    out = np.clip(pre, -4.0, 4.0)
    if g_out is None:
        return out, mag * r, None
    mask = (pre >= -4.0) & (pre <= 4.0)
    gl = (g_out * mask * r).astype(np.float32)
    (dv, dwp, dwn), mags = oracle.backward(v, wp, wn, gl, ti, td, dmin, scale, vsat, with_mag=True)
    dls = float((g_out * mask * idiff * r).astype(np.float64).sum())  # d/d log_scale of R = R exp(s)
    return out, mag * r, (dv, dwp, dwn, dls, mags)


def test_physical_ffn_block_under_autocast_matches_oracle_composition():
    from isa_b200.operators.cim import PhysicalFFN
    torch.manual_seed(0)
    d, hdim, b, n = 64, 256, 3, 41
    ffn = PhysicalFFN(d, hdim).cuda()
    with torch.no_grad():
        ffn.input_mapping.set_affine(0.8, 1.6)
        ffn.fc1.set_r_tia(2.0e4)
        ffn.fc2.set_r_tia(6.0e3)
        ffn.adc_affine_scale.uniform_(0.5, 1.5)
        ffn.adc_affine_shift.uniform_(-0.2, 0.2)
    x = torch.randn(b, n, d, device="cuda")
    g = torch.randn(b, n, d, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = ffn(x)
    assert y.dtype == torch.float32  # the CIM block stays fp32 under autocast
    y.backward(g)

    tabs = _tables(ffn.fc1.cfg)
    xs = x.reshape(-1, d).cpu().numpy()
    gs = g.reshape(-1, d).cpu().numpy()
    s, t = float(ffn.input_mapping.scale), float(ffn.input_mapping.shift)
    pre_v = (xs * np.float32(s) + np.float32(t)).astype(np.float32)
    v = np.clip(pre_v, 0.0, 4.0).astype(np.float32)
    h1, _, _ = _cim_oracle(ffn.fc1, v, None, tabs)
    h2, mag2, _ = _cim_oracle(ffn.fc2, h1, None, tabs)
    a = ffn.adc_affine_scale.detach().cpu().numpy()
    c = ffn.adc_affine_shift.detach().cpu().numpy()
    want = h2 * a + c
    assert_close_scaled(y.detach().reshape(-1, d).cpu().numpy(), want, mag2 * np.abs(a) + 1e-30,
                        what="block output")
    # backward through the composition
    _, _, (dh1, dwp2, dwn2, dls2, (_, mwp2, mwn2)) = _cim_oracle(ffn.fc2, h1, (gs * a).astype(np.float32), tabs)
    _, _, (dv, dwp1, dwn1, dls1, (mv, mwp1, mwn1)) = _cim_oracle(ffn.fc1, v, dh1.astype(np.float32), tabs)
    assert_close_scaled(ffn.fc2.vth_pos.grad.cpu().numpy(), dwp2, mwp2, what="fc2 dVth_pos")
    assert_close_scaled(ffn.fc2.vth_neg.grad.cpu().numpy(), dwn2, mwn2, what="fc2 dVth_neg")
    # fc1's upstream gradient already carries fc2's rounding; its sums cancel
    # less, so compare norm-wise at the same 1e-5 level
    for got, exp, name in ((ffn.fc1.vth_pos.grad, dwp1, "fc1 dVth_pos"), (ffn.fc1.vth_neg.grad, dwn1, "fc1 dVth_neg")):
        assert _rel(got.cpu(), torch.from_numpy(exp)) < 1e-4, name
    dx_map = dv * ((pre_v >= 0.0) & (pre_v <= 4.0))
    assert _rel(ffn.input_mapping.scale.grad.cpu(), torch.tensor((dx_map * xs).sum())) < 1e-4
    assert _rel(ffn.input_mapping.shift.grad.cpu(), torch.tensor(dx_map.sum())) < 1e-4
    assert _rel(ffn.fc2.r_tia_log_scale.grad.cpu(), torch.tensor([dls2])) < 1e-4
    assert _rel(ffn.fc1.r_tia_log_scale.grad.cpu(), torch.tensor([dls1])) < 1e-4
    assert _rel(ffn.adc_affine_scale.grad.cpu(), torch.from_numpy((gs * h2).sum(0))) < 1e-5
    assert _rel(ffn.adc_affine_shift.grad.cpu(), torch.from_numpy(gs.sum(0))) < 1e-6


# ------------------------------------------------- against the reference ----

def _compare_modules(ours, ref, x, g, tol, what):
    ref.load_state_dict(ours.state_dict(), strict=True)
    xo = x.clone().requires_grad_(True)
    xr = x.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16):
        yo = ours(xo)
        yr = ref(xr)
    assert _rel(yo.float(), yr.float()) < tol, f"{what} output {_rel(yo.float(), yr.float())}"
    yo.float().backward(g)
    yr.float().backward(g)
    assert _rel(xo.grad, xr.grad) < tol, f"{what} input grad"
    pr = dict(ref.named_parameters())
    for name, p in ours.named_parameters():
        q = pr[name]
        if p.grad is None and q.grad is None:
            continue
        assert _rel(p.grad, q.grad) < tol, f"{what} grad {name}: {_rel(p.grad, q.grad)}"


@pytest.mark.parametrize("kind", ["physical", "hybrid"])
def test_ffn_blocks_match_reference_gpu_path(kind):
    ref_cim = _reference()
    from isa_b200.operators import cim as our_cim
    torch.manual_seed(1)
    cls_o = our_cim.PhysicalFFN if kind == "physical" else our_cim.HybridFFN
    cls_r = ref_cim.PhysicalFFN if kind == "physical" else ref_cim.HybridFFN
    ours = cls_o(96, 384).cuda()
    with torch.no_grad():
        ours.input_mapping.set_affine(0.7, 1.8)
        ours.fc1.set_r_tia(2.0e4)
        if kind == "physical":
            ours.fc2.set_r_tia(5.0e3)
    ref = cls_r(96, 384).cuda()
    x = torch.randn(4, 64, 96, device="cuda")
    g = torch.randn(4, 64, 96, device="cuda")
    _compare_modules(ours, ref, x, g, 2e-2, f"{kind} FFN")


@pytest.mark.parametrize("kind", ["physical", "hybrid"])
def test_gpt2_model_matches_reference_gpu_path(kind):
    _reference()
    from isa.language.config import ModelConfig as RefConfig
    from isa.language.models import GPT2Model as RefGPT

    from isa_b200.language import GPT2Model, ModelConfig
    torch.manual_seed(2)
    cfg = ModelConfig.from_preset("tiny", kind, max_seq_len=64)
    cfg.depth = 2
    rcfg = RefConfig.from_preset("tiny", kind, max_seq_len=64)
    rcfg.depth = 2
    ours = GPT2Model(cfg).cuda()
    ref = RefGPT(rcfg).cuda()
    ids = torch.randint(0, cfg.vocab_size, (4, 64), device="cuda")
    ref.load_state_dict(ours.state_dict(), strict=True)

    def loss_of(model):
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(ids[:, :-1])
            return logits, torch.nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]),
                                                             ids[:, 1:].reshape(-1))

    lo, l_o = loss_of(ours)
    lr, l_r = loss_of(ref)
    assert _rel(lo.float(), lr.float()) < 2e-2
    l_o.backward()
    l_r.backward()
    pr = dict(ref.named_parameters())
    for name, p in ours.named_parameters():
        if p.grad is not None:
            assert _rel(p.grad, pr[name].grad) < 2e-2, f"{kind} grad {name}: {_rel(p.grad, pr[name].grad)}"


def test_reference_model_with_patched_backend_matches_unpatched():
    ref_cim = _reference()
    from isa.language.config import ModelConfig as RefConfig
    from isa.language.models import GPT2Model as RefGPT

    from isa_b200.kernels.transformer_ffn.ekv_lut import cuda_lut_ekv_matmul
    torch.manual_seed(3)
    rcfg = RefConfig.from_preset("tiny", "physical", max_seq_len=64)
    rcfg.depth = 2
    model = RefGPT(rcfg).cuda()
    ids = torch.randint(0, rcfg.vocab_size, (4, 64), device="cuda")

    def run():
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            logits = model(ids[:, :-1])
            loss = torch.nn.functional.cross_entropy(logits.float().reshape(-1, logits.shape[-1]),
                                                     ids[:, 1:].reshape(-1))
        loss.backward()
        return logits.detach().float(), {n: p.grad.clone() for n, p in model.named_parameters()
                                         if p.grad is not None}

    base_logits, base_grads = run()
    original = ref_cim.triton_lut_ekv_matmul
    ref_cim.triton_lut_ekv_matmul = cuda_lut_ekv_matmul
    try:
        logits, grads = run()
    finally:
        ref_cim.triton_lut_ekv_matmul = original
    assert _rel(logits, base_logits) < 2e-2
    assert grads.keys() == base_grads.keys()
    for n in grads:
        assert _rel(grads[n], base_grads[n]) < 2e-2, f"{n}: {_rel(grads[n], base_grads[n])}"
