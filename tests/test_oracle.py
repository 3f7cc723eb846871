"""The CPU oracle, pinned against the reference's own kernels (golden vectors
minted by tests/golden/make_golden.py from the reference Triton kernels)."""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._util import GOLDEN, GOLDEN_CASES, assert_close_scaled, bf16_bits_to_f32, geometry, load_golden


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_oracle_forward_matches_reference_triton(case):
    g = load_golden(case)
    dmin, scale, size = geometry(g)
    ti = bf16_bits_to_f32(g["table_i"])
    out, mag = oracle.forward(g["x"], g["wpos"], g["wneg"], ti, dmin, scale, float(g["v_sat"]),
                              float(g["out_min"]), float(g["out_max"]), with_mag=True)
    assert_close_scaled(out, g["out"], mag, what=f"{case} forward")


@pytest.mark.parametrize("case", GOLDEN_CASES)
def test_oracle_backward_matches_reference_triton(case):
    g = load_golden(case)
    dmin, scale, size = geometry(g)
    ti, td = bf16_bits_to_f32(g["table_i"]), bf16_bits_to_f32(g["table_ddelta"])
    (gx, gwp, gwn), (mx, mwp, mwn) = oracle.backward(
        g["x"], g["wpos"], g["wneg"], g["grad_out"], ti, td, dmin, scale, float(g["v_sat"]), with_mag=True)
    # The reference Triton backward uses the q0(1-a)+q1 a lerp and true
    # division; the oracle follows the CUDA backward (fmaf lerp, reciprocal).
    # Both are fp32-rounding apart.
    assert_close_scaled(gx, g["grad_x"], mx, what=f"{case} grad_x")
    assert_close_scaled(gwp, g["grad_wpos"], mwp, what=f"{case} grad_wpos")
    assert_close_scaled(gwn, g["grad_wneg"], mwn, what=f"{case} grad_wneg")


@pytest.mark.parametrize("size", [8192, 4096])
def test_oracle_index_selection_is_bit_exact(size):
    """Reference _lut_lookup on table[j] = j, reproduced bit for bit."""
    with np.load(GOLDEN / "golden_index.npz") as z:
        delta = z[f"delta_t{size}"]
        want = z[f"lookup_t{size}"]
        dmin64, dmax64 = float(z[f"dmin_t{size}"]), float(z[f"dmax_t{size}"])
    dmin = float(np.float32(dmin64))
    scale = float(np.float32((size - 1) / (dmax64 - dmin64)))
    for idx, a in (oracle.lut_index(delta, size, dmin, scale), oracle.lut_index_np(delta, size, dmin, scale)):
        i1 = np.minimum(idx + 1, size - 1)
        t = np.arange(size, dtype=np.float32)
        got = t[idx] * (np.float32(1) - a) + t[i1] * a
        np.testing.assert_array_equal(got.astype(np.float32), want)


def test_lut_builder_bit_identical_to_reference():
    from isa_b200.approximations.delta_lut import _cpu_lut_cached, build_lut_tables_cpu
    from isa_b200.device_models.config import make_flash_transistor_ekv_config

    for case in GOLDEN_CASES:
        g = load_golden(case)
        cfg = make_flash_transistor_ekv_config(default_lut_size=int(g["size"]))
        cfg["LUT_DELTA_SIZE"] = int(g["size"])
        ti, td = build_lut_tables_cpu(cfg)
        np.testing.assert_array_equal(ti.view(torch.int16).numpy().view(np.uint16), g["table_i"])
        np.testing.assert_array_equal(td.view(torch.int16).numpy().view(np.uint16), g["table_ddelta"])
    with np.load(GOLDEN / "golden_lut_testkey.npz") as z:
        key = tuple(float(v) for v in z["key"][:-1]) + (int(z["key"][-1]),)
        ti, td = _cpu_lut_cached(key)
        np.testing.assert_array_equal(ti.view(torch.int16).numpy().view(np.uint16), z["table_i"])
        np.testing.assert_array_equal(td.view(torch.int16).numpy().view(np.uint16), z["table_ddelta"])


def test_lut_builder_matches_formula_loosely():
    """The reference's own builder test (tests/test_flash_formula.py:56-84): bf16
    table vs the fp32 formula at rtol 8e-3 / atol 3e-3."""
    import torch.nn.functional as F

    from isa_b200.approximations.delta_lut import _cpu_lut_cached

    n, u_t, i_s, v_d = 4.1360, 0.026, 0.75875, 0.1
    key = (n, 8.2624, i_s, u_t, v_d, -1.0, 3.0, 257)
    table, _ = _cpu_lut_cached(key)
    delta = torch.linspace(-1.0, 3.0, 257, dtype=torch.float32)
    inv = 1.0 / (2.0 * n * u_t)
    expected = i_s * (F.softplus(delta * inv).square() - F.softplus((delta - v_d) * inv).square())
    assert torch.allclose(table.float(), expected, rtol=8.0e-3, atol=3.0e-3)


@pytest.mark.parametrize("case", ["exact_small", "exact_ragged"])
def test_exact_oracle_matches_reference_exact_triton(case):
    g = load_golden(case)
    inv = 1.0 / (2.0 * float(g["n"]) * float(g["U_T"]))
    args = (inv, float(g["V_D"]), float(g["I_S"]), float(g["V_sat"]))
    out, mag = oracle.exact_forward(g["x"], g["wpos"], g["wneg"], *args, with_mag=True)
    assert_close_scaled(out, g["out"], mag, what=f"{case} exact forward")
    (gx, gwp, gwn), (mx, mwp, mwn) = oracle.exact_backward(g["x"], g["wpos"], g["wneg"], g["grad_out"], *args,
                                                           with_mag=True)
    assert_close_scaled(gx, g["grad_x"], mx, what=f"{case} exact grad_x")
    assert_close_scaled(gwp, g["grad_wpos"], mwp, what=f"{case} exact grad_wpos")
    assert_close_scaled(gwn, g["grad_wneg"], mwn, what=f"{case} exact grad_wneg")
