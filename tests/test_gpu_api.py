"""Autograd-level behaviour of the drop-in entry points, and a seeded random
parity sweep over shapes, input distributions and table sizes."""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._util import assert_close_scaled
from tests.test_gpu_parity import check_all, cfg_tables

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _cfg(size=4096):
    from isa_b200 import make_flash_transistor_ekv_config
    c = make_flash_transistor_ekv_config(size)
    c["LUT_DELTA_SIZE"] = size
    return c


def test_dtypes_layouts_and_partial_grads():
    from isa_b200.kernels.transformer_ffn.ekv_lut import triton_lut_ekv_matmul
    cfg = _cfg()
    torch.manual_seed(0)
    x = torch.randn(64, 40, device="cuda")
    wp = 2.5 + 0.1 * torch.rand(30, 40, device="cuda")
    wn = 2.5 + 0.1 * torch.rand(30, 40, device="cuda")
    ref = triton_lut_ekv_matmul(x, wp, wn, cfg)
    # non-contiguous inputs give the same result
    xt = x.t().contiguous().t()
    assert not xt.is_contiguous()
    torch.testing.assert_close(triton_lut_ekv_matmul(xt, wp, wn, cfg), ref, rtol=0, atol=0)
    # bf16 input: computed in fp32 (as the reference upcasts), fp32 output, bf16 input gradient
    xb = x.to(torch.bfloat16).requires_grad_(True)
    out = triton_lut_ekv_matmul(xb, wp, wn, cfg)
    assert out.dtype == torch.float32
    torch.testing.assert_close(out, triton_lut_ekv_matmul(xb.detach().float(), wp, wn, cfg), rtol=0, atol=0)
    out.sum().backward()
    assert xb.grad.dtype == torch.bfloat16
    # gradients only where requested
    for need in ((True, False, False), (False, True, True), (False, True, False)):
        xx, pp, nn_ = (t.clone().requires_grad_(r) for t, r in zip((x, wp, wn), need))
        triton_lut_ekv_matmul(xx, pp, nn_, cfg).sum().backward()
        for t, r in zip((xx, pp, nn_), need):
            assert (t.grad is not None) == r


CASES = [(int(m), int(k), int(o), int(t), d) for m, k, o, t, d in zip(
    np.random.default_rng(123).integers(1, 400, 24), np.random.default_rng(124).integers(1, 150, 24),
    np.random.default_rng(125).integers(1, 300, 24), np.random.default_rng(126).choice([257, 1000, 4096, 8192, 16384], 24),
    np.random.default_rng(127).choice(["normal", "mapped", "signed", "wide"], 24))]


@pytest.mark.parametrize("m,k,o,size,dist", CASES)
def test_random_sweep(m, k, o, size, dist):
    rng = np.random.default_rng(m * 7 + k * 11 + o)
    if dist == "normal":
        x = rng.standard_normal((m, k))
    elif dist == "mapped":
        x = np.clip(rng.standard_normal((m, k)) + 2, 0, 4)
    elif dist == "signed":
        x = np.clip(3 * rng.standard_normal((m, k)), -4, 4)
    else:
        x = rng.uniform(-10, 10, (m, k))
    spread = 2.5 if dist == "wide" else 0.2
    wp = 2.5 + rng.uniform(-spread, spread, (o, k))
    wn = 2.5 + rng.uniform(-spread, spread, (o, k))
    g = rng.standard_normal((m, o))
    f = np.float32
    check_all(x.astype(f), wp.astype(f), wn.astype(f), g.astype(f), *cfg_tables(size), tag=f"{m},{k},{o} T={size} {dist}")
