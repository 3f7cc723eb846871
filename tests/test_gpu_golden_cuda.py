"""Parity with the reference's DEFAULT GPU backward.

The fixtures ``golden_cuda_*.npz`` were minted on a B200 by
``tests/golden/make_golden_cuda.py`` from the unmodified reference: its Triton
forward (``ekv_lut_triton.py:37-62``) and its CUDA shared backward
(``cuda/ekv_cuda.cu:193-341``, selected by ``CUDA_SHARED_BACKWARD``), on the
inputs of the Triton-minted golden cases and on benchmark config 1 at full
size.  Our kernels run through the C ABI on the same inputs.  Tolerance as for
every LUT parity check: 1e-5 of the summed |terms| of each output (the sums
cancel, so a bound relative to the output itself would be meaningless).
"""

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._util import GOLDEN, assert_close_scaled, bf16_bits_to_f32
from tests.test_gpu_parity import CFG_V_SAT, cfg_tables, gpu_backward, gpu_forward, pack

pytestmark = pytest.mark.gpu

CASES = ["small_t4096", "small_t8192", "ragged_clamp", "odd_t257", "c1_slice", "config1"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from isa_b200 import build
    build.build_library()


def test_fixtures_present():
    missing = [c for c in CASES if not (GOLDEN / f"golden_cuda_{c}.npz").exists()]
    assert not missing, f"minted fixtures missing: {missing}"


@pytest.mark.parametrize("case", CASES)
def test_reference_cuda_backward(case):
    path = GOLDEN / f"golden_cuda_{case}.npz"
    if not path.exists():
        pytest.skip(f"{path.name} not minted")
    with np.load(path) as z:
        gold = {k: z[k] for k in z.files}
    tib, tdb, dmin, scale, size = cfg_tables(int(gold["size"]))
    lut = pack(tib, tdb)
    ti, td = bf16_bits_to_f32(tib), bf16_bits_to_f32(tdb)
    x, wp, wn, g = gold["x"], gold["wpos"], gold["wneg"], gold["grad_out"]
    out = gpu_forward(x, wp, wn, lut, dmin, scale, size)
    _, mag = oracle.forward(x, wp, wn, ti, dmin, scale, CFG_V_SAT, with_mag=True)
    assert_close_scaled(out, gold["out"], mag, what=f"{case} forward vs reference Triton")
    gx, gwp, gwn = gpu_backward(x, wp, wn, g, lut, dmin, scale, size)
    _, (mx, mwp, mwn) = oracle.backward(x, wp, wn, g, ti, td, dmin, scale, CFG_V_SAT, with_mag=True)
    assert_close_scaled(gx, gold["grad_x"], mx, what=f"{case} grad_x vs reference CUDA")
    assert_close_scaled(gwp, gold["grad_wpos"], mwp, what=f"{case} grad_wpos vs reference CUDA")
    assert_close_scaled(gwn, gold["grad_wneg"], mwn, what=f"{case} grad_wneg vs reference CUDA")
