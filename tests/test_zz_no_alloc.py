"""The allocation-free backward entry point (cimekv_backward_noalloc).

Some callers of this operator cannot allocate device memory around it (a host
runtime without a device allocator, code confined to a memory pool it does not
own, plugins that must not grow the footprint per call), so they cannot provide
the workspace cimekv_backward asks for.  The no-allocation variant uses a fixed
scratch array inside the library instead.  These tests call it through the C
ABI and compare it with cimekv_backward, twice in a row, since every call
reuses the same scratch.  The file name makes pytest collect it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from tests._util import assert_close_scaled, bf16_bits_to_f32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from isa_b200 import build
    build.build_library()


def _setup(m, k, o, size, seed):
    from tests.test_gpu_parity import cfg_tables, pack
    tib, tdb, dmin, scale, _ = cfg_tables(size)
    lut = pack(tib, tdb)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(m, k, device="cuda", generator=gen)
    wp = 2.5 + (torch.rand(o, k, device="cuda", generator=gen) * 2 - 1) * 0.10712
    wn = 2.5 + (torch.rand(o, k, device="cuda", generator=gen) * 2 - 1) * 0.10712
    return lut, (tib, tdb), dmin, scale, x, wp, wn, gen


def _both(x, wp, wn, g, lut, dmin, scale, size):
    from isa_b200 import _lib
    v_sat = 8.2624
    m, k = x.shape
    o = wp.shape[0]
    ref = [torch.empty_like(x), torch.empty_like(wp), torch.empty_like(wn)]
    ws = torch.empty(_lib.backward_workspace_bytes(m, k, o, size), dtype=torch.uint8, device="cuda")
    _lib.backward(x, wp, wn, g, lut, size, dmin, scale, v_sat, *ref, ws)
    got = [torch.full_like(x, float("nan")), torch.full_like(wp, float("nan")), torch.full_like(wn, float("nan"))]
    _lib.backward_noalloc(x, wp, wn, g, lut, size, dmin, scale, v_sat, *got)
    torch.cuda.synchronize()
    return [t.cpu().numpy() for t in ref], [t.cpu().numpy() for t in got]


@pytest.mark.parametrize("shape,size", [((300, 70, 130), 4096), ((32768, 384, 1536), 4096),
                                        ((8320, 256, 1024), 8192)])
def test_noalloc_matches_backward_two_calls_in_a_row(shape, size):
    m, k, o = shape
    lut, (tib, tdb), dmin, scale, x, wp, wn, gen = _setup(m, k, o, size, seed=m + o)
    dd = float(np.abs(bf16_bits_to_f32(tdb)).max())
    for call in range(2):  # the second call reuses the scratch the first one left
        g = torch.randn(m, o, device="cuda", generator=gen)
        (rx, rwp, rwn), (gx, gwp, gwn) = _both(x, wp, wn, g, lut, dmin, scale, size)
        # dX does not go through the scratch: same kernel, same result.
        np.testing.assert_array_equal(gx, rx)
        # dVth: same cells, possibly fewer token splits, so a different order
        # of the final fp32 sum; bound by sum_m |g| * max|dI/dV|.
        bound = g.abs().sum(0).unsqueeze(1).expand(o, k).cpu().numpy() * dd
        assert_close_scaled(gwp, rwp, bound, rtol=2e-6, what=f"call {call} dWpos")
        assert_close_scaled(gwn, rwn, bound, rtol=2e-6, what=f"call {call} dWneg")
        if m * k * o < 5e6:  # small case: also against the oracle at the suite's tolerance
            ti, td = bf16_bits_to_f32(tib), bf16_bits_to_f32(tdb)
            (ox, owp, own), (mx, mwp, mwn) = oracle.backward(
                x.cpu().numpy(), wp.cpu().numpy(), wn.cpu().numpy(), g.cpu().numpy(), ti, td, dmin, scale,
                8.2624, with_mag=True)
            assert_close_scaled(gx, ox, mx, what="noalloc grad_x vs oracle")
            assert_close_scaled(gwp, owp, mwp, what="noalloc grad_wpos vs oracle")
            assert_close_scaled(gwn, own, mwn, what="noalloc grad_wneg vs oracle")


def test_noalloc_rejects_layers_beyond_its_scratch():
    from isa_b200 import _lib
    lib = _lib.load()
    dummy = ctypes.c_void_p(256)
    # 4096 x 1100 thresholds need 2*4096*1100*4 B > 32 MiB of scratch per split.
    rc = lib.cimekv_backward_noalloc(dummy, dummy, dummy, dummy, dummy, 64, 1100, 4096, 4096,
                                     -9.0, 315.0, 8.2624, None, dummy, dummy, None)
    assert rc == 4
    assert b"scratch" in lib.cimekv_last_error()
