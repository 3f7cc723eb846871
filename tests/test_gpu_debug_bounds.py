"""Bounds audit of the table lookups: the debug library variant (built with
CIMEKV_DEBUG_BOUNDS=1) checks every shared-memory table index of the forward
and backward kernels against the table size and counts violations.  Adversarial
inputs (coordinates exactly on and just beyond both table edges, infinities,
NaN, ragged shapes) must produce zero violations, and the debug build's outputs
must be bit-identical to the release build's."""

import numpy as np
import pytest
import torch

from tests.test_gpu_parity import CFG_V_SAT, cfg_tables, pack

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def libs():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from isa_b200 import _lib, build
    build.build_library()
    dbg = _lib.open_variant(build.build_library(debug=True))
    rel = _lib.load()
    assert dbg.cimekv_debug_build() == 1 and rel.cimekv_debug_build() == 0
    dbg.cimekv_debug_oob_count(1)
    return rel, dbg


def _edge_values(dmin, scale, size, n, rng):
    """dV values whose table coordinate sits on, just inside and just outside
    both table edges, plus random in-range and far out-of-range values."""
    f32 = np.float32
    lo = f32(dmin)
    hi = f32(dmin + (size - 1) / scale)
    cands = [lo, np.nextafter(lo, f32(-np.inf)), np.nextafter(lo, f32(np.inf)),
             hi, np.nextafter(hi, f32(-np.inf)), np.nextafter(hi, f32(np.inf)),
             f32(dmin + size / scale), f32(dmin - 1 / scale), f32(1e30), f32(-1e30)]
    vals = rng.choice(np.array(cands, dtype=np.float32), n)
    mix = rng.random(n)
    vals = np.where(mix < 0.3, rng.uniform(lo, hi, n).astype(np.float32), vals)
    return vals.astype(np.float32)


def _run(lib, x, wp, wn, g, lut, dmin, scale, size):
    m, k = x.shape
    o = wp.shape[0]
    out = torch.full((m, o), float("nan"), device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.cimekv_forward(x.data_ptr(), wp.data_ptr(), wn.data_ptr(), lut.data_ptr(), m, k, o, size,
                              dmin, scale, CFG_V_SAT, -4.0, 4.0, out.data_ptr(), stream) == 0
    gx = torch.full_like(x, float("nan"))
    gwp = torch.full_like(wp, float("nan"))
    gwn = torch.full_like(wn, float("nan"))
    ws_bytes = lib.cimekv_backward_workspace_bytes(m, k, o, size)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    assert lib.cimekv_backward(x.data_ptr(), wp.data_ptr(), wn.data_ptr(), g.data_ptr(), lut.data_ptr(),
                               m, k, o, size, dmin, scale, CFG_V_SAT, gx.data_ptr(), gwp.data_ptr(),
                               gwn.data_ptr(), ws.data_ptr(), ws_bytes, stream) == 0
    torch.cuda.synchronize()
    return out, gx, gwp, gwn


def _same_bits(a, b):
    return torch.equal(a.view(torch.int32), b.view(torch.int32))


@pytest.mark.parametrize("shape,size", [((67, 33, 45), 16), ((129, 97, 130), 257), ((300, 64, 96), 4096),
                                        ((1025, 130, 70), 8192), ((64, 24, 3072), 16384), ((3, 1, 1), 8192)])
def test_no_out_of_bounds_index_on_edge_inputs(libs, shape, size):
    rel, dbg = libs
    m, k, o = shape
    tib, tdb, dmin, scale, _ = cfg_tables(size)
    lut = pack(tib, tdb)
    rng = np.random.default_rng(size + m)
    wp = (2.5 + rng.uniform(-0.1, 0.1, (o, k))).astype(np.float32)
    wn = (2.5 + rng.uniform(-0.1, 0.1, (o, k))).astype(np.float32)
    # x = w + dV for the positive column 0 so the edge coordinates hit exactly;
    # the other columns see nearby coordinates on both sides of the edges
    x = (wp[0][None, :] + _edge_values(dmin, scale, size, m * k, rng).reshape(m, k)).astype(np.float32)
    x[rng.random((m, k)) < 0.02] = np.inf
    x[rng.random((m, k)) < 0.02] = -np.inf
    x[rng.random((m, k)) < 0.02] = np.nan
    g = rng.standard_normal((m, o)).astype(np.float32)
    args = [torch.from_numpy(a).cuda() for a in (x, wp, wn, g)]
    want = _run(rel, *args, lut, dmin, scale, size)
    got = _run(dbg, *args, lut, dmin, scale, size)
    assert dbg.cimekv_debug_oob_count(1) == 0, "table index outside [0, T)"
    for a, b, what in zip(got, want, ("forward", "grad_x", "grad_wpos", "grad_wneg")):
        assert _same_bits(a, b), f"{what}: debug and release builds differ"

