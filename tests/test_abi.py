"""The C-ABI library loads and exports every entry point include/*.h declares.
No compute calls here (no GPU); only the argument checks that run before any
CUDA call."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_symbols():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(cimekv_\w+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    from isa_b200 import build, _lib
    build.build_library()
    return _lib.load()


def test_header_declares_entry_points():
    assert {"cimekv_forward", "cimekv_backward", "cimekv_lut_pack"} <= set(declared_symbols())


def test_every_declared_symbol_is_exported(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), name


def test_binding_covers_header():
    from isa_b200 import _lib
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_host_side_argument_checks(lib):
    assert lib.cimekv_abi_version() == 1
    assert lib.cimekv_lut_bytes(4096) == 4096 * 8
    assert lib.cimekv_lut_bytes(1) == 0
    assert lib.cimekv_lut_bytes(1 << 20) == 0
    rc = lib.cimekv_forward(None, None, None, None, -1, 4, 4, 4096, -9.0, 315.0, 8.26, -4.0, 4.0, None, None)
    assert rc == 1 and b"negative" in lib.cimekv_last_error()
    rc = lib.cimekv_forward(None, None, None, None, 4, 4, 4, 1 << 20, -9.0, 315.0, 8.26, -4.0, 4.0, None, None)
    assert rc == 2
    rc = lib.cimekv_backward(None, None, None, None, None, 4, 4, 4, 4096, -9.0, 315.0, 8.26,
                             None, ctypes.c_void_p(16), None, None, 0, None)
    assert rc == 1 and b"both" in lib.cimekv_last_error()


def test_operator_refuses_cpu_tensors():
    torch = pytest.importorskip("torch")
    from isa_b200.kernels.transformer_ffn.ekv_lut import cuda_lut_ekv_matmul
    from isa_b200 import FLASH_TRANSISTOR_EKV_CONFIG as cfg
    x = torch.zeros(4, 8)
    w = torch.full((3, 8), 2.5)
    with pytest.raises(RuntimeError, match="CUDA"):
        cuda_lut_ekv_matmul(x, w, w, cfg)


def test_debug_variant_exports_the_same_symbols():
    """The bounds-checking build (CIMEKV_DEBUG_BOUNDS=1) is a drop-in for the
    release library and says which one it is."""
    from isa_b200 import _lib, build
    dbg = _lib.open_variant(build.build_library(debug=True))
    for name in declared_symbols():
        assert hasattr(dbg, name), name
    assert dbg.cimekv_debug_build() == 1
    assert _lib.load().cimekv_debug_build() == 0
