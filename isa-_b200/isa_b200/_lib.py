"""ctypes binding of ``libcimekv.so`` (the C ABI in ``include/cimekv.h``).

Every wrapper takes torch tensors, checks them the way the reference's
``check_float_cuda_contiguous`` does (``ekv_cuda.cu:343-347``: CUDA, float32,
contiguous) and raises ``RuntimeError`` carrying ``cimekv_last_error()`` when
the library reports a failure.  There is no fallback: without the library the
import of this module fails.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(os.environ.get("CIMEKV_LIB", Path(__file__).resolve().parent / "_lib" / "libcimekv.so"))

_c_int, _c_float, _c_size, _vp = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_void_p

# name -> (restype, argtypes); mirrors include/cimekv.h
SIGNATURES = {
    "cimekv_abi_version": (_c_int, []),
    "cimekv_last_error": (ctypes.c_char_p, []),
    "cimekv_lut_bytes": (_c_size, [_c_int]),
    "cimekv_lut_pack": (_c_int, [_vp, _vp, _c_int, _vp, _vp]),
    "cimekv_forward": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                _c_float, _c_float, _c_float, _c_float, _c_float, _vp, _vp]),
    "cimekv_forward_tia": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                    _c_float, _c_float, _c_float, _c_float, _c_float, _vp,
                                    _c_float, _c_float, _vp, _vp, _vp]),
    "cimekv_tia_workspace_bytes": (_c_size, [ctypes.c_longlong]),
    "cimekv_tia_backward": (_c_int, [_vp, _vp, _vp, ctypes.c_longlong, _c_float, _c_float, _vp, _vp, _vp,
                                     _c_size, _vp]),
    "cimekv_backward_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, _c_int]),
    "cimekv_backward": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                 _c_float, _c_float, _c_float, _vp, _vp, _vp, _vp, _c_size, _vp]),
    "cimekv_backward_noalloc": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int,
                                         _c_float, _c_float, _c_float, _vp, _vp, _vp, _vp]),
    "cimekv_exact_forward": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_float, _c_float, _c_float,
                                      _c_float, _vp, _vp]),
    "cimekv_exact_backward_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int]),
    "cimekv_exact_backward": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_float, _c_float, _c_float,
                                       _c_float, _vp, _vp, _vp, _vp, _c_size, _vp]),
    "cimekv_measured_forward": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                         _c_float, _c_float, _vp, _c_float, _c_float, _vp, _vp, _vp]),
    "cimekv_measured_backward_x": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int,
                                            _c_float, _c_float, _vp, _c_float, _c_float, _vp, _vp, _vp, _vp]),
    "cimekv_lut_index": (_c_int, [_vp, _c_int, _c_int, _c_float, _c_float, _vp, _vp, _vp]),
    "cimekv_debug_build": (_c_int, []),
    "cimekv_debug_oob_count": (ctypes.c_uint, [_c_int]),
    "cimekv_fp32_probe": (_c_int, [_vp, _c_int, _c_int, ctypes.POINTER(ctypes.c_longlong), _vp]),
}

_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load the library once (raises if it has not been built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not _LIB_PATH.exists():
                raise RuntimeError(
                    f"libcimekv.so not found at {_LIB_PATH}; build it with `python -m isa_b200.build` "
                    "(there is no CPU fallback for the CIM operator)"
                )
            lib = ctypes.CDLL(str(_LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def open_variant(path) -> ctypes.CDLL:
    """Open another build of the library (e.g. the bounds-checking
    libcimekv_debug.so) side by side with the default one, with the same
    prototypes. The wrappers in this module keep using the default library."""
    lib = ctypes.CDLL(str(path))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


def library_path() -> Path:
    return _LIB_PATH


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().cimekv_last_error().decode(errors="replace")
        raise RuntimeError(f"{what} failed (status {rc}): {msg}")


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(stream) -> int | None:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    return stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream)


def check_float_cuda_contiguous(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise RuntimeError(f"{name} must be float32")
    if not t.is_contiguous():
        raise RuntimeError(f"{name} must be contiguous")


def lut_bytes(table_size: int) -> int:
    n = load().cimekv_lut_bytes(int(table_size))
    if n == 0:
        raise RuntimeError(f"unsupported LUT size {table_size}")
    return int(n)


def lut_pack(table_i: torch.Tensor, table_ddelta: torch.Tensor, table_size: int, packed: torch.Tensor,
             stream=None) -> None:
    for t, n in ((table_i, "table_i"), (table_ddelta, "table_ddelta")):
        if not t.is_cuda or t.dtype != torch.bfloat16 or not t.is_contiguous() or t.numel() != table_size:
            raise RuntimeError(f"{n} must be a contiguous CUDA bf16 tensor of {table_size} entries")
    rc = load().cimekv_lut_pack(_ptr(table_i), _ptr(table_ddelta), int(table_size), _ptr(packed), _stream(stream))
    _check(rc, "cimekv_lut_pack")


def forward(x, wpos, wneg, lut, table_size, delta_min, delta_scale, v_sat, out_min, out_max, out,
            stream=None) -> None:
    m, k = x.shape
    o = wpos.shape[0]
    rc = load().cimekv_forward(_ptr(x), _ptr(wpos), _ptr(wneg), _ptr(lut), m, k, o, int(table_size),
                               delta_min, delta_scale, v_sat, out_min, out_max, _ptr(out), _stream(stream))
    _check(rc, "cimekv_forward")


def forward_tia(x, wpos, wneg, lut, table_size, delta_min, delta_scale, v_sat, idiff_min, idiff_max, r_tia,
                out_min, out_max, idiff, out, stream=None) -> None:
    m, k = x.shape
    o = wpos.shape[0]
    rc = load().cimekv_forward_tia(_ptr(x), _ptr(wpos), _ptr(wneg), _ptr(lut), m, k, o, int(table_size),
                                   delta_min, delta_scale, v_sat, idiff_min, idiff_max, _ptr(r_tia),
                                   out_min, out_max, _ptr(idiff), _ptr(out), _stream(stream))
    _check(rc, "cimekv_forward_tia")


def tia_backward(grad_out, idiff, r_tia, out_min, out_max, grad_idiff, grad_r_tia, stream=None) -> None:
    n = idiff.numel()
    ws = torch.empty(int(load().cimekv_tia_workspace_bytes(n)), dtype=torch.uint8, device=idiff.device)
    rc = load().cimekv_tia_backward(_ptr(grad_out), _ptr(idiff), _ptr(r_tia), n, out_min, out_max,
                                    _ptr(grad_idiff), _ptr(grad_r_tia), _ptr(ws), ws.numel(), _stream(stream))
    _check(rc, "cimekv_tia_backward")


def backward_workspace_bytes(m: int, k: int, o: int, table_size: int) -> int:
    return int(load().cimekv_backward_workspace_bytes(int(m), int(k), int(o), int(table_size)))


def backward(x, wpos, wneg, grad_out, lut, table_size, delta_min, delta_scale, v_sat,
             grad_x, grad_wpos, grad_wneg, workspace, stream=None) -> None:
    m, k = x.shape
    o = wpos.shape[0]
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = load().cimekv_backward(_ptr(x), _ptr(wpos), _ptr(wneg), _ptr(grad_out), _ptr(lut), m, k, o,
                                int(table_size), delta_min, delta_scale, v_sat,
                                _ptr(grad_x), _ptr(grad_wpos), _ptr(grad_wneg),
                                _ptr(workspace), ws_bytes, _stream(stream))
    _check(rc, "cimekv_backward")


def backward_noalloc(x, wpos, wneg, grad_out, lut, table_size, delta_min, delta_scale, v_sat,
                     grad_x, grad_wpos, grad_wneg, stream=None) -> None:
    """cimekv_backward without a workspace: uses the library's fixed scratch."""
    m, k = x.shape
    o = wpos.shape[0]
    rc = load().cimekv_backward_noalloc(_ptr(x), _ptr(wpos), _ptr(wneg), _ptr(grad_out), _ptr(lut), m, k, o,
                                        int(table_size), delta_min, delta_scale, v_sat,
                                        _ptr(grad_x), _ptr(grad_wpos), _ptr(grad_wneg), _stream(stream))
    _check(rc, "cimekv_backward_noalloc")


def exact_forward(x, wpos, wneg, inv_2nut, v_d, i_s, v_sat, out, stream=None) -> None:
    m, k = x.shape
    o = wpos.shape[0]
    rc = load().cimekv_exact_forward(_ptr(x), _ptr(wpos), _ptr(wneg), m, k, o, inv_2nut, v_d, i_s, v_sat,
                                     _ptr(out), _stream(stream))
    _check(rc, "cimekv_exact_forward")


def exact_backward_workspace_bytes(m: int, k: int, o: int) -> int:
    return int(load().cimekv_exact_backward_workspace_bytes(int(m), int(k), int(o)))


def exact_backward(x, wpos, wneg, grad_out, inv_2nut, v_d, i_s, v_sat, grad_x, grad_wpos, grad_wneg, workspace,
                   stream=None) -> None:
    m, k = x.shape
    o = wpos.shape[0]
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = load().cimekv_exact_backward(_ptr(x), _ptr(wpos), _ptr(wneg), _ptr(grad_out), m, k, o,
                                      inv_2nut, v_d, i_s, v_sat, _ptr(grad_x), _ptr(grad_wpos), _ptr(grad_wneg),
                                      _ptr(workspace), ws_bytes, _stream(stream))
    _check(rc, "cimekv_exact_backward")


def measured_forward(x, pos_idx, neg_idx, vg, coef, lookup_min, lookup_max, r_tia, out_min, out_max, idiff, out,
                     stream=None) -> None:
    m, k = x.shape
    o = pos_idx.shape[0]
    s_, g_ = coef.shape[0], vg.numel()
    rc = load().cimekv_measured_forward(_ptr(x), _ptr(pos_idx), _ptr(neg_idx), _ptr(vg), _ptr(coef), m, k, o, s_, g_,
                                        lookup_min, lookup_max, _ptr(r_tia), out_min, out_max, _ptr(idiff), _ptr(out),
                                        _stream(stream))
    _check(rc, "cimekv_measured_forward")


def measured_backward_x(x, pos_idx, neg_idx, vg, coef, lookup_min, lookup_max, r_tia, out_min, out_max, idiff,
                        grad_out, grad_x, stream=None) -> None:
    m, k = x.shape
    o = pos_idx.shape[0]
    s_, g_ = coef.shape[0], vg.numel()
    rc = load().cimekv_measured_backward_x(_ptr(x), _ptr(pos_idx), _ptr(neg_idx), _ptr(vg), _ptr(coef), m, k, o,
                                           s_, g_, lookup_min, lookup_max, _ptr(r_tia), out_min, out_max,
                                           _ptr(idiff), _ptr(grad_out), _ptr(grad_x), _stream(stream))
    _check(rc, "cimekv_measured_backward_x")


def lut_index(delta: torch.Tensor, table_size: int, delta_min: float, delta_scale: float,
              stream=None) -> tuple[torch.Tensor, torch.Tensor]:
    check_float_cuda_contiguous(delta, "delta")
    index = torch.empty(delta.shape, dtype=torch.int32, device=delta.device)
    alpha = torch.empty(delta.shape, dtype=torch.float32, device=delta.device)
    rc = load().cimekv_lut_index(_ptr(delta), delta.numel(), int(table_size), delta_min, delta_scale,
                                 _ptr(index), _ptr(alpha), _stream(stream))
    _check(rc, "cimekv_lut_index")
    return index, alpha


def fp32_probe(sink: torch.Tensor, iters: int, blocks: int, stream=None) -> int:
    """Launch the FFMA probe; returns the lane-ops it issues."""
    ops = ctypes.c_longlong(0)
    rc = load().cimekv_fp32_probe(_ptr(sink), int(iters), int(blocks), ctypes.byref(ops), _stream(stream))
    _check(rc, "cimekv_fp32_probe")
    return int(ops.value)
