"""ctypes front end of the C oracle (``cimekv_oracle.c``) — TEST INFRASTRUCTURE ONLY.

The C code restates the reference LUT forward (Triton ``_forward_kernel``,
``ekv_lut_triton.py:26-62``) and the reference CUDA shared-memory backward
(``ekv_cuda.cu:59-87,193-341``).  ``lut_index_np`` restates the index rule in
numpy as an independent second implementation for cross-checks.
"""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "_build" / "liboracle_cimekv.so"

_lib = None


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB.exists():
            build()
        lib = ctypes.CDLL(str(LIB))
        f, i, vp = ctypes.c_float, ctypes.c_int, ctypes.c_void_p
        lib.oracle_max_threads.restype = i
        lib.oracle_lut_index.argtypes = [vp, i, i, f, f, vp, vp]
        lib.oracle_forward.argtypes = [vp, vp, vp, vp, i, i, i, i, f, f, f, f, f, vp, vp, i]
        lib.oracle_backward.argtypes = [vp, vp, vp, vp, vp, vp, i, i, i, i, f, f, f,
                                        vp, vp, vp, vp, vp, vp, i]
        d = ctypes.c_double
        lib.oracle_exact_forward.argtypes = [vp, vp, vp, i, i, i, d, d, d, d, vp, vp, i]
        lib.oracle_exact_backward.argtypes = [vp, vp, vp, vp, i, i, i, d, d, d, d, vp, vp, vp, vp, vp, vp, i]
        _lib = lib
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


def max_threads() -> int:
    return int(load().oracle_max_threads())


def lut_index(delta, table_size: int, delta_min: float, scale: float):
    d = _f32(delta).ravel()
    idx = np.empty(d.shape, np.int32)
    alpha = np.empty(d.shape, np.float32)
    load().oracle_lut_index(_p(d), d.size, int(table_size), float(delta_min), float(scale), _p(idx), _p(alpha))
    return idx, alpha


def lut_index_np(delta, table_size: int, delta_min: float, scale: float):
    """Index rule in numpy fp32 (ekv_lut_triton.py:27-31)."""
    d = _f32(delta)
    f = (d - np.float32(delta_min)) * np.float32(scale)
    f = np.minimum(np.maximum(f, np.float32(0.0)), np.float32(table_size - 1))
    i0 = np.trunc(f).astype(np.int32)
    return i0, (f - i0.astype(np.float32)).astype(np.float32)


def forward(x, wp, wn, table_i, delta_min, scale, v_sat, out_min=-4.0, out_max=4.0, nthreads=0,
            with_mag=False):
    x, wp, wn, ti = _f32(x), _f32(wp), _f32(wn), _f32(table_i)
    m, k = x.shape
    o = wp.shape[0]
    out = np.empty((m, o), np.float32)
    mag = np.empty((m, o), np.float32) if with_mag else None
    load().oracle_forward(_p(x), _p(wp), _p(wn), _p(ti), m, k, o, ti.size, float(delta_min), float(scale),
                          float(v_sat), float(out_min), float(out_max), _p(out), _p(mag), int(nthreads))
    return (out, mag) if with_mag else out


def backward(x, wp, wn, g, table_i, table_dd, delta_min, scale, v_sat, need_x=True, need_w=True,
             nthreads=0, with_mag=False):
    x, wp, wn, g = _f32(x), _f32(wp), _f32(wn), _f32(g)
    ti, td = _f32(table_i), _f32(table_dd)
    m, k = x.shape
    o = wp.shape[0]
    gx = np.empty((m, k), np.float32) if need_x else None
    gwp = np.empty((o, k), np.float32) if need_w else None
    gwn = np.empty((o, k), np.float32) if need_w else None
    mx = np.empty((m, k), np.float32) if (with_mag and need_x) else None
    mwp = np.empty((o, k), np.float32) if (with_mag and need_w) else None
    mwn = np.empty((o, k), np.float32) if (with_mag and need_w) else None
    load().oracle_backward(_p(x), _p(wp), _p(wn), _p(g), _p(ti), _p(td), m, k, o, ti.size, float(delta_min),
                           float(scale), float(v_sat), _p(gx), _p(gwp), _p(gwn), _p(mx), _p(mwp), _p(mwn),
                           int(nthreads))
    if with_mag:
        return (gx, gwp, gwn), (mx, mwp, mwn)
    return gx, gwp, gwn


def exact_consts(cfg) -> tuple[float, float, float, float]:
    """(1/(2 n U_T), V_D, I_S, V_sat) of a cfg dict, as the reference computes them."""
    return 1.0 / (2.0 * float(cfg["n"]) * float(cfg["U_T"])), float(cfg["V_D"]), float(cfg["I_S"]), float(cfg["V_sat"])


def exact_forward(x, wp, wn, inv, vd, i_s, v_sat, nthreads=0, with_mag=False):
    """Exact-formula forward in fp64 (flash_transistor.py:27-41 semantics)."""
    x, wp, wn = _f32(x), _f32(wp), _f32(wn)
    m, k = x.shape
    o = wp.shape[0]
    out = np.empty((m, o), np.float32)
    mag = np.empty((m, o), np.float32) if with_mag else None
    load().oracle_exact_forward(_p(x), _p(wp), _p(wn), m, k, o, inv, vd, i_s, v_sat, _p(out), _p(mag), int(nthreads))
    return (out, mag) if with_mag else out


def exact_backward(x, wp, wn, g, inv, vd, i_s, v_sat, need_x=True, need_w=True, nthreads=0, with_mag=False):
    """Exact-formula gradients in fp64 (flash_transistor.py:44-82 semantics)."""
    x, wp, wn, g = _f32(x), _f32(wp), _f32(wn), _f32(g)
    m, k = x.shape
    o = wp.shape[0]
    gx = np.empty((m, k), np.float32) if need_x else None
    gwp = np.empty((o, k), np.float32) if need_w else None
    gwn = np.empty((o, k), np.float32) if need_w else None
    mx = np.empty((m, k), np.float32) if (with_mag and need_x) else None
    mwp = np.empty((o, k), np.float32) if (with_mag and need_w) else None
    mwn = np.empty((o, k), np.float32) if (with_mag and need_w) else None
    load().oracle_exact_backward(_p(x), _p(wp), _p(wn), _p(g), m, k, o, inv, vd, i_s, v_sat, _p(gx), _p(gwp),
                                 _p(gwn), _p(mx), _p(mwp), _p(mwn), int(nthreads))
    if with_mag:
        return (gx, gwp, gwn), (mx, mwp, mwn)
    return gx, gwp, gwn
