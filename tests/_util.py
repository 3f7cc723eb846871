"""Shared helpers of the test suite: golden fixtures and tolerance checks."""

from __future__ import annotations

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"

# fp32 parity bar: |got - want| <= RTOL * (sum of |terms|) + FLOOR * max(sum of |terms|).
# The sums are of cancelling differences, so the tolerance scales with the
# magnitude of the summed terms rather than with the (possibly tiny) result.
# FLOOR only matters for entries ~1e8 below the tensor's largest magnitude
# (e.g. dV far below the table, where terms are subnormal and reciprocal vs
# division rounding differs completely).
RTOL = 1e-5
FLOOR = 1e-8


def load_golden(name: str) -> dict:
    with np.load(GOLDEN / f"golden_{name}.npz") as z:
        return {k: z[k] for k in z.files}


GOLDEN_CASES = ["small_t8192", "small_t4096", "ragged_clamp", "odd_t257", "c1_slice"]


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def geometry(g: dict):
    """(dmin_f32, scale_f32, size) exactly as the kernels receive them."""
    size = int(g["size"])
    dmin = float(np.float32(g["delta_min"]))
    scale = float(np.float32((size - 1) / (float(g["delta_max"]) - float(g["delta_min"]))))
    return dmin, scale, size


def assert_close_scaled(got, want, mag, rtol=RTOL, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    mag = np.asarray(mag, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    floor = FLOOR * (float(mag.max()) if mag.size else 0.0) + np.finfo(np.float32).tiny
    err = np.abs(got - want)
    bound = rtol * mag + floor
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err / bound), err.shape)
        raise AssertionError(
            f"{what}: {bad.sum()} of {bad.size} outside rtol={rtol}*mag; worst at {i}: "
            f"got {got[i]!r} want {want[i]!r} mag {mag[i]!r}"
        )
