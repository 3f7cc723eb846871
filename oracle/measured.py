"""fp64 restatement of the measured-codebook forward — TEST INFRASTRUCTURE ONLY.

Follows src/isa/measured_deployment/operator.py: per-segment slopes and
intercepts (:119-123), clamp of the input to the lookup range and
right-bisect segment selection (:171-196), sum over inputs of
x*(slope_p - slope_n) + (icpt_p - icpt_n), then * r_tia and the signed clamp
(:198-203).  The input gradient is the analytic derivative of that
piecewise-linear map (what autograd of the reference's masked GEMMs gives).
"""

from __future__ import annotations

import numpy as np


def coefficients(vg, currents):
    vg = np.asarray(vg, np.float64)
    cur = np.asarray(currents, np.float64)
    slopes = (cur[:, 1:] - cur[:, :-1]) / (vg[1:] - vg[:-1])[None, :]
    return slopes, cur[:, :-1] - slopes * vg[None, :-1]


def forward(x, vg, currents, pos, neg, lookup_min, lookup_max, r_tia, lo=-4.0, hi=4.0):
    """Returns (out, idiff, mag) with mag = sum |x da| + |db| per output."""
    x = np.asarray(x, np.float64)
    a, b = coefficients(vg, currents)
    xc = np.clip(x, lookup_min, lookup_max)
    seg = np.clip(np.searchsorted(np.asarray(vg, np.float64), xc, side="right") - 1, 0, len(vg) - 2)
    pos = np.asarray(pos, np.int64)
    neg = np.asarray(neg, np.int64)
    m, k = x.shape
    o = pos.shape[0]
    idiff = np.zeros((m, o))
    mag = np.zeros((m, o))
    for kk in range(k):
        s = seg[:, kk][:, None]          # [m,1]
        da = a[pos[:, kk][None, :], s] - a[neg[:, kk][None, :], s]   # [m,o]
        db = b[pos[:, kk][None, :], s] - b[neg[:, kk][None, :], s]
        term = xc[:, kk][:, None] * da + db
        idiff += term
        mag += np.abs(xc[:, kk][:, None] * da) + np.abs(db)
    return np.clip(idiff * r_tia, lo, hi), idiff, mag


def backward_x(x, vg, currents, pos, neg, lookup_min, lookup_max, r_tia, grad_out, lo=-4.0, hi=4.0):
    """(grad_x, mag) of the measured forward."""
    x = np.asarray(x, np.float64)
    a, _ = coefficients(vg, currents)
    _, idiff, _ = forward(x, vg, currents, pos, neg, lookup_min, lookup_max, r_tia, lo, hi)
    v = idiff * r_tia
    gm = np.asarray(grad_out, np.float64) * r_tia * ((v >= lo) & (v <= hi))
    xc = np.clip(x, lookup_min, lookup_max)
    seg = np.clip(np.searchsorted(np.asarray(vg, np.float64), xc, side="right") - 1, 0, len(vg) - 2)
    pos = np.asarray(pos, np.int64)
    neg = np.asarray(neg, np.int64)
    gx = np.zeros_like(x)
    mag = np.zeros_like(x)
    for kk in range(x.shape[1]):
        s = seg[:, kk][:, None]
        da = a[pos[:, kk][None, :], s] - a[neg[:, kk][None, :], s]
        gx[:, kk] = (gm * da).sum(1)
        mag[:, kk] = np.abs(gm * da).sum(1)
    inside = (x >= lookup_min) & (x <= lookup_max)
    return gx * inside, mag


def bin_ids(x, lookup_min, lookup_max, bins):
    """Input bin of every element, with the reference's fp32 arithmetic
    (operator.py:176-188): clamp to the lookup range, (x - min) * (bins-1)/(max-min),
    round half to even, clamp to [0, bins-1]; one bin maps everything to bin 0."""
    xf = np.clip(np.asarray(x, np.float32), np.float32(lookup_min), np.float32(lookup_max))
    if bins == 1:
        return np.zeros(xf.shape, np.int64)
    scale = np.float32((bins - 1) / (lookup_max - lookup_min))
    t = (xf - np.float32(lookup_min)).astype(np.float32) * scale
    return np.clip(np.round(t.astype(np.float32)), 0, bins - 1).astype(np.int64)


def forward_binned(x, vg, currents, pos, neg, lookup_min, lookup_max, r_tia, bins, centers, lo=-4.0, hi=4.0):
    """Binned-input measured forward (operator.py:99-110, 176-188) in fp64:
    every curve evaluated at the bin centres (currents_at, :147-161), the per-cell
    difference of the pos / neg devices at the input's bin, summed over inputs,
    then * r_tia and the signed clamp.  Returns (out, idiff, mag)."""
    vg = np.asarray(vg, np.float64)
    cur = np.asarray(currents, np.float64)
    c = np.clip(np.asarray(centers, np.float64), vg[0], vg[-1])
    upper = np.clip(np.searchsorted(vg, c, side="right"), 1, len(vg) - 1)
    lower = upper - 1
    alpha = (c - vg[lower]) / (vg[upper] - vg[lower])
    table = cur[:, lower] + alpha[None, :] * (cur[:, upper] - cur[:, lower])  # [S][bins]
    ids = bin_ids(x, lookup_min, lookup_max, bins)
    pos = np.asarray(pos, np.int64)
    neg = np.asarray(neg, np.int64)
    m, k = ids.shape
    o = pos.shape[0]
    idiff = np.zeros((m, o))
    mag = np.zeros((m, o))
    for kk in range(k):
        b = ids[:, kk][:, None]
        vp = table[pos[:, kk][None, :], b]
        vn = table[neg[:, kk][None, :], b]
        idiff += vp - vn
        mag += np.abs(vp) + np.abs(vn)
    return np.clip(idiff * r_tia, lo, hi), idiff, mag
