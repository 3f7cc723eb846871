"""Golden vectors of the reference's binned-input measured codebook.

Run where the reference source tree is available (NOT on the GPU box):

    python tests/golden/make_golden_binned.py /path/to/reference

Imports ``DeploymentAwareCIMLinear`` from ``<reference>/src`` and runs its
measured forward on CPU with ``configure_codebook(..., vin_lut_bins=B)``
(measured_deployment/operator.py:88-110 builds the per-bin difference
currents, :176-188 bins the inputs and sums them with masked GEMMs).  Inputs are
seeded and stored next to the outputs in ``golden_measured_binned*.npz``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    sys.path.insert(0, str(Path(ref_root) / "src"))
    import torch

    from isa.measured_deployment.operator import DeploymentAwareCIMLinear

    rng = np.random.default_rng(2024)
    cases = (("measured_binned", (40, 48, 36), 33, 32), ("measured_binned_one", (7, 9, 11), 9, 1),
             ("measured_binned_ragged", (19, 37, 45), 12, 257))
    for name, (m, k, o), g_pts, bins in cases:
        torch.manual_seed(13)
        layer = DeploymentAwareCIMLinear(k, o)
        layer.set_r_tia(2.0e4)
        vg = np.sort(rng.uniform(-0.5, 4.5, g_pts)).astype(np.float32)
        vg[0], vg[-1] = -0.5, 4.5
        base = np.exp(rng.uniform(-14, -11, (24, 1))) * np.cumsum(rng.uniform(0.0, 1.0, (24, g_pts)), axis=1)
        currents = base.astype(np.float32)
        layer.configure_codebook(torch.from_numpy(vg), torch.from_numpy(currents), vin_lut_bins=bins)
        pos = rng.integers(0, 24, (o, k)).astype(np.int16)
        neg = rng.integers(0, 24, (o, k)).astype(np.int16)
        layer.set_assignment(torch.from_numpy(pos), torch.from_numpy(neg))
        layer.set_forward_mode("measured")
        x = rng.uniform(-1.0, 5.0, (1, m, k)).astype(np.float32)
        with torch.no_grad():
            out = layer(torch.from_numpy(x))
        np.savez_compressed(HERE / f"golden_{name}.npz", x=x[0], vg=vg, currents=currents, pos=pos, neg=neg,
                            r_tia=np.float64(2.0e4), bins=np.int64(bins), out=out.numpy()[0],
                            bin_centers=layer.bin_centers.numpy(),
                            lookup_min=np.float64(layer.lookup_min), lookup_max=np.float64(layer.lookup_max))
        print(f"{name} saved")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden_binned.py <reference source tree>")
    main(sys.argv[1])
