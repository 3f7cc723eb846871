"""Golden vectors from the reference's DEFAULT GPU backward.

The reference's default backward for the LUT path (``CUDA_SHARED_BACKWARD``
true, ``device_models/config.py:37``) is its JIT-built CUDA extension
(``kernels/transformer_ffn/cuda/ekv_cuda.cu:193-341``, ``grad_x_shared`` and
``grad_w_shared``), reached through ``LUTTritonEKVMatmulFn.backward``
(``ekv_lut_triton.py:176-200``).  It needs a GPU, so this script runs on a GPU
box against the unmodified reference package installed in ``baseline/_ref``:

    python tests/golden/make_golden_cuda.py [out_dir]

It re-runs the reference on the inputs stored in the Triton-minted fixtures
(``golden_<case>.npz``, written by make_golden.py) and on benchmark config 1 at
full size, and writes ``golden_cuda_<case>.npz`` holding the inputs, the
reference's Triton forward output and its CUDA-backward gradients.
"""

from __future__ import annotations

import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
CASES = ("small_t4096", "small_t8192", "ragged_clamp", "odd_t257", "c1_slice")


def main(out_dir: Path) -> None:
    sys.path.insert(0, str(REPO / "baseline" / "_ref"))
    os.environ.setdefault("EKV_CUDA_SHARED_BACKWARD", "1")
    import torch

    from isa.device_models.config import make_flash_transistor_ekv_config
    from isa.kernels.transformer_ffn import ekv_lut_triton as ref
    from isa.operators.cim import CIMLinear

    assert torch.cuda.is_available(), "needs a GPU"
    dev = torch.device("cuda", 0)
    out_dir.mkdir(parents=True, exist_ok=True)

    def run(name, x, wp, wn, g, size):
        t0 = time.time()
        cfg = make_flash_transistor_ekv_config(default_lut_size=size)
        cfg["LUT_DELTA_SIZE"] = int(size)
        cfg["CUDA_SHARED_BACKWARD"] = True
        xt = torch.from_numpy(x).to(dev).requires_grad_(True)
        pt = torch.from_numpy(wp).to(dev).requires_grad_(True)
        nt = torch.from_numpy(wn).to(dev).requires_grad_(True)
        out = ref.triton_lut_ekv_matmul(xt, pt, nt, cfg)
        out.backward(torch.from_numpy(g).to(dev))
        torch.cuda.synchronize()
        np.savez_compressed(
            out_dir / f"golden_cuda_{name}.npz", x=x, wpos=wp, wneg=wn, grad_out=g, size=np.int64(size),
            out=out.detach().cpu().numpy(), grad_x=xt.grad.cpu().numpy(),
            grad_wpos=pt.grad.cpu().numpy(), grad_wneg=nt.grad.cpu().numpy())
        print(f"{name}: M,K,O={x.shape[0]},{x.shape[1]},{wp.shape[0]} T={size} ({time.time() - t0:.1f}s)", flush=True)

    for case in CASES:
        d = np.load(HERE / f"golden_{case}.npz")
        run(case, d["x"], d["wpos"], d["wneg"], d["grad_out"], int(d["size"]))

    # Benchmark config 1 at full size: x[256,192] ~ N(0,1) seed 0, one
    # CIMLinear(192, 768) built under seed 1 (its default init), grad ~ N(0,1)
    # seed 3, T = 8192.
    torch.manual_seed(0)
    x = torch.randn(256, 192).numpy()
    torch.manual_seed(1)
    lin = CIMLinear(192, 768)
    torch.manual_seed(3)
    g = torch.randn(256, 768).numpy()
    run("config1", x, lin.vth_pos.detach().numpy().copy(), lin.vth_neg.detach().numpy().copy(), g, 8192)


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else HERE)
