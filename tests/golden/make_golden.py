"""Generate golden vectors from the reference's own LUT kernels.

Run in a container that has the reference source tree (NOT on the GPU box):

    python tests/golden/make_golden.py /path/to/reference

It imports the reference package from ``<reference>/src`` and runs its Triton
kernels on CPU through the Triton interpreter (``TRITON_INTERPRET=1``):
  * ``LUTTritonEKVMatmulFn`` forward (``_forward_kernel``) and, with
    ``EKV_CUDA_SHARED_BACKWARD=0``, its Triton backward (``_grad_x_kernel``,
    ``_grad_w_kernel``) — ekv_lut_triton.py:37-218;
  * ``_lut_lookup`` on an index-revealing table (ekv_lut_triton.py:26-34);
  * the LUT builder ``_cpu_lut_cached`` (delta_lut.py:12-35).
Inputs are seeded and stored next to the outputs in ``golden_*.npz`` so the
tests need nothing but these files.
"""

from __future__ import annotations

import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(ref_root: str) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    os.environ["EKV_CUDA_SHARED_BACKWARD"] = "0"
    sys.path.insert(0, str(Path(ref_root) / "src"))
    import torch
    import triton
    import triton.language as tl

    from isa.approximations.delta_lut import _cpu_lut_cached, get_ekv_lut_tables
    from isa.device_models.config import make_flash_transistor_ekv_config
    from isa.kernels.transformer_ffn import ekv_lut_triton as ref
    from isa.operators.cim import CIMLinear

    globals()["ref"] = ref  # the probe kernel below resolves names in module globals

    def cfg_for(size: int) -> dict:
        cfg = make_flash_transistor_ekv_config(default_lut_size=size)
        cfg["LUT_DELTA_SIZE"] = size
        cfg["CUDA_SHARED_BACKWARD"] = False  # Triton backward (CUDA one needs a GPU)
        return cfg

    def geometry(cfg: dict):
        v_min = float(cfg.get("V_signed_min", -4.0))
        v_max = float(cfg.get("V_signed_max", 4.0))
        dmin = float(cfg.get("LUT_DELTA_MIN", v_min - float(cfg.get("V_TH_MAX", 5.0))))
        dmax = float(cfg.get("LUT_DELTA_MAX", v_max - float(cfg.get("V_TH_MIN", 0.0))))
        size = int(cfg["LUT_DELTA_SIZE"])
        return dmin, dmax, size

    def run_case(name, x, wp, wn, g, cfg):
        t0 = time.time()
        xt = torch.from_numpy(x).requires_grad_(True)
        pt = torch.from_numpy(wp).requires_grad_(True)
        nt = torch.from_numpy(wn).requires_grad_(True)
        out = ref.triton_lut_ekv_matmul(xt, pt, nt, cfg)
        out.backward(torch.from_numpy(g))
        ti, td = get_ekv_lut_tables(cfg, torch.device("cpu"))
        dmin, dmax, size = geometry(cfg)
        np.savez_compressed(
            HERE / f"golden_{name}.npz",
            x=x, wpos=wp, wneg=wn, grad_out=g,
            out=out.detach().numpy(), grad_x=xt.grad.numpy(),
            grad_wpos=pt.grad.numpy(), grad_wneg=nt.grad.numpy(),
            table_i=ti.view(torch.int16).numpy().view(np.uint16),
            table_ddelta=td.view(torch.int16).numpy().view(np.uint16),
            delta_min=np.float64(dmin), delta_max=np.float64(dmax), size=np.int64(size),
            v_sat=np.float64(cfg["V_sat"]),
            out_min=np.float64(cfg["V_signed_min"]), out_max=np.float64(cfg["V_signed_max"]),
        )
        print(f"{name}: M,K,O={x.shape[0]},{x.shape[1]},{wp.shape[0]} T={size} ({time.time() - t0:.1f}s)")

    def vth_init(o, k, seed_p, seed_n, cfg):
        # CIMLinear's default init (centered_random, eps_k=0.5; cim.py:113-138):
        # vth_pos from a module built under seed_p, vth_neg from one under seed_n.
        torch.manual_seed(seed_p)
        wp = CIMLinear(k, o, cfg).vth_pos.detach().numpy().copy()
        torch.manual_seed(seed_n)
        wn = CIMLinear(k, o, cfg).vth_neg.detach().numpy().copy()
        return wp.astype(np.float32), wn.astype(np.float32)

    rng = np.random.default_rng(20261201)

    # 1-2. Small shapes at both production table sizes, CIMLinear init.
    for size in (8192, 4096):
        cfg = cfg_for(size)
        m, k, o = 32, 64, 64
        x = rng.standard_normal((m, k)).astype(np.float32)
        wp, wn = vth_init(o, k, 1, 2, cfg)
        g = rng.standard_normal((m, o)).astype(np.float32)
        run_case(f"small_t{size}", x, wp, wn, g, cfg)

    # 3. Ragged shape, inputs that drive dV past both table ends (clamp paths).
    cfg = cfg_for(4096)
    m, k, o = 19, 37, 45
    x = rng.uniform(-8.0, 8.0, (m, k)).astype(np.float32)
    wp = rng.uniform(0.0, 5.0, (o, k)).astype(np.float32)
    wn = rng.uniform(0.0, 5.0, (o, k)).astype(np.float32)
    g = rng.standard_normal((m, o)).astype(np.float32)
    run_case("ragged_clamp", x, wp, wn, g, cfg)

    # 4. Odd, small table (T=257) with voltage-mapped inputs in [0, 4].
    cfg = cfg_for(257)
    m, k, o = 24, 40, 33
    x = np.clip(rng.standard_normal((m, k)) + 2.0, 0.0, 4.0).astype(np.float32)
    wp, wn = vth_init(o, k, 5, 6, cfg)
    g = rng.standard_normal((m, o)).astype(np.float32)
    run_case("odd_t257", x, wp, wn, g, cfg)

    # 5. A slice of config 1 (x[256,192] ~ N(0,1) seed 0, Vth seeds 1/2,
    #    grad ~ N(0,1) seed 3, T=8192): the first 16 tokens, all 768 outputs.
    cfg = cfg_for(8192)
    torch.manual_seed(0)
    x_full = torch.randn(256, 192).numpy()
    wp, wn = vth_init(768, 192, 1, 2, cfg)
    torch.manual_seed(3)
    g_full = torch.randn(256, 768).numpy()
    run_case("c1_slice", x_full[:16].copy(), wp, wn, g_full[:16].copy(), cfg)

    # 6. Index selection: reference _lut_lookup on table[j] = j (exact in fp32)
    #    over dV values that sit on and next to table nodes and beyond both ends.
    @triton.jit
    def lookup_probe(table, delta, out, n, DMIN: tl.constexpr, DMAX: tl.constexpr, SIZE: tl.constexpr,
                     BLOCK: tl.constexpr):
        offs = tl.program_id(0) * BLOCK + tl.arange(0, BLOCK)
        mask = offs < n
        d = tl.load(delta + offs, mask=mask, other=0.0)
        tl.store(out + offs, ref._lut_lookup(table, d, DMIN, DMAX, SIZE), mask=mask)

    probes = {}
    for size in (8192, 4096):
        cfg = cfg_for(size)
        dmin, dmax, size = geometry(cfg)
        step = (dmax - dmin) / (size - 1)
        nodes = dmin + step * rng.integers(0, size, 4000)
        near = np.concatenate([
            nodes, np.nextafter(nodes.astype(np.float32), np.float32(-np.inf)),
            np.nextafter(nodes.astype(np.float32), np.float32(np.inf)),
            rng.uniform(dmin - 3.0, dmax + 3.0, 8000),
            [dmin, dmax, dmin - 1e-7, dmax + 1e-7, -100.0, 100.0, 0.0],
        ]).astype(np.float32)
        table = torch.arange(size, dtype=torch.float32)
        out = torch.empty(near.size, dtype=torch.float32)
        lookup_probe[(triton.cdiv(near.size, 256),)](table, torch.from_numpy(near), out, near.size,
                                                      dmin, dmax, size, BLOCK=256)
        probes[f"delta_t{size}"] = near
        probes[f"lookup_t{size}"] = out.numpy()
        probes[f"dmin_t{size}"] = np.float64(dmin)
        probes[f"dmax_t{size}"] = np.float64(dmax)
    np.savez_compressed(HERE / "golden_index.npz", **probes)
    print("index probes saved")

    # 7. Reference LUT builder at the reference test's key (tests/test_flash_formula.py:56-84).
    key = (4.1360, 8.2624, 0.75875, 0.026, 0.1, -1.0, 3.0, 257)
    ti, td = _cpu_lut_cached(key)
    np.savez_compressed(HERE / "golden_lut_testkey.npz",
                        key=np.array(key, dtype=np.float64),
                        table_i=ti.view(torch.int16).numpy().view(np.uint16),
                        table_ddelta=td.view(torch.int16).numpy().view(np.uint16))
    print("builder golden saved")

    # 8. Exact-formula path: the reference's exact Triton kernels
    #    (ekv_triton.py:69-150, TritonEKVMatmulFn) on two small cases.
    from isa.kernels.transformer_ffn import ekv_triton as ref_exact
    for name, (m, k, o), lo, hi in (("exact_small", (32, 48, 40), -1.0, 1.0),
                                    ("exact_ragged", (19, 37, 45), -4.0, 4.0)):
        cfg = cfg_for(4096)
        x = rng.uniform(lo, hi, (m, k)).astype(np.float32) + 2.5
        wp, wn = vth_init(o, k, 7, 8, cfg)
        g = rng.standard_normal((m, o)).astype(np.float32)
        xt = torch.from_numpy(x).requires_grad_(True)
        pt = torch.from_numpy(wp).requires_grad_(True)
        nt = torch.from_numpy(wn).requires_grad_(True)
        out = ref_exact.triton_ekv_matmul(xt, pt, nt, cfg)
        out.backward(torch.from_numpy(g))
        np.savez_compressed(HERE / f"golden_{name}.npz", x=x, wpos=wp, wneg=wn, grad_out=g,
                            out=out.detach().numpy(), grad_x=xt.grad.numpy(), grad_wpos=pt.grad.numpy(),
                            grad_wneg=nt.grad.numpy(), n=np.float64(cfg["n"]), U_T=np.float64(cfg["U_T"]),
                            V_D=np.float64(cfg["V_D"]), I_S=np.float64(cfg["I_S"]), V_sat=np.float64(cfg["V_sat"]))
        print(f"{name} saved")

    # 8b. State-dict layout of the reference modules (checkpoint compatibility).
    import json
    from isa.operators.cim import HybridFFN, PhysicalFFN
    layout = {}
    for name, mod in (("CIMLinear", CIMLinear(12, 20)), ("PhysicalFFN", PhysicalFFN(12, 20)),
                      ("HybridFFN", HybridFFN(12, 20))):
        layout[name] = {k: [list(v.shape), str(v.dtype)] for k, v in mod.state_dict().items()}
    (HERE / "reference_state_dict_layout.json").write_text(json.dumps(layout, indent=1, sort_keys=True))
    print("state-dict layout saved")

    # 9. Measured-codebook forward (measured_deployment/operator.py:163-206),
    #    plain torch on CPU: 24 curves on a non-uniform Vg grid, random
    #    assignment, inputs partly outside the lookup range; autograd dX.
    from isa.measured_deployment.operator import DeploymentAwareCIMLinear
    for name, (m, k, o), g_pts in (("measured_small", (40, 48, 36), 33), ("measured_ragged", (19, 37, 45), 9)):
        torch.manual_seed(11)
        layer = DeploymentAwareCIMLinear(k, o)
        layer.set_r_tia(2.0e4)
        vg = np.sort(rng.uniform(-0.5, 4.5, g_pts)).astype(np.float32)
        vg[0], vg[-1] = -0.5, 4.5
        base = np.exp(rng.uniform(-14, -11, (24, 1))) * np.cumsum(rng.uniform(0.0, 1.0, (24, g_pts)), axis=1)
        currents = base.astype(np.float32)
        layer.configure_codebook(torch.from_numpy(vg), torch.from_numpy(currents))
        pos = rng.integers(0, 24, (o, k)).astype(np.int16)
        neg = rng.integers(0, 24, (o, k)).astype(np.int16)
        layer.set_assignment(torch.from_numpy(pos), torch.from_numpy(neg))
        layer.set_forward_mode("measured")
        x = rng.uniform(-1.0, 5.0, (1, m, k)).astype(np.float32)
        xt = torch.from_numpy(x).requires_grad_(True)
        out = layer(xt)
        g = rng.standard_normal(out.shape).astype(np.float32)
        out.backward(torch.from_numpy(g))
        np.savez_compressed(HERE / f"golden_{name}.npz", x=x[0], vg=vg, currents=currents, pos=pos, neg=neg,
                            r_tia=np.float64(2.0e4), out=out.detach().numpy()[0], grad_out=g[0],
                            grad_x=xt.grad.numpy()[0], lookup_min=np.float64(layer.lookup_min),
                            lookup_max=np.float64(layer.lookup_max))
        print(f"{name} saved")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: make_golden.py <reference source tree>")
    main(sys.argv[1])
