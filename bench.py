#!/usr/bin/env python
"""Benchmark of the Flash-EKV CIM FFN hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload gpt_m_ffn]

One step = forward + backward of one Physical FFN block (VoltageMapping ->
CIMLinear -> CIMLinear -> ADC affine) on the workload's tokens, bf16 autocast
around the block (the CIM path stays fp32), followed at N > 1 by the one
gradient all-reduce of data-parallel training.  Metric: fwd+bwd cell-evals/s,
one cell = one (token, input, output) triple of a CIM projection.
Per-GPU work is fixed (weak scaling): every rank processes the full token
count of the workload.

Prints ONE JSON line (rank 0).  The reference arm (``--impl reference``) times
the CPU restatement of the reference LUT path (oracle/) on the host cores on a
bounded token sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (ROOT, ROOT / "isa-_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

WORKLOADS = {
    # benchmark config 3: Physical GPT-M FFN block, batch 32 x seq 1024, T = 4096
    "gpt_m_ffn": dict(model="Physical GPT-M FFN block", d=384, hidden=1536, batch=32, seq=1024, lut=4096),
    # benchmark config 2: Physical ViT-M FFN block, batch 128 x 65 tokens, T = 8192
    "vit_m_ffn": dict(model="Physical ViT-M FFN block", d=256, hidden=1024, batch=128, seq=65, lut=8192),
    # Config 3, Hybrid variant: CIM up projection + bf16 digital nn.Linear down projection
    "gpt_m_ffn_hybrid": dict(model="Hybrid GPT-M FFN block", d=384, hidden=1536, batch=32, seq=1024, lut=4096,
                             hybrid=True),
    # Config 3 with the exact-formula path (cfg ekv_approx="exact"; the LUT is the default)
    "gpt_m_ffn_exact": dict(model="Physical GPT-M FFN block, exact EKV formula", d=384, hidden=1536, batch=32,
                            seq=1024, lut=4096, approx="exact"),
    # Measured-codebook fc1 (DeploymentAwareCIMLinear "measured" mode) at the ViT-L fc1 shape:
    # 256 images x 197 tokens, 384 -> 1536, 24 measured curves on a 33-point Vg grid
    "vit_l_fc1_measured": dict(model="ViT-L fc1, measured 24-state codebook", d=384, hidden=1536, batch=256,
                               seq=197, lut=8192, measured=True),
    # benchmark config 5: Physical ViT-L training step, 224x224 images, patch 16 (197 tokens), global batch 256
    "vit_l_step": dict(model="Physical ViT-L (d=384, 6 heads, 12 layers, hidden 1536, 200 classes)", d=384,
                       hidden=1536, batch=256, seq=197, lut=8192, layers=12),
    # benchmark config 4: Physical GPT-L full training step, global batch 64 x 1024 (strong scaling)
    "gpt_l_step": dict(model="Physical GPT-L (d=768, ffn 3072, 12 layers, 12 heads, vocab 50257)", d=768,
                       hidden=3072, batch=64, seq=1024, lut=4096, layers=12),
}

OPS_FWD, OPS_BWD = 16, 24  # algorithmic FP32 lane-ops per cell (forward, fused backward)
L2_FLUSH_BYTES = 256 << 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "reference_gpu"], default="ours",
                    help="reference_gpu: informational run of the unmodified reference's own GPU path "
                         "(Triton forward + JIT CUDA backward) installed in baseline/_ref")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="gpt_m_ffn")
    ap.add_argument("--cpu-sample-tokens", type=int, default=1024,
                    help="tokens of the CPU baseline sample (our arm)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the GPT-L step sub-record and the reference-GPU comparison of the default line")
    ap.add_argument("--gpt-l-steps", type=int, default=3, help="timed steps of the GPT-L and ViT-L sub-records")
    return ap.parse_args()


def cells_per_token(wl) -> int:
    """CIM cells per token: both projections (Physical) or the up projection only (Hybrid)."""
    return (1 if wl.get("hybrid") else 2) * wl["d"] * wl["hidden"]


# ------------------------------------------------------------------ clocks --

class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}

        def num(s):
            try:
                return float(s)
            except ValueError:
                return None
        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": num(rows[0][2]), "samples": len(rows), "reasons": reasons,
                "power_w_max": max((num(r[3]) or 0.0) for r in rows)}


# ------------------------------------------------------------- helpers ----

def host_cores() -> int:
    """Host threads this process may use (its CPU affinity), independent of
    OMP_NUM_THREADS, which torchrun sets to 1 for every rank."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return {}


def fp32_peak(dev) -> dict:
    """FFMA lane-op throughput of this GPU: burst (best single launch) and
    sustained (back-to-back launches for ~2 s, the regime of a long step)."""
    import torch

    from isa_b200 import _lib

    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    sink = torch.zeros(1, device=dev)
    blocks, iters = sms * 8, 4000
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        ops = _lib.fp32_probe(sink, iters, blocks)
    best = float("inf")
    for _ in range(5):
        s.record()
        ops = _lib.fp32_probe(sink, iters, blocks)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    n = max(1, int(2000.0 / best))
    s.record()
    for _ in range(n):
        _lib.fp32_probe(sink, iters, blocks)
    e.record()
    e.synchronize()
    return {"burst": ops / (best * 1e-3), "sustained": n * ops / (s.elapsed_time(e) * 1e-3)}


def make_ffn(wl, dev, seed=0, reference=False):
    import torch

    if reference:
        # The unmodified reference package (pip-installed into baseline/_ref),
        # through its own public module API: Triton LUT forward, JIT-built CUDA
        # shared-memory backward (its defaults).
        ref_dir = ROOT / "baseline" / "_ref"
        if not (ref_dir / "isa").exists():
            raise SystemExit("baseline/_ref is not installed")
        sys.path.insert(0, str(ref_dir))
        from isa.device_models.config import make_flash_transistor_ekv_config
        from isa.operators.cim import PhysicalFFN
    else:
        from isa_b200 import make_flash_transistor_ekv_config
        from isa_b200.operators.cim import HybridFFN, PhysicalFFN

    cfg = make_flash_transistor_ekv_config(default_lut_size=wl["lut"])
    cfg["LUT_DELTA_SIZE"] = wl["lut"]
    cfg["ekv_approx"] = wl.get("approx", "lut")
    torch.manual_seed(seed)
    if wl.get("hybrid"):
        if reference:
            from isa.operators.cim import HybridFFN
        return HybridFFN(wl["d"], wl["hidden"], cfg).to(dev), cfg
    return PhysicalFFN(wl["d"], wl["hidden"], cfg).to(dev), cfg


def ffn_step(ffn, x, gseed, allreduce):
    import torch

    for p in ffn.parameters():
        p.grad = None
    with torch.autocast("cuda", dtype=torch.bfloat16):
        z = ffn(x)
    loss = (z.float() * gseed).sum()
    loss.backward()
    if allreduce:
        from isa_b200.distributed import allreduce_gradients
        allreduce_gradients(ffn.parameters())
    return loss


def time_kernels(ffn, cfg, x, dev, reps=5):
    """CUDA-event time of one forward and one backward launch per projection
    (the stream the library launches on is torch's current stream)."""
    import torch

    from isa_b200 import _lib
    from isa_b200.approximations.delta_lut import get_packed_lut, lut_geometry

    geo = lut_geometry(cfg)
    lut = get_packed_lut(cfg, dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    res = {}
    with torch.no_grad():
        x1 = x.reshape(-1, x.shape[-1]).float().clamp(0, 4).contiguous()
        h = torch.empty(x1.shape[0], ffn.fc1.out_features, device=dev)
        _lib.forward(x1, ffn.fc1.vth_pos, ffn.fc1.vth_neg, lut, geo.size, geo.delta_min_f32, geo.scale,
                     float(cfg["V_sat"]), -4.0, 4.0, h)
        h = (h * ffn.fc1.r_tia).clamp(-4, 4).contiguous()
        from isa_b200.operators.cim import CIMLinear
        for name, lin, xin in (("fc1", ffn.fc1, x1), ("fc2", ffn.fc2, h)):
            if not isinstance(lin, CIMLinear):  # Hybrid: digital down projection
                continue
            m, k = xin.shape
            o = lin.out_features
            out = torch.empty(m, o, device=dev)
            g = torch.randn(m, o, device=dev)
            gx, gwp, gwn = torch.empty_like(xin), torch.empty_like(lin.vth_pos), torch.empty_like(lin.vth_neg)
            ws = torch.empty(_lib.backward_workspace_bytes(m, k, o, geo.size), dtype=torch.uint8, device=dev)
            t = {"fwd": [], "bwd": []}
            for i in range(reps + 1):
                for kind in ("fwd", "bwd"):
                    flush.zero_()
                    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    s.record()
                    if kind == "fwd":
                        _lib.forward(xin, lin.vth_pos, lin.vth_neg, lut, geo.size, geo.delta_min_f32, geo.scale,
                                     float(cfg["V_sat"]), -4.0, 4.0, out)
                    else:
                        _lib.backward(xin, lin.vth_pos, lin.vth_neg, g, lut, geo.size, geo.delta_min_f32,
                                      geo.scale, float(cfg["V_sat"]), gx, gwp, gwn, ws)
                    e.record()
                    e.synchronize()
                    if i > 0:
                        t[kind].append(s.elapsed_time(e))
            res[name] = {"cells": m * k * o, "fwd_ms": statistics.median(t["fwd"]),
                         "bwd_ms": statistics.median(t["bwd"])}
    return res


def cpu_sample(wl, tokens, nthreads=0, seed=0):
    """Oracle (CPU restatement of the reference LUT path) fwd+bwd of both
    projections of the block on `tokens` tokens.  Returns (cells, seconds)."""
    import numpy as np
    import torch

    from isa_b200 import make_flash_transistor_ekv_config
    from isa_b200.approximations.delta_lut import build_lut_tables_cpu, lut_geometry
    from isa_b200.operators.cim import CIMLinear
    from oracle import oracle

    cfg = make_flash_transistor_ekv_config(default_lut_size=wl["lut"])
    cfg["LUT_DELTA_SIZE"] = wl["lut"]
    geo = lut_geometry(cfg)
    ti, td = (t.float().numpy() for t in build_lut_tables_cpu(cfg))
    torch.manual_seed(seed)
    fc1, fc2 = CIMLinear(wl["d"], wl["hidden"], cfg), CIMLinear(wl["hidden"], wl["d"], cfg)
    rng = np.random.default_rng(seed)
    x = np.clip(rng.standard_normal((tokens, wl["d"])), 0, 4).astype(np.float32)
    args = (geo.delta_min_f32, geo.scale, float(cfg["V_sat"]))
    w1 = (fc1.vth_pos.detach().numpy(), fc1.vth_neg.detach().numpy())
    w2 = (fc2.vth_pos.detach().numpy(), fc2.vth_neg.detach().numpy())
    g2 = rng.standard_normal((tokens, wl["d"])).astype(np.float32)
    t0 = time.perf_counter()
    h = oracle.forward(x, *w1, ti, *args, nthreads=nthreads)
    h = np.clip(h * np.float32(1e5), -4, 4).astype(np.float32)
    oracle.forward(h, *w2, ti, *args, nthreads=nthreads)
    g1, _, _ = oracle.backward(h, *w2, g2, ti, td, *args, nthreads=nthreads)
    oracle.backward(x, *w1, g1 * np.float32(1e5), ti, td, *args, nthreads=nthreads)
    return tokens * cells_per_token(wl), time.perf_counter() - t0


def reference_pytorch_cpu(wl, tokens=64, seed=0) -> dict:
    """The reference's own PyTorch CPU path (its CIMLinear CPU branch: the exact
    EKV formula, then autograd), fwd+bwd of the unmodified reference block from
    baseline/_ref on `tokens` tokens with all host threads.  Informational: it
    evaluates the exact formula, not the LUT, so it is not the parity oracle."""
    import torch

    if not (ROOT / "baseline" / "_ref" / "isa").exists():
        return {"unavailable": "baseline/_ref (the pip-installed reference) is not present"}
    ffn, _ = make_ffn(wl, "cpu", seed=seed, reference=True)
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(1, tokens, wl["d"], generator=gen)
    g = torch.randn(1, tokens, wl["d"], generator=gen)
    xw = torch.randn(1, min(tokens, 16), wl["d"], generator=gen)
    ffn(xw).backward(torch.ones_like(xw))  # warm-up
    ffn.zero_grad(set_to_none=True)
    t0 = time.perf_counter()
    ffn(x).backward(g)
    sec = time.perf_counter() - t0
    cells = tokens * cells_per_token(wl)
    return {"value": cells / sec / 1e9, "unit": "Gcell-evals/s", "cores": torch.get_num_threads(),
            "kind": "reference", "sample": f"{tokens} tokens, one fwd+bwd of the reference block on CPU, "
                                           f"{sec:.1f} s", "formula": "exact EKV (the reference's CPU branch)"}


# ------------------------------------------------------------ our arm -----

def extras_wanted(args) -> bool:
    return args.impl == "ours" and args.workload == "gpt_m_ffn" and not args.no_extras


def _bench_subprocess(argv, timeout=900) -> dict:
    """One bench.py invocation in a fresh process; its JSON line, or why not."""
    cmd = [sys.executable, str(ROOT / "bench.py"), *argv, "--no-cpu-baseline", "--no-extras"]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, cwd=str(ROOT),
                           env={**os.environ, "WORLD_SIZE": "1", "RANK": "0", "LOCAL_RANK": "0"})
    except subprocess.TimeoutExpired:
        return {"unavailable": f"timed out after {timeout} s: {' '.join(argv)}"}
    for line in reversed(r.stdout.splitlines()):
        if line.startswith("{"):
            try:
                return json.loads(line)
            except ValueError:
                break
    tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
    return {"unavailable": f"exit {r.returncode}: {tail[0][:300]}"}


def reference_gpu_comparison(args, ours_rec) -> dict:
    """The reference's own GPU path (unmodified package in baseline/_ref: Triton
    LUT forward, JIT-built CUDA shared backward) on the same GPU and workload,
    Physical (config 3) and Hybrid (config 3, Hybrid variant), each in a
    subprocess; with our/reference ratios of the device-timed step rates."""
    if not (ROOT / "baseline" / "_ref" / "isa").exists():
        return {"unavailable": "baseline/_ref (the pip-installed reference) is not present"}
    steps, warm = str(min(args.steps, 10)), str(max(args.warmup, 3))
    out = {}
    ref_p = _bench_subprocess(["--impl", "reference_gpu", "--workload", "gpt_m_ffn", "--steps", steps,
                               "--warmup", warm])
    ours_h = _bench_subprocess(["--impl", "ours", "--workload", "gpt_m_ffn_hybrid", "--steps", steps,
                                "--warmup", warm])
    ref_h = _bench_subprocess(["--impl", "reference_gpu", "--workload", "gpt_m_ffn_hybrid", "--steps", steps,
                               "--warmup", warm])
    for key, ref, ours in (("physical", ref_p, ours_rec), ("hybrid", ref_h, ours_h)):
        ent = {"reference": {k: ref.get(k) for k in ("value", "unit", "ms_per_step", "clocks", "unavailable")
                             if k in ref},
               "ours": {k: ours.get(k) for k in ("value", "unit", "ms_per_step", "unavailable") if k in ours}}
        if "value" in ref and "value" in ours:
            ent["ratio_ours_over_reference"] = ours["value"] / ref["value"]
        out[key] = ent
    out["note"] = ("reference: unmodified package from baseline/_ref through its module API (Triton _forward_kernel, "
                   "CUDA grad_x_shared/grad_w_shared), same workload, same device-event timing")
    return out


def run_ours(args, wl):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    refgpu = args.impl == "reference_gpu"
    exact = wl.get("approx") == "exact"
    ffn, cfg = make_ffn(wl, dev, reference=refgpu)
    B, S, d = wl["batch"], wl["seq"], wl["d"]
    gen = torch.Generator(device=dev).manual_seed(1234 + rank)
    x = torch.randn(B, S, d, device=dev, generator=gen)  # post-LayerNorm scale
    gseed = torch.randn(B, S, d, device=dev, generator=gen)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    allreduce = world > 1

    for _ in range(max(args.warmup, 3)):
        ffn_step(ffn, x, gseed, allreduce)
    barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier()
        for i in range(args.steps):
            flush.zero_()
            starts[i].record()
            ffn_step(ffn, x, gseed, allreduce)
            ends[i].record()
        barrier()
    ms_rank = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    t = torch.tensor([ms_rank], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_total = float(t.item())
    tokens = B * S
    cells_step = tokens * cells_per_token(wl)
    value = world * cells_step * args.steps / (ms_total * 1e-3)

    # End to end through the public module API: the step's input from pinned
    # host memory, the loss back to the host, every step.
    x_host = x.cpu().pin_memory()
    loss_host = torch.empty((), pin_memory=True)
    for _ in range(2):
        ffn_step(ffn, x_host.to(dev, non_blocking=True), gseed, allreduce)
    barrier()
    # The next step's input is copied on a side stream while this step computes
    # (double-buffered), and this step's end event waits for that copy, so every
    # host->device copy lies inside a timed interval (step 0 copies its own).
    e_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    e_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    main = torch.cuda.current_stream(dev)
    copy_stream = torch.cuda.Stream(device=dev)
    xbuf = [torch.empty_like(x), torch.empty_like(x)]
    copied = [torch.cuda.Event(), torch.cuda.Event()]
    used = [torch.cuda.Event(), torch.cuda.Event()]
    for i in range(args.steps):
        flush.zero_()
        e_starts[i].record()
        b = i % 2
        if i == 0:
            xbuf[b].copy_(x_host, non_blocking=True)
        else:
            main.wait_event(copied[b])
        if i + 1 < args.steps:
            nb = (i + 1) % 2
            with torch.cuda.stream(copy_stream):
                if i >= 1:
                    copy_stream.wait_event(used[nb])  # step i-1 is done with that buffer
                xbuf[nb].copy_(x_host, non_blocking=True)
                copied[nb].record(copy_stream)
        loss = ffn_step(ffn, xbuf[b], gseed, allreduce)
        used[b].record(main)
        loss_host.copy_(loss.detach(), non_blocking=True)
        if i + 1 < args.steps:
            main.wait_event(copied[(i + 1) % 2])
        e_ends[i].record()
    barrier()
    e_ms = torch.tensor([sum(s.elapsed_time(e) for s, e in zip(e_starts, e_ends))], device=dev)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e_value = world * cells_step * args.steps / (float(e_ms.item()) * 1e-3)

    kern = time_kernels(ffn, cfg, x, dev) if rank == 0 and not refgpu and not exact else None
    # Second half of the headline metric, measured in the same invocation on the
    # same ranks: the Physical GPT-L training step at a fixed global batch.
    gpt_l = vit_l = None
    if extras_wanted(args) and not refgpu and not exact and not wl.get("hybrid"):
        del ffn
        torch.cuda.empty_cache()
        gpt_l = gpt_l_measure(WORKLOADS["gpt_l_step"], world, rank, local, dev, args.gpt_l_steps,
                              min(args.warmup, 3))
        torch.cuda.empty_cache()
        vit_l = vit_l_measure(WORKLOADS["vit_l_step"], world, rank, local, dev, args.gpt_l_steps,
                              min(args.warmup, 3))
    peak = fp32_peak(dev) if rank == 0 else None
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not refgpu and not exact:
        cores = host_cores()
        c, sec = cpu_sample(wl, args.cpu_sample_tokens, nthreads=cores)
        cpu = {"value": c / sec / 1e9, "unit": "Gcell-evals/s", "cores": cores, "kind": "port",
               "sample": f"{args.cpu_sample_tokens} tokens of the block (both projections, fwd+bwd), "
                         f"oracle/cimekv_oracle.c with OpenMP, {sec:.1f} s"}
    cpu_ref = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and not refgpu:
        cpu_ref = reference_pytorch_cpu(wl)
    if world > 1:
        dist.barrier()
    if rank == 0 and (refgpu or exact):
        rec = {"metric": "CIM-FFN fwd+bwd Gcell-evals/s", "value": value / 1e9, "unit": "Gcell-evals/s",
               "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_total / args.steps,
               "higher_is_better": True, "scaling": "weak", "dtype": "f32", "impl": args.impl,
               "config": {"workload": args.workload, "model": wl["model"], "tokens_per_gpu": tokens,
                          "lut_size": wl["lut"], "parallelism": f"dp{world}"},
               "tokens_per_s": world * tokens * args.steps / (ms_total * 1e-3),
               "step_frac_of_fp32_peak": value / world * (OPS_FWD + OPS_BWD) / peak["sustained"],
               "e2e": {"value": e2e_value / 1e9, "unit": "Gcell-evals/s"},
               "clocks": clocks.summary(), "cpu_reference_pytorch": cpu_ref,
               "note": ("unmodified reference package from baseline/_ref through its module API, same workload "
                        "and timing" if refgpu else "exact-formula kernels of this build")}
        print(json.dumps(rec), flush=True)
    elif rank == 0:
        clk = clocks.summary()
        # Dominant kernel: the one with the largest total time per step.
        per = []
        for name, k in kern.items():
            per.append((k["fwd_ms"], f"{name}.fwd", k["cells"] * OPS_FWD))
            per.append((k["bwd_ms"], f"{name}.bwd", k["cells"] * OPS_BWD))
        dom_ms, dom_name, dom_ops = max(per)
        pk = peak["sustained"]
        achieved = dom_ops / (dom_ms * 1e-3)
        traffic, co_bound = None, None
        tf = ROOT / "profiles" / "traffic.json"
        if tf.exists():
            try:
                prof = json.loads(tf.read_text()).get(args.workload, {})
                traffic = prof.get(dom_name)
                l1 = prof.get("l1_wavefront_frac", {}).get(dom_name)
                if l1 is not None:
                    co_bound = {"resource": "L1 shared-memory data pipe (table gathers)", "frac": l1,
                                "source": "ncu capture of this kernel (committed traffic record)",
                                "captured_at_commit": prof.get("commit")}
            except ValueError:
                traffic = None
        kernel_ms = sum(k["fwd_ms"] + k["bwd_ms"] for k in kern.values())
        rec = {
            "metric": "CIM-FFN fwd+bwd Gcell-evals/s",
            "value": value / 1e9,
            "unit": "Gcell-evals/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_total / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic: x ~ N(0,1) (post-LayerNorm scale), Vth ~ U(2.5 +- 0.107) (CIMLinear init), "
                    "upstream grad ~ N(0,1)",
            "config": {"workload": args.workload, "model": wl["model"], "global_batch": wl["batch"] * world,
                       "seq_len": wl["seq"], "tokens_per_gpu": tokens, "d": wl["d"], "hidden": wl["hidden"],
                       "lut_size": wl["lut"], "autocast": "bf16 (CIM path fp32)", "parallelism": f"dp{world}",
                       "l2": "flushed (256 MiB write) before every timed step"},
            "tokens_per_s": world * tokens * args.steps / (ms_total * 1e-3),
            "e2e": {"value": e2e_value / 1e9, "unit": "Gcell-evals/s",
                    "h2d_bytes_per_step": x_host.numel() * x_host.element_size(),
                    "d2h_bytes_per_step": loss_host.numel() * loss_host.element_size()},
            "roofline": {"bound": "fp32_issue", "kernel": dom_name, "achieved": achieved / 1e12,
                         "peak": pk / 1e12, "unit": "Tlane-op/s", "frac": achieved / pk, "traffic": traffic, "co_bound": co_bound,
                         "peak_source": "measured FFMA probe (cimekv_fp32_probe), sustained",
                         "peak_burst": peak["burst"] / 1e12,
                         "step_frac": value / world * (OPS_FWD + OPS_BWD) / pk,
                         "kernel_share_of_step": kernel_ms / (ms_total / args.steps),
                         "kernels_ms": kern,
                         "ops_per_cell": {"fwd": OPS_FWD, "bwd": OPS_BWD},
                         "hbm_peak_gbs": measured_peaks().get("hbm_gbs")},
            "cpu_baseline": cpu,
            "cpu_reference_pytorch": cpu_ref,
            "clocks": clk,
            "gpu_launches": 10 * args.steps,  # per projection: fwd, tia_bwd, sum_partials, bwd, bwd_reduce
            "impl": "ours",
        }
        if gpt_l is not None:
            rec["gpt_l_step"] = gpt_l
        if vit_l is not None:
            rec["vit_l_step"] = vit_l
        if extras_wanted(args) and world == 1:
            rec["reference_gpu"] = reference_gpu_comparison(args, rec)
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------------------------ reference arm -----

def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # rank 0 alone times the host CPU path

    tokens = 128  # bounded sample per step: ~1 s of CPU work on 8 cores
    for _ in range(max(args.warmup, 1)):
        cpu_sample(wl, tokens, nthreads=host_cores())
    total_c, total_s = 0, 0.0
    for i in range(args.steps):
        c, s = cpu_sample(wl, tokens, nthreads=host_cores(), seed=i)
        total_c += c
        total_s += s
    v = total_c / total_s / 1e9
    cores = host_cores()
    rec = {
        "metric": "CIM-FFN fwd+bwd Gcell-evals/s", "value": v, "unit": "Gcell-evals/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_s * 1e3 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic, same distributions as our arm",
        "config": {"workload": args.workload, "model": wl["model"], "tokens_per_step_sample": tokens,
                   "d": wl["d"], "hidden": wl["hidden"], "lut_size": wl["lut"], "parallelism": "host CPU"},
        "impl": "reference",
        "cpu_baseline": {"value": v, "unit": "Gcell-evals/s", "cores": cores, "kind": "port",
                         "sample": f"{tokens} tokens of the block per step (both projections, fwd+bwd): "
                                   "CPU restatement of the reference LUT path, oracle/cimekv_oracle.c, OpenMP"},
        "e2e": {"value": v, "unit": "Gcell-evals/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "cpu_reference_pytorch": reference_pytorch_cpu(wl),
    }
    print(json.dumps(rec), flush=True)


def run_vit_l(args, wl):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    rec = vit_l_measure(wl, world, rank, local, dev, args.steps, args.warmup)
    if rec is not None:
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.destroy_process_group()


def vit_l_measure(wl, world, rank, local, dev, steps, warmup):
    """Full Physical ViT-L training step (fp16 autocast + GradScaler, DDP,
    clip, AdamW, clamp_vth); the global batch is fixed and split across the ranks
    of the (already initialised) process group.  Returns rank 0's record."""
    import torch
    import torch.distributed as dist

    from isa_b200.harness.vit import PhysicalViT, ViTConfig, train_step

    per = wl["batch"] // world
    torch.manual_seed(0)
    model = PhysicalViT(ViTConfig()).to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4)
    scaler = torch.amp.GradScaler("cuda")
    cims = model.cim_layers()
    net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local]) if world > 1 else model
    gen = torch.Generator(device="cpu").manual_seed(200 + rank)
    img_host = torch.randn(per, 3, 224, 224, generator=gen).pin_memory()
    lab_host = torch.randint(0, 200, (per,), generator=gen).pin_memory()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(max(warmup, 3)):
        train_step(net, opt, scaler, img_host.to(dev), lab_host.to(dev), cims)
    barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    loss_host = torch.empty((), pin_memory=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier()
        for s_, e_ in ev:
            s_.record()
            loss = train_step(net, opt, scaler, img_host.to(dev, non_blocking=True),
                              lab_host.to(dev, non_blocking=True), cims)
            loss_host.copy_(loss, non_blocking=True)
            e_.record()
        barrier()
    t = torch.tensor([sum(s_.elapsed_time(e_) for s_, e_ in ev)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    images = wl["batch"] * steps
    rec = None
    if rank == 0:
        cells = images * wl["seq"] * wl["layers"] * cells_per_token(wl)
        rec = {"metric": "Physical ViT-L train images/s", "value": images / (ms * 1e-3), "unit": "images/s",
               "n_gpus": world, "steps": steps, "warmup": max(warmup, 3), "ms_per_step": ms / steps,
               "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
               "dtype": "f32 CIM / fp16 digital", "data": "synthetic images ~ N(0,1), uniform labels, random init",
               "config": {"workload": "vit_l_step", "model": wl["model"], "global_batch": wl["batch"],
                          "tokens_per_image": wl["seq"], "parallelism": f"dp{world}", "lut_size": wl["lut"]},
               "tokens_per_s": images * wl["seq"] / (ms * 1e-3),
               "cim_gcell_evals_per_s": cells / (ms * 1e-3) / 1e9,
               "e2e": {"value": images / (ms * 1e-3), "unit": "images/s",
                       "h2d_bytes_per_step": img_host.numel() * 4 + lab_host.numel() * 8, "d2h_bytes_per_step": 4},
               "loss": float(loss_host), "clocks": clocks.summary(), "impl": "ours"}
    del net, model, opt
    torch.cuda.empty_cache()
    return rec


def gpt_l_measure(wl, world, rank, local, dev, steps, warmup):
    """Full Physical GPT-L training step (forward, backward, DDP all-reduce,
    clip, AdamW, clamp_vth); the global batch is fixed and split across the
    ranks of the (already initialised) process group.  Returns rank 0's record."""
    import torch
    import torch.distributed as dist

    from isa_b200.harness.gpt import GPTConfig, PhysicalGPT, train_step

    if wl["batch"] % world:
        raise SystemExit(f"global batch {wl['batch']} does not split over {world} ranks")
    per = wl["batch"] // world
    torch.manual_seed(0)
    model = PhysicalGPT(GPTConfig()).to(dev)
    opt = model.optimizer()
    cims = model.cim_layers()
    net = model
    if world > 1:
        net = torch.nn.parallel.DistributedDataParallel(model, device_ids=[local])
    gen = torch.Generator(device="cpu").manual_seed(100 + rank)
    ids_host = torch.randint(0, 50257, (per, wl["seq"] + 1), generator=gen).pin_memory()
    ids = ids_host.to(dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(max(warmup, 2)):
        train_step(net, opt, ids, cims)
    barrier()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    loss_host = torch.empty((), pin_memory=True)
    with ClockSampler(torch.cuda.current_device()) as clocks:
        barrier()
        for s_, e_ in ev:
            s_.record()
            # public-API step with the batch copied from pinned host memory and
            # the loss read back: device time and e2e coincide for this step
            loss = train_step(net, opt, ids_host.to(dev, non_blocking=True), cims)
            loss_host.copy_(loss, non_blocking=True)
            e_.record()
        barrier()
    t = torch.tensor([sum(s_.elapsed_time(e_) for s_, e_ in ev)], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item())
    tokens = wl["batch"] * wl["seq"] * steps
    del net, model, opt
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    cells = tokens * wl["layers"] * cells_per_token(wl)
    return {"metric": "Physical GPT-L train tokens/s", "value": tokens / (ms * 1e-3), "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": max(warmup, 2), "ms_per_step": ms / steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32 CIM / bf16 digital",
            "data": "synthetic token ids uniform in [0, 50257), random-init weights",
            "config": {"workload": "gpt_l_step", "model": wl["model"], "global_batch": wl["batch"],
                       "per_gpu_batch": per, "seq_len": wl["seq"], "parallelism": f"dp{world}",
                       "lut_size": wl["lut"], "l2": "working set >> L2 (activations of 64k tokens)"},
            "cim_gcell_evals_per_s": cells / (ms * 1e-3) / 1e9,
            "e2e": {"value": tokens / (ms * 1e-3), "unit": "tokens/s",
                    "h2d_bytes_per_step": ids_host.numel() * ids_host.element_size(), "d2h_bytes_per_step": 4},
            "loss": float(loss_host), "clocks": clocks.summary(),
            "gpu_launches": 10 * wl["layers"] * steps, "impl": "ours"}


def run_gpt_l(args, wl):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    rec = gpt_l_measure(wl, world, rank, local, dev, args.steps, args.warmup)
    if rec is not None:
        print(json.dumps(rec), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_measured(args, wl):
    """fc1 in measured mode: forward (per-cell codebook gather, fused TIA) and
    input gradient; the reference arm runs its own module (masked GEMM per
    active segment, measured_deployment/operator.py:163-206)."""
    import numpy as np
    import torch

    ref = args.impl == "reference_gpu"
    if ref:
        sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
        from isa.measured_deployment.operator import DeploymentAwareCIMLinear
    else:
        from isa_b200.operators.measured import DeploymentAwareCIMLinear
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rng = np.random.default_rng(0)
    torch.manual_seed(0)
    layer = DeploymentAwareCIMLinear(wl["d"], wl["hidden"]).to(dev)
    layer.set_r_tia(2.0e4)
    g_pts = 33
    vg = np.linspace(-0.5, 4.5, g_pts).astype(np.float32)
    cur = (np.exp(rng.uniform(-14, -11, (24, 1))) * np.cumsum(rng.uniform(0, 1, (24, g_pts)), axis=1)).astype(np.float32)
    layer.configure_codebook(torch.from_numpy(vg), torch.from_numpy(cur))
    pos = torch.from_numpy(rng.integers(0, 24, (wl["hidden"], wl["d"])).astype(np.int16))
    neg = torch.from_numpy(rng.integers(0, 24, (wl["hidden"], wl["d"])).astype(np.int16))
    layer.set_assignment(pos, neg)
    layer.set_forward_mode("measured")
    x = (torch.rand(wl["batch"], wl["seq"], wl["d"], device=dev) * 4.0).requires_grad_(True)
    g = torch.randn(wl["batch"], wl["seq"], wl["hidden"], device=dev)

    def step():
        x.grad = None
        layer(x).backward(g)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    s_, e_ = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s_.record()
    for _ in range(args.steps):
        step()
    e_.record()
    e_.synchronize()
    ms = s_.elapsed_time(e_) / args.steps
    cells = wl["batch"] * wl["seq"] * wl["d"] * wl["hidden"]
    print(json.dumps({"metric": "measured fc1 fwd+dX Gcell-evals/s", "value": cells / (ms * 1e-3) / 1e9,
                      "unit": "Gcell-evals/s", "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
                      "impl": args.impl, "config": {"workload": args.workload, "tokens": wl["batch"] * wl["seq"],
                                                    "d": wl["d"], "hidden": wl["hidden"], "states": 24,
                                                    "grid_points": g_pts}}), flush=True)


def main():
    args = parse()
    wl = WORKLOADS[args.workload]
    if wl.get("measured"):
        run_measured(args, wl)
        return
    if args.workload == "vit_l_step":
        run_vit_l(args, wl)
        return
    if args.workload == "gpt_l_step":
        if args.impl != "ours":
            raise SystemExit("gpt_l_step is measured for this build only")
        run_gpt_l(args, wl)
        return
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
