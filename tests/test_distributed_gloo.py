"""Token-sharded data parallelism on CPU ranks (gloo, world size 2): the
sharded dVth summed by the package's all-reduce equals the single-process
dVth of the whole batch (oracle arithmetic stands in for the kernels)."""

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, result_path):
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "isa-_b200")]
    from isa_b200.distributed import allreduce_gradients, shard_rows
    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(0)
    m, k, o = 96, 24, 40
    x = rng.standard_normal((m, k)).astype(np.float32)
    wp = (2.5 + rng.uniform(-.1, .1, (o, k))).astype(np.float32)
    wn = (2.5 + rng.uniform(-.1, .1, (o, k))).astype(np.float32)
    g = rng.standard_normal((m, o)).astype(np.float32)
    ti = np.linspace(0, 1e-6, 4096, dtype=np.float32)
    td = np.linspace(1e-6, 0, 4096, dtype=np.float32)
    sl = shard_rows(m, rank, world)
    _, gwp, gwn = oracle.backward(x[sl], wp, wn, g[sl], ti, td, -9.0, 315.0, 8.2624, need_x=False)
    pp = torch.nn.Parameter(torch.zeros(o, k))
    pn = torch.nn.Parameter(torch.zeros(o, k))
    pp.grad, pn.grad = torch.from_numpy(gwp), torch.from_numpy(gwn)
    allreduce_gradients([pp, pn], average=False)
    if rank == 0:
        _, fwp, fwn = oracle.backward(x, wp, wn, g, ti, td, -9.0, 315.0, 8.2624, need_x=False)
        np.savez(result_path, gwp=pp.grad.numpy(), gwn=pn.grad.numpy(), fwp=fwp, fwn=fwn)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_dvth_allreduce_equals_full_batch(tmp_path):
    out = str(tmp_path / "r.npz")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    r = np.load(out)
    np.testing.assert_allclose(r["gwp"], r["fwp"], rtol=1e-6, atol=1e-12)
    np.testing.assert_allclose(r["gwn"], r["fwn"], rtol=1e-6, atol=1e-12)


def test_shard_rows_cover_exactly():
    from isa_b200.distributed import shard_rows
    for n in (0, 1, 7, 64, 65537):
        for w in (1, 2, 3, 8):
            idx = np.concatenate([np.arange(n)[shard_rows(n, r, w)] for r in range(w)])
            np.testing.assert_array_equal(idx, np.arange(n))


def _failing_worker(rank, world, port, result_path):
    """Rank 1 dies before the gradient exchange; rank 0 must get an error from
    its collective within the process-group timeout instead of hanging."""
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "isa-_b200")]
    from isa_b200.distributed import allreduce_gradients

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(0)  # a rank that leaves between steps
    p = torch.nn.Parameter(torch.zeros(4))
    p.grad = torch.ones(4)
    try:
        allreduce_gradients([p])
        outcome = "completed"
    except Exception as exc:  # noqa: BLE001 - any collective error is the detection signal
        outcome = "error: " + type(exc).__name__
    Path(result_path).write_text(outcome)


def test_lost_rank_is_detected_by_collective_timeout(tmp_path):
    out = tmp_path / "r.txt"
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, str(out))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    assert out.exists() and out.read_text().startswith("error"), out.read_text() if out.exists() else "no result"
