"""Data-parallel exchange on CPU ranks (gloo, world size 2): batch sharding of a
DCNv2 layer with one bucketed all-reduce of grad_weight / grad_bias reproduces
the full-batch gradients (the per-rank backward here is the float64 oracle; on
GPUs it is the CUDA operator, the exchange is the same code), and a rank that
fails before the collective makes the other rank's collective fail instead of hang."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=20):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _shard_worker(rank, world, port, q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    import oracle
    from dcn_cases import Case, make_inputs
    from dcnv2_b200.dp import GradBucket
    _init(rank, world, port)
    try:
        c = Case("dp", 4, 8, 9, 9, 12, 3, 3)
        x, w, b, off, m, gy = [t.double().numpy() for t in make_inputs(c)]
        per = c.B // world
        sl = slice(rank * per, (rank + 1) * per)
        g = oracle.backward(x[sl], w, off[sl], m[sl], gy[sl], 1, 1)
        pw = torch.nn.Parameter(torch.zeros(w.shape, dtype=torch.float64))
        pb = torch.nn.Parameter(torch.zeros(b.shape, dtype=torch.float64))
        pw.grad = torch.from_numpy(g[3].copy())
        pb.grad = torch.from_numpy(g[4].copy())
        GradBucket([pw, pb]).allreduce(average=False)
        full = oracle.backward(x, w, off, m, gy, 1, 1)
        errw = float(np.abs(pw.grad.numpy() - full[3]).max() / np.abs(full[3]).max())
        errb = float(np.abs(pb.grad.numpy() - full[4]).max() / np.abs(full[4]).max())
        q.put((rank, errw, errb))
    finally:
        dist.destroy_process_group()


def _failing_worker(rank, world, port, q):
    _init(rank, world, port, timeout_s=5)
    if rank == 1:
        q.put((rank, "left before the collective"))
        q.close()
        q.join_thread()
        os._exit(0)  # the rank dies between steps, none of its work in flight
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, f"error: {type(e).__name__}"))


def _run(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_batch_sharded_grads_allreduce_equal_full_batch():
    res = _run(_shard_worker)
    assert len(res) == 2
    for _, errw, errb in res:
        assert errw < 1e-6 and errb < 1e-6  # the bucket is float32


def test_dead_rank_fails_collective_instead_of_hanging():
    res = dict(_run(_failing_worker))
    assert res[1] == "left before the collective"
    assert res[0].startswith("error")


def _overlap_worker(rank, world, port, q):
    """Two small layers; the buckets start from the backward hooks (overlap) and
    the averaged gradients equal the full-batch mean on every rank."""
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    from dcnv2_b200.dp import GradBucket
    _init(rank, world, port)
    try:
        torch.manual_seed(0)
        layers = [torch.nn.Linear(6, 5).double(), torch.nn.Linear(5, 3).double()]
        x = torch.randn(8, 6, dtype=torch.float64, generator=torch.Generator().manual_seed(1))
        per = 8 // world
        red = GradBucket(layers, overlap=True, average=True)
        errs = []
        for _step in range(2):   # hooks re-arm after every allreduce()
            for lay in layers:
                lay.zero_grad(set_to_none=True)
            h = x[rank * per:(rank + 1) * per]
            for lay in layers:
                h = torch.tanh(lay(h))
            h.sum().backward()
            red.allreduce()
            got = [p.grad.clone() for lay in layers for p in lay.parameters()]
            for lay in layers:
                lay.zero_grad(set_to_none=True)
            h = x
            for lay in layers:
                h = torch.tanh(lay(h))
            (h.sum() / world).backward()
            ref = [p.grad.clone() for lay in layers for p in lay.parameters()]
            errs.append(max(float((a - b).abs().max()) for a, b in zip(got, ref)))
        q.put((rank, max(errs)))
    finally:
        dist.destroy_process_group()


def test_overlapped_buckets_average_equals_full_batch():
    res = _run(_overlap_worker)
    assert len(res) == 2
    for _, err in res:
        assert err < 1e-6, err   # fp32 bucket
