"""Data-parallel training over NCCL on 2 GPUs (skipped with fewer): every rank
runs the CUDA operator on its shard of the batch and the weight / bias gradients
are all-reduced; the result must equal the 1-GPU full-batch gradients.

* the operator alone (`_C.dcn_v2_backward` + `allreduce_tensors`), fp32 and
  bf16: summed gW / gB against the full batch on one GPU (fp32: 1e-5, the two
  partial fp32 sums are added in another order; bf16: 1e-2, each rank rounds
  its partial gradient to bf16 before the sum);
* a stack of two `DCN` modules with `GradBucket(overlap=True)`, whose per-layer
  all-reduces start from backward hooks: every parameter gradient (predictor
  convs included) against the full-batch gradient / world size.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import sys
    import datetime
    import torch.distributed as dist
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, root)
    sys.path.insert(0, os.path.join(root, "tests"))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    torch.backends.cudnn.allow_tf32 = False
    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from dcn_cases import Case, make_inputs, rel_err
        from dcnv2_b200 import _C
        from dcnv2_b200.dp import GradBucket, allreduce_tensors
        from dcnv2_b200.modules import DCN
        out = {}
        # ---- the operator on batch shards
        c = Case("dp", 4, 64, 24, 24, 96, 3, 3)
        per = c.B // world
        for name, dt, tol in (("fp32", torch.float32, 1e-5), ("bf16", torch.bfloat16, 1e-2)):
            x, w, b, off, m, gy = [t.to(dt).to(dev) for t in make_inputs(c)]
            sl = slice(rank * per, (rank + 1) * per)
            g = _C.dcn_v2_backward(x[sl], w, m[sl], off[sl], b, gy[sl], 1, 1, 1, 1)
            gw, gb = allreduce_tensors([g[3], g[4]], average=False)
            full = _C.dcn_v2_backward(x, w, m, off, b, gy, 1, 1, 1, 1)
            torch.cuda.synchronize()
            out[f"op_{name}"] = (max(rel_err(gw.cpu().numpy(), full[3].float().cpu().numpy()),
                                     rel_err(gb.cpu().numpy(), full[4].float().cpu().numpy())), tol)
        # ---- a stack of DCN modules, buckets overlapped with the backward
        torch.manual_seed(5)
        layers = [DCN(32, 32, 3, stride=1, padding=1).to(dev) for _ in range(2)]
        with torch.no_grad():
            for lay in layers:
                lay.conv_offset_mask.weight.normal_(0, 0.05)
                lay.conv_offset_mask.bias.normal_(0, 0.3)
        gen = torch.Generator().manual_seed(9)
        X = torch.randn(4, 32, 16, 16, generator=gen).to(dev)
        GY = torch.randn(4, 32, 16, 16, generator=gen).to(dev)
        bucket = GradBucket(layers, overlap=True, average=True)

        def run(xx, gg):
            for lay in layers:
                lay.zero_grad(set_to_none=True)
            h = xx
            for i, lay in enumerate(layers):
                h = lay(h)
                if i + 1 < len(layers):
                    h = torch.relu(h)
            h.backward(gg)

        sl = slice(rank * 2, rank * 2 + 2)
        errs = []
        for _ in range(2):   # the hooks re-arm after every allreduce()
            run(X[sl], GY[sl])
            bucket.allreduce()
            got = [p.grad.clone() for lay in layers for p in lay.parameters()]
            bucket.detach()
            run(X, GY)
            ref = [p.grad / world for lay in layers for p in lay.parameters()]
            errs.append(max(rel_err(a.cpu().numpy(), r.cpu().numpy()) for a, r in zip(got, ref)))
            bucket = GradBucket(layers, overlap=True, average=True)
        out["stack_overlap"] = (max(errs), 1e-4)
        q.put((rank, out))
    except Exception as e:  # noqa: BLE001
        q.put((rank, {"error": (repr(e), 0.0)}))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_nccl_two_gpus_shards_equal_full_batch():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for rank, out in res:
        assert "error" not in out, out
        for k, (err, tol) in out.items():
            assert err <= tol, f"rank {rank} {k}: {err} > {tol}"
