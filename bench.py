"""Benchmark of the DCNv2 operator: one step = forward + backward of one DCNv2
layer (the reference README's shape by default: B=8, C=64, 128x128, Co=256, 3x3,
stride 1, pad 1) on seeded synthetic data, per GPU.  With N GPUs every rank runs
its own batch (weak scaling) and the weight/bias gradients are summed over the
ranks with one NCCL all-reduce per step (the data-parallel exchange).

Prints ONE JSON line (rank 0).  Throughput unit: README-formula TFLOP/s, where a
forward counts B*Ho*Wo*Co*(10*k*k*C + 2*k*k) FLOPs (reference README.md:17) and a
forward+backward step counts three times that.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--dtype bf16|fp16|fp32]
  python bench.py --impl reference ...   # the CPU port of the reference path

Timing: per-step CUDA events on the launching stream, L2 flushed (256 MiB write)
before every step outside the events, max over ranks; SM clocks sampled with
nvidia-smi during the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

# The bench's stdout is one JSON line.  Whatever the libraries print (NCCL's
# version banner, warnings) goes to stderr: file descriptor 1 is pointed at
# stderr and the JSON line is written to a duplicate of the original stdout.
os.environ.setdefault("NCCL_DEBUG", "WARN")
os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
sys.stdout.flush()
_JSON_OUT = os.fdopen(os.dup(1), "w")
os.dup2(2, 1)
import torch  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (B, C, H, W, Co, k, stride, pad, dil, dg, off_std)
    "readme": (8, 64, 128, 128, 256, 3, 1, 1, 1, 1, 1.5),
    # the README layer at batch 2: the small case for ncu captures
    "readme_b2": (2, 64, 128, 128, 256, 3, 1, 1, 1, 1, 1.5),
    # the other layer shapes of the benchmark configurations (run with --dtype
    # of the configuration: fp16 for the ResNet-50 stages, bf16 for c512_dg4)
    "resnet_s1": (16, 128, 64, 64, 128, 3, 1, 1, 1, 1, 1.5),
    "resnet_s2": (16, 256, 32, 32, 256, 3, 1, 1, 1, 1, 1.5),
    "resnet_s3": (16, 512, 16, 16, 512, 3, 1, 1, 1, 1, 1.5),
    "c512_dg4": (32, 512, 32, 32, 512, 3, 1, 1, 1, 4, 2.0),
    "edge_k5": (4, 96, 97, 131, 160, 5, 2, 4, 2, 2, 8.0),
    # the 1x1 deformable conv of the reference's CIFAR training demo (bottleneck
    # 256 -> 64 channels at 32x32, batch 128; train.py:56-73)
    "k1_cifar": (128, 256, 32, 32, 64, 1, 1, 0, 1, 1, 1.5),
}
# stacks of DCN modules (offset/mask predicted by a plain 3x3 conv, ReLU between),
# the global batch split over the ranks: one data-parallel training step per step
STACKS = {
    "stack3": {"global_batch": 256, "C": 256, "H": 64, "W": 64, "layers": 3, "k": 3, "off_std": 1.5},
}
DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def readme_flops(B, C, Ho, Wo, Co, k):
    """README.md:17 forward FLOP count."""
    return B * Ho * Wo * Co * (10.0 * k * k * C + 2.0 * k * k)


def gemm_flops(B, C, Ho, Wo, Co, k):
    """Algorithmic tensor-core work of one GEMM pass: 2*Co*C*k*k*B*Ho*Wo."""
    return 2.0 * Co * C * k * k * B * Ho * Wo


def out_hw(H, W, k, s, p, d):
    return (H + 2 * p - (d * (k - 1) + 1)) // s + 1, (W + 2 * p - (d * (k - 1) + 1)) // s + 1


def make_inputs(wl, dtype, device, seed):
    B, C, H, W, Co, k, s, p, d, dg, off_std = wl
    Ho, Wo = out_hw(H, W, k, s, p, d)
    g = lambda i: torch.Generator().manual_seed(1000 * seed + i)  # noqa: E731
    x = torch.randn(B, C, H, W, generator=g(0))
    w = torch.randn(Co, C, k, k, generator=g(1)) * (2.0 / (C * k * k)) ** 0.5
    b = torch.randn(Co, generator=g(2)) * 0.01
    off = torch.randn(B, 2 * dg * k * k, Ho, Wo, generator=g(3)) * off_std
    m = torch.sigmoid(torch.randn(B, dg * k * k, Ho, Wo, generator=g(4)))
    gy = torch.randn(B, Co, Ho, Wo, generator=g(5))
    ts = [x, w, b, off, m, gy]
    if device is None:
        return ts
    return [t.to(dtype).to(device) for t in ts]


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return {"hbm_gbs": float(pk["hbm_gbs"]), "bf16_tflops": float(pk["bf16_tflops"])}, "measured"
    except Exception:
        return dict(PEAKS_FALLBACK), "fallback"


def load_traffic(kernel, workload, dtype):
    """DRAM bytes per launch of `kernel` from a committed ncu summary, or None."""
    path = os.path.join(ROOT, "profiles", f"traffic_{workload}_{dtype}.txt")
    try:
        with open(path) as f:
            for line in f:
                parts = line.split()
                if len(parts) >= 2 and parts[0] == kernel:
                    return float(parts[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        load = sorted(sm)[len(sm) // 2:] if sm else []
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def host_threads():
    """Host threads this process may use (torchrun sets OMP_NUM_THREADS=1 for its workers)."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_port_step(wl, B_sample):
    """One forward+backward of the C port of the reference path (float32, OpenMP)."""
    import oracle
    oracle.set_threads(host_threads())
    x, w, b, off, m, gy = [t.numpy() for t in make_inputs(wl, None, None, 0)]
    _, C, H, W, Co, k, s, p, d, dg, _ = wl
    sl = slice(0, B_sample)
    t0 = time.perf_counter()
    oracle.forward(x[sl], w, b, off[sl], m[sl], s, p, d, dg, dtype=np.float32)
    oracle.backward(x[sl], w, off[sl], m[sl], gy[sl], s, p, d, dg, dtype=np.float32)
    return time.perf_counter() - t0


def cpu_baseline(wl, budget_s=20.0):
    """Times the CPU port on a bounded sample of the workload (rank 0, N=1 only)."""
    import oracle
    B = wl[0]
    t1 = cpu_port_step(wl, 1)  # also warms the library
    bs = int(max(1, min(B, (budget_s / 3) // max(t1, 1e-3))))
    times = [cpu_port_step(wl, bs) for _ in range(2)]
    t = min(times)
    C, H, W, Co, k, s, p, d = wl[1], wl[2], wl[3], wl[4], wl[5], wl[6], wl[7], wl[8]
    Ho, Wo = out_hw(H, W, k, s, p, d)
    flops = 3 * readme_flops(bs, C, Ho, Wo, Co, k)
    return {"value": flops / t / 1e12, "unit": "TFLOP/s (README formula, fwd+bwd)",
            "cores": oracle.num_threads(), "kind": "port",
            "sample": f"batch {bs} of {B} (fwd+bwd, float32), best of 2, {t:.3f} s per sample"}


def cpu_torchvision(wl, budget_s=20.0):
    """torchvision.ops.deform_conv2d on the host cores (float32, forward + backward) on a
    bounded sample of the workload: the CPU path the benchmark configuration names."""
    try:
        import torchvision
        from torchvision.ops import deform_conv2d
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"torchvision not importable: {e}"}
    torch.set_num_threads(host_threads())
    B, C, H, W, Co, k, s, p, d, dg, _ = wl
    x, w, b, off, m, gy = make_inputs(wl, None, None, 0)

    def one(bs):
        xs, offs, ms = [t[:bs].clone().requires_grad_(True) for t in (x, off, m)]
        ws, bias = w.clone().requires_grad_(True), b.clone().requires_grad_(True)
        t0 = time.perf_counter()
        y = deform_conv2d(xs, offs, ws, bias, stride=(s, s), padding=(p, p), dilation=(d, d), mask=ms)
        y.backward(gy[:bs])
        return time.perf_counter() - t0

    t1 = one(1)
    bs = int(max(1, min(B, (budget_s / 3) // max(t1, 1e-3))))
    t = min(one(bs) for _ in range(2))
    Ho, Wo = out_hw(H, W, k, s, p, d)
    return {"value": 3 * readme_flops(bs, C, Ho, Wo, Co, k) / t / 1e12,
            "unit": "TFLOP/s (README formula, fwd+bwd)", "cores": torch.get_num_threads(),
            "kind": f"torchvision {torchvision.__version__} deform_conv2d (CPU)",
            "sample": f"batch {bs} of {B} (fwd+bwd, float32), best of 2, {t:.3f} s per sample"}


def run_reference(args, wl, rank):
    """--impl reference: the CPU port of the reference path on the host cores."""
    if rank != 0:
        return
    import oracle
    B = wl[0]
    C, H, W, Co, k, s, p, d = wl[1], wl[2], wl[3], wl[4], wl[5], wl[6], wl[7], wl[8]
    Ho, Wo = out_hw(H, W, k, s, p, d)
    t1 = cpu_port_step(wl, 1)
    # keep the whole run to about two minutes
    per_step = 120.0 / max(1, args.steps + args.warmup)
    bs = int(max(1, min(B, per_step // max(t1, 1e-3))))
    for _ in range(args.warmup):
        cpu_port_step(wl, bs)
    ts = [cpu_port_step(wl, bs) for _ in range(args.steps)]
    t = sum(ts) / len(ts)
    val = 3 * readme_flops(bs, C, Ho, Wo, Co, k) / t / 1e12
    line = {
        "impl": "reference", "metric": "dcnv2_fwd_bwd_readme_tflops", "value": val,
        "unit": "TFLOP/s (README formula, fwd+bwd)", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t * 1e3 * B / bs, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_of(args, wl),
        "cpu_baseline": {"value": val, "unit": "TFLOP/s (README formula, fwd+bwd)",
                         "cores": oracle.num_threads(), "kind": "port",
                         "sample": f"batch {bs} of {B} per step (fwd+bwd, float32 C port of the "
                                   "reference arithmetic; the reference has no CPU kernel)"},
        "e2e": {"value": val, "unit": "TFLOP/s (README formula, fwd+bwd)",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_gpu": reference_gpu(wl, args),
    }
    print(json.dumps(line), file=_JSON_OUT, flush=True)


def reference_gpu(wl, args):
    """Context for the reference arm: the reference's own CUDA operator (com.cu +
    ext.cpp compiled for sm_100a by oracle/build_ref.py into oracle/_ref) timed on
    this GPU, float32 (its only dtype), forward + backward of the same layer, CUDA
    events, L2 flushed before every step.  The reference handles neither dilation
    nor deformable groups, so other workloads report it as unavailable."""
    import glob
    import importlib.machinery
    import importlib.util
    B, C, H, W, Co, k, s, p, d, dg, _ = wl
    if d != 1 or dg != 1:
        return {"unavailable": "the reference operator implements neither dilation nor deformable groups"}
    if not torch.cuda.is_available():
        return {"unavailable": "no CUDA device"}
    so = glob.glob(os.path.join(ROOT, "oracle", "_ref", "Conv2d_ref*.so"))
    if not so:
        return {"unavailable": "oracle/_ref not built (python oracle/build_ref.py <reference checkout>)"}
    try:
        loader = importlib.machinery.ExtensionFileLoader("Conv2d_ref", so[0])
        spec = importlib.util.spec_from_loader("Conv2d_ref", loader)
        ref = importlib.util.module_from_spec(spec)
        loader.exec_module(ref)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"oracle/_ref does not load: {e}"[:200]}
    dev = torch.device("cuda", 0)
    x, w, b, off, m, gy = make_inputs(wl, torch.float32, dev, seed=0)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def step():
        ref.dcn_v2_forward(x, w, m, off, b, s, s, p, p)
        ref.dcn_v2_backward(x, w, m, off, b, gy, s, s, p, p)

    def timed(fn, n):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        torch.cuda.synchronize()
        for i in range(n):
            flush.zero_()
            ev[i][0].record()
            fn()
            ev[i][1].record()
        torch.cuda.synchronize()
        return sum(a.elapsed_time(b_) for a, b_ in ev) / n

    n = max(3, min(args.steps, 20))
    for _ in range(3):
        step()
    ms = timed(step, n)
    ms_fwd = timed(lambda: ref.dcn_v2_forward(x, w, m, off, b, s, s, p, p), n)
    Ho, Wo = out_hw(H, W, k, s, p, d)
    return {"ms_per_step": ms, "fwd_ms": ms_fwd,
            "value": 3 * readme_flops(B, C, Ho, Wo, Co, k) / (ms * 1e-3) / 1e12,
            "unit": "TFLOP/s (README formula, fwd+bwd)", "dtype": "f32", "steps": n,
            "kind": "reference com.cu/ext.cpp built for sm_100a (oracle/_ref), on this GPU"}


def make_timer(world, dev, stream, flush):
    """Per-step CUDA events on `stream`, L2 flushed before every step (outside the
    events), barrier before and after, max over ranks; returns ms per step."""
    import torch.distributed as dist

    def timed(fn, n):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(n)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(n):
            flush.zero_()
            ev[i][0].record(stream)
            fn()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = sum(a.elapsed_time(b_) for a, b_ in ev)
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()) / n
    return timed


def run_stack(args):
    """Data-parallel training step of a stack of DCN modules (the reference's `DCN`
    module API: offset/mask predictor conv, sigmoid mask, DCNv2 op), ReLU between
    layers, the global batch split over the ranks (strong scaling), every layer's
    weight and bias gradients (the predictor's included) averaged over the ranks by
    NCCL, one bucket per layer started as soon as that layer's backward is done."""
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from dcnv2_b200 import _lib
    from dcnv2_b200.dp import GradBucket
    from dcnv2_b200.modules import DCN

    cfg = STACKS[args.workload]
    dtype = DTYPES[args.dtype]
    G, C, H, W, L, k = cfg["global_batch"], cfg["C"], cfg["H"], cfg["W"], cfg["layers"], cfg["k"]
    if G % world != 0:
        raise SystemExit(f"global batch {G} does not split over {world} ranks")
    Bl = G // world
    torch.manual_seed(1234)                       # the same parameters on every rank
    layers = [DCN(C, C, k, stride=1, padding=k // 2).to(dev) for _ in range(L)]
    gen = torch.Generator().manual_seed(100 + rank)
    x = torch.randn(Bl, C, H, W, generator=gen).to(dev, dtype)
    gy = torch.randn(Bl, C, H, W, generator=gen).to(dev, dtype)
    if args.channels_last:
        # channels-last activations end to end: the predictor convs and the DCN
        # operator (DCN_NHWC layout) pass them on without layout passes
        x = x.contiguous(memory_format=torch.channels_last)
        gy = gy.contiguous(memory_format=torch.channels_last)
    with torch.no_grad():
        # predictor: random init scaled so the offsets have the configured std
        h = x.float()
        for lay in layers:
            lay.conv_offset_mask.weight.normal_()
            lay.conv_offset_mask.bias.zero_()
            o = lay.conv_offset_mask(h)[:, : 2 * k * k]
            lay.conv_offset_mask.weight.mul_(cfg["off_std"] / float(o.std()))
            h = torch.relu(torch.nn.functional.conv2d(h, lay.weight, lay.bias, padding=k // 2))
        for lay in layers:
            lay.to(dtype)
            if args.channels_last:
                lay.to(memory_format=torch.channels_last)
    # each layer's gradients are all-reduced as soon as its backward has produced
    # them, overlapping the backward of the layers below (not under graph capture)
    bucket = GradBucket(layers, overlap=world > 1 and not args.graph, average=True)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    timed = make_timer(world, dev, stream, flush)

    def step(xin, gin):
        for lay in layers:
            for prm in lay.parameters():
                prm.grad = None
        hh = xin
        for i, lay in enumerate(layers):
            hh = lay(hh)
            if i + 1 < L:
                hh = torch.relu(hh)
        hh.backward(gin)
        if world > 1:
            bucket.allreduce()

    for _ in range(args.warmup):
        step(x, gy)
    torch.cuda.synchronize()
    run_step = lambda: step(x, gy)  # noqa: E731
    if args.graph:
        # the whole step (predictor convs, DCN kernels, autograd, all-reduce) as one
        # CUDA graph replayed on the launching stream; x and gy are its static inputs
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                step(x, gy)
        stream.wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step(x, gy)
        torch.cuda.synchronize()
        run_step = graph.replay
        for _ in range(args.warmup):
            run_step()
        torch.cuda.synchronize()
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    clocks = ClockSampler(vis.split(",")[local] if vis else local)
    clocks.start()
    ms_step = timed(run_step, args.steps)
    _lib.trace_reset()
    _lib.trace_enable(True)
    timed(lambda: step(x, gy), args.steps)   # eager (the trace records library launches)
    _lib.trace_enable(False)
    trace = _lib.trace_collect()
    # end to end: the rank's inputs from pinned host memory, the last layer's weight
    # gradient back to the host, every step
    hx, hgy = x.cpu().pin_memory(), gy.cpu().pin_memory()
    dx, dgy = torch.empty_like(x), torch.empty_like(gy)
    hgw = torch.empty(layers[-1].weight.shape, dtype=dtype).pin_memory()

    def e2e_step():
        if args.graph:   # the graph's static inputs receive the copies
            x.copy_(hx, non_blocking=True)
            gy.copy_(hgy, non_blocking=True)
            run_step()
        else:
            dx.copy_(hx, non_blocking=True)
            dgy.copy_(hgy, non_blocking=True)
            step(dx, dgy)
        hgw.copy_(layers[-1].weight.grad, non_blocking=True)

    for _ in range(2):
        e2e_step()
    ms_e2e = timed(e2e_step, args.steps)
    clk = clocks.stop()

    flops_rank = L * 3 * readme_flops(Bl, C, H, W, C, k)
    value = world * flops_rank / (ms_step * 1e-3) / 1e12
    gflop = L * gemm_flops(Bl, C, H, W, C, k)   # one GEMM pass of every layer
    layer_wl = (Bl, C, H, W, C, k, 1, k // 2, 1, 1, cfg["off_std"])
    roofline, launches = roofline_of(trace, args.steps, layer_wl, dtype, L, args.workload, args.dtype)
    kernels = {kname: (n, tot) for kname, (n, tot) in trace.items()}
    line = {
        "metric": "dcnv2_fwd_bwd_readme_tflops", "value": value,
        "unit": "TFLOP/s (README formula, fwd+bwd of every DCN layer)", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": args.dtype, "data": "synthetic (seeded)",
        "config": {"workload": f"{args.workload}: {L} x DCN({C},{C},{k}x{k},pad {k // 2}) + ReLU, "
                               f"{H}x{W}, global batch {G}, {Bl} per rank, fwd+bwd+all-reduce",
                   "global_batch": G, "parallelism": f"dp{world}",
                   "l2": "flushed before every step (256 MiB write)", "offset_std_px": cfg["off_std"],
                   "cuda_graph": bool(args.graph), "channels_last": bool(args.channels_last)},
        "fwd_bwd_gemm_tflops": world * 3 * gflop / (ms_step * 1e-3) / 1e12,
        "kernels_ms_per_step": {kk: v[1] / args.steps for kk, v in kernels.items()},
        "roofline": roofline,
        "clocks": clk,
        "e2e": {"value": world * flops_rank / (ms_e2e * 1e-3) / 1e12,
                "unit": "TFLOP/s (README formula, fwd+bwd of every DCN layer)",
                "h2d_bytes_per_step": 2 * x.numel() * x.element_size(),
                "d2h_bytes_per_step": hgw.numel() * hgw.element_size(), "ms_per_step": ms_e2e},
        "gpu_launches": int(launches),
    }
    if rank == 0:
        print(json.dumps(line), file=_JSON_OUT, flush=True)
    if world > 1:
        dist.destroy_process_group()


def roofline_of(trace, steps, wl, dtype, layers_per_step, workload, dtype_name):
    """Roofline of the dominant kernel of a traced run: the tensor-core kernels against
    the measured bf16 dense peak with the algorithmic FLOPs of one GEMM pass; the SIMT
    scatter against the measured HBM copy bandwidth with its algorithmic bytes.
    `wl` is one layer's shape; a step runs
    `layers_per_step` such layers.  Returns (roofline, library launches in the run)."""
    B, C, H, W, Co, k, s, p, d, dg, _ = wl
    Ho, Wo = out_hw(H, W, k, s, p, d)
    peaks, peak_kind = load_peaks()
    kernels = {kname: (n, tot) for kname, (n, tot) in trace.items()}
    dom = max(kernels, key=lambda kk: kernels[kk][1])
    n_dom, tot_dom = kernels[dom]
    per_launch_ms = tot_dom / n_dom
    launches_per_layer = n_dom / steps / layers_per_step   # > 1 when the backward runs in chunks
    esz = torch.tensor([], dtype=dtype).element_size()
    K2 = k * k
    if dom in ("forward", "backward_data", "backward_weight"):
        gflop = gemm_flops(B, C, Ho, Wo, Co, k) / launches_per_layer
        work, bound, unit, peak = gflop, "tensor", "TFLOP/s", peaks["bf16_tflops"]
        basis = f"2*Co*C*k*k*B*Ho*Wo = {gflop:.4g} FLOP per launch"
        achieved = work / (per_launch_ms * 1e-3) / 1e12
    else:
        # scatter: read gcol (P*K2*C), x (B*C*H*W), offset+mask (3*K2*P); read+write the
        # fp32 grad_input accumulator (2 * 4*B*C*H*W); write grad_offset+grad_mask (3*K2*P)
        # and the sampled columns for the weight gradient (P*K2*C operands, hi+lo for f32)
        P = B * Ho * Wo
        nsplit = 2 if esz == 4 else 1
        nbytes = (P * K2 * C * esz + B * C * H * W * esz + 6 * K2 * P * esz + 8 * B * C * H * W
                  + P * K2 * C * 2 * nsplit) / launches_per_layer
        work, bound, unit, peak = nbytes, "hbm", "GB/s", peaks["hbm_gbs"]
        basis = (f"algorithmic bytes {nbytes:.4g} per launch (gcol, x, offset/mask, fp32 grad_input acc, "
                 "outputs, columns)")
        achieved = work / (per_launch_ms * 1e-3) / 1e9
    roofline = {"kernel": dom, "bound": bound, "achieved": achieved, "peak": peak, "unit": unit,
                "frac": achieved / peak,
                "peak_source": f"{peak_kind} ({'bf16 dense, burst' if bound == 'tensor' else 'HBM copy'})",
                "traffic": load_traffic(dom, workload, dtype_name), "algorithmic": basis}
    # library kernels in the traced run (the accumulator memset is a runtime call)
    launches = sum(n for kk, (n, _) in kernels.items() if kk != "zero_accumulators")
    return roofline, launches


def config_of(args, wl):
    B, C, H, W, Co, k, s, p, d, dg, off_std = wl
    return {"workload": f"{args.workload}: B={B}/gpu C={C} {H}x{W} Co={Co} {k}x{k} s{s} p{p} "
                        f"d{d} dg{dg}, fwd+bwd", "global_batch": B * args.gpus,
            "parallelism": f"dp{args.gpus}", "l2": "flushed before every step (256 MiB write)",
            "offset_std_px": off_std, "channels_last": bool(getattr(args, "channels_last", False)),
            "backward_reuses_packed_input": not getattr(args, "no_reuse", False)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--dtype", default="bf16", choices=list(DTYPES))
    ap.add_argument("--workload", default="readme", choices=list(WORKLOADS) + list(STACKS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-reuse", action="store_true",
                    help="the backward packs the input again instead of reusing the forward's")
    ap.add_argument("--no-fp32", action="store_true",
                    help="skip the float32 step reported beside a 16-bit run")
    ap.add_argument("--channels-last", action="store_true",
                    help="channels-last activations (the operator's NHWC layout)")
    ap.add_argument("--graph", action="store_true",
                    help="stack workloads: capture the training step in a CUDA graph and replay it")
    ap.add_argument("--launch-only", type=int, default=0, metavar="N",
                    help="run N forward+backward calls without timing and exit (for ncu)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.workload in STACKS:
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the stack workloads have no CPU "
                                  "reference arm; use the single-layer workloads"}), file=_JSON_OUT, flush=True)
            return
        run_stack(args)
        return
    wl = WORKLOADS[args.workload]

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, wl, rank)
        return

    import torch.distributed as dist
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    from dcnv2_b200 import _C, _lib
    from dcnv2_b200.dp import allreduce_tensors

    dtype = DTYPES[args.dtype]
    B, C, H, W, Co, k, s, p, d, dg, _ = wl
    Ho, Wo = out_hw(H, W, k, s, p, d)
    x, w, b, off, m, gy = make_inputs(wl, dtype, dev, seed=rank)
    if args.channels_last:
        # the operator's NHWC layout: every activation tensor channels-last
        x, off, m, gy = [t.contiguous(memory_format=torch.channels_last) for t in (x, off, m, gy)]
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    reuse = not args.no_reuse

    def step(x, off, m, gy):
        # one workspace for the pair, so the backward reuses the input the forward
        # packed (what the autograd modules do); --no-reuse packs it twice
        ws = _C.backward_workspace(x, w, s, s, p, p, d, d, dg) if reuse else None
        y = _C.dcn_v2_forward(x, w, m, off, b, s, s, p, p, d, d, dg, workspace=ws)
        gi, goff, gm, gw, gb = _C.dcn_v2_backward(x, w, m, off, b, gy, s, s, p, p, d, d, dg,
                                                  workspace=ws, input_packed=reuse)
        if world > 1:  # the data-parallel exchange: one bucketed all-reduce
            gw, gb = allreduce_tensors([gw, gb])
        return y, gw, gb

    def timed(fn, n):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(n)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        for i in range(n):
            flush.zero_()
            ev[i][0].record(stream)
            fn()
            ev[i][1].record(stream)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        ms = sum(a.elapsed_time(b_) for a, b_ in ev)
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()) / n

    if args.launch_only:
        for _ in range(args.launch_only):
            step(x, off, m, gy)
        torch.cuda.synchronize()
        print("launch-only done", flush=True)
        return

    # warm-up
    for _ in range(args.warmup):
        step(x, off, m, gy)
    torch.cuda.synchronize()

    # timed region (device-resident inputs), kernels traced with CUDA events
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
    clocks = ClockSampler(vis.split(",")[local] if vis else local)
    clocks.start()
    ms_step = timed(lambda: step(x, off, m, gy), args.steps)
    # the same steps again with every kernel bracketed by CUDA events (the
    # per-kernel breakdown and the roofline; the brackets themselves add about
    # 2 us per launch, so the step time above is taken without them)
    _lib.trace_reset()
    _lib.trace_enable(True)
    ms_step_traced = timed(lambda: step(x, off, m, gy), args.steps)
    _lib.trace_enable(False)
    trace = _lib.trace_collect()
    # forward alone (reported beside the step)
    ms_fwd = timed(lambda: _C.dcn_v2_forward(x, w, m, off, b, s, s, p, p, d, d, dg), args.steps)

    # end to end through the public API: pinned host inputs -> device -> result to host
    hx, hoff, hm, hgy = [t.cpu().pin_memory() for t in (x, off, m, gy)]
    hgw = torch.empty(w.shape, dtype=torch.float32 if world > 1 else w.dtype).pin_memory()
    hgb = torch.empty(b.shape, dtype=hgw.dtype).pin_memory()
    dx, doff, dm, dgy = [torch.empty_like(t) for t in (x, off, m, gy)]
    h2d = sum(t.numel() * t.element_size() for t in (hx, hoff, hm, hgy))
    d2h = hgw.numel() * hgw.element_size() + hgb.numel() * hgb.element_size()

    def e2e_step():
        for dst, src in ((dx, hx), (doff, hoff), (dm, hm), (dgy, hgy)):
            dst.copy_(src, non_blocking=True)
        _, gw_, gb_ = step(dx, doff, dm, dgy)
        hgw.copy_(gw_, non_blocking=True)
        hgb.copy_(gb_, non_blocking=True)

    for _ in range(2):
        e2e_step()
    ms_e2e_serial = timed(e2e_step, args.steps)

    # the same end-to-end steps as a training loop runs them: the host->device
    # copies of step i+1 go on a copy stream while step i computes (inputs double
    # buffered; every step still copies its own inputs in and its result out)
    copy_stream = torch.cuda.Stream(dev)
    hosts = (hx, hoff, hm, hgy)
    bufs = [[torch.empty_like(t) for t in (x, off, m, gy)] for _ in range(2)]
    copied = [torch.cuda.Event() for _ in range(2)]
    used = [torch.cuda.Event() for _ in range(2)]

    def e2e_pipelined(n):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        copy_stream.wait_stream(stream)

        def load(i):
            with torch.cuda.stream(copy_stream):
                if i >= 2:
                    copy_stream.wait_event(used[i % 2])
                for dst, src in zip(bufs[i % 2], hosts):
                    dst.copy_(src, non_blocking=True)
                copied[i % 2].record(copy_stream)

        load(0)
        for i in range(n):
            if i + 1 < n:
                load(i + 1)
            flush.zero_()
            stream.wait_event(copied[i % 2])
            _, gw_, gb_ = step(*bufs[i % 2])
            used[i % 2].record(stream)
            hgw.copy_(gw_, non_blocking=True)
            hgb.copy_(gb_, non_blocking=True)
        t1.record(stream)
        torch.cuda.synchronize()
        t = torch.tensor([t0.elapsed_time(t1)], device=dev, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item()) / n

    e2e_pipelined(3)
    ms_e2e = e2e_pipelined(args.steps)
    step_flops = 3 * readme_flops(B, C, Ho, Wo, Co, k)
    value = world * step_flops / (ms_step * 1e-3) / 1e12
    gflop = gemm_flops(B, C, Ho, Wo, Co, k)

    # the same step in float32, the precision of the benchmark configuration
    # (configs[0]) and of the reference operator, timed the same way
    fp32_leg = None
    if args.dtype != "fp32" and not args.no_fp32:
        x32, w32, b32, off32, m32, gy32 = make_inputs(wl, torch.float32, dev, seed=rank)

        def step32():
            ws = _C.backward_workspace(x32, w32, s, s, p, p, d, d, dg) if reuse else None
            _C.dcn_v2_forward(x32, w32, m32, off32, b32, s, s, p, p, d, d, dg, workspace=ws)
            gi_, go_, gm_, gw_, gb_ = _C.dcn_v2_backward(x32, w32, m32, off32, b32, gy32, s, s, p, p, d, d, dg,
                                                         workspace=ws, input_packed=reuse)
            if world > 1:
                allreduce_tensors([gw_, gb_])

        for _ in range(args.warmup):
            step32()
        ms32 = timed(step32, args.steps)
        ms32_fwd = timed(lambda: _C.dcn_v2_forward(x32, w32, m32, off32, b32, s, s, p, p, d, d, dg), args.steps)
        fp32_leg = {"ms_per_step": ms32, "value": world * step_flops / (ms32 * 1e-3) / 1e12,
                    "unit": "TFLOP/s (README formula, fwd+bwd)",
                    "fwd_bwd_gemm_tflops": world * 3 * gflop / (ms32 * 1e-3) / 1e12,
                    "fwd_ms": ms32_fwd,
                    "note": "float32 tensors; every GEMM operand split into bf16 hi + lo, three MMAs"}
        del x32, w32, b32, off32, m32, gy32
    clk = clocks.stop()
    e2e_value = world * step_flops / (ms_e2e * 1e-3) / 1e12

    roofline, launches = roofline_of(trace, args.steps, wl, dtype, 1, args.workload, args.dtype)
    kernels = {kname: (n, tot) for kname, (n, tot) in trace.items()}

    line = {
        "metric": "dcnv2_fwd_bwd_readme_tflops", "value": value,
        "unit": "TFLOP/s (README formula, fwd+bwd)", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": args.dtype, "data": "synthetic (seeded)",
        "config": config_of(args, wl),
        "fwd_ms": ms_fwd, "fwd_readme_tflops": readme_flops(B, C, Ho, Wo, Co, k) / (ms_fwd * 1e-3) / 1e12,
        "fwd_bwd_gemm_tflops": world * 3 * gflop / (ms_step * 1e-3) / 1e12,
        "kernels_ms_per_step": {kk: v[1] / args.steps for kk, v in kernels.items()},
        "ms_per_step_traced": ms_step_traced,
        "roofline": roofline,
        "clocks": clk,
        "e2e": {"value": e2e_value, "unit": "TFLOP/s (README formula, fwd+bwd)",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": ms_e2e,
                "pipelined": "copies of step i+1 overlap step i on a second stream; the 256 MiB L2 "
                             "flush is also written before every step",
                "serial_ms_per_step": ms_e2e_serial},
        "gpu_launches": int(launches),
    }
    if fp32_leg is not None:
        line["fp32"] = fp32_leg
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(wl)
        line["cpu_torchvision"] = cpu_torchvision(wl)
    if rank == 0:
        print(json.dumps(line), file=_JSON_OUT, flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
