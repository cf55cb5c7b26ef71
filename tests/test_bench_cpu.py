"""bench.py on CPU: the reference arm's JSON line, the stack workload's reference
line, and the roofline arithmetic on a synthetic kernel trace."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                         capture_output=True, text=True, timeout=600, check=True)
    lines = [ln for ln in out.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, out.stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _run("--impl", "reference", "--steps", "1", "--warmup", "3", "--workload", "readme_b2")
    assert d["impl"] == "reference"
    assert d["value"] > 0 and d["higher_is_better"] is True
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["value"] == d["value"]


def test_stack_reference_unavailable():
    d = _run("--impl", "reference", "--workload", "stack3")
    assert d["impl"] == "reference" and "unavailable" in d


def test_roofline_of_branches():
    sys.path.insert(0, ROOT)
    import bench
    import torch
    wl = bench.WORKLOADS["readme"]
    # one step: forward 0.1 ms (tensor bound), scatter 0.25 ms over two chunk launches
    trace = {"forward": (1, 0.1), "backward_scatter": (2, 0.25)}
    roof, launches = bench.roofline_of(trace, 1, wl, torch.bfloat16, 1, "readme", "bf16")
    assert roof["kernel"] == "backward_scatter" and roof["bound"] == "hbm"
    B, C, H, W, Co, k = wl[:6]
    P = B * H * W
    nbytes = (P * k * k * C * 2 + B * C * H * W * 2 + 6 * k * k * P * 2 + 8 * B * C * H * W
              + P * k * k * C * 2) / 2             # per launch (two chunks)
    assert abs(roof["achieved"] - nbytes / 0.125e-3 / 1e9) < 1e-6
    assert "l2_reduction" not in roof
    assert launches == 3
    trace = {"forward": (3, 0.3), "backward_scatter": (3, 0.1)}   # 3 layers per step
    roof, _ = bench.roofline_of(trace, 1, wl, torch.bfloat16, 3, "readme", "bf16")
    gflop = bench.gemm_flops(B, C, H, W, Co, k)
    assert roof["bound"] == "tensor" and abs(roof["achieved"] - gflop / 0.1e-3 / 1e12) < 1e-6
