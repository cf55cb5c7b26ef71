"""Generates float64 golden vectors with torchvision.ops.deform_conv2d (CPU) for
dilation > 1 and deformable groups > 1 -- the same arithmetic as the reference
(checked to 1e-15 where both apply), extended to the arguments the reference
kernels ignore.

    python tests/golden/make_tv_golden.py --out tests/golden
"""
import argparse
import os
import sys

import numpy as np
import torch
from torchvision.ops import deform_conv2d

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from golden_cases import TV_CASES, make  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    for case in TV_CASES:
        name, B, C, H, W, Co, kh, kw, s, p, d, dg, _ = case
        arrs = make(case, integer_offsets=False)
        x, w, b, off, m, gy = [torch.from_numpy(a).requires_grad_(True) for a in arrs]
        y = deform_conv2d(x, off, w, b, stride=s, padding=p, dilation=d, mask=m)
        y.backward(gy.detach())
        out = {"x": arrs[0], "w": arrs[1], "b": arrs[2], "offset": arrs[3], "mask": arrs[4],
               "grad_out": arrs[5], "y": y.detach().numpy(), "grad_input": x.grad.numpy(),
               "grad_offset": off.grad.numpy(), "grad_mask": m.grad.numpy(),
               "grad_weight": w.grad.numpy(), "grad_bias": b.grad.numpy(),
               "params": np.array([s, p, d, dg], dtype=np.int64)}
        np.savez_compressed(os.path.join(args.out, f"{name}.npz"), **out)
        print("wrote", name)


if __name__ == "__main__":
    main()
