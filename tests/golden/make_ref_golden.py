"""Generates golden vectors from the reference's own CUDA kernels.

Runs on a GPU box with the reference extension prebuilt into oracle/_ref
(``python oracle/build_ref.py <reference checkout>``).  Inputs are rounded to
float32 (the reference's only dtype) and stored with the reference's forward
output and all five gradients in ``<out>/<case>.npz``.

    python tests/golden/make_ref_golden.py --out tests/golden
"""
import argparse
import glob
import importlib.machinery
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, HERE)
from golden_cases import REF_CASES, make  # noqa: E402


def load_ref():
    so = glob.glob(os.path.join(ROOT, "oracle", "_ref", "Conv2d_ref*.so"))
    if not so:
        raise SystemExit("oracle/_ref/Conv2d_ref*.so missing (python oracle/build_ref.py <ref>)")
    loader = importlib.machinery.ExtensionFileLoader("Conv2d_ref", so[0])
    spec = importlib.util.spec_from_loader("Conv2d_ref", loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    os.makedirs(args.out, exist_ok=True)
    torch.backends.cuda.matmul.allow_tf32 = False
    ref = load_ref()
    for case in REF_CASES:
        name, B, C, H, W, Co, kh, kw, s, p, d, dg, _ = case
        assert d == 1 and dg == 1
        x, w, b, off, m, gy = [a.astype(np.float32) for a in make(case)]
        cu = [torch.from_numpy(a).cuda() for a in (x, w, b, off, m, gy)]
        y = ref.dcn_v2_forward(cu[0], cu[1], cu[4], cu[3], cu[2], s, s, p, p)
        grads = ref.dcn_v2_backward(cu[0], cu[1], cu[4], cu[3], cu[2], cu[5], s, s, p, p)
        torch.cuda.synchronize()
        out = {"x": x, "w": w, "b": b, "offset": off, "mask": m, "grad_out": gy,
               "y": y.cpu().numpy()}
        for k, g in zip(["grad_input", "grad_offset", "grad_mask", "grad_weight", "grad_bias"], grads):
            out[k] = g.cpu().numpy()
        out["params"] = np.array([s, p, d, dg], dtype=np.int64)
        np.savez_compressed(os.path.join(args.out, f"{name}.npz"), **out)
        print("wrote", name, {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
