"""Seeded synthetic DCNv2 problems shared by the tests (shapes of the benchmark
configurations scaled down so the float64 oracle finishes in seconds)."""
from __future__ import annotations

import dataclasses

import numpy as np
import torch


@dataclasses.dataclass(frozen=True)
class Case:
    name: str
    B: int
    C: int
    H: int
    W: int
    Co: int
    kh: int
    kw: int
    stride: int = 1
    pad: int = 1
    dil: int = 1
    dg: int = 1
    off_std: float = 1.5
    mask_std: float = 1.0
    bias: bool = True

    def out_hw(self):
        ho = (self.H + 2 * self.pad - (self.dil * (self.kh - 1) + 1)) // self.stride + 1
        wo = (self.W + 2 * self.pad - (self.dil * (self.kw - 1) + 1)) // self.stride + 1
        return ho, wo


def make_inputs(c: Case, seed: int = 0):
    """float32 CPU tensors x, weight, bias, offset, mask, grad_out (fixed seeds per
    tensor: 0 x, 1 weight, 2 bias, 3 offset, 4 mask, 5 grad_out; shifted by `seed`)."""
    ho, wo = c.out_hw()
    K2 = c.kh * c.kw

    def g(s):
        return torch.Generator().manual_seed(1000 * seed + s)

    x = torch.randn(c.B, c.C, c.H, c.W, generator=g(0))
    fan_in = c.C * K2
    w = torch.randn(c.Co, c.C, c.kh, c.kw, generator=g(1)) * (2.0 / fan_in) ** 0.5
    b = torch.randn(c.Co, generator=g(2)) * 0.01 if c.bias else None
    off = torch.randn(c.B, 2 * c.dg * K2, ho, wo, generator=g(3)) * c.off_std
    m = torch.sigmoid(torch.randn(c.B, c.dg * K2, ho, wo, generator=g(4)) * c.mask_std)
    gy = torch.randn(c.B, c.Co, ho, wo, generator=g(5))
    return x, w, b, off, m, gy


def rel_err(a, b) -> float:
    """max|a - b| / max|b| (the tests' error metric; elementwise relative error is
    undefined where the reference is ~0)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.abs(b).max() if b.size else 0.0
    if den == 0.0:
        return float(np.abs(a).max()) if a.size else 0.0
    return float(np.abs(a - b).max() / den)


# parity cases: (case, dtypes)
SMALL = [
    Case("readme_small", 2, 64, 16, 16, 256, 3, 3),
    Case("c_odd", 1, 24, 11, 13, 40, 3, 3, off_std=2.0),
    Case("stride2_pad0", 2, 64, 17, 15, 64, 3, 3, stride=2, pad=0),
    Case("dg4_bf", 1, 128, 8, 8, 128, 3, 3, dg=4, off_std=2.0),
    Case("edge_c4", 1, 96, 21, 27, 160, 5, 5, stride=2, pad=4, dil=2, dg=2, off_std=8.0,
         mask_std=3.0),
    Case("k1_nopad", 2, 64, 9, 9, 64, 1, 1, pad=0),
    Case("co512_c512", 1, 512, 6, 6, 512, 3, 3),
    Case("nobias", 1, 32, 7, 9, 48, 3, 2, bias=False),
    # 64-pixel blocks inside one image (H*Wo % 64 == 0): for 16-bit types the
    # GEMMs read grad_output directly and the weight-gradient kernel sums grad_bias
    Case("direct_co100", 3, 32, 8, 16, 100, 3, 3),
    Case("direct_co40", 2, 16, 8, 8, 40, 3, 3, off_std=2.0),
    # one-pixel-high / -wide images: the clamped 2x2 corner block degenerates
    Case("thin_h1", 2, 16, 1, 9, 24, 3, 3),
    Case("thin_w1", 1, 16, 6, 1, 24, 3, 3, off_std=2.0),
    # images large enough for the forward's input windows (Wo % 16 == 0,
    # W >= 24, H >= 16; Ho = 20: a partial last tile row) and the tile scatter
    Case("win_20x32", 2, 64, 20, 32, 96, 3, 3, off_std=2.0),
    Case("win_k1", 2, 64, 16, 32, 64, 1, 1, pad=0),
]


def record(test: str, errs: dict, tol: float) -> None:
    """Appends the achieved errors of a parity test as one JSON line to the file
    named by DCN_PARITY_LOG (when set), so the margins of a GPU run can be read
    back and tabulated."""
    import json
    import os
    path = os.environ.get("DCN_PARITY_LOG")
    if not path:
        return
    with open(path, "a") as f:
        f.write(json.dumps({"test": test, "tol": tol, "errors": errs}) + "\n")
