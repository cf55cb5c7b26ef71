"""Golden-vector cases (small, seeded).  REF_CASES run on the reference's own CUDA
kernels (deformable_groups 1, dilation 1, equal pads: what the reference supports);
TV_CASES run on torchvision.ops.deform_conv2d in float64 (dilation and deformable
groups, which the reference kernels ignore).  TV_CASES use non-integer offsets:
at integer sample coordinates torchvision's grad_offset takes a different one-sided
difference than the reference (com.cu:388-429), whose formula this repository follows."""

# (name, B, C, H, W, Co, kh, kw, stride, pad, dil, dg, off_std)
REF_CASES = [
    ("ref_k3_s1_p1", 2, 16, 9, 9, 32, 3, 3, 1, 1, 1, 1, 1.5),
    ("ref_k3_s2_p0_odd", 1, 8, 11, 13, 24, 3, 3, 2, 0, 1, 1, 2.5),
    ("ref_k1_p0", 2, 32, 8, 8, 64, 1, 1, 1, 0, 1, 1, 1.0),
    ("ref_k5_p2_far", 1, 12, 10, 7, 20, 5, 5, 1, 2, 1, 1, 4.0),
    ("ref_k7_s2_p3", 1, 64, 14, 14, 256, 7, 7, 2, 3, 1, 1, 1.5),
]

TV_CASES = [
    ("tv_dil2_dg2", 2, 8, 11, 9, 12, 3, 3, 1, 2, 2, 2, 2.0),
    ("tv_k5_s2_d2_dg2", 1, 12, 17, 19, 10, 5, 5, 2, 4, 2, 2, 8.0),
    ("tv_dg4_k3x2", 1, 16, 7, 10, 8, 3, 2, 1, 1, 1, 4, 1.5),
]


def make(case, seed=0, integer_offsets=True):
    """float64 numpy inputs x, w, b, offset, mask, grad_out for one case."""
    import numpy as np
    name, B, C, H, W, Co, kh, kw, s, p, d, dg, off_std = case
    rng = np.random.default_rng(seed + sum(map(ord, name)))
    Ho = (H + 2 * p - (d * (kh - 1) + 1)) // s + 1
    Wo = (W + 2 * p - (d * (kw - 1) + 1)) // s + 1
    x = rng.standard_normal((B, C, H, W))
    w = rng.standard_normal((Co, C, kh, kw)) * (2.0 / (C * kh * kw)) ** 0.5
    b = rng.standard_normal(Co) * 0.01
    off = rng.standard_normal((B, 2 * dg * kh * kw, Ho, Wo)) * off_std
    m = 1.0 / (1.0 + np.exp(-rng.standard_normal((B, dg * kh * kw, Ho, Wo))))
    gy = rng.standard_normal((B, Co, Ho, Wo))
    if integer_offsets:
        # integer-valued offsets on a quarter of the samples hit exact corners / edges
        off[..., ::2, ::2] = np.round(off[..., ::2, ::2])
    return x, w, b, off, m, gy
