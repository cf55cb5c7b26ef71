"""Build the reference's own CUDA extension into ``oracle/_ref`` (test infrastructure).

The reference operator (TseLin-Liu/DCNv2, ``com.cu`` + ``ext.cpp``, the sources its
``setup.py:24`` builds) is compiled from the files where they lie in the reference
checkout, with torch's extension builder, for sm_100.  Nothing from the reference is
copied into this repository: the only outputs are the object files and the
``Conv2d_ref*.so`` module under ``oracle/_ref/`` (git-ignored, shipped to GPU boxes
with the rest of the tree).

The module is used only as a checker: by ``tests/golden/make_ref_golden.py`` to pin
the C oracle against the reference's real kernels on a B200, and by GPU parity
tests when the ``.so`` is present.  It is never on the product path.

Usage: ``python oracle/build_ref.py REFERENCE_DIR`` (or with ``DCN_REFERENCE_DIR``
set in the environment).
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")


def build(ref_dir: str) -> None:
    src = [os.path.join(ref_dir, "com.cu"), os.path.join(ref_dir, "ext.cpp")]
    for s in src:
        if not os.path.exists(s):
            raise FileNotFoundError(s)
    os.makedirs(OUT, exist_ok=True)
    os.environ.setdefault("TORCH_CUDA_ARCH_LIST", "10.0")
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load

    load(
        name="Conv2d_ref",
        sources=src,
        extra_include_paths=[ref_dir],
        extra_cuda_cflags=["-O3", "-gencode", "arch=compute_100a,code=sm_100a"],
        build_directory=OUT,
        verbose=False,
    )
    print("built", [f for f in os.listdir(OUT) if f.endswith(".so")])


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("DCN_REFERENCE_DIR")
    if not ref:
        raise SystemExit("usage: build_ref.py REFERENCE_DIR (or set DCN_REFERENCE_DIR)")
    build(ref)
