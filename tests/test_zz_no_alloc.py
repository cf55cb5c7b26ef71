"""dcn_forward_noalloc: the forward for callers that may not allocate GPU memory
(for example code running while a framework records a stream into a graph,
runtimes whose memory is fixed at start-up, or plugins whose host owns every
buffer).  It takes its scratch from a fixed array inside the library instead of
a caller-provided workspace.

Checked here through the C ABI: two calls in a row (different inputs, so the
second call must not depend on what the first left in the shared scratch) give
the same output as the workspace-taking dcn_forward, within the parity
tolerances of the other GPU tests; oversized problems are rejected.  This file
is collected last so that a run stopping at the first failure has already run
every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from dcn_cases import Case, make_inputs, rel_err

TOL = {torch.float32: 1e-4, torch.bfloat16: 1e-2}


def _desc(lib_mod, c, dtype):
    code = {torch.float32: lib_mod.DCN_F32, torch.bfloat16: lib_mod.DCN_BF16}[dtype]
    return lib_mod.DcnDesc(c.B, c.C, c.H, c.W, c.Co, c.kh, c.kw, c.stride, c.stride, c.pad, c.pad,
                           c.dil, c.dil, c.dg, code, 1)


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32], ids=["bf16", "fp32"])
def test_noalloc_matches_workspace_forward_twice(dtype):
    from dcnv2_b200 import _lib
    lib = _lib.lib
    cases = [Case("na_a", 2, 64, 20, 18, 96, 3, 3, off_std=2.0),
             Case("na_b", 1, 48, 13, 17, 40, 3, 3, stride=2, pad=2, dil=2, dg=2, off_std=3.0)]
    dev = torch.device("cuda:0")
    stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    for seed, c in enumerate(cases):
        x, w, b, off, m, _ = [t.to(dtype).to(dev) for t in make_inputs(c, seed=seed + 7)]
        d = _desc(_lib, c, dtype)
        ho, wo = c.out_hw()
        ref = torch.empty(c.B, c.Co, ho, wo, dtype=dtype, device=dev)
        out = torch.full_like(ref, float("nan"))
        nbytes = lib.dcn_forward_workspace_size(ctypes.byref(d))
        assert 0 < nbytes <= _lib.NOALLOC_SCRATCH_BYTES
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        rc = lib.dcn_forward(ctypes.byref(d), _p(x), _p(w), _p(m), _p(off), _p(b), _p(ref), _p(ws),
                             nbytes, stream)
        assert rc == 0, _lib.strerror(rc)
        rc = lib.dcn_forward_noalloc(ctypes.byref(d), _p(x), _p(w), _p(m), _p(off), _p(b), _p(out),
                                     stream)
        assert rc == 0, _lib.strerror(rc)
        torch.cuda.synchronize()
        err = rel_err(out.float().cpu().numpy(), ref.float().cpu().numpy())
        assert np.isfinite(out.float().cpu().numpy()).all()
        assert err <= TOL[dtype], f"{c.name}: {err}"


@pytest.mark.gpu
def test_noalloc_rejects_problems_beyond_its_scratch():
    from dcnv2_b200 import _lib
    c = Case("huge", 64, 256, 128, 128, 256, 3, 3)   # packed input alone is 512 MiB in bf16
    d = _desc(_lib, c, torch.bfloat16)
    assert _lib.lib.dcn_forward_workspace_size(ctypes.byref(d)) > _lib.NOALLOC_SCRATCH_BYTES
    rc = _lib.lib.dcn_forward_noalloc(ctypes.byref(d), None, None, None, None, None, None, None)
    assert rc == _lib.DCN_E_SCRATCH_LIMIT
    assert "scratch" in _lib.strerror(rc)
