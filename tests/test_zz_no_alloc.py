"""The allocation-free scan backward (hclsm_ssm_scan_bwd_noalloc).

It exists for callers that cannot allocate device memory at the moment they run
the backward — host callbacks, allocator hooks, runtimes with a fixed memory
plan — so it keeps its scratch in a fixed device array instead of a workspace.
This test calls it through the C ABI twice in a row (the array keeps the
previous call's contents) and compares it with the workspace entry point.
It sits in its own file, collected last.
"""
import ctypes

import numpy as np
import pytest
import torch

from hclsm_b200 import _lib
from hclsm_b200.kernels.ssm_scan_kernel import scan_bwd_raw
from hclsm_b200.workloads import scan_inputs

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a = a.double().cpu().numpy()
    b = b.double().cpu().numpy()
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def _noalloc(d, gated, dtype):
    lib = _lib.load()
    x = d["x"]
    nseq, L, Dn = x.shape
    S = d["B"].shape[-1]
    out = dict(dx=torch.empty_like(x), ddt=torch.empty_like(x), dB=torch.empty_like(d["B"]),
               dC=torch.empty_like(d["C"]), dA=torch.empty(Dn, S, device=x.device),
               dD=torch.empty(Dn, device=x.device) if gated else None,
               dz=torch.empty_like(x) if gated else None)
    p = _lib.ptr
    rc = lib.hclsm_ssm_scan_bwd_noalloc(
        p(x), p(d["dt"]), p(d["A_log"]), p(d["B"]), p(d["C"]), p(d.get("D")), p(d.get("z")), p(d["dy"]),
        p(out["dx"]), p(out["ddt"]), p(out["dA"]), p(out["dB"]), p(out["dC"]), p(out["dD"]), p(out["dz"]),
        nseq, L, Dn, S, _lib.dtype_code(dtype), 0, _lib.stream_ptr(x.device))
    assert rc == 0, rc
    return [out[k] for k in ("dx", "ddt", "dA", "dB", "dC", "dD", "dz")]


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-5)])
@pytest.mark.parametrize("gated", [False, True])
def test_noalloc_matches_workspace_entry(dtype, tol, gated):
    lib = _lib.load()
    assert lib.hclsm_ssm_scan_bwd_noalloc_max_scratch() == 48 << 20
    cases = [scan_inputs(8, 64, 256, 16, dtype=dtype, seed=5, device="cuda", gated=gated),
             scan_inputs(3, 40, 136, 8, dtype=dtype, seed=6, device="cuda", gated=gated)]
    for d in cases:  # two calls in a row, different shapes, shared scratch
        ref = scan_bwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], d["dy"], d.get("D"), d.get("z"))
        got = _noalloc(d, gated, dtype)
        torch.cuda.synchronize()
        for g, r in zip(got, ref):
            if r is not None:
                assert _rel(g, r) <= tol
    # and the first case again after the second overwrote the scratch
    d = cases[0]
    ref = scan_bwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], d["dy"], d.get("D"), d.get("z"))
    got = _noalloc(d, gated, dtype)
    for g, r in zip(got, ref):
        if r is not None:
            assert _rel(g, r) <= tol


def test_noalloc_rejects_oversize():
    lib = _lib.load()
    d = scan_inputs(2, 8, 64, 16, dtype=torch.bfloat16, seed=1, device="cuda")
    big_nseq = 1 << 20  # needs far more than 48 MiB of scratch; nothing is launched
    p = _lib.ptr
    rc = lib.hclsm_ssm_scan_bwd_noalloc(p(d["x"]), p(d["dt"]), p(d["A_log"]), p(d["B"]), p(d["C"]), None, None,
                                        p(d["dy"]), p(d["x"]), p(d["x"]), p(d["A_log"]), p(d["B"]), p(d["C"]),
                                        None, None, big_nseq, 8, 64, 16, _lib.BF16, 0,
                                        _lib.stream_ptr(d["x"].device))
    assert rc == 4  # HCLSM_ERR_WORKSPACE
