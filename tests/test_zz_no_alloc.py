"""The allocation-free scan backward (hclsm_ssm_scan_bwd_noalloc).

It exists for callers that cannot allocate device memory at the moment they run
the backward — host callbacks, allocator hooks, runtimes with a fixed memory
plan — so it keeps its scratch in a fixed device array instead of a workspace.
Both entry points run the same kernels on the same inputs, so the results must
be bit-identical: the test calls the new entry point through the C ABI twice in
a row (the array keeps the previous call's contents), for every flag
combination, and compares it with the workspace entry point with torch.equal;
one case is also checked against the CPU oracle.  It sits in its own file,
collected last.
"""
import numpy as np
import pytest
import torch

from hclsm_b200 import _lib
from hclsm_b200.kernels.ssm_scan_kernel import scan_bwd_raw
from hclsm_b200.workloads import scan_inputs

pytestmark = pytest.mark.gpu

CLAMP, SOFTPLUS = 1, 2  # HCLSM_SCAN_CLAMP, HCLSM_SCAN_DT_SOFTPLUS


def _noalloc(d, gated, dtype, flags):
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
        nseq, L, Dn, S, _lib.dtype_code(dtype), flags, _lib.stream_ptr(x.device))
    assert rc == 0, rc
    return [out[k] for k in ("dx", "ddt", "dA", "dB", "dC", "dD", "dz")]


def _workspace(d, flags):
    return scan_bwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], d["dy"], d.get("D"), d.get("z"),
                        clamp=bool(flags & CLAMP), dt_softplus=bool(flags & SOFTPLUS))


def _same(got, ref):
    for g, r in zip(got, ref):
        assert (g is None) == (r is None)
        if r is not None:
            assert torch.equal(g, r)


@pytest.mark.parametrize("flags", [0, CLAMP, SOFTPLUS, CLAMP | SOFTPLUS])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("gated", [False, True])
def test_noalloc_matches_workspace_entry(dtype, gated, flags):
    lib = _lib.load()
    assert lib.hclsm_ssm_scan_bwd_noalloc_max_scratch() == 48 << 20
    cases = [scan_inputs(8, 64, 256, 16, dtype=dtype, seed=5, device="cuda", gated=gated),
             scan_inputs(3, 40, 136, 8, dtype=dtype, seed=6, device="cuda", gated=gated)]
    for d in cases:  # two calls in a row, different shapes, shared scratch
        _same(_noalloc(d, gated, dtype, flags), _workspace(d, flags))
    # the first case again after the second overwrote the scratch
    _same(_noalloc(cases[0], gated, dtype, flags), _workspace(cases[0], flags))
    torch.cuda.synchronize()


@pytest.mark.parametrize("dtype,tol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-5)])
def test_noalloc_matches_oracle(dtype, tol):
    from oracle import scan as oscan

    # unclamped: with A_log ~ U(0, ln 16) the clamp of exp(A_log) to [1e-6, 1]
    # binds everywhere and would zero dA_log
    d = scan_inputs(4, 48, 128, 16, dtype=dtype, seed=9, device="cuda", gated=True)
    for _ in range(2):
        got = _noalloc(d, True, dtype, 0)
    torch.cuda.synchronize()
    o = {k: v.float().cpu().numpy() for k, v in d.items()}
    ref = oscan.scan_bwd(o["x"], o["dt"], o["A_log"], o["B"], o["C"], o["dy"], o["D"], o["z"], clamp=False)
    for g, name in zip(got, ("dx", "ddt", "dA_log", "dB", "dC", "dD", "dz")):
        g = g.double().cpu().numpy()
        r = ref[name].astype(np.float64)
        assert np.abs(g - r).max() / np.abs(r).max() <= tol, name


def _call(lib, d, nseq, L, Dn, S, dtype, flags, ws=None):
    p = _lib.ptr
    args = (p(d["x"]), p(d["dt"]), p(d["A_log"]), p(d["B"]), p(d["C"]), None, None, p(d["dy"]), p(d["x"]),
            p(d["x"]), p(d["A_log"]), p(d["B"]), p(d["C"]), None, None, nseq, L, Dn, S, dtype, flags)
    st = _lib.stream_ptr(d["x"].device)
    if ws is None:
        return lib.hclsm_ssm_scan_bwd_noalloc(*args, st)
    return lib.hclsm_ssm_scan_bwd(*args, _lib.ptr(ws), ws.numel(), st)


def test_noalloc_rejects_like_workspace_entry():
    lib = _lib.load()
    d = scan_inputs(2, 8, 64, 16, dtype=torch.bfloat16, seed=1, device="cuda")
    ws = torch.empty(64 << 20, dtype=torch.uint8, device="cuda")
    # oversize: needs far more than 48 MiB of scratch; nothing is launched
    assert _call(lib, d, 1 << 20, 8, 64, 16, _lib.BF16, 0) == 4  # HCLSM_ERR_WORKSPACE
    # invalid arguments: the same status as the workspace entry point
    for nseq, L, Dn, S, dt, fl in ((2, 8, 0, 16, _lib.BF16, 0), (2, 8, 64, 0, _lib.BF16, 0),
                                   (2, 8, 64, 100, _lib.BF16, 0), (2, 8, 64, 16, 7, 0),
                                   (2, 8, 64, 16, _lib.BF16, 8), (-1, 8, 64, 16, _lib.BF16, 0)):
        want = _call(lib, d, nseq, L, Dn, S, dt, fl, ws=ws)
        assert want != 0
        assert _call(lib, d, nseq, L, Dn, S, dt, fl) == want, (nseq, L, Dn, S, dt, fl)
    torch.cuda.synchronize()
