"""bf16 GEMM with fused epilogue on tcgen05 (``hclsm_gemm_bf16``)."""
from __future__ import annotations

import torch

from .. import _lib

EPI = {"none": 0, "relu": 1, "resid": 2}


def gemm_bf16(a, w, *, bias=None, epilogue="none", resid=None, clamp=0.0, out_f32=True, out_bf16=False):
    """act(a @ w.T + bias [+ resid]) with a (M, K) and w (N, K) bf16; returns
    (fp32 result or None, bf16 result or None)."""
    _lib.require_cuda(a, w)
    a = a.contiguous()
    w = w.contiguous()
    M, K = a.shape
    N = w.shape[0]
    of = torch.empty(M, N, dtype=torch.float32, device=a.device) if out_f32 else None
    ob = torch.empty(M, N, dtype=torch.bfloat16, device=a.device) if out_bf16 else None
    rc = _lib.load().hclsm_gemm_bf16(_lib.ptr(a), _lib.ptr(w), M, N, K, EPI[epilogue], _lib.ptr(bias),
                                     _lib.ptr(resid), _lib.ptr(of), _lib.ptr(ob), float(clamp),
                                     _lib.stream_ptr(a.device))
    _lib.check(rc, "hclsm_gemm_bf16")
    return of, ob
