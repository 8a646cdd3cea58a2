"""Selective SSM scan on B200 — drop-in for hclsm/kernels/ssm_scan_kernel.py.

``ssm_scan_fn(x, dt, A_log, B, C, backend="auto")`` keeps the reference
signature (ssm_scan_kernel.py:394-421).  Keyword-only extras keep reference
semantics at their defaults:

* ``clamp`` — ``None`` (default) follows the reference dispatcher: the CUDA
  paths (Triton / parallel, :168-290) do not clamp, so ``clamp=False``.  Pass
  ``clamp=True`` for the arithmetic of ``sequential_ssm_scan`` (:42-86), which is
  also what the model's inline scan does (hclsm/dynamics/level0_ssm.py:82-99).
* ``D`` (d_inner,) and ``z`` (like x): ``y = (scan + D*x) * silu(z)``.

Computation is fp32 for fp32 and bf16 inputs; the output has x's dtype and the
gradients have their inputs' dtypes (A_log / D gradients are fp32), as in the
reference's ``_TritonSSMScan`` (:292-377).
"""
from __future__ import annotations

import torch

from .. import _lib

__all__ = ["ssm_scan_fn", "ssm_scan", "scan_fwd_raw", "scan_bwd_raw", "bwd_workspace_bytes", "states_bytes"]


def _io_dtype(*ts):
    dts = {t.dtype for t in ts if t is not None}
    if dts == {torch.bfloat16}:
        return torch.bfloat16
    return torch.float32


def _prep(t, dt):
    if t is None:
        return None
    t = t.to(dt) if t.dtype != dt else t
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def _check_shapes(x, dt, A_log, B, C, D, z):
    if x.dim() != 3:
        raise ValueError(f"x must be (batch, T, d_inner), got {tuple(x.shape)}")
    nseq, L, Dn = x.shape
    if dt.shape != x.shape:
        raise ValueError("dt must have x's shape")
    if B.dim() != 3 or B.shape[:2] != x.shape[:2] or C.shape != B.shape:
        raise ValueError("B and C must be (batch, T, d_state)")
    S = B.shape[-1]
    if A_log.shape != (Dn, S):
        raise ValueError(f"A_log must be (d_inner, d_state) = {(Dn, S)}")
    if D is not None and D.shape != (Dn,):
        raise ValueError("D must be (d_inner,)")
    if z is not None and z.shape != x.shape:
        raise ValueError("z must have x's shape")
    return nseq, L, Dn, S


def states_bytes(nseq, L, Dn, S, dtype) -> int:
    """Bytes of the forward's state snapshots for the backward (0 where that
    path does not apply: it needs bf16, 9 <= d_state <= 16, even d_inner)."""
    return int(_lib.load().hclsm_ssm_scan_states_size(nseq, L, Dn, S, _lib.dtype_code(dtype)))


def _flags(clamp, dt_softplus):
    """The scan entry points' flags argument: bit 0 clamped arithmetic, bit 1
    softplus applied to the raw dt inside the kernel."""
    return int(bool(clamp)) | (2 if dt_softplus else 0)


def scan_fwd_raw(x, dt, A_log, B, C, D=None, z=None, clamp=False, out=None, states=None, dt_softplus=False):
    """One forward call through the C ABI; tensors must already be prepared.
    With ``states`` (a uint8 tensor of ``states_bytes(...)`` bytes) the forward
    also keeps h every 10 steps for ``scan_bwd_raw(..., states=...)``.  With
    ``dt_softplus`` dt is the raw projection and softplus is applied inside."""
    nseq, L, Dn, S = x.shape[0], x.shape[1], x.shape[2], B.shape[-1]
    flags = _flags(clamp, dt_softplus)
    y = out if out is not None else torch.empty_like(x)
    lib = _lib.load()
    if states is not None:
        rc = lib.hclsm_ssm_scan_fwd_states(_lib.ptr(x), _lib.ptr(dt), _lib.ptr(A_log), _lib.ptr(B), _lib.ptr(C),
                                           _lib.ptr(D), _lib.ptr(z), _lib.ptr(y), nseq, L, Dn, S,
                                           _lib.dtype_code(x.dtype), flags, _lib.ptr(states),
                                           states.numel() * states.element_size(), _lib.stream_ptr(x.device))
        _lib.check(rc, "hclsm_ssm_scan_fwd_states")
        return y
    rc = lib.hclsm_ssm_scan_fwd(_lib.ptr(x), _lib.ptr(dt), _lib.ptr(A_log), _lib.ptr(B), _lib.ptr(C),
                                _lib.ptr(D), _lib.ptr(z), _lib.ptr(y), nseq, L, Dn, S,
                                _lib.dtype_code(x.dtype), flags, _lib.stream_ptr(x.device))
    _lib.check(rc, "hclsm_ssm_scan_fwd")
    return y


def bwd_workspace_bytes(nseq, L, Dn, S) -> int:
    return int(_lib.load().hclsm_ssm_scan_bwd_workspace_size(nseq, L, Dn, S))


def scan_bwd_raw(x, dt, A_log, B, C, dy, D=None, z=None, clamp=False, workspace=None, states=None,
                 dt_softplus=False):
    """Gradients (dx, ddt, dA_log, dB, dC, dD, dz); with ``dt_softplus`` ddt is
    the gradient of the raw dt."""
    nseq, L, Dn, S = x.shape[0], x.shape[1], x.shape[2], B.shape[-1]
    flags = _flags(clamp, dt_softplus)
    lib = _lib.load()
    ws_bytes = bwd_workspace_bytes(nseq, L, Dn, S)
    if ws_bytes == 0 and nseq * L > 0:
        raise NotImplementedError(
            f"hclsm_b200 scan backward: d_state={S}, L={L} outside the supported range")
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=x.device)
    dx = torch.empty_like(x)
    ddt = torch.empty_like(x)
    dB = torch.empty_like(B)
    dC = torch.empty_like(C)
    dA = torch.empty(Dn, S, dtype=torch.float32, device=x.device)
    dD = torch.empty(Dn, dtype=torch.float32, device=x.device) if D is not None else None
    dz = torch.empty_like(x) if z is not None else None
    if states is not None:
        rc = lib.hclsm_ssm_scan_bwd_states(_lib.ptr(x), _lib.ptr(dt), _lib.ptr(A_log), _lib.ptr(B), _lib.ptr(C),
                                           _lib.ptr(D), _lib.ptr(z), _lib.ptr(dy), _lib.ptr(dx), _lib.ptr(ddt),
                                           _lib.ptr(dA), _lib.ptr(dB), _lib.ptr(dC), _lib.ptr(dD), _lib.ptr(dz),
                                           nseq, L, Dn, S, _lib.dtype_code(x.dtype), flags,
                                           _lib.ptr(states), states.numel() * states.element_size(),
                                           _lib.ptr(workspace), workspace.numel(), _lib.stream_ptr(x.device))
        _lib.check(rc, "hclsm_ssm_scan_bwd_states")
        return dx, ddt, dA, dB, dC, dD, dz
    rc = lib.hclsm_ssm_scan_bwd(_lib.ptr(x), _lib.ptr(dt), _lib.ptr(A_log), _lib.ptr(B), _lib.ptr(C),
                                _lib.ptr(D), _lib.ptr(z), _lib.ptr(dy), _lib.ptr(dx), _lib.ptr(ddt),
                                _lib.ptr(dA), _lib.ptr(dB), _lib.ptr(dC), _lib.ptr(dD), _lib.ptr(dz),
                                nseq, L, Dn, S, _lib.dtype_code(x.dtype), flags,
                                _lib.ptr(workspace), workspace.numel(), _lib.stream_ptr(x.device))
    _lib.check(rc, "hclsm_ssm_scan_bwd")
    return dx, ddt, dA, dB, dC, dD, dz


class _SSMScan(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, dt, A_log, B, C, D, z, clamp, dt_softplus):
        _lib.require_cuda(x, dt, A_log, B, C, D, z)
        _check_shapes(x, dt, A_log, B, C, D, z)
        io = _io_dtype(x, dt, B, C, z)
        xs, dts, Bs, Cs, zs = (_prep(t, io) for t in (x, dt, B, C, z))
        As = _prep(A_log, torch.float32)
        Ds = _prep(D, torch.float32)
        # when a gradient will be asked for and the packed path applies, the
        # forward keeps state snapshots so the backward skips its forward sweep
        st = None
        if any(ctx.needs_input_grad[:7]):
            nb = states_bytes(xs.shape[0], xs.shape[1], xs.shape[2], Bs.shape[-1], xs.dtype)
            if nb > 0:
                st = torch.empty(nb, dtype=torch.uint8, device=xs.device)
        y = scan_fwd_raw(xs, dts, As, Bs, Cs, Ds, zs, clamp, states=st, dt_softplus=dt_softplus)
        ctx.save_for_backward(xs, dts, As, Bs, Cs, Ds, zs, st)
        ctx.clamp = clamp
        ctx.dt_softplus = dt_softplus
        ctx.in_dtypes = (x.dtype, dt.dtype, A_log.dtype, B.dtype, C.dtype,
                         None if D is None else D.dtype, None if z is None else z.dtype)
        return y.to(x.dtype)

    @staticmethod
    def backward(ctx, gy):
        xs, dts, As, Bs, Cs, Ds, zs, st = ctx.saved_tensors
        dy = _prep(gy, xs.dtype)
        grads = scan_bwd_raw(xs, dts, As, Bs, Cs, dy, Ds, zs, ctx.clamp, states=st, dt_softplus=ctx.dt_softplus)
        out = []
        for g, dtp in zip(grads, ctx.in_dtypes):
            out.append(None if g is None or dtp is None else g.to(dtp))
        return (*out, None, None)


def ssm_scan(x, dt, A_log, B, C, *, clamp=False, D=None, z=None, dt_softplus=False):
    """Selective scan on sm_100a; differentiable in every tensor argument.
    ``dt_softplus``: dt is the raw projection, softplus(dt) is taken inside the
    kernel (and its gradient is the raw dt's)."""
    return _SSMScan.apply(x, dt, A_log, B, C, D, z, bool(clamp), bool(dt_softplus))


def ssm_scan_fn(x, dt, A_log, B, C, backend: str = "auto", *, clamp=None, D=None, z=None, dt_softplus=False):
    """Drop-in for ``hclsm.kernels.ssm_scan_fn`` (ssm_scan_kernel.py:394).

    ``backend`` accepts the reference's names ("auto", "triton", "parallel",
    "sequential") plus "b200"; every one runs the B200 kernel.  "sequential"
    selects the clamped arithmetic of ``sequential_ssm_scan`` unless ``clamp``
    is given, all others the unclamped arithmetic of the reference's CUDA paths.
    """
    if backend not in ("auto", "b200", "triton", "parallel", "sequential"):
        raise ValueError(f"unknown backend {backend!r}")
    if clamp is None:
        clamp = backend == "sequential"
    return ssm_scan(x, dt, A_log, B, C, clamp=clamp, D=D, z=z, dt_softplus=dt_softplus)
