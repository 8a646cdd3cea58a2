"""The library's entry points as PyTorch dispatcher operators (``torch.ops.hclsm_b200.*``).

Registered with ``torch.library.custom_op``: each op validates its inputs,
allocates outputs on the current device and stream, calls the C ABI, and turns
a status code into ``ValueError`` / ``NotImplementedError`` / ``RuntimeError``.
CUDA tensors only (no CPU kernel is registered).  Every op has a fake
(shape-only) implementation, so ``torch.compile`` can trace through them, and
``ssm_scan_fwd`` has a registered autograd formula:

* ``ssm_scan_fwd(x, dt, A_log, B, C, D, z, flags, keep_states) -> (y, states)``
  (hclsm/kernels/ssm_scan_kernel.py:394 ``ssm_scan_fn``); ``flags`` as the C
  ABI's (1 clamped arithmetic, 2 softplus of a raw dt); ``states`` holds the
  forward's snapshots for the backward when ``keep_states`` and the path
  applies, else it is empty;
* ``ssm_scan_bwd(x, dt, A_log, B, C, dy, D, z, flags, states)
  -> [dx, ddt, dA_log, dB, dC, dD, dz]`` (empty tensors for absent D / z);
* ``slot_attn_core(Q, K, V, scale, clamp, eps, return_attn) -> (out, attn)``
  (slot_attention_kernel.py:265-291, forward);
* ``event_compact(mask) -> (idx, pos, counts, meta)``,
  ``event_gather(states, idx, counts, meta, n_frames, pad_k)``,
  ``event_scatter(states, upd, pos, counts, pad_k)``,
  ``event_mha(qkv, key_pad, frames, T, H, HD, scale)``
  (sparse_event_attn.py:93-188, level1_event.py:33-54).

Scan inputs must already share one dtype (fp32 or bf16: x, dt, B, C, z) with
A_log and D in fp32, and be contiguous; ``hclsm_b200.kernels.ssm_scan`` does
that preparation for Python callers.
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
from torch import Tensor

from . import _lib
from .kernels import sparse_event_attn as _ev
from .kernels import ssm_scan_kernel as _scan
from .kernels.slot_attention_kernel import slot_attention_core as _slot_core

__all__ = ["ssm_scan_fwd", "ssm_scan_bwd", "slot_attn_core", "event_compact", "event_gather", "event_scatter",
           "event_mha"]

_NS = "hclsm_b200"


def _check_scan(x, dt, A_log, B, C, D, z):
    _lib.require_cuda(x, dt, A_log, B, C, D, z)
    io = x.dtype
    if io not in (torch.float32, torch.bfloat16):
        raise ValueError("ssm_scan: x must be float32 or bfloat16")
    for name, t in (("dt", dt), ("B", B), ("C", C), ("z", z)):
        if t is not None and t.dtype != io:
            raise ValueError(f"ssm_scan: {name} must have x's dtype ({io})")
    if A_log.dtype != torch.float32 or (D is not None and D.dtype != torch.float32):
        raise ValueError("ssm_scan: A_log and D must be float32")
    for t in (x, dt, A_log, B, C, D, z):
        if t is not None and not t.is_contiguous():
            raise ValueError("ssm_scan: inputs must be contiguous")
    _scan._check_shapes(x, dt, A_log, B, C, D, z)


@torch.library.custom_op(f"{_NS}::ssm_scan_fwd", mutates_args=())
def ssm_scan_fwd(x: Tensor, dt: Tensor, A_log: Tensor, B: Tensor, C: Tensor, D: Optional[Tensor],
                 z: Optional[Tensor], flags: int, keep_states: bool) -> Tuple[Tensor, Tensor]:
    _check_scan(x, dt, A_log, B, C, D, z)
    nseq, L, Dn = x.shape
    nb = _scan.states_bytes(nseq, L, Dn, B.shape[-1], x.dtype) if keep_states else 0
    states = torch.empty(nb, dtype=torch.uint8, device=x.device)
    y = _scan.scan_fwd_raw(x, dt, A_log, B, C, D, z, clamp=bool(flags & 1), dt_softplus=bool(flags & 2),
                           states=states if nb > 0 else None)
    return y, states


@ssm_scan_fwd.register_fake
def _(x, dt, A_log, B, C, D, z, flags, keep_states):
    nseq, L, Dn = x.shape
    nb = _scan.states_bytes(nseq, L, Dn, B.shape[-1], x.dtype) if keep_states else 0  # a host-side query
    return torch.empty_like(x), x.new_empty(nb, dtype=torch.uint8)


@torch.library.custom_op(f"{_NS}::ssm_scan_bwd", mutates_args=())
def ssm_scan_bwd(x: Tensor, dt: Tensor, A_log: Tensor, B: Tensor, C: Tensor, dy: Tensor, D: Optional[Tensor],
                 z: Optional[Tensor], flags: int, states: Tensor) -> List[Tensor]:
    _check_scan(x, dt, A_log, B, C, D, z)
    dy = dy.to(x.dtype).contiguous()
    g = _scan.scan_bwd_raw(x, dt, A_log, B, C, dy, D, z, clamp=bool(flags & 1), dt_softplus=bool(flags & 2),
                           states=states if states.numel() > 0 else None)
    # absent gradients as distinct empty tensors (outputs may not alias)
    return [g[0], g[1], g[2], g[3], g[4], g[5] if g[5] is not None else x.new_empty(0),
            g[6] if g[6] is not None else x.new_empty(0)]


@ssm_scan_bwd.register_fake
def _(x, dt, A_log, B, C, dy, D, z, flags, states):
    return [torch.empty_like(x), torch.empty_like(x), torch.empty_like(A_log), torch.empty_like(B),
            torch.empty_like(C), torch.empty_like(D) if D is not None else x.new_empty(0),
            torch.empty_like(z) if z is not None else x.new_empty(0)]


def _scan_setup(ctx, inputs, output):
    x, dt, A_log, B, C, D, z, flags, keep_states = inputs
    ctx.save_for_backward(x, dt, A_log, B, C, D, z, output[1])
    ctx.flags = flags


def _scan_backward(ctx, gy, gstates):
    x, dt, A_log, B, C, D, z, states = ctx.saved_tensors
    g = ssm_scan_bwd(x, dt, A_log, B, C, gy, D, z, ctx.flags, states)
    return (g[0], g[1], g[2], g[3], g[4], g[5] if D is not None else None, g[6] if z is not None else None,
            None, None)


torch.library.register_autograd(f"{_NS}::ssm_scan_fwd", _scan_backward, setup_context=_scan_setup)


@torch.library.custom_op(f"{_NS}::slot_attn_core", mutates_args=())
def slot_attn_core(Q: Tensor, K: Tensor, V: Tensor, scale: float, clamp: float, eps: float,
                   return_attn: bool) -> Tuple[Tensor, Tensor]:
    out, attn = _slot_core(Q, K, V, scale, clamp=clamp, eps=eps, return_attn=return_attn)
    return out, attn if attn is not None else out.new_empty(0)


@slot_attn_core.register_fake
def _(Q, K, V, scale, clamp, eps, return_attn):
    dt = torch.bfloat16 if {Q.dtype, K.dtype, V.dtype} == {torch.bfloat16} else torch.float32
    F, N, D = Q.shape
    out = Q.new_empty((F, N, D), dtype=dt)
    attn = Q.new_empty((F, N, K.shape[1]), dtype=torch.float32 if dt == torch.float32 else dt) if return_attn \
        else Q.new_empty(0, dtype=dt)
    return out, attn


@torch.library.custom_op(f"{_NS}::event_compact", mutates_args=())
def event_compact(mask: Tensor) -> Tuple[Tensor, Tensor, Tensor, Tensor]:
    _lib.require_cuda(mask)
    idx, pos, counts, meta = _ev.event_compact(mask)
    return idx, pos, counts, meta


@event_compact.register_fake
def _(mask):
    B, T = mask.shape
    i32 = torch.int32
    return (mask.new_empty(max(B * T, 1), dtype=i32), mask.new_empty(max(B * T, 1), dtype=i32),
            mask.new_empty(max(B, 1), dtype=i32), mask.new_empty(2, dtype=i32))


@torch.library.custom_op(f"{_NS}::event_gather", mutates_args=())
def event_gather(states: Tensor, idx: Tensor, counts: Tensor, meta: Tensor, n_frames: int, pad_k: int) -> Tensor:
    _lib.require_cuda(states, idx, counts, meta)
    return _ev.event_gather(states.contiguous(), idx, counts, meta, n_frames, pad_k=pad_k)


@event_gather.register_fake
def _(states, idx, counts, meta, n_frames, pad_k):
    B, T, N, D = states.shape
    return states.new_empty((n_frames, N, D))


@torch.library.custom_op(f"{_NS}::event_scatter", mutates_args=())
def event_scatter(states: Tensor, upd: Tensor, pos: Tensor, counts: Tensor, pad_k: int) -> Tensor:
    _lib.require_cuda(states, upd, pos, counts)
    return _ev.event_scatter(states.contiguous(), upd.to(states.dtype), pos, counts, pad_k=pad_k)


@event_scatter.register_fake
def _(states, upd, pos, counts, pad_k):
    return torch.empty_like(states)


@torch.library.custom_op(f"{_NS}::event_mha", mutates_args=())
def event_mha(qkv: Tensor, key_pad: Optional[Tensor], frames: int, T: int, H: int, HD: int, scale: float) -> Tensor:
    _lib.require_cuda(qkv, key_pad)
    if qkv.dtype not in (torch.float32, torch.bfloat16) or not qkv.is_contiguous():
        raise ValueError("event_mha: qkv must be contiguous float32 or bfloat16")
    kp = None if key_pad is None else key_pad.to(torch.uint8).contiguous()
    out = torch.empty(frames * T, H * HD, dtype=qkv.dtype, device=qkv.device)
    rc = _lib.load().hclsm_event_mha(_lib.ptr(qkv), _lib.ptr(kp), _lib.ptr(out), frames, T, H, HD, float(scale),
                                     _lib.dtype_code(qkv.dtype), _lib.stream_ptr(qkv.device))
    _lib.check(rc, "hclsm_event_mha")
    return out


@event_mha.register_fake
def _(qkv, key_pad, frames, T, H, HD, scale):
    return qkv.new_empty((frames * T, H * HD))
