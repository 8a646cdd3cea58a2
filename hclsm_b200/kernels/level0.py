"""Level0SSM around its SSM blocks (hclsm/dynamics/level0_ssm.py:159-220): the
global track's masked mean over objects and the nan_to_num / clamp / mask
epilogue, each one sm_100a kernel pass, differentiable in the states."""
from __future__ import annotations

import torch

from .. import _lib

__all__ = ["masked_mean_pool", "level0_epilogue", "level0_forward"]


def _c(t):
    return t if t.is_contiguous() else t.contiguous()


def _mask_f32(mask, B, N):
    if mask is None:
        return None
    m = _c(mask.detach().to(torch.float32))
    if m.shape != (B, N):
        raise ValueError(f"obj_mask must be ({B}, {N})")
    return m


class _Pool(torch.autograd.Function):
    @staticmethod
    def forward(ctx, obj, mask):
        B, N, T, D = obj.shape
        m = _mask_f32(mask, B, N)
        odt = torch.promote_types(obj.dtype, mask.dtype) if mask is not None else obj.dtype
        x = _c(obj)
        out = torch.empty(B, T, D, dtype=odt, device=obj.device)
        rc = _lib.load().hclsm_l0_pool(_lib.ptr(x), _lib.dtype_code(x.dtype), _lib.ptr(m), _lib.ptr(out),
                                       _lib.dtype_code(odt), B, N, T * D, _lib.stream_ptr(obj.device))
        _lib.check(rc, "hclsm_l0_pool")
        w = (m / m.sum(1, keepdim=True).clamp(min=1.0)) if m is not None else None
        ctx.save_for_backward(w)
        ctx.N, ctx.in_dtype = N, obj.dtype
        return out

    @staticmethod
    def backward(ctx, g):
        (w,) = ctx.saved_tensors
        if w is None:
            gx = (g / ctx.N).unsqueeze(1).expand(-1, ctx.N, -1, -1)
        else:
            gx = g.unsqueeze(1) * w[:, :, None, None]
        return gx.to(ctx.in_dtype), None


class _Epilogue(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, mask):
        B, N, T, D = x.shape
        m = _mask_f32(mask, B, N)
        odt = torch.promote_types(x.dtype, mask.dtype) if mask is not None else x.dtype
        xc = _c(x)
        out = torch.empty(B, N, T, D, dtype=odt, device=x.device)
        rc = _lib.load().hclsm_l0_epilogue(_lib.ptr(xc), _lib.dtype_code(xc.dtype), _lib.ptr(m), _lib.ptr(out),
                                           _lib.dtype_code(odt), B, N, T * D, _lib.stream_ptr(x.device))
        _lib.check(rc, "hclsm_l0_epilogue")
        ctx.save_for_backward(xc, m)
        return out

    @staticmethod
    def backward(ctx, g):
        x, m = ctx.saved_tensors
        B, N, T, D = x.shape
        gc = _c(g)
        gx = torch.empty_like(x)
        rc = _lib.load().hclsm_l0_epilogue_bwd(_lib.ptr(x), _lib.dtype_code(x.dtype), _lib.ptr(m), _lib.ptr(gc),
                                               _lib.dtype_code(gc.dtype), _lib.ptr(gx), B, N, T * D,
                                               _lib.stream_ptr(x.device))
        _lib.check(rc, "hclsm_l0_epilogue_bwd")
        return gx, None


def masked_mean_pool(obj_states, obj_mask=None):
    """(B, N, T, D) -> (B, T, D): sum_n mask obj / max(sum_n mask, 1), or the
    mean over objects without a mask (level0_ssm.py:175-180).  A mask that
    needs its own gradient takes the reference's formula."""
    _lib.require_cuda(obj_states, obj_mask)
    if obj_mask is not None and obj_mask.requires_grad and torch.is_grad_enabled():
        n_alive = obj_mask.sum(dim=1, keepdim=True).clamp(min=1.0)
        return (obj_states * obj_mask[:, :, None, None]).sum(dim=1) / n_alive[:, :, None]
    return _Pool.apply(obj_states, obj_mask)


def level0_epilogue(x, obj_mask=None):
    """clamp(nan_to_num(x, 0, 100, -100), -100, 100) * mask in one pass
    (level0_ssm.py:210-218); x (B, N, T, D)."""
    _lib.require_cuda(x, obj_mask)
    if obj_mask is not None and obj_mask.requires_grad and torch.is_grad_enabled():
        y = torch.clamp(torch.nan_to_num(x, nan=0.0, posinf=100.0, neginf=-100.0), min=-100.0, max=100.0)
        return y * obj_mask[:, :, None, None]
    return _Epilogue.apply(x, obj_mask)


def level0_forward(mod, obj_states, obj_mask=None):
    """Level0SSM.forward (level0_ssm.py:159-220) with the pooling and the
    epilogue as kernels; the blocks are the module's own (patched by install()
    to the fused scan path when they are SimplifiedSSMBlocks)."""
    B, N, T, D = obj_states.shape
    global_out = masked_mean_pool(obj_states, obj_mask)
    for block in mod.global_blocks:
        if mod.use_gradient_checkpointing and mod.training:
            global_out = torch.utils.checkpoint.checkpoint(block, global_out, use_reentrant=False)
        else:
            global_out = block(global_out)
    global_cond = mod.condition_proj(global_out)
    x = (obj_states + global_cond.unsqueeze(1)).reshape(B * N, T, D)
    for block in mod.object_blocks:
        if mod.use_gradient_checkpointing and mod.training:
            x = torch.utils.checkpoint.checkpoint(block, x, use_reentrant=False)
        else:
            x = block(x)
    return level0_epilogue(x.reshape(B, N, T, D), obj_mask)
