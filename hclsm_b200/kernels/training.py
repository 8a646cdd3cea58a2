"""Training mode of the slot-attention iteration and of the Level-1 event
transformer: autograd Functions whose forward and backward run this library's
kernels (the weight products and their gradients are library GEMMs).

* ``slot_iteration_train`` — DynamicSlotAttention._iteration_step
  (hclsm/objects/dynamic_slots.py:98-131) differentiable in the slots, k, v and
  every parameter it uses.
* ``level1_train`` — Level1EventDynamics.forward's stack
  (hclsm/dynamics/level1_event.py:85-133: proj_in, EventTransformerBlocks,
  norm, proj_out) differentiable in the frames and every parameter.
* ``event_gather_train`` / ``event_scatter_train`` — HierarchyManager's
  gather_events / scatter_events (hclsm/dynamics/hierarchy_manager.py:42-118)
  with their gradients: the gather's is a scatter into zeros, the scatter's a
  gather (updates) and the incoming gradient with the event frames zeroed
  (base states).

Arithmetic follows the module's: ``dtype`` bfloat16 runs the weight products
on bf16 operands with fp32 accumulation (the reference under bf16 autocast),
float32 runs everything in fp32 (the reference without autocast).
"""
from __future__ import annotations

import torch

from .. import _lib
from .slot_attention_kernel import _c, gru_cell, layernorm, residual_clamp, slot_attention_core

__all__ = ["colsum", "layernorm_bwd", "gru_cell_bwd", "slot_softmax_bwd", "residual_clamp_bwd", "relu_bwd",
           "swiglu_bwd", "event_mha_bwd", "slot_iteration_train", "level1_train", "event_gather_train",
           "event_scatter_train", "layer_norm"]

F32 = torch.float32


# ---- wrappers of the backward kernels ----------------------------------------------------
def colsum(a):
    a = _c(a.float())
    C = a.shape[-1]
    rows = a.numel() // C
    out = torch.empty(C, dtype=F32, device=a.device)
    lib = _lib.load()
    ws = torch.empty(max(lib.hclsm_colsum_workspace_size(C), 1), dtype=torch.uint8, device=a.device)
    _lib.check(lib.hclsm_colsum(_lib.ptr(a), _lib.ptr(out), rows, C, _lib.ptr(ws), ws.numel(),
                                _lib.stream_ptr(a.device)), "hclsm_colsum")
    return out


def layernorm_bwd(x, w, dy, eps=1e-5, dx=None, want_affine=True):
    """(dx, dw, db) of nn.LayerNorm; with ``dx`` given the input gradient is
    added to it in place."""
    x = _c(x.float())
    dy = _c(dy.float())
    D = x.shape[-1]
    rows = x.numel() // D
    acc = dx is not None
    if dx is None:
        dx = torch.empty(x.shape, dtype=F32, device=x.device)
    dw = torch.empty(D, dtype=F32, device=x.device) if (want_affine and w is not None) else None
    db = torch.empty(D, dtype=F32, device=x.device) if want_affine else None
    lib = _lib.load()
    nws = lib.hclsm_layernorm_bwd_workspace_size(rows, D)
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=x.device)
    _lib.check(lib.hclsm_layernorm_bwd(_lib.ptr(x), _lib.ptr(w), _lib.ptr(dy), _lib.ptr(dx), _lib.ptr(dw),
                                       _lib.ptr(db), rows, D, float(eps), int(acc), _lib.ptr(ws), ws.numel(),
                                       _lib.stream_ptr(x.device)), "hclsm_layernorm_bwd")
    return dx, dw, db


def gru_cell_bwd(gi, gh, b_ih, b_hh, h, dh_new):
    H = h.shape[-1]
    rows = h.numel() // H
    d_gi = torch.empty(rows, 3 * H, dtype=F32, device=h.device)
    d_gh = torch.empty_like(d_gi)
    dh = torch.empty(rows, H, dtype=F32, device=h.device)
    dh_new = _c(dh_new.float())
    _lib.check(_lib.load().hclsm_gru_cell_bwd(_lib.ptr(gi), _lib.ptr(gh), _lib.ptr(b_ih), _lib.ptr(b_hh),
                                              _lib.ptr(h), _lib.ptr(dh_new), _lib.ptr(d_gi), _lib.ptr(d_gh),
                                              _lib.ptr(dh), rows, H, _lib.stream_ptr(h.device)),
               "hclsm_gru_cell_bwd")
    return d_gi, d_gh, dh


def slot_softmax_bwd(dots, d_attn, scale, clamp, eps, dtype):
    """(attn, d_dots) in ``dtype`` from dots = q k^T (F, N, M) fp32 and d_attn."""
    F_, N, M = dots.shape
    attn = torch.empty(F_, N, M, dtype=dtype, device=dots.device)
    d_dots = torch.empty_like(attn)
    _lib.check(_lib.load().hclsm_slot_softmax_bwd(_lib.ptr(_c(dots)), _lib.ptr(_c(d_attn.float())), _lib.ptr(attn),
                                                  _lib.ptr(d_dots), F_, N, M, float(scale), float(clamp), float(eps),
                                                  _lib.dtype_code(dtype), _lib.stream_ptr(dots.device)),
               "hclsm_slot_softmax_bwd")
    return attn, d_dots


def residual_clamp_bwd(h, m, b, dout, clamp):
    C = h.shape[-1]
    dpre = torch.empty(h.shape, dtype=F32, device=h.device)
    _lib.check(_lib.load().hclsm_residual_clamp_bwd(_lib.ptr(h), _lib.ptr(m), _lib.ptr(b), _lib.ptr(_c(dout.float())),
                                                    _lib.ptr(dpre), h.numel() // C, C, float(clamp),
                                                    _lib.stream_ptr(h.device)), "hclsm_residual_clamp_bwd")
    return dpre


def relu_bwd(y, dy, out_dtype=F32):
    dx = torch.empty(y.shape, dtype=out_dtype, device=y.device)
    _lib.check(_lib.load().hclsm_relu_bwd(_lib.ptr(y), _lib.dtype_code(y.dtype), _lib.ptr(_c(dy.float())),
                                          _lib.ptr(dx), _lib.dtype_code(out_dtype), y.numel(),
                                          _lib.stream_ptr(y.device)), "hclsm_relu_bwd")
    return dx


def swiglu_bwd(u, ds, out_dtype=F32):
    rows, C2 = u.shape
    du = torch.empty(rows, C2, dtype=out_dtype, device=u.device)
    _lib.check(_lib.load().hclsm_swiglu_bwd(_lib.ptr(u), _lib.ptr(_c(ds.float())), _lib.ptr(du), rows, C2 // 2,
                                            _lib.dtype_code(out_dtype), _lib.stream_ptr(u.device)),
               "hclsm_swiglu_bwd")
    return du


def event_mha_bwd(qkv, key_pad, dout, frames, T, H, HD, scale):
    dqkv = torch.empty(qkv.shape, dtype=qkv.dtype, device=qkv.device)
    _lib.check(_lib.load().hclsm_event_mha_bwd(_lib.ptr(qkv), _lib.ptr(key_pad), _lib.ptr(_c(dout.float())),
                                               _lib.ptr(dqkv), frames, T, H, HD, float(scale),
                                               _lib.dtype_code(qkv.dtype), _lib.stream_ptr(qkv.device)),
               "hclsm_event_mha_bwd")
    return dqkv


def _lp(w, dt):
    """w in the arithmetic dtype ``dt``.  For bf16 the cast of a parameter is
    kept on the parameter and reused while its version counter is unchanged
    (the three refinement steps and their backward passes of one training
    step share one cast; an optimizer's in-place update bumps the version).
    As for the inference caches, in-place changes that bypass the version
    counter (``w.data`` edits) are not seen."""
    if w.dtype == dt:
        return w
    if dt == F32:
        return w.float()
    ent = getattr(w, "_hclsm_lp", None)
    if ent is not None and ent[0] == w._version and ent[1] == dt and ent[2] == w.data_ptr():
        return ent[3]
    cast = w.detach().to(dt)
    try:
        w._hclsm_lp = (w._version, dt, w.data_ptr(), cast)
    except (AttributeError, RuntimeError):
        pass
    return cast


def _mm(a, b, dt):
    """a @ b with fp32 output: fp32 operands for dt = fp32, bf16 operands
    (fp32 accumulation) for dt = bf16."""
    if dt == F32:
        return torch.mm(a.float(), b.float())
    return torch.mm(a.to(dt), b.to(dt), out_dtype=F32)


def _wgrad(g, x, dt):
    """Weight gradient g^T x (out, in) in fp32."""
    return _mm(g.t(), x, dt)


# ---- nn.LayerNorm ----------------------------------------------------------------------
class _LayerNorm(torch.autograd.Function):
    """nn.LayerNorm over the last dimension on this library's kernels: the
    forward row kernel (fp32 statistics) and the backward row kernel plus
    the deterministic two-stage column sums for the affine gradients."""

    @staticmethod
    def forward(ctx, x, w, b, eps, out_dtype):
        w32 = w.float().contiguous() if w is not None else None
        b32 = b.float().contiguous() if b is not None else None
        xs = _c(x)
        ctx.save_for_backward(xs, w32)
        ctx.eps, ctx.dtypes = eps, (x.dtype, None if w is None else w.dtype, None if b is None else b.dtype)
        return layernorm(xs, w32, b32, eps, out_dtype)

    @staticmethod
    def backward(ctx, dy):
        x, w32 = ctx.saved_tensors
        xd, wd, bd = ctx.dtypes
        affine = ctx.needs_input_grad[1] or ctx.needs_input_grad[2]
        dx, dw, db = layernorm_bwd(x, w32, dy, ctx.eps, want_affine=affine)
        return (dx.to(xd) if ctx.needs_input_grad[0] else None,
                dw.to(wd) if (dw is not None and ctx.needs_input_grad[1]) else None,
                db.to(bd) if (db is not None and ctx.needs_input_grad[2]) else None, None, None)


def layer_norm(mod, x):
    """``mod(x)`` for an nn.LayerNorm over the last dimension, on this
    library's kernels (forward and backward).  Under CUDA autocast the output
    is fp32, as torch runs layer_norm in fp32 there; otherwise x's dtype."""
    _lib.require_cuda(x)
    if tuple(mod.normalized_shape) != (x.shape[-1],):
        raise ValueError("hclsm_b200.layer_norm normalises the last dimension only")
    out = F32 if torch.is_autocast_enabled("cuda") else x.dtype
    with torch.autocast("cuda", enabled=False):
        return _LayerNorm.apply(x, mod.weight, mod.bias, float(mod.eps), out)


# ---- slot-attention iteration ------------------------------------------------------------
class _SlotIteration(torch.autograd.Function):
    @staticmethod
    def forward(ctx, slots, k, v, wq, w_ih, w_hh, b_ih, b_hh, lna_w, lna_b, lnm_w, lnm_b, w1, b1, w2, b2, dt, scale):
        F_, N, D = slots.shape
        R = F_ * N
        s2 = _c(slots.reshape(R, D).float())
        kd, vd = _c(k.to(dt)), _c(v.to(dt))
        b_ih32, b_hh32, b2_32 = b_ih.float().contiguous(), b_hh.float().contiguous(), b2.float().contiguous()
        sn = layernorm(s2, lna_w.float().contiguous(), lna_b.float().contiguous(), out_dtype=dt)
        q = torch.mm(sn, _lp(wq, dt).t()).reshape(F_, N, D)
        upd, _ = slot_attention_core(q, kd, vd, scale, clamp=30.0, eps=0.0, return_attn=False)
        s_dt = s2 if dt == F32 else s2.to(dt)
        gi = _c(_mm(upd.reshape(R, D), _lp(w_ih, dt).t(), dt))
        gh = _c(_mm(s_dt, _lp(w_hh, dt).t(), dt))
        h = gru_cell(gi, gh, b_ih32, b_hh32, s2)
        mln = layernorm(h, lnm_w.float().contiguous(), lnm_b.float().contiguous(), out_dtype=dt)
        m1 = torch._addmm_activation(b1.to(dt), mln, _lp(w1, dt).t())
        m2 = _c(_mm(m1, _lp(w2, dt).t(), dt))
        out = residual_clamp(h, m2, b2_32, 50.0)
        ctx.save_for_backward(s2, s_dt, kd, vd, sn, q, upd, gi, gh, h, mln, m1, m2, wq, w_ih, w_hh, b_ih32, b_hh32,
                              lna_w, lnm_w, w1, w2, b2_32)
        ctx.dt, ctx.scale, ctx.shape = dt, scale, (F_, N, D)
        ctx.in_dtypes = (slots.dtype, k.dtype, v.dtype)
        return out.reshape(F_, N, D)

    @staticmethod
    def backward(ctx, dout):
        (s2, s_dt, kd, vd, sn, q, upd, gi, gh, h, mln, m1, m2, wq, w_ih, w_hh, b_ih32, b_hh32, lna_w, lnm_w, w1, w2,
         b2_32) = ctx.saved_tensors
        dt, scale = ctx.dt, ctx.scale
        F_, N, D = ctx.shape
        R = F_ * N
        # clamp(h + mlp + b2): residual and the MLP's output bias
        dpre = residual_clamp_bwd(h, m2, b2_32, dout.reshape(R, D), 50.0)
        # each fp32 gradient is cast to the product dtype once, for both of
        # its products (weight gradient and input gradient)
        db2 = colsum(dpre)
        dpre_l = dpre.to(dt)
        dW2 = _wgrad(dpre_l, m1, dt)
        dm1 = relu_bwd(m1, _mm(dpre_l, _lp(w2, dt), dt), F32)
        db1 = colsum(dm1)
        dm1_l = dm1.to(dt)
        dW1 = _wgrad(dm1_l, mln, dt)
        dmln = _mm(dm1_l, _lp(w1, dt), dt)
        dh, dlnm_w, dlnm_b = layernorm_bwd(h, lnm_w.float().contiguous(), dmln, dx=dpre.clone())
        # GRUCell
        d_gi, d_gh, ds = gru_cell_bwd(gi, gh, b_ih32, b_hh32, s2, dh)
        db_ih, db_hh = colsum(d_gi), colsum(d_gh)
        d_gi, d_gh = d_gi.to(dt), d_gh.to(dt)
        dW_ih = _wgrad(d_gi, upd.reshape(R, D), dt)
        dW_hh = _wgrad(d_gh, s_dt, dt)
        d_upd = _mm(d_gi, _lp(w_ih, dt), dt).reshape(F_, N, D)
        ds += _mm(d_gh, _lp(w_hh, dt), dt)
        # attention core: softmax over slots of clamp(scale q k^T), weighted sum of v
        if dt == F32:
            d_attn = torch.bmm(d_upd, vd.transpose(1, 2))
            dots = torch.bmm(q, kd.transpose(1, 2))
        else:
            du = d_upd.to(dt)
            d_attn = torch.bmm(du, vd.transpose(1, 2), out_dtype=F32)
            dots = torch.bmm(q, kd.transpose(1, 2), out_dtype=F32)
        attn, d_dots = slot_softmax_bwd(dots, d_attn, scale, 30.0, 0.0, dt)
        if dt == F32:
            dv = torch.bmm(attn.transpose(1, 2), d_upd)
            dq = torch.bmm(d_dots, kd)
            dk = torch.bmm(d_dots.transpose(1, 2), q)
        else:
            dv = torch.bmm(attn.transpose(1, 2), du, out_dtype=F32)
            dq = torch.bmm(d_dots, kd, out_dtype=F32)
            dk = torch.bmm(d_dots.transpose(1, 2), q, out_dtype=F32)
        dq = dq.reshape(R, D).to(dt)
        dWq = _wgrad(dq, sn, dt)
        dsn = _mm(dq, _lp(wq, dt), dt)
        ds, dlna_w, dlna_b = layernorm_bwd(s2, lna_w.float().contiguous(), dsn, dx=ds)
        sdt, kdt, vdt = ctx.in_dtypes
        return (ds.reshape(F_, N, D).to(sdt), dk.to(kdt), dv.to(vdt), dWq.to(wq.dtype), dW_ih.to(w_ih.dtype),
                dW_hh.to(w_hh.dtype), db_ih, db_hh, dlna_w, dlna_b, dlnm_w, dlnm_b, dW1.to(w1.dtype), db1,
                dW2.to(w2.dtype), db2, None, None)


def slot_iteration_train(mod, slots, k, v, dtype):
    """One differentiable _iteration_step of DynamicSlotAttention ``mod``
    (parameter names of dynamic_slots.py:44-83).  Returns fp32 slots."""
    _lib.require_cuda(slots, k, v)
    return _SlotIteration.apply(slots, k, v, mod.project_q.weight, mod.gru.weight_ih, mod.gru.weight_hh,
                                mod.gru.bias_ih, mod.gru.bias_hh, mod.norm_pre_attn.weight, mod.norm_pre_attn.bias,
                                mod.norm_slots.weight, mod.norm_slots.bias, mod.mlp[0].weight, mod.mlp[0].bias,
                                mod.mlp[2].weight, mod.mlp[2].bias, dtype, float(mod.scale))


# ---- Level-1 event transformer -----------------------------------------------------------
_PER_LAYER = 9  # norm1.w, norm1.b, attn.in_proj_weight, attn.out_proj.weight, norm2.w, norm2.b, w1, w3, w2


class _Level1(torch.autograd.Function):
    @staticmethod
    def forward(ctx, frames, key_pad, n_heads, dt, w_in, w_out, nw, nb, *layer_params):
        n, N, Ds = frames.shape
        R = n * N
        E = w_in.shape[0]
        H = n_heads
        hd = E // H
        lib = _lib.load()
        fr = _c(frames.reshape(R, Ds))
        x = _c(_mm(fr, _lp(w_in, dt).t(), dt))
        saved = [fr]
        nl = len(layer_params) // _PER_LAYER
        for i in range(nl):
            n1w, n1b, wqkv, wo, n2w, n2b, w1, w3, w2 = layer_params[i * _PER_LAYER:(i + 1) * _PER_LAYER]
            h1 = layernorm(x, n1w.float().contiguous(), n1b.float().contiguous(), out_dtype=dt)
            qkv = _c(torch.mm(h1, _lp(wqkv, dt).t()))
            a = torch.empty(R, E, dtype=dt, device=x.device)
            _lib.check(lib.hclsm_event_mha(_lib.ptr(qkv), _lib.ptr(key_pad), _lib.ptr(a), n, N, H, hd,
                                           float(hd ** -0.5), _lib.dtype_code(dt), _lib.stream_ptr(x.device)),
                       "hclsm_event_mha")
            x1 = residual_clamp(x, _c(_mm(a, _lp(wo, dt).t(), dt)), None, 0.0)
            h2 = layernorm(x1, n2w.float().contiguous(), n2b.float().contiguous(), out_dtype=dt)
            u = _c(_mm(h2, torch.cat([_lp(w1, dt), _lp(w3, dt)], 0).t(), dt))
            F_ = u.shape[1] // 2
            s = torch.empty(R, F_, dtype=dt, device=x.device)
            _lib.check(lib.hclsm_swiglu(_lib.ptr(u), _lib.dtype_code(u.dtype), _lib.ptr(s), R, F_, _lib.dtype_code(dt),
                                        _lib.stream_ptr(x.device)), "hclsm_swiglu")
            saved += [x, h1, qkv, a, x1, h2, u, s]
            x = residual_clamp(x1, _c(_mm(s, _lp(w2, dt).t(), dt)), None, 0.0)
        hf = layernorm(x, nw.float().contiguous(), nb.float().contiguous(), out_dtype=dt)
        y = _mm(hf, _lp(w_out, dt).t(), dt)
        saved += [x, hf]
        ctx.save_for_backward(*saved, w_in, w_out, nw, *layer_params)
        ctx.meta = (n, N, Ds, E, H, hd, nl, dt, frames.dtype)
        ctx.key_pad = key_pad
        return y.reshape(n, N, -1).to(frames.dtype)

    @staticmethod
    def backward(ctx, dy):
        n, N, Ds, E, H, hd, nl, dt, fdt = ctx.meta
        R = n * N
        sv = ctx.saved_tensors
        fr = sv[0]
        per = sv[1:1 + 8 * nl]
        xL, hf = sv[1 + 8 * nl], sv[2 + 8 * nl]
        w_in, w_out, nw = sv[3 + 8 * nl:6 + 8 * nl]
        lp = sv[6 + 8 * nl:]
        dy = _c(dy.reshape(R, -1).float())
        g_out = _wgrad(dy, hf, dt)
        dx, g_nw, g_nb = layernorm_bwd(xL, nw.float().contiguous(), _mm(dy, _lp(w_out, dt), dt))
        grads = [None] * len(lp)
        for i in reversed(range(nl)):
            x, h1, qkv, a, x1, h2, u, s = per[8 * i:8 * i + 8]
            n1w, n1b, wqkv, wo, n2w, n2b, w1, w3, w2 = lp[i * _PER_LAYER:(i + 1) * _PER_LAYER]
            # x2 = x1 + w2(swiglu(w13 LN2(x1)))
            g_w2 = _wgrad(dx, s, dt)
            du = swiglu_bwd(u, _mm(dx, _lp(w2, dt), dt), F32)
            g_w13 = _wgrad(du, h2, dt)
            Fh = du.shape[1] // 2
            dx1, g_n2w, g_n2b = layernorm_bwd(x1, n2w.float().contiguous(), _mm(du, torch.cat([_lp(w1, dt), _lp(w3, dt)], 0), dt),
                                              dx=dx.clone())
            # x1 = x + out_proj(mha(in_proj LN1(x)))
            g_wo = _wgrad(dx1, a, dt)
            dqkv = event_mha_bwd(qkv, ctx.key_pad, _mm(dx1, _lp(wo, dt), dt), n, N, H, hd, hd ** -0.5)
            g_wqkv = _wgrad(dqkv, h1, dt)
            dx, g_n1w, g_n1b = layernorm_bwd(x, n1w.float().contiguous(), _mm(dqkv, _lp(wqkv, dt), dt), dx=dx1)
            grads[i * _PER_LAYER:(i + 1) * _PER_LAYER] = [g_n1w, g_n1b, g_wqkv.to(wqkv.dtype), g_wo.to(wo.dtype),
                                                          g_n2w, g_n2b, g_w13[:Fh].to(w1.dtype),
                                                          g_w13[Fh:].to(w3.dtype), g_w2.to(w2.dtype)]
        g_in = _wgrad(dx, fr, dt)
        dfr = _mm(dx, _lp(w_in, dt), dt).reshape(n, N, Ds).to(fdt)
        return (dfr, None, None, None, g_in.to(w_in.dtype), g_out.to(w_out.dtype), g_nw, g_nb, *grads)


def level1_params(mod):
    """(w_in, w_out, norm.w, norm.b, per-layer params) of a Level1EventDynamics."""
    lp = []
    for blk in mod.blocks:
        lp += [blk.norm1.weight, blk.norm1.bias, blk.attn.in_proj_weight, blk.attn.out_proj.weight,
               blk.norm2.weight, blk.norm2.bias, blk.ffn.w1.weight, blk.ffn.w3.weight, blk.ffn.w2.weight]
    return [mod.proj_in.weight, mod.proj_out.weight, mod.norm.weight, mod.norm.bias] + lp


def level1_train(mod, frames, key_padding_mask, dtype):
    """Level1EventDynamics ``mod``'s stack on (n, N, d_slot) frames,
    differentiable; key_padding_mask (n, N) bool (True = dead slot) or None."""
    _lib.require_cuda(frames)
    kp = None if key_padding_mask is None else _c(key_padding_mask.to(torch.uint8))
    heads = mod.blocks[0].attn.num_heads
    return _Level1.apply(frames, kp, heads, dtype, *level1_params(mod))


# ---- gather / scatter --------------------------------------------------------------------
class _Gather(torch.autograd.Function):
    @staticmethod
    def forward(ctx, states, idx, pos, counts, meta, K):
        from .sparse_event_attn import event_gather

        B, T, N, D = states.shape
        ctx.save_for_backward(pos, counts)
        ctx.K, ctx.shape = K, states.shape
        return event_gather(_c(states), idx, counts, meta, B * K, pad_k=K).reshape(B, K, N, D)

    @staticmethod
    def backward(ctx, g):
        from .sparse_event_attn import event_scatter

        pos, counts = ctx.saved_tensors
        B, T, N, D = ctx.shape
        zeros = torch.zeros(ctx.shape, dtype=g.dtype, device=g.device)
        ds = event_scatter(zeros, _c(g.reshape(B * ctx.K, N, D)), pos, counts, pad_k=ctx.K)
        return ds, None, None, None, None, None


class _Scatter(torch.autograd.Function):
    @staticmethod
    def forward(ctx, base, upd, idx, pos, counts, meta, K):
        from .sparse_event_attn import event_scatter

        B, T, N, D = base.shape
        ctx.save_for_backward(idx, pos, counts, meta)
        ctx.K, ctx.shape, ctx.upd_dtype = K, base.shape, upd.dtype
        return event_scatter(_c(base), _c(upd.reshape(B * K, N, D).to(base.dtype)), pos, counts, pad_k=K)

    @staticmethod
    def backward(ctx, g):
        from .sparse_event_attn import event_gather, event_scatter

        idx, pos, counts, meta = ctx.saved_tensors
        B, T, N, D = ctx.shape
        K = ctx.K
        g = _c(g)
        d_base = event_scatter(g, torch.zeros(B * K, N, D, dtype=g.dtype, device=g.device), pos, counts, pad_k=K)
        d_upd = event_gather(g, idx, counts, meta, B * K, pad_k=K).reshape(B, K, N, D).to(ctx.upd_dtype)
        return d_base, d_upd, None, None, None, None, None


def event_gather_train(states, idx, pos, counts, meta, K):
    return _Gather.apply(states, idx, pos, counts, meta, K)


def event_scatter_train(base, upd, idx, pos, counts, meta, K):
    return _Scatter.apply(base, upd, idx, pos, counts, meta, K)
