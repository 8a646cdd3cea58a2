"""Slot attention on B200 — drop-in for hclsm/kernels/slot_attention_kernel.py
and for DynamicSlotAttention._iteration_step (hclsm/objects/dynamic_slots.py:98-131).

* ``slot_attention_fn(Q, K, V, scale=None, backend="auto")`` keeps the reference
  signature (slot_attention_kernel.py:324-355) and returns ``(out, attn)`` with
  the softmax over the SLOT axis.  The forward runs the fused sm_100a core;
  the backward applies the reference's own formulas (:215-236) with this
  library's softmax-over-slots backward kernel and batched library GEMMs.  ``eps`` (keyword) adds to the softmax denominator: 0 for the
  naive/compiled reference paths, 1e-8 for its Triton path (:126).
* ``slot_attention_iteration(slots, k, v, params)`` runs one full refinement
  step — LayerNorm, W_q, the attention core with the +-30 logit clamp, GRUCell,
  the residual LayerNorm-MLP and the +-50 clamp — with the attention core and
  every element-wise stage in this library's kernels and the five weight
  products as library GEMMs (bf16 operands, fp32 outputs).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from .. import _lib

__all__ = ["slot_attention_fn", "slot_attention_core", "SlotIterationParams", "slot_attention_iteration", "slot_attn_iter",
           "fold_query_into_keys", "key_value_weights", "project_keys_values",
           "layernorm", "gru_cell", "bias_act", "residual_clamp"]


def _c(t):
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


def slot_attention_core(Q, K, V, scale=None, *, clamp=0.0, eps=0.0, return_attn=True, attn_fp32=None, out=None):
    """Forward only.  Q (F, N, D), K/V (F, M, D) on CUDA, fp32 or bf16.  ``out``
    (optional): a contiguous (F, N, D) tensor of the I/O dtype to write into."""
    _lib.require_cuda(Q, K, V)
    if Q.dim() != 3 or K.dim() != 3 or V.shape != K.shape or Q.shape[0] != K.shape[0] or Q.shape[2] != K.shape[2]:
        raise ValueError("expected Q (B, N, D) and K, V (B, M, D)")
    dt = torch.bfloat16 if {Q.dtype, K.dtype, V.dtype} == {torch.bfloat16} else torch.float32
    Q, K, V = (_c(t.to(dt)) for t in (Q, K, V))
    F, N, D = Q.shape
    M = K.shape[1]
    if scale is None:
        scale = D ** -0.5
    if out is None:
        out = torch.empty(F, N, D, dtype=dt, device=Q.device)
    elif out.shape != (F, N, D) or out.dtype != dt or not out.is_contiguous() or out.data_ptr() % 16:
        raise ValueError("out must be a contiguous, 16-byte aligned (F, N, D) tensor of the I/O dtype")
    if attn_fp32 is None:
        attn_fp32 = dt == torch.float32
    attn = None
    if return_attn:
        attn = torch.empty(F, N, M, dtype=torch.float32 if attn_fp32 else dt, device=Q.device)
    rc = _lib.load().hclsm_slot_attn_core(_lib.ptr(Q), _lib.ptr(K), _lib.ptr(V), _lib.ptr(out), _lib.ptr(attn),
                                          F, N, M, D, float(scale), float(clamp), float(eps),
                                          _lib.dtype_code(dt), int(bool(attn_fp32)), _lib.stream_ptr(Q.device))
    _lib.check(rc, "hclsm_slot_attn_core")
    return out, attn


class _SlotAttn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, V, scale, eps):
        out, attn = slot_attention_core(Q, K, V, scale, eps=eps, attn_fp32=True)
        ctx.save_for_backward(Q, K, V)
        ctx.scale, ctx.eps = scale, eps
        return out.to(Q.dtype), attn if Q.dtype == torch.float32 else attn.to(Q.dtype)

    @staticmethod
    def backward(ctx, grad_out, grad_attn):
        # the reference's backward (slot_attention_kernel.py:215-236): the
        # probabilities are recomputed from Q K^T and the softmax-over-slots
        # backward runs in this library's kernel; the contractions are batched
        # library GEMMs in fp32
        from .training import slot_softmax_bwd

        Q, K, V = ctx.saved_tensors
        f = torch.float32
        Qf, Kf, Vf = Q.to(f), K.to(f), V.to(f)
        go = grad_out.to(f)
        d_attn = torch.bmm(go, Vf.transpose(1, 2))
        if grad_attn is not None:
            d_attn = d_attn + grad_attn.to(f)
        dots = torch.bmm(Qf, Kf.transpose(1, 2))
        attn, d_dots = slot_softmax_bwd(dots, d_attn, ctx.scale, 0.0, ctx.eps, f)
        dQ = torch.bmm(d_dots, Kf).to(Q.dtype)
        dK = torch.bmm(d_dots.transpose(1, 2), Qf).to(K.dtype)
        dV = torch.bmm(attn.transpose(1, 2), go).to(V.dtype)
        return dQ, dK, dV, None, None


def slot_attention_fn(Q, K, V, scale=None, backend: str = "auto", *, eps: float | None = None):
    """Drop-in for ``hclsm.kernels.slot_attention_fn``: returns (out, attn) with
    the softmax over slots.  Every backend name runs the B200 core; ``eps``
    defaults to the reference backend's value (1e-8 for "triton", else 0)."""
    if backend not in ("auto", "b200", "triton", "compiled", "naive"):
        raise ValueError(f"unknown backend {backend!r}")
    if scale is None:
        scale = Q.shape[-1] ** -0.5
    if eps is None:
        eps = 1e-8 if backend == "triton" else 0.0
    return _SlotAttn.apply(Q, K, V, float(scale), float(eps))


# ---- element-wise stages -------------------------------------------------------------
def layernorm(x, w=None, b=None, eps=1e-5, out_dtype=torch.float32):
    x = _c(x.float())
    rows, D = x.numel() // x.shape[-1], x.shape[-1]
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    rc = _lib.load().hclsm_layernorm(_lib.ptr(x), _lib.ptr(w), _lib.ptr(b), _lib.ptr(y), rows, D, float(eps),
                                     _lib.dtype_code(out_dtype), _lib.stream_ptr(x.device))
    _lib.check(rc, "hclsm_layernorm")
    return y


def gru_cell(gi, gh, b_ih, b_hh, h, out=None):
    H = h.shape[-1]
    rows = h.numel() // H
    out = torch.empty_like(h) if out is None else out
    rc = _lib.load().hclsm_gru_cell(_lib.ptr(gi), _lib.ptr(gh), _lib.ptr(b_ih), _lib.ptr(b_hh), _lib.ptr(h),
                                    _lib.ptr(out), rows, H, _lib.stream_ptr(h.device))
    _lib.check(rc, "hclsm_gru_cell")
    return out


def bias_act(x, b, act="relu", out_dtype=torch.bfloat16):
    C = x.shape[-1]
    y = torch.empty(x.shape, dtype=out_dtype, device=x.device)
    rc = _lib.load().hclsm_bias_act(_lib.ptr(x), _lib.ptr(b), _lib.ptr(y), x.numel() // C, C,
                                    1 if act == "relu" else 0, _lib.dtype_code(out_dtype), _lib.stream_ptr(x.device))
    _lib.check(rc, "hclsm_bias_act")
    return y


def residual_clamp(h, m, b, clamp=50.0, out=None, out_bf16=None):
    C = h.shape[-1]
    out = torch.empty_like(h) if out is None else out
    rc = _lib.load().hclsm_residual_clamp(_lib.ptr(h), _lib.ptr(m), _lib.ptr(b), _lib.ptr(out), _lib.ptr(out_bf16),
                                          h.numel() // C, C, float(clamp), _lib.stream_ptr(h.device))
    _lib.check(rc, "hclsm_residual_clamp")
    return out


def gru_cell_ln(gi, gh, b_ih, b_hh, h, ln_w, ln_b, ln_dtype, eps=1e-5):
    """(GRUCell state fp32, LayerNorm of it in ln_dtype) in one pass; the gate
    products gi and gh are fp32 or bf16 (both the same)."""
    H = h.shape[-1]
    rows = h.numel() // H
    if gi.dtype != gh.dtype:
        raise TypeError("hclsm_b200: gru_cell_ln wants gi and gh of one dtype")
    out = torch.empty_like(h)
    ln = torch.empty(h.shape, dtype=ln_dtype, device=h.device)
    rc = _lib.load().hclsm_gru_cell_ln(_lib.ptr(gi), _lib.ptr(gh), _lib.dtype_code(gi.dtype), _lib.ptr(b_ih), _lib.ptr(b_hh), _lib.ptr(h),
                                       _lib.ptr(out), _lib.ptr(ln_w), _lib.ptr(ln_b), _lib.ptr(ln),
                                       _lib.dtype_code(ln_dtype), rows, H, float(eps), _lib.stream_ptr(h.device))
    _lib.check(rc, "hclsm_gru_cell_ln")
    return out, ln


def residual_clamp_ln(h, m, b, clamp, ln_w, ln_b, ln_dtype, out_bf16=None, eps=1e-5):
    """(clamp(h + m + b) fp32, LayerNorm of it in ln_dtype) in one pass; m is
    fp32 or bf16; the optional bf16 copy of the first goes to out_bf16."""
    C = h.shape[-1]
    out = torch.empty_like(h)
    ln = torch.empty(h.shape, dtype=ln_dtype, device=h.device)
    rc = _lib.load().hclsm_residual_clamp_ln(_lib.ptr(h), _lib.ptr(m), _lib.dtype_code(m.dtype), _lib.ptr(b), _lib.ptr(out), _lib.ptr(out_bf16),
                                             _lib.ptr(ln_w), _lib.ptr(ln_b), _lib.ptr(ln), _lib.dtype_code(ln_dtype),
                                             h.numel() // C, C, float(clamp), float(eps), _lib.stream_ptr(h.device))
    _lib.check(rc, "hclsm_residual_clamp_ln")
    return out, ln


# ---- the fused refinement step -------------------------------------------------------
@dataclass
class SlotIterationParams:
    """Parameters of DynamicSlotAttention used by _iteration_step (names as in
    hclsm/objects/dynamic_slots.py:44-83), prepared once: weights in ``dtype``
    (transposed for x @ W^T), biases and LayerNorm affines in fp32.  ``dtype``
    is the arithmetic of the weight products: bfloat16 (the reference under
    bf16 autocast; fp32 accumulation and outputs) or float32 (the reference
    without autocast: every product in fp32)."""
    wq_t: torch.Tensor
    w_ih_t: torch.Tensor
    w_hh_t: torch.Tensor
    b_ih: torch.Tensor
    b_hh: torch.Tensor
    w1_t: torch.Tensor
    b1: torch.Tensor
    w2_t: torch.Tensor
    b2: torch.Tensor
    ln_attn_w: torch.Tensor
    ln_attn_b: torch.Tensor
    ln_mlp_w: torch.Tensor
    ln_mlp_b: torch.Tensor
    scale: float
    b1_bf16: torch.Tensor | None = None  # the MLP's first bias for the fused GEMM epilogue (bf16 path)
    dtype: torch.dtype = torch.bfloat16
    w_gru_t: torch.Tensor | None = None  # (2, D, 3D): [W_ih^T, W_hh^T] for one batched product (bf16 path)

    @classmethod
    def from_state(cls, sd: dict, device, d_slot: int | None = None, dtype=torch.bfloat16):
        if dtype not in (torch.bfloat16, torch.float32):
            raise TypeError(f"hclsm_b200: slot iteration dtype {dtype} (bfloat16 or float32)")

        def w(name):
            return sd[name].detach().to(device=device, dtype=dtype).t().contiguous()

        def f(name):
            return sd[name].detach().to(device=device, dtype=torch.float32).contiguous()

        D = d_slot or sd["project_q.weight"].shape[0]
        b1 = f("mlp.0.bias")
        return cls(w("project_q.weight"), w("gru.weight_ih"), w("gru.weight_hh"), f("gru.bias_ih"),
                   f("gru.bias_hh"), w("mlp.0.weight"), b1, w("mlp.2.weight"), f("mlp.2.bias"),
                   f("norm_pre_attn.weight"), f("norm_pre_attn.bias"), f("norm_slots.weight"),
                   f("norm_slots.bias"), D ** -0.5, b1.to(torch.bfloat16) if dtype == torch.bfloat16 else None,
                   dtype, torch.stack([w("gru.weight_ih"), w("gru.weight_hh")]) if dtype == torch.bfloat16 else None)

    @classmethod
    def from_module(cls, mod, dtype=torch.bfloat16):
        return cls.from_state(dict(mod.named_parameters()), next(mod.parameters()).device, mod.d_slot, dtype)


def _mm(a, w_t):
    if a.dtype == torch.float32:
        return torch.mm(a, w_t)
    return torch.mm(a, w_t, out_dtype=torch.float32)


def slot_attention_iteration(slots, k, v, p: SlotIterationParams, slots_lp=None, pair=None):
    """One _iteration_step (dynamic_slots.py:98-131).  slots (F, N, D) fp32 (the
    carried state), k and v (F, M, D) in ``p.dtype``.  Returns (slots_new fp32,
    a bf16 copy of it on the bf16 path, else None)."""
    out, out_lp, _ = _iteration(slots, k, v, p, slots_lp, pair, None, False)
    return out, out_lp


def fold_query_into_keys(project_k_weight, project_q_weight, dtype=torch.bfloat16):
    """The key projection with W_q folded in: (d_input, d_slot) = W_k^T W_q.

    project_q and project_k have no bias (dynamic_slots.py:51-53), so the
    attention logits of _iteration_step (:113-117) are
    LN(s) W_q^T (x W_k^T)^T = LN(s) (x W_k^T W_q)^T: keys projected with this
    weight (k' = x @ it, once per forward) let every refinement step feed the
    normalised slots to the attention core directly, without its own W_q
    product.  The product is formed in fp32 and rounded to ``dtype`` once."""
    wk = project_k_weight.detach().float()
    wq = project_q_weight.detach().float()
    return (wk.t() @ wq).to(dtype).contiguous()


def key_value_weights(project_k_weight, project_v_weight, project_q_weight=None, dtype=torch.bfloat16):
    """(2, d_input, d_slot): [W_k^T (or W_k^T W_q, see fold_query_into_keys),
    W_v^T] for project_keys_values."""
    wk = (fold_query_into_keys(project_k_weight, project_q_weight, dtype) if project_q_weight is not None
          else project_k_weight.detach().t().to(dtype))
    return torch.stack([wk, project_v_weight.detach().t().to(dtype)]).contiguous()


def project_keys_values(x, w_kv):
    """k and v (dynamic_slots.py:152-154) of x (F, M, d_input) as one batched
    library GEMM over the stacked weights (x is read through a stride-0 batch
    view, not copied); both outputs contiguous (F, M, d_slot)."""
    F, M, Din = x.shape
    kv = torch.bmm(x.reshape(1, F * M, Din).expand(2, -1, -1), w_kv)
    return kv[0].view(F, M, -1), kv[1].view(F, M, -1)


def _iteration(slots, k, v, p: SlotIterationParams, slots_lp, pair, sn, want_next_sn, keys_folded=False):
    """The step with its row stages fused: LayerNorm (skipped when ``sn``, the
    normalised slots, is given), W_q, the attention core, the GRU gate
    products, GRUCell + norm_slots LayerNorm (one kernel), the MLP, and
    residual + clamp (+ the next step's norm_pre_attn LayerNorm when
    ``want_next_sn``; one kernel).  Returns (slots_new fp32, bf16 copy or None,
    next sn or None).

    bf16 path with ``pair`` (a (2, F*N, D) bf16 buffer whose [1] holds the
    slots in bf16): the attention core writes its updates into pair[0], both
    GRU gate products run as one batched GEMM over pair and the stacked
    [W_ih^T, W_hh^T], and the new slots' bf16 copy lands in pair[1] for the
    next iteration."""
    F, N, D = slots.shape
    R = F * N
    dt = p.dtype
    s2 = slots.reshape(R, D)
    lp = dt == torch.bfloat16
    if lp and slots_lp is None and pair is None:
        slots_lp = s2.to(torch.bfloat16)
    if sn is None:
        sn = layernorm(s2, p.ln_attn_w, p.ln_attn_b, out_dtype=dt)
    if keys_folded:  # k holds x W_k^T W_q: the logits need LN(s) only
        q = sn.reshape(F, N, D)
    else:
        q = torch.mm(sn.reshape(R, D), p.wq_t).reshape(F, N, D)
    if lp and pair is not None and p.w_gru_t is not None:
        slot_attention_core(q, k, v, p.scale, clamp=30.0, eps=0.0, return_attn=False, out=pair[0].view(F, N, D))
        # gate products rounded to bf16, as the reference's GRUCell receives
        # them under bf16 autocast (gate arithmetic and state stay fp32)
        g2 = torch.bmm(pair, p.w_gru_t)
        gi, gh = g2[0], g2[1]
    else:
        upd, _ = slot_attention_core(q, k, v, p.scale, clamp=30.0, eps=0.0, return_attn=False)
        gi = _mm(upd.reshape(R, D), p.w_ih_t)
        gh = _mm(slots_lp.reshape(R, D) if lp else s2, p.w_hh_t)
    fuse = D % 128 == 0 and D <= 1024  # the row-fused kernels' shapes
    if fuse:
        h, m = gru_cell_ln(gi, gh, p.b_ih, p.b_hh, s2, p.ln_mlp_w, p.ln_mlp_b, dt)
    else:
        h = gru_cell(gi.float(), gh.float(), p.b_ih, p.b_hh, s2)
        m = layernorm(h, p.ln_mlp_w, p.ln_mlp_b, out_dtype=dt)
    if lp and p.b1_bf16 is not None:
        # bias + ReLU in the library GEMM's epilogue, bf16 out (the MLP runs in
        # the autocast dtype in the reference)
        m = torch._addmm_activation(p.b1_bf16, m, p.w1_t)
    elif not lp:
        m = torch._addmm_activation(p.b1, m, p.w1_t)  # fp32 throughout
    else:
        m = bias_act(_mm(m, p.w1_t), p.b1, "relu", torch.bfloat16)
    sn_fused = want_next_sn and fuse
    # the MLP output in bf16 where the fused residual kernel reads it (the
    # reference's MLP output under autocast); fp32 otherwise
    m = torch.mm(m, p.w2_t) if (lp and sn_fused) else _mm(m, p.w2_t)
    if lp:
        out_lp = pair[1] if pair is not None else torch.empty(R, D, dtype=torch.bfloat16, device=slots.device)
    else:
        out_lp = None
    sn_next = None
    if sn_fused:
        out, sn_next = residual_clamp_ln(h, m, p.b2, 50.0, p.ln_attn_w, p.ln_attn_b, dt, out_bf16=out_lp)
    else:
        out = residual_clamp(h, m, p.b2, 50.0, out_bf16=out_lp)
    return out.reshape(F, N, D), (out_lp.reshape(F, N, D) if lp else None), sn_next


def slot_attention_iterations(slots, k, v, p: SlotIterationParams, n_iterations: int, keys_folded: bool = False):
    """``n_iterations`` refinement steps.  With ``keys_folded`` the keys are
    x @ fold_query_into_keys(W_k, W_q) instead of x W_k^T and no step runs the
    W_q product."""
    s = slots.float().contiguous()
    k = _c(k.to(p.dtype))
    v = _c(v.to(p.dtype))
    F, N, D = s.shape
    pair, sl, sn = None, None, None
    if p.dtype == torch.bfloat16 and p.w_gru_t is not None and (F * N * D * 2) % 16 == 0:
        pair = torch.empty(2, F * N, D, dtype=torch.bfloat16, device=s.device)
        pair[1].copy_(s.reshape(F * N, D))
    for i in range(n_iterations):
        s, sl, sn = _iteration(s, k, v, p, sl, pair, sn, i + 1 < n_iterations, keys_folded)
    return s


def slot_attn_iter(slots, k, v, p: SlotIterationParams, out_bf16=None):
    """One _iteration_step through the single C entry point
    hclsm_slot_attn_iter (bf16 weight products).  slots (F, N, D) fp32, k and
    v (F, M, D) bf16.  Returns the new slots (fp32); their bf16 copy goes to
    ``out_bf16`` when given."""
    if p.dtype != torch.bfloat16:
        raise TypeError("hclsm_slot_attn_iter runs bf16 weight products (SlotIterationParams dtype bfloat16)")
    _lib.require_cuda(slots, k, v)
    s = _c(slots.float())
    k, v = _c(k.to(torch.bfloat16)), _c(v.to(torch.bfloat16))
    F, N, D = s.shape
    M = k.shape[1]
    lib = _lib.load()
    ws = torch.empty(max(lib.hclsm_slot_attn_iter_workspace_size(F, N, D), 1), dtype=torch.uint8, device=s.device)
    w = _lib.SlotIterWeights(*[_lib.ptr(t) for t in (p.wq_t, p.w_ih_t, p.w_hh_t, p.b_ih, p.b_hh, p.w1_t, p.b1_bf16,
                                                      p.w2_t, p.b2, p.ln_attn_w, p.ln_attn_b, p.ln_mlp_w, p.ln_mlp_b)])
    out = torch.empty_like(s)
    rc = lib.hclsm_slot_attn_iter(_lib.ptr(s), _lib.ptr(k), _lib.ptr(v), ctypes.byref(w), _lib.ptr(out),
                                  _lib.ptr(out_bf16), F, N, M, D, _lib.ptr(ws), ws.numel(), _lib.stream_ptr(s.device))
    _lib.check(rc, "hclsm_slot_attn_iter")
    return out
