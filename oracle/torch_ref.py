"""PyTorch CPU restatement of the reference's own CPU code paths (TEST
INFRASTRUCTURE ONLY: the timed CPU baseline of ``bench.py`` and a cross-check
in ``tests/``).  The reference runs these as PyTorch ops on the host when no
GPU kernel applies; restated op for op (same loops, same temporaries, same
autograd graph) they cost what the reference's CPU path costs on the same
cores.  Pinned against the golden vectors the reference produced
(``tests/test_oracle_golden.py``).

* ``sequential_ssm_scan`` — hclsm/kernels/ssm_scan_kernel.py:42-86 (the CPU
  dispatch of ``ssm_scan_fn``): clamp exp(A_log) to [1e-6, 1] and dt to
  [1e-3, 1], a Python loop over time with (batch, d_inner, d_state)
  temporaries, fp32; differentiable through autograd as in the reference.
* ``iteration_step`` — hclsm/objects/dynamic_slots.py:98-131.
* ``level1_event`` — hclsm/dynamics/level1_event.py:85-133 (proj_in, pre-LN
  blocks with nn.MultiheadAttention semantics and SwiGLU, LayerNorm, proj_out).
* ``naive_sparse_event_attention`` — hclsm/kernels/sparse_event_attn.py:35-86.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def sequential_ssm_scan(x, dt, A_log, B, C):
    batch, T, d_inner = x.shape
    d_state = B.shape[-1]
    A = -A_log.exp().clamp(min=1e-6, max=1.0)
    x_f, B_f, C_f = x.float(), B.float(), C.float()
    dt_f = dt.float().clamp(min=1e-3, max=1.0)
    h = torch.zeros(batch, d_inner, d_state, dtype=torch.float32, device=x.device)
    ys = []
    for t in range(T):
        dA = torch.exp(torch.clamp(dt_f[:, t, :, None] * A[None], min=-20.0, max=0.0))
        dBt = dt_f[:, t, :, None] * B_f[:, t, None, :]
        h = dA * h + dBt * x_f[:, t, :, None]
        ys.append((h * C_f[:, t, None, :]).sum(dim=-1))
    return torch.stack(ys, dim=1).to(x.dtype)


def iteration_step(slots, k, v, W):
    """W: parameter name -> tensor (DynamicSlotAttention's names)."""
    Fr, N, D = slots.shape
    sn = F.layer_norm(slots, (D,), W.get("norm_pre_attn.weight"), W.get("norm_pre_attn.bias"))
    q = F.linear(sn, W["project_q.weight"])
    logits = torch.clamp(torch.bmm(q, k.transpose(1, 2)) * D ** -0.5, -30.0, 30.0)
    attn = torch.softmax(logits, dim=1)
    upd = torch.bmm(attn, v)
    h = torch.gru_cell(upd.reshape(-1, D), slots.reshape(-1, D), W["gru.weight_ih"], W["gru.weight_hh"],
                       W["gru.bias_ih"], W["gru.bias_hh"]).reshape(Fr, N, D)
    m = F.layer_norm(h, (D,), W.get("norm_slots.weight"), W.get("norm_slots.bias"))
    m = F.linear(F.relu(F.linear(m, W["mlp.0.weight"], W["mlp.0.bias"])), W["mlp.2.weight"], W["mlp.2.bias"])
    return torch.clamp(h + m, -50.0, 50.0)


def _mha(x, w_in, w_out, heads, key_padding_mask=None):
    n, N, E = x.shape
    hd = E // heads
    q, k, v = F.linear(x, w_in).chunk(3, dim=-1)

    def split(t):
        return t.reshape(n, N, heads, hd).transpose(1, 2)

    q, k, v = split(q), split(k), split(v)
    s = torch.matmul(q * hd ** -0.5, k.transpose(-1, -2))
    if key_padding_mask is not None:
        s = s.masked_fill(key_padding_mask[:, None, None, :], float("-inf"))
    o = torch.matmul(torch.softmax(s, dim=-1), v).transpose(1, 2).reshape(n, N, E)
    return F.linear(o, w_out)


def level1_event(frames, W, heads, layers, key_padding_mask=None):
    x = F.linear(frames, W["proj_in.weight"])
    E = x.shape[-1]
    for i in range(layers):
        p = f"blocks.{i}."
        h = F.layer_norm(x, (E,), W.get(p + "norm1.weight"), W.get(p + "norm1.bias"))
        x = x + _mha(h, W[p + "attn.in_proj_weight"], W[p + "attn.out_proj.weight"], heads, key_padding_mask)
        h = F.layer_norm(x, (E,), W.get(p + "norm2.weight"), W.get(p + "norm2.bias"))
        x = x + F.linear(F.silu(F.linear(h, W[p + "ffn.w1.weight"])) * F.linear(h, W[p + "ffn.w3.weight"]),
                         W[p + "ffn.w2.weight"])
    x = F.layer_norm(x, (E,), W.get("norm.weight"), W.get("norm.bias"))
    return F.linear(x, W["proj_out.weight"])


def naive_sparse_event_attention(states, event_mask, attn_fn):
    out = states.clone()
    for b in range(states.shape[0]):
        idx = torch.nonzero(event_mask[b] > 0.5).flatten()
        if len(idx):
            out[b, idx] = attn_fn(states[b, idx])
    return out
