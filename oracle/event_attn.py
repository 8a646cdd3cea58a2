"""Sparse event attention oracle (TEST INFRASTRUCTURE ONLY).

* ``naive_sparse_event_attention`` restates hclsm/kernels/sparse_event_attn.py:35-86:
  gather the event timesteps of each video in ascending time, run ``attn_fn`` on
  every gathered frame, write the results back; other timesteps are unchanged.
* ``level1_event`` restates Level1EventDynamics.forward (hclsm/dynamics/level1_event.py:85-133)
  for one batch of frames: proj_in -> n_layers x [pre-LN MHA + residual,
  pre-LN SwiGLU + residual] -> LayerNorm -> proj_out.
"""
from __future__ import annotations

import numpy as np

from .nn import layernorm, mha, silu


def naive_sparse_event_attention(states, event_mask, attn_fn, max_events=None):
    states = np.asarray(states, np.float32)
    mask = np.asarray(event_mask)
    out = states.copy()
    Bn = states.shape[0]
    for b in range(Bn):
        idx = np.nonzero(mask[b] > 0.5)[0]
        if max_events is not None:
            idx = idx[:max_events]
        if len(idx):
            out[b, idx] = attn_fn(states[b, idx])
    return out


def level1_event(frames, W, n_heads, n_layers, key_padding_mask=None):
    """frames: (F, N, d_slot) -> (F, N, d_slot).  W uses Level1EventDynamics's
    parameter names; key_padding_mask (F, N) True marks dead slots."""
    x = np.asarray(frames, np.float32) @ W["proj_in.weight"].T
    for i in range(n_layers):
        p = f"blocks.{i}."
        h = layernorm(x, W.get(p + "norm1.weight"), W.get(p + "norm1.bias"))
        x = x + mha(h, W[p + "attn.in_proj_weight"], W[p + "attn.out_proj.weight"], n_heads, key_padding_mask)
        h = layernorm(x, W.get(p + "norm2.weight"), W.get(p + "norm2.bias"))
        f = silu(h @ W[p + "ffn.w1.weight"].T) * (h @ W[p + "ffn.w3.weight"].T)
        x = x + f @ W[p + "ffn.w2.weight"].T
    x = layernorm(x, W.get("norm.weight"), W.get("norm.bias"))
    return (x @ W["proj_out.weight"].T).astype(np.float32)
