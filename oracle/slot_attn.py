"""Slot-attention oracle (TEST INFRASTRUCTURE ONLY).

* ``naive_slot_attention`` restates hclsm/kernels/slot_attention_kernel.py:265-291
  (softmax over the SLOT axis, weighted sum of values).
* ``iteration_step`` restates DynamicSlotAttention._iteration_step,
  hclsm/objects/dynamic_slots.py:98-131, with the parameter names of that module.
"""
from __future__ import annotations

import numpy as np

from .nn import gru_cell, layernorm, softmax


def naive_slot_attention(Q, K, V, scale=None):
    Q, K, V = (np.asarray(t, np.float32) for t in (Q, K, V))
    if scale is None:
        scale = Q.shape[-1] ** -0.5
    logits = (Q @ K.transpose(0, 2, 1)) * np.float32(scale)
    attn = softmax(logits, axis=1)
    return (attn @ V).astype(np.float32), attn


def iteration_step(slots, k, v, W, clamp_logits=30.0, clamp_slots=50.0):
    """One refinement step.  W maps parameter names of DynamicSlotAttention
    (``project_q.weight``, ``gru.weight_ih`` ...) to arrays."""
    slots, k, v = (np.asarray(t, np.float32) for t in (slots, k, v))
    Fr, N, D = slots.shape
    scale = np.float32(D ** -0.5)
    sn = layernorm(slots, W.get("norm_pre_attn.weight"), W.get("norm_pre_attn.bias"))
    q = sn @ W["project_q.weight"].T
    logits = np.clip((q @ k.transpose(0, 2, 1)) * scale, -clamp_logits, clamp_logits)
    attn = softmax(logits, axis=1)
    updates = attn @ v
    h = gru_cell(updates.reshape(-1, D), slots.reshape(-1, D), W["gru.weight_ih"], W["gru.weight_hh"],
                 W["gru.bias_ih"], W["gru.bias_hh"]).reshape(Fr, N, D)
    m = layernorm(h, W.get("norm_slots.weight"), W.get("norm_slots.bias"))
    m = np.maximum(m @ W["mlp.0.weight"].T + W["mlp.0.bias"], 0.0)
    m = m @ W["mlp.2.weight"].T + W["mlp.2.bias"]
    return np.clip(h + m, -clamp_slots, clamp_slots).astype(np.float32)
