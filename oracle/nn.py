"""Small numpy building blocks shared by the oracle modules (TEST INFRASTRUCTURE ONLY).

Each follows the PyTorch module the reference uses: nn.LayerNorm (eps 1e-5),
nn.GRUCell (gate order r, z, n), nn.MultiheadAttention (bias=False,
batch_first, key_padding_mask), F.silu.
"""
from __future__ import annotations

import numpy as np


def layernorm(x, w=None, b=None, eps=1e-5):
    x = np.asarray(x, np.float32)
    mu = x.mean(-1, keepdims=True)
    var = ((x - mu) ** 2).mean(-1, keepdims=True)
    y = (x - mu) / np.sqrt(var + eps)
    if w is not None:
        y = y * w
    if b is not None:
        y = y + b
    return y.astype(np.float32)


def sigmoid(x):
    return (1.0 / (1.0 + np.exp(-x))).astype(np.float32)


def silu(x):
    return (x * sigmoid(x)).astype(np.float32)


def softmax(x, axis):
    m = x.max(axis=axis, keepdims=True)
    e = np.exp(x - m)
    return (e / e.sum(axis=axis, keepdims=True)).astype(np.float32)


def gru_cell(x, h, w_ih, w_hh, b_ih, b_hh):
    """torch.nn.GRUCell: r, z, n gates stacked in that order."""
    gi = x @ w_ih.T + b_ih
    gh = h @ w_hh.T + b_hh
    H = h.shape[-1]
    r = sigmoid(gi[..., :H] + gh[..., :H])
    z = sigmoid(gi[..., H:2 * H] + gh[..., H:2 * H])
    n = np.tanh(gi[..., 2 * H:] + r * gh[..., 2 * H:])
    return ((1.0 - z) * n + z * h).astype(np.float32)


def mha(x, in_proj_weight, out_proj_weight, n_heads, key_padding_mask=None):
    """nn.MultiheadAttention(bias=False, batch_first=True) self-attention.

    x: (B, N, E); key_padding_mask: (B, N) bool, True = ignore that key."""
    Bn, N, E = x.shape
    hd = E // n_heads
    qkv = x @ in_proj_weight.T
    q, k, v = qkv[..., :E], qkv[..., E:2 * E], qkv[..., 2 * E:]

    def split(t):
        return t.reshape(Bn, N, n_heads, hd).transpose(0, 2, 1, 3)

    q, k, v = split(q), split(k), split(v)
    s = (q @ k.transpose(0, 1, 3, 2)) / np.float32(np.sqrt(hd))
    if key_padding_mask is not None:
        s = np.where(key_padding_mask[:, None, None, :], -np.inf, s)
    a = softmax(s, axis=-1)
    o = (a @ v).transpose(0, 2, 1, 3).reshape(Bn, N, E)
    return (o @ out_proj_weight.T).astype(np.float32)
