"""Seeded parameters for the tiny-preset model fixture (model_golden.npz).

Each parameter is drawn from a generator seeded by its qualified name, so the
fixture stores no weights: the generator (make_golden.py, with the reference)
and the GPU test (with stand-in modules of the same parameter names) draw the
same tensors independently of module order.
"""
from __future__ import annotations

import zlib

import torch


def seeded_param(qualname: str, shape) -> torch.Tensor:
    g = torch.Generator().manual_seed(zlib.crc32(qualname.encode()) + 7)
    leaf = qualname.rsplit(".", 1)[-1]
    if leaf == "A_log":
        return torch.empty(shape).uniform_(-1.0, 0.5, generator=g)
    r = torch.randn(shape, generator=g)
    if "norm" in qualname and leaf == "weight":
        return 1.0 + 0.05 * r
    if len(shape) >= 2:
        return r * 0.05
    return r * 0.02


def load_seeded(prefix: str, module) -> None:
    """Overwrite every parameter of ``module`` with seeded_param(prefix + name)."""
    with torch.no_grad():
        for name, p in module.named_parameters():
            p.copy_(seeded_param(f"{prefix}.{name}", tuple(p.shape)))


def grad_sample(name: str, g):
    """The stored part of a parameter gradient: all of it up to 65536
    elements, else every 16th element of the flattened tensor."""
    flat = g.reshape(-1)
    return flat if flat.numel() <= 65536 else flat[::16]
