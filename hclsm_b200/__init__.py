"""hclsm_b200 — B200-native (sm_100a) hot path of the HCLSM world model.

Drop-in replacements for ``hclsm.kernels`` (same call signatures):

    from hclsm_b200.kernels import ssm_scan_fn, slot_attention_fn, sparse_event_attn_fn

``hclsm_b200.install()`` patches a loaded ``hclsm`` package so the model's own
call sites use these kernels.
"""
from __future__ import annotations

from . import _lib
from .kernels import ssm_scan_fn  # noqa: F401
from .graphs import GraphedStep  # noqa: F401

__version__ = "0.1.0"


def native_version() -> int:
    return _lib.load().hclsm_version()


def device_error() -> int:
    """Synchronise, then return and clear the first device-side error code."""
    return _lib.load().hclsm_device_error()
