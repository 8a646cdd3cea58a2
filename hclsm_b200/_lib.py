"""ctypes binding of ``libhclsm_b200.so`` (the C ABI declared in include/hclsm_b200.h).

The library is the only compute path: there is no CPU or PyTorch fallback.  A
missing library or a non-CUDA tensor raises.
"""
from __future__ import annotations

import ctypes
import os

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libhclsm_b200.so")

F32, BF16 = 0, 1
_STATUS = {
    1: (ValueError, "unsupported shape"),
    2: (TypeError, "unsupported dtype"),
    3: (ValueError, "misaligned pointer"),
    4: (ValueError, "workspace missing or too small"),
    5: (RuntimeError, "CUDA launch failed"),
    6: (RuntimeError, "device-side wait timed out"),
    7: (NotImplementedError, "input outside what this build supports"),
    8: (ValueError, "required pointer is NULL"),
}

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_sz = ctypes.c_size_t

# name -> (restype, argtypes)
SIGNATURES = {
    "hclsm_version": (ctypes.c_int, []),
    "hclsm_device_error": (ctypes.c_int, []),
    "hclsm_selftest_wait_timeout": (ctypes.c_int, [ctypes.c_uint32, _vp, _vp]),
    "hclsm_ssm_scan_fwd": (ctypes.c_int, [_vp] * 8 + [_i64, _i32, _i32, _i32, _i32, _i32, _vp]),
    "hclsm_ssm_scan_bwd_workspace_size": (_sz, [_i64, _i32, _i32, _i32]),
    "hclsm_ssm_scan_bwd": (ctypes.c_int, [_vp] * 15 + [_i64, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp]),
    "hclsm_ssm_scan_states_size": (_sz, [_i64, _i32, _i32, _i32, _i32]),
    "hclsm_ssm_scan_fwd_states": (ctypes.c_int, [_vp] * 8 + [_i64, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp]),
    "hclsm_ssm_scan_bwd_states": (ctypes.c_int, [_vp] * 15 + [_i64, _i32, _i32, _i32, _i32, _i32, _vp, _sz, _vp,
                                                              _sz, _vp]),
    "hclsm_l0_pool": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i32, _i32, _i32, _i64, _vp]),
    "hclsm_l0_epilogue": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i32, _i32, _i32, _i64, _vp]),
    "hclsm_l0_epilogue_bwd": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i32, _vp, _i32, _i32, _i64, _vp]),
    "hclsm_slot_attn_core": (ctypes.c_int, [_vp] * 5 + [_i32] * 4 + [ctypes.c_float] * 3 + [_i32, _i32, _vp]),
    "hclsm_layernorm": (ctypes.c_int, [_vp] * 4 + [_i64, _i32, ctypes.c_float, _i32, _vp]),
    "hclsm_gru_cell": (ctypes.c_int, [_vp] * 6 + [_i64, _i32, _vp]),
    "hclsm_bias_act": (ctypes.c_int, [_vp] * 3 + [_i64, _i32, _i32, _i32, _vp]),
    "hclsm_residual_clamp": (ctypes.c_int, [_vp] * 5 + [_i64, _i32, ctypes.c_float, _vp]),
    "hclsm_event_detect": (ctypes.c_int, [_vp, _vp, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "hclsm_event_compact": (ctypes.c_int, [_vp, _i32, _i32, _i32] + [_vp] * 5),
    "hclsm_event_gather": (ctypes.c_int, [_vp] * 5 + [_i64, _i32, _i32, _i64, _i32, _vp]),
    "hclsm_event_scatter": (ctypes.c_int, [_vp] * 5 + [_i64, _i64, _i32, _i32, _i32, _vp]),
    "hclsm_event_mha": (ctypes.c_int, [_vp] * 3 + [_i32] * 4 + [ctypes.c_float, _i32, _vp]),
    "hclsm_swiglu": (ctypes.c_int, [_vp, _i32, _vp, _i64, _i32, _i32, _vp]),
    "hclsm_slot_attn_iter_workspace_size": (_sz, [_i32] * 3),
    "hclsm_slot_attn_iter": (ctypes.c_int, [_vp] * 6 + [_i32] * 4 + [_vp, _sz, _vp]),
    "hclsm_gru_cell_ln": (ctypes.c_int, [_vp, _vp, _i32] + [_vp] * 7 + [_i32, _i64, _i32, ctypes.c_float, _vp]),
    "hclsm_residual_clamp_ln": (ctypes.c_int, [_vp, _vp, _i32] + [_vp] * 6 + [_i32, _i64, _i32, ctypes.c_float,
                                                                           ctypes.c_float, _vp]),
    "hclsm_colsum_workspace_size": (_sz, [_i32]),
    "hclsm_colsum": (ctypes.c_int, [_vp, _vp, _i64, _i32, _vp, _sz, _vp]),
    "hclsm_layernorm_bwd_workspace_size": (_sz, [_i64, _i32]),
    "hclsm_layernorm_bwd": (ctypes.c_int, [_vp] * 6 + [_i64, _i32, ctypes.c_float, _i32, _vp, _sz, _vp]),
    "hclsm_gru_cell_bwd": (ctypes.c_int, [_vp] * 9 + [_i64, _i32, _vp]),
    "hclsm_slot_softmax_bwd": (ctypes.c_int, [_vp] * 4 + [_i32] * 3 + [ctypes.c_float] * 3 + [_i32, _vp]),
    "hclsm_residual_clamp_bwd": (ctypes.c_int, [_vp] * 5 + [_i64, _i32, ctypes.c_float, _vp]),
    "hclsm_relu_bwd": (ctypes.c_int, [_vp, _i32, _vp, _vp, _i32, _i64, _vp]),
    "hclsm_swiglu_bwd": (ctypes.c_int, [_vp, _vp, _vp, _i64, _i32, _i32, _vp]),
    "hclsm_event_mha_bwd": (ctypes.c_int, [_vp] * 4 + [_i32] * 4 + [ctypes.c_float, _i32, _vp]),
    "hclsm_ssm_scan_bwd_noalloc_max_scratch": (_sz, []),
    "hclsm_ssm_scan_bwd_noalloc": (ctypes.c_int, [_vp] * 15 + [_i64, _i32, _i32, _i32, _i32, _i32, _vp]),
}

class SlotIterWeights(ctypes.Structure):
    """hclsm_slot_iter_weights (include/hclsm_b200.h)."""
    _fields_ = [(n, ctypes.c_void_p) for n in ("wq_t", "w_ih_t", "w_hh_t", "b_ih", "b_hh", "w1_t", "b1", "w2_t", "b2",
                                                "ln_attn_w", "ln_attn_b", "ln_mlp_w", "ln_mlp_b")]


_lib = None


def load() -> ctypes.CDLL:
    """Load the library (building nothing); raise if it is absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"hclsm_b200: native library {LIB_PATH} is missing; build it with "
                "`python -m hclsm_b200.build` (there is no fallback path)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != 0:
        exc, msg = _STATUS.get(rc, (RuntimeError, f"status {rc}"))
        raise exc(f"{what}: {msg} (hclsm status {rc})")


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_ptr(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return F32
    if dt == torch.bfloat16:
        return BF16
    raise TypeError(f"hclsm_b200: dtype {dt} not supported (float32 or bfloat16)")


def require_cuda(*tensors) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("hclsm_b200 ops run on CUDA tensors only (no CPU fallback)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError("hclsm_b200: all tensors must be on the same device")
    return dev
