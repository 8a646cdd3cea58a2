"""Selective-scan oracle (TEST INFRASTRUCTURE ONLY).

ctypes wrapper over ``scan_oracle.c`` (a C restatement of
hclsm/kernels/ssm_scan_kernel.py: sequential_ssm_scan :42-86 when ``clamp`` is
true, parallel_ssm_scan_pytorch :168-218 / _TritonSSMScan :292-377 otherwise).
Sequences are split across host threads; the C code is single-threaded.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_f = ctypes.POINTER(ctypes.c_float)
_d = ctypes.POINTER(ctypes.c_double)


def build() -> str:
    """Compile the C oracle with the committed Makefile (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        lib = ctypes.CDLL(_LIB_PATH)
        lib.oracle_scan_fwd.argtypes = [_f] * 8 + [ctypes.c_int64] + [ctypes.c_int] * 4
        lib.oracle_scan_fwd.restype = None
        lib.oracle_scan_bwd.argtypes = [_f] * 13 + [_d, _d, ctypes.c_int64] + [ctypes.c_int] * 4
        lib.oracle_scan_bwd.restype = None
        _lib = lib
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(_f)


def _f32(a):
    return None if a is None else np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _split(nseq: int, threads: int):
    threads = max(1, min(threads, nseq))
    step = (nseq + threads - 1) // threads
    return [(s, min(nseq, s + step)) for s in range(0, nseq, step)]


def default_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def scan_fwd(x, dt, A_log, B, C, D=None, z=None, clamp=False, threads=None):
    """y = (scan(x, dt, A_log, B, C) + D*x) * silu(z), all fp32 numpy."""
    lib = _load()
    x, dt, A_log, B, C, D, z = map(_f32, (x, dt, A_log, B, C, D, z))
    nseq, L, Dn = x.shape
    S = B.shape[-1]
    y = np.empty_like(x)
    threads = threads or default_threads()

    def run(rng):
        s0, s1 = rng
        sl = slice(s0, s1)
        lib.oracle_scan_fwd(_p(x[sl]), _p(dt[sl]), _p(A_log), _p(B[sl]), _p(C[sl]), _p(D),
                            _p(None if z is None else z[sl]), _p(y[sl]), s1 - s0, L, Dn, S, int(bool(clamp)))

    parts = _split(nseq, threads)
    if len(parts) == 1:
        run(parts[0])
    else:
        with ThreadPoolExecutor(len(parts)) as ex:
            list(ex.map(run, parts))
    return y


def scan_bwd(x, dt, A_log, B, C, dy, D=None, z=None, clamp=False, threads=None):
    """Gradients of y_out w.r.t. every input.  Returns a dict of fp32 arrays."""
    lib = _load()
    x, dt, A_log, B, C, D, z, dy = map(_f32, (x, dt, A_log, B, C, D, z, dy))
    nseq, L, Dn = x.shape
    S = B.shape[-1]
    dx = np.empty_like(x)
    ddt = np.empty_like(x)
    dB = np.empty_like(B)
    dC = np.empty_like(C)
    dz = np.empty_like(x) if z is not None else None
    threads = threads or default_threads()
    parts = _split(nseq, threads)
    gAs = [np.zeros((Dn, S), np.float64) for _ in parts]
    gDs = [np.zeros((Dn,), np.float64) for _ in parts]

    def run(i):
        s0, s1 = parts[i]
        sl = slice(s0, s1)
        lib.oracle_scan_bwd(_p(x[sl]), _p(dt[sl]), _p(A_log), _p(B[sl]), _p(C[sl]), _p(D),
                            _p(None if z is None else z[sl]), _p(dy[sl]), _p(dx[sl]), _p(ddt[sl]),
                            _p(dB[sl]), _p(dC[sl]), _p(None if dz is None else dz[sl]),
                            gAs[i].ctypes.data_as(_d), gDs[i].ctypes.data_as(_d),
                            s1 - s0, L, Dn, S, int(bool(clamp)))

    if len(parts) == 1:
        run(0)
    else:
        with ThreadPoolExecutor(len(parts)) as ex:
            list(ex.map(run, range(len(parts))))
    gA = np.sum(gAs, axis=0)
    e = np.exp(A_log.astype(np.float64))
    fac = -e
    if clamp:
        fac = np.where((e >= 1e-6) & (e <= 1.0), fac, 0.0)
    out = dict(dx=dx, ddt=ddt, dB=dB, dC=dC, dA_log=(gA * fac).astype(np.float32))
    if D is not None:
        out["dD"] = np.sum(gDs, axis=0).astype(np.float32)
    if z is not None:
        out["dz"] = dz
    return out
