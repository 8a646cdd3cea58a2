"""The C-ABI library loads without a GPU and exports every entry point that
include/hclsm_b200.h declares (no compute calls)."""
import ctypes
import os
import re

from hclsm_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "hclsm_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(hclsm_[a-z0-9_]+)\s*\(", src)))


def test_every_declared_symbol_is_exported():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = _declared()
    assert "hclsm_ssm_scan_fwd" in names and "hclsm_ssm_scan_bwd" in names
    for n in names:
        assert hasattr(lib, n), n


def test_python_binding_covers_header():
    assert set(_declared()) == set(_lib.SIGNATURES)


def test_version_and_workspace_query_on_host():
    lib = _lib.load()
    assert lib.hclsm_version() >= 1
    assert lib.hclsm_ssm_scan_bwd_workspace_size(256, 64, 768, 16) > 0
    assert lib.hclsm_ssm_scan_bwd_workspace_size(2, 16, 32, 128) == 0  # d_state > 64: unsupported
