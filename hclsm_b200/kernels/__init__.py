"""Mirror of ``hclsm.kernels`` (hclsm/kernels/__init__.py:9-35) backed by sm_100a kernels."""
from .ssm_scan_kernel import ssm_scan_fn, ssm_scan  # noqa: F401

__all__ = ["ssm_scan_fn", "ssm_scan"]
