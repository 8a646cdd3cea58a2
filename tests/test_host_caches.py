"""Host-side caches of the training path (no GPU needed)."""
import torch

from hclsm_b200.kernels.training import _lp


def test_weight_cast_cache_follows_the_version_counter():
    """The bf16 cast of a parameter is reused while its version is unchanged
    and redone after an in-place (optimizer-style) update; fp32 needs none."""
    w = torch.nn.Parameter(torch.randn(8, 4))
    a = _lp(w, torch.bfloat16)
    assert _lp(w, torch.bfloat16) is a and torch.equal(a, w.detach().to(torch.bfloat16))
    with torch.no_grad():
        w.mul_(2.0)
    b = _lp(w, torch.bfloat16)
    assert b is not a and torch.equal(b, w.detach().to(torch.bfloat16))
    assert _lp(w, torch.float32) is w
