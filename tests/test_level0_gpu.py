"""Level0SSM around its blocks: the masked mean over objects and the
nan_to_num / clamp / mask epilogue kernels against torch's own ops, and the
patched Level0SSM.forward against the reference's golden vectors (fp32:
1e-5 relative to the exact answer; rel = max|err| / max|ref|)."""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import rel_err
from hclsm_b200 import install as inst
from hclsm_b200.kernels.level0 import level0_epilogue, level0_forward, masked_mean_pool
from hclsm_b200.workloads import SSMBlockModule

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "level0_golden.npz")


def _ref_pool(x, m):
    if m is None:
        return x.mean(dim=1)
    n_alive = m.sum(dim=1, keepdim=True).clamp(min=1.0)
    return (x * m[:, :, None, None]).sum(dim=1) / n_alive[:, :, None]


def _ref_epi(x, m):
    y = torch.clamp(torch.nan_to_num(x, nan=0.0, posinf=100.0, neginf=-100.0), min=-100.0, max=100.0)
    return y if m is None else y * m[:, :, None, None]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("masked", [False, True])
def test_pool_and_epilogue_vs_torch(dtype, masked):
    g = torch.Generator().manual_seed(3)
    B, N, T, D = 3, 5, 7, 24
    x = (torch.randn(B, N, T, D, generator=g) * 80).to(dtype).cuda()
    x.view(-1)[::97] = float("nan")
    x.view(-1)[5::131] = float("inf")
    x.view(-1)[9::151] = float("-inf")
    m = (torch.rand(B, N, generator=g) < 0.6).float().cuda() if masked else None
    if masked:
        m[1] = 0.0  # a video with no live object
    xf = torch.nan_to_num(x.float(), nan=0.0)  # the pool's input has no nan in the model
    xp = xf.clamp(-1e4, 1e4).to(dtype)
    pool = masked_mean_pool(xp, m)
    ref = _ref_pool(xp, m)
    assert pool.dtype == ref.dtype
    assert rel_err(pool.float().cpu().numpy(), ref.float().cpu().numpy()) < (1e-6 if dtype == torch.float32 else 1e-2)
    epi = level0_epilogue(x, m)
    eref = _ref_epi(x, m)
    assert epi.dtype == eref.dtype and torch.equal(epi, eref)
    # gradients
    x1 = x.clone().requires_grad_(True)
    x2 = x.clone().requires_grad_(True)
    dy = torch.randn(eref.shape, generator=g).to(eref.dtype).cuda()
    level0_epilogue(x1, m).backward(dy)
    _ref_epi(x2, m).backward(dy)
    assert torch.equal(x1.grad, x2.grad)
    p1 = xp.clone().requires_grad_(True)
    p2 = xp.clone().requires_grad_(True)
    dp = torch.randn(ref.shape, generator=g).to(ref.dtype).cuda()
    masked_mean_pool(p1, m).backward(dp)
    _ref_pool(p2, m).backward(dp)
    assert rel_err(p1.grad.float().cpu().numpy(), p2.grad.float().cpu().numpy()) < 1e-2


class _Block(SSMBlockModule):
    def forward(self, x):
        return inst._ssm_block_forward(self, x)


class _Level0(nn.Module):
    def __init__(self, d_slot=32, d_state=16, n_blocks=2):
        super().__init__()
        self.use_gradient_checkpointing = False
        self.object_blocks = nn.ModuleList([_Block(d_slot, d_state) for _ in range(n_blocks)])
        self.global_blocks = nn.ModuleList([_Block(d_slot, d_state) for _ in range(n_blocks)])
        self.condition_proj = nn.Linear(d_slot, d_slot, bias=False)


@pytest.mark.parametrize("case", ["l0m", "l0"])
def test_patched_level0_matches_reference_golden(case):
    """Forward and every gradient against the exact answer (the reference
    module run in float64 by the fixture generator), and against the
    reference's own fp32 result within 1e-5 plus that result's distance from
    the exact answer.  Against the exact answer the bar is 1e-5, except 2e-5
    in the masked case: there the gradient of the first global block's A_log
    (a sum over the two videos' ten steps of products that carry the masked
    mean of inputs reaching 400) is ill-conditioned in fp32 -- the reference's
    fp32 result on the CPU is 9.9e-6 from exact, the same formula in plain
    PyTorch fp32 on the GPU 1.23e-5, this library 1.61e-5."""
    g = np.load(GOLD)
    mod = _Level0().cuda()
    with torch.no_grad():
        for name, p in mod.named_parameters():
            p.copy_(torch.from_numpy(g[f"l0w/{name}"]))
    x = torch.from_numpy(g[f"{case}/x"]).cuda().requires_grad_(True)
    m = torch.from_numpy(g[f"{case}/mask"]).cuda() if f"{case}/mask" in g.files else None
    y = level0_forward(mod, x, m)
    y.backward(torch.from_numpy(g[f"{case}/dy"]).cuda())
    pairs = [("y", y.detach(), g[f"{case}/y"], g[f"{case}/y64"]),
             ("dx", x.grad, g[f"{case}/dx"], g[f"{case}/dx64"])]
    pairs += [(name, p.grad, g[f"{case}/g/{name}"], g[f"{case}/g64/{name}"]) for name, p in mod.named_parameters()]
    for name, got, ref32, ref64 in pairs:
        got = got.cpu().numpy()
        assert rel_err(got, ref64) < (2e-5 if case == "l0m" else 1e-5), (name, rel_err(got, ref64))
        assert rel_err(got, ref32) < 1e-5 + rel_err(ref32, ref64), name
