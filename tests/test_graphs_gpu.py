"""A whole training step captured as one CUDA graph (hclsm_b200.graphs):
the graphed forward + backward of the slot-attention iteration (3 refinement
steps at config-2 shapes) and of the SimplifiedSSMBlock (config-1 shapes,
bf16 autocast) must give exactly the eager step's gradients, also after new
inputs are copied into the captured tensors."""
import pytest
import torch

from hclsm_b200.graphs import GraphedStep
from hclsm_b200.workloads import SlotIterModule, slot_inputs, ssm_block_inputs

pytestmark = pytest.mark.gpu


def _grads(params):
    return [p.grad.clone() for p in params]


def _same(a, b):
    assert len(a) == len(b)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


def test_graphed_slot_training_step():
    from hclsm_b200.kernels.training import slot_iteration_train

    dev = torch.device("cuda")
    d = slot_inputs(F=16, seed=11, device=dev)
    W = d["weights"]
    mod = SlotIterModule.from_weights(W, 384, dev)
    k = torch.nn.functional.linear(d["inputs"], W["project_k.weight"]).to(torch.bfloat16)
    v = torch.nn.functional.linear(d["inputs"], W["project_v.weight"]).to(torch.bfloat16)
    w = torch.randn(d["slots"].shape, device=dev)
    leaves = [t.detach().clone().requires_grad_(True) for t in (d["slots"], k, v)]
    params = leaves + list(mod.parameters())

    def step():
        s = leaves[0]
        for _ in range(3):
            s = slot_iteration_train(mod, s, leaves[1], leaves[2], torch.bfloat16)
        (s * w).sum().backward()

    def eager():
        for p in params:
            p.grad = None
        step()
        torch.cuda.synchronize()
        return _grads(params)

    ref = eager()
    g = GraphedStep(step, params)
    g.replay()
    torch.cuda.synchronize()
    _same(_grads(params), ref)
    # new slots copied into the captured input, replayed twice
    with torch.no_grad():
        leaves[0].mul_(0.5).add_(0.1)
    ref2 = eager()
    g = GraphedStep(step, params)
    for _ in range(2):
        g()
    torch.cuda.synchronize()
    _same(_grads(params), ref2)


def test_graphed_ssm_block_step():
    from hclsm_b200.install import _ssm_block_forward

    blk, x = ssm_block_inputs(nseq=32, seed=30, device="cuda")
    x.requires_grad_(True)
    params = [x] + list(blk.parameters())

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=False):
            y = _ssm_block_forward(blk, x)
        y.float().sum().backward()

    for p in params:
        p.grad = None
    step()
    torch.cuda.synchronize()
    ref = _grads(params)
    g = GraphedStep(step, params)
    g.replay()
    torch.cuda.synchronize()
    _same(_grads(params), ref)
