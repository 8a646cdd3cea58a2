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


def test_graphed_event_training_step():
    """Gather -> Level-1 stack -> scatter, forward + backward, with the event
    compaction (a host read of the event count) done before the capture."""
    from hclsm_b200.kernels.sparse_event_attn import event_compact
    from hclsm_b200.kernels.training import event_gather_train, event_scatter_train, level1_train
    from hclsm_b200.workloads import Level1Module, event_inputs

    dev = torch.device("cuda")
    e = event_inputs(B=3, T=16, N=8, D=64, heads=2, layers=2, p=0.3, seed=4, device=dev)
    mod = Level1Module.from_weights(e["weights"], e["heads"], e["layers"], dev)
    states = e["states"].to(torch.bfloat16).requires_grad_(True)
    B, T, N, D = states.shape
    idx, pos, counts, meta = event_compact(e["mask"])
    K = max(int(meta[1].item()), 1)
    w = torch.randn(B, T, N, D, device=dev)
    params = [states] + list(mod.parameters())

    def step():
        ev = event_gather_train(states, idx, pos, counts, meta, K)
        upd = level1_train(mod, ev.reshape(B * K, N, D), None, torch.bfloat16)
        out = event_scatter_train(states, upd.reshape(B, K, N, D), idx, pos, counts, meta, K)
        (out.float() * w).sum().backward()

    for p in params:
        p.grad = None
    step()
    torch.cuda.synchronize()
    ref = _grads(params)
    g = GraphedStep(step, params)
    g.replay()
    torch.cuda.synchronize()
    _same(_grads(params), ref)
