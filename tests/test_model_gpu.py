"""The hot-path call sites of the reference's own tiny-preset HCLSMWorldModel
(hclsm/model.py:200-412), replayed through install()'s patched methods.

tests/golden/model_golden.npz holds what the unpatched reference recorded at
each call site during one forward and backward of the whole model on CPU in
fp32 (tests/golden/make_golden.py, model_cases): the inputs, outputs and
upstream gradients of DynamicSlotAttention, Level0SSM, the EventDetector's
decision, HierarchyManager.gather_events, Level1EventDynamics and
HierarchyManager.scatter_events, and the parameter gradients of those
modules.  The modules' weights come from name-seeded generators
(tests/golden/model_weights.py), so stand-ins with the reference's parameter
names regenerate them here.  Each stage runs on its recorded inputs with the
patched method and is compared at 1e-5 relative (fp32): outputs, the input
gradients that only that module produces, and every parameter gradient.
"""
import os
import sys

import numpy as np
import pytest
import torch

from conftest import rel_err
from hclsm_b200.kernels.level0 import level0_forward
from test_level0_gpu import _Level0
from test_train_gpu import _DSA, _HM, _L1

sys.path.insert(0, os.path.join(os.path.dirname(__file__), "golden"))
from model_weights import grad_sample, load_seeded  # noqa: E402

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "model_golden.npz")
TOL = 1e-5


def _t(g, k, grad=False):
    t = torch.from_numpy(g[f"m/{k}"]).cuda()
    return t.requires_grad_(True) if grad else t


def _check_param_grads(mod, g, prefix, skip=(), only=None):
    n = 0
    for name, p in mod.named_parameters():
        if name in skip or (only is not None and name not in only):
            continue
        key = f"m/{prefix}/g/{name}"
        if key not in g.files:
            assert p.grad is None or not p.grad.abs().any(), name
            continue
        assert p.grad is not None, name
        got = grad_sample(name, p.grad.detach()).cpu().numpy()
        ref = g[key]
        if name == "norm_pre_attn.bias":
            # a cancellation residue (softmax over slots): compare on the scale
            # of the same LayerNorm's weight gradient
            err = np.abs(got - ref).max() / np.abs(g[f"m/{prefix}/g/norm_pre_attn.weight"]).max()
        else:
            err = rel_err(got, ref)
        assert err < TOL, (prefix, name, err)
        n += 1
    assert n > 0


def test_slot_attention_stage():
    g = np.load(GOLD)
    slots0 = _t(g, "sa/slots0", grad=True)  # the draw of the model's _init_slots, as a leaf
    mod = _DSA(128, 16, 3, 256, slots0=slots0).cuda()
    load_seeded("sa", mod)
    inputs = _t(g, "sa/inputs", grad=True)
    slots, alive = mod(inputs)
    assert rel_err(slots.detach().cpu().numpy(), g["m/sa/slots"]) < TOL
    assert rel_err(alive.detach().cpu().numpy(), g["m/sa/alive"]) < TOL
    # the gradient recorded on the slots tensor is its total, the existence
    # head's path (alive = sigmoid(head(slots)), taken inside the module)
    # included; so the slots are back-propagated alone, and the existence
    # head's own parameters from alive's gradient
    slots.backward(_t(g, "sa/slots/grad"), retain_graph=True)
    assert rel_err(inputs.grad.cpu().numpy(), g["m/sa/inputs/grad"]) < TOL
    head = {n for n, _ in mod.named_parameters() if n.startswith("existence_head.")}
    init = {"slot_mu", "slot_log_sigma"}
    _check_param_grads(mod, g, "sa", skip=head | init)
    # _init_slots draws slots0 = mu + exp(log_sigma) * eps (dynamic_slots.py:86-96):
    # d mu = sum of d slots0, d log_sigma = sum of d slots0 * (slots0 - mu)
    gs0 = slots0.grad
    mu = mod.slot_mu.detach()
    assert rel_err(gs0.sum((0, 1)).cpu().numpy(), g["m/sa/g/slot_mu"]) < TOL
    assert rel_err((gs0 * (slots0.detach() - mu)).sum((0, 1)).cpu().numpy(), g["m/sa/g/slot_log_sigma"]) < TOL
    mod.zero_grad(set_to_none=True)
    alive.backward(_t(g, "sa/alive/grad"))
    _check_param_grads(mod, g, "sa", only=head)


def test_level0_stage():
    g = np.load(GOLD)
    mod = _Level0(d_slot=128, d_state=32, n_blocks=2).cuda()
    load_seeded("l0", mod)
    x = _t(g, "l0/x", grad=True)
    y = level0_forward(mod, x, _t(g, "l0/mask"))
    assert rel_err(y.detach().cpu().numpy(), g["m/l0/y"]) < TOL
    y.backward(_t(g, "l0/y/grad"))
    assert rel_err(x.grad.cpu().numpy(), g["m/l0/x/grad"]) < TOL
    _check_param_grads(mod, g, "l0")


def test_event_stages():
    from hclsm_b200.kernels.sparse_event_attn import event_detect

    g = np.load(GOLD)
    # the detector's decision from the model's own probabilities and threshold
    mask = event_detect(_t(g, "ed/probs"), _t(g, "ed/thr"))
    assert torch.equal(mask.cpu(), torch.from_numpy(g["m/ed/mask"]))
    assert torch.equal(mask.cpu(), torch.from_numpy(g["m/g/mask"]))
    hm = _HM()
    states = _t(g, "g/states")
    ev, pad, kmax = hm.gather_events(states, mask)
    assert torch.equal(ev.cpu(), torch.from_numpy(g["m/g/ev"]))
    assert torch.equal(pad.cpu(), torch.from_numpy(g["m/g/pad"]))
    l1 = _L1(128, 256, int(g["m/n_heads"]), 2).cuda()
    load_seeded("l1", l1)
    x = _t(g, "l1/x", grad=True)
    y = l1(x, _t(g, "l1/pad"), _t(g, "l1/obj_mask"))
    assert rel_err(y.detach().cpu().numpy(), g["m/l1/y"]) < TOL
    y.backward(_t(g, "l1/y/grad"))
    _check_param_grads(l1, g, "l1")
    base = _t(g, "s/base", grad=True)
    upd = _t(g, "s/upd", grad=True)
    out = hm.scatter_events(base, upd, mask)
    assert torch.equal(out.detach().cpu(), torch.from_numpy(g["m/s/y"]))
    out.backward(_t(g, "s/y/grad"))
    assert torch.equal(upd.grad.cpu(), torch.from_numpy(g["m/s/upd/grad"]))
