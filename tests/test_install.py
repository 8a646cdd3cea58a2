"""install() patches the reference's call sites (checked on a stand-in package
with the reference's module layout; no compute), and the patched call sites
match the reference's golden vectors on the GPU."""
import os
import types

import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import rel_err
import hclsm_b200
from hclsm_b200 import install as inst

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _fake_hclsm():
    def mod(**kw):
        return types.SimpleNamespace(**kw)

    def f(*a, **k):
        return "reference"

    class Block:
        def forward(self, x):
            return "reference"

    class DSA:
        def _iteration_step(self, s, k, v):
            return "reference"

        def forward(self, inputs, return_attention=False):
            return "reference"

    class HM:
        def gather_events(self, s, m):
            return "reference"

        def scatter_events(self, b, u, m):
            return "reference"

    class L1:
        def forward(self, e, p=None, o=None):
            return "reference"

    class L0:
        def forward(self, s, m=None):
            return "reference"

    class ED:
        def forward(self, s):
            return "reference"

    kernels = mod(ssm_scan_fn=f, slot_attention_fn=f, sparse_event_attn_fn=f,
                  ssm_scan_kernel=mod(ssm_scan_fn=f), slot_attention_kernel=mod(slot_attention_fn=f),
                  sparse_event_attn=mod(sparse_event_attn_fn=f))
    dyn = mod(level0_ssm=mod(SimplifiedSSMBlock=Block, Level0SSM=L0), hierarchy_manager=mod(HierarchyManager=HM),
              level1_event=mod(Level1EventDynamics=L1), event_detector=mod(EventDetector=ED))
    objs = mod(dynamic_slots=mod(DynamicSlotAttention=DSA))
    return mod(kernels=kernels, dynamics=dyn, objects=objs), (Block, DSA, HM, L1)


def test_install_patches_and_uninstall_restores():
    pkg, (Block, DSA, HM, L1) = _fake_hclsm()
    orig = Block.forward
    done = inst.install(pkg)
    done2 = inst.install(pkg)  # idempotent
    assert done == done2 and len(done) == 14
    assert pkg.kernels.ssm_scan_fn is hclsm_b200.kernels.ssm_scan_fn
    assert pkg.kernels.ssm_scan_kernel.ssm_scan_fn is hclsm_b200.kernels.ssm_scan_fn
    assert Block.forward is not orig
    inst.uninstall()
    assert Block.forward is orig
    assert pkg.kernels.ssm_scan_fn(None) == "reference"
    assert DSA()._iteration_step(None, None, None) == "reference"


class _Block(nn.Module):
    """Attribute layout of SimplifiedSSMBlock (level0_ssm.py:34-56)."""

    def __init__(self, d_model, d_state):
        super().__init__()
        di = 2 * d_model
        self.in_proj = nn.Linear(d_model, di, bias=False)
        self.gate_proj = nn.Linear(d_model, di, bias=False)
        self.dt_proj = nn.Linear(di, di, bias=True)
        self.B_proj = nn.Linear(di, d_state, bias=False)
        self.C_proj = nn.Linear(di, d_state, bias=False)
        self.A_log = nn.Parameter(torch.zeros(di, d_state))
        self.out_proj = nn.Linear(di, d_model, bias=False)
        self.norm = nn.LayerNorm(d_model)


@pytest.mark.gpu
def test_patched_ssm_block_matches_reference_golden():
    g = np.load(os.path.join(GOLD, "scan_golden.npz"))
    blk = _Block(32, 16).cuda()
    with torch.no_grad():
        for name, p in blk.named_parameters():
            p.copy_(torch.from_numpy(g[f"blk/w/{name}"]))
    x = torch.from_numpy(g["blk/x"]).cuda().requires_grad_(True)
    y = inst._ssm_block_forward(blk, x)
    assert rel_err(y.detach().cpu().numpy(), g["blk/y"]) < 1e-5
    y.backward(torch.from_numpy(g["blk/dy"]).cuda())
    assert rel_err(x.grad.cpu().numpy(), g["blk/dx"]) < 1e-5
    for name, p in blk.named_parameters():
        assert rel_err(p.grad.cpu().numpy(), g[f"blk/g/{name}"]) < 1e-5, name


class _DSA(nn.Module):
    """Parameter layout of DynamicSlotAttention used by _iteration_step."""

    def __init__(self, D):
        super().__init__()
        self.d_slot = D
        self.project_q = nn.Linear(D, D, bias=False)
        self.gru = nn.GRUCell(D, D)
        self.norm_slots = nn.LayerNorm(D)
        self.mlp = nn.Sequential(nn.Linear(D, 4 * D), nn.ReLU(), nn.Linear(4 * D, D))
        self.norm_pre_attn = nn.LayerNorm(D)


@pytest.mark.gpu
def test_patched_iteration_step_matches_reference_golden():
    g = np.load(os.path.join(GOLD, "slot_golden.npz"))
    m = _DSA(64).cuda()
    sd = {k[len("iter/w/"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("iter/w/")}
    with torch.no_grad():
        for name, p in m.named_parameters():
            p.copy_(sd[name])
    step = inst._make_iteration_step(lambda *a: None)
    s = torch.from_numpy(g["iter/slots0"]).cuda()
    k, v = (torch.from_numpy(g[f"iter/{n}"]).cuda() for n in ("k", "v"))
    with torch.no_grad():
        for i in range(3):
            s = step(m, s, k, v)
    assert s.dtype == torch.float32
    assert rel_err(s.cpu().numpy(), g["iter/slots3"]) < 1e-5  # fp32 module and inputs: fp32 arithmetic


REF = os.environ.get("HCLSM_REFERENCE", "/root/reference")


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "hclsm")), reason="reference source tree not present")
def test_install_on_the_real_reference_package():
    """install() on the reference package itself (imported from its source
    tree, CPU only, no compute): every documented call site is replaced by this
    library's function, and uninstall() restores the reference's own."""
    import importlib
    import sys

    sys.path.insert(0, REF)
    try:
        hclsm = importlib.import_module("hclsm")
        importlib.import_module("hclsm.kernels")
        l0 = importlib.import_module("hclsm.dynamics.level0_ssm")
        ds = importlib.import_module("hclsm.objects.dynamic_slots")
        hm = importlib.import_module("hclsm.dynamics.hierarchy_manager")
        l1 = importlib.import_module("hclsm.dynamics.level1_event")
        ed = importlib.import_module("hclsm.dynamics.event_detector")
        before = {(c, n): getattr(c, n) for c, n in (
            (l0.SimplifiedSSMBlock, "forward"), (l0.Level0SSM, "forward"),
            (ds.DynamicSlotAttention, "_iteration_step"), (ds.DynamicSlotAttention, "forward"),
            (hm.HierarchyManager, "gather_events"), (hm.HierarchyManager, "scatter_events"),
            (l1.Level1EventDynamics, "forward"), (ed.EventDetector, "forward"))}
        done = inst.install(hclsm)
        try:
            assert len(done) == 14, done
            assert hclsm.kernels.ssm_scan_fn is hclsm_b200.kernels.ssm_scan_fn
            assert hclsm.kernels.ssm_scan_kernel.ssm_scan_fn is hclsm_b200.kernels.ssm_scan_fn
            assert hclsm.kernels.slot_attention_fn is hclsm_b200.kernels.slot_attention_fn
            assert hclsm.kernels.sparse_event_attn_fn is hclsm_b200.kernels.sparse_event_attn_fn
            for (c, n), f in before.items():
                assert getattr(c, n) is not f, (c.__name__, n)
            assert l0.SimplifiedSSMBlock.forward is inst._ssm_block_forward
        finally:
            inst.uninstall()
        for (c, n), f in before.items():
            assert getattr(c, n) is f
    finally:
        sys.path.remove(REF)
