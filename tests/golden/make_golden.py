"""Generate golden vectors from the reference implementation itself.

Run in a container that has the reference source tree (pure Python + torch):

    python tests/golden/make_golden.py --reference <path to RightNow-AI/hclsm>

Writes ``tests/golden/*.npz``.  Each case stores its inputs and the reference's
outputs, computed on CPU in fp32 by the reference functions named in the key.
The oracle (``oracle/``) is pinned against these files by
``tests/test_oracle_golden.py``; nothing at test or bench time needs the
reference tree.
"""
from __future__ import annotations

import argparse
import copy
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _np(t):
    return t.detach().cpu().float().numpy().copy()


def scan_cases():
    from hclsm.kernels import ssm_scan_kernel as sk

    out = {}
    # (a) the reference test fixtures, tests/test_kernels.py:120-128 distributions
    shapes = [(2, 16, 32, 8), (1, 8, 64, 16), (4, 32, 16, 4)]
    for ci, (Bn, T, d, s) in enumerate(shapes):
        g = torch.Generator().manual_seed(100 + ci)
        x = torch.randn(Bn, T, d, generator=g)
        dt = torch.rand(Bn, T, d, generator=g).abs() + 0.01
        A_log = torch.randn(d, s, generator=g)
        Bp = torch.randn(Bn, T, s, generator=g)
        C = torch.randn(Bn, T, s, generator=g)
        dy = torch.randn(Bn, T, d, generator=g)
        out.update(_scan_case(sk, f"test{ci}", x, dt, A_log, Bp, C, dy))
    # (b) BASELINE value distributions (configs 0/1/4) at a small size
    g = torch.Generator().manual_seed(7)
    Bn, T, d, s = 4, 24, 64, 16
    x = torch.randn(Bn, T, d, generator=g)
    dt = F.softplus(torch.randn(Bn, T, d, generator=g) - 2.0)
    A_log = torch.empty(d, s).uniform_(0.0, float(np.log(16.0)), generator=g)
    Bp = torch.randn(Bn, T, s, generator=g)
    C = torch.randn(Bn, T, s, generator=g)
    dy = torch.randn(Bn, T, d, generator=g)
    Dv = torch.randn(d, generator=g)
    z = torch.randn(Bn, T, d, generator=g)
    out.update(_scan_case(sk, "base", x, dt, A_log, Bp, C, dy, Dv=Dv, z=z))
    return out


def _scan_case(sk, name, x, dt, A_log, Bp, C, dy, Dv=None, z=None):
    o = {f"{name}/x": _np(x), f"{name}/dt": _np(dt), f"{name}/A_log": _np(A_log), f"{name}/B": _np(Bp),
         f"{name}/C": _np(C), f"{name}/dy": _np(dy)}
    # forward: sequential (CPU dispatch; clamped) and parallel (GPU semantics)
    o[f"{name}/y_sequential"] = _np(sk.sequential_ssm_scan(x, dt, A_log, Bp, C))
    o[f"{name}/y_parallel"] = _np(sk.parallel_ssm_scan_pytorch(x, dt, A_log, Bp, C))
    # backward: autograd through both
    for tag, fn in (("sequential", sk.sequential_ssm_scan), ("parallel", sk.parallel_ssm_scan_pytorch)):
        leaves = [t.clone().requires_grad_(True) for t in (x, dt, A_log, Bp, C)]
        y = fn(*leaves)
        y.backward(dy)
        for k, t in zip(("dx", "ddt", "dA_log", "dB", "dC"), leaves):
            o[f"{name}/{k}_{tag}"] = _np(t.grad)
    # backward: _TritonSSMScan.backward called directly (its body is PyTorch)
    if hasattr(sk, "_TritonSSMScan"):
        class Ctx:
            pass
        ctx = Ctx()
        ctx.saved_tensors = (x.float(), dt.float(), A_log, Bp.float(), C.float(), None)
        grads = sk._TritonSSMScan.backward(ctx, dy)
        for k, t in zip(("dx", "ddt", "dA_log", "dB", "dC"), grads):
            o[f"{name}/{k}_tritonbwd"] = _np(t)
    if Dv is not None:
        # composed extension: y_out = (scan + D*x) * silu(z), gate form of
        # hclsm/dynamics/level0_ssm.py:73,104 — built from the reference scan
        o[f"{name}/D"] = _np(Dv)
        o[f"{name}/z"] = _np(z)
        leaves = [t.clone().requires_grad_(True) for t in (x, dt, A_log, Bp, C, Dv, z)]
        xs, dts, As, Bs, Cs, Ds, zs = leaves
        y = (sk.parallel_ssm_scan_pytorch(xs, dts, As, Bs, Cs) + Ds * xs) * F.silu(zs)
        y.backward(dy)
        o[f"{name}/y_gated"] = _np(y)
        for k, t in zip(("dx", "ddt", "dA_log", "dB", "dC", "dD", "dz"), leaves):
            o[f"{name}/{k}_gated"] = _np(t.grad)
    return o


def block_cases():
    """SimplifiedSSMBlock forward and input/parameter gradients
    (hclsm/dynamics/level0_ssm.py:30-107), weights drawn so the clamps bind."""
    from hclsm.dynamics.level0_ssm import SimplifiedSSMBlock

    g = torch.Generator().manual_seed(500)
    blk = SimplifiedSSMBlock(d_model=32, d_state=16)
    with torch.no_grad():
        for name, p in blk.named_parameters():
            if name.startswith("norm"):
                continue
            if name == "A_log":
                p.copy_(torch.empty(p.shape).uniform_(-1.0, 0.5, generator=g))  # some exp(A_log) > 1: clamp binds
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.3)
    x = torch.randn(6, 12, 32, generator=g, requires_grad=True)
    dy = torch.randn(6, 12, 32, generator=g)
    y = blk(x)
    y.backward(dy)
    out = {"blk/x": _np(x), "blk/dy": _np(dy), "blk/y": _np(y), "blk/dx": _np(x.grad)}
    for name, p in blk.named_parameters():
        out[f"blk/w/{name}"] = _np(p)
        out[f"blk/g/{name}"] = _np(p.grad)
    return out


def level0_cases():
    """Level0SSM forward and gradients (hclsm/dynamics/level0_ssm.py:126-220)
    with SimplifiedSSMBlocks, a mask with dead objects and inputs large enough
    that the epilogue's +-100 clamp binds; and the same module without a mask."""
    from hclsm.config import Level0Config
    from hclsm.dynamics.level0_ssm import Level0SSM

    g = torch.Generator().manual_seed(600)
    mod = Level0SSM(Level0Config(d_state=16, n_blocks=2, expand_ratio=2), d_slot=32)
    with torch.no_grad():
        for name, p in mod.named_parameters():
            if "norm" in name:
                continue
            if name.endswith("A_log"):
                p.copy_(torch.empty(p.shape).uniform_(-1.0, 0.5, generator=g))
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.2)
    out = {}
    for case, use_mask in (("l0m", True), ("l0", False)):
        x = torch.randn(2, 3, 10, 32, generator=g)
        x[0, 0, 4, :6] = 400.0  # carried by the residuals past the clamp
        x.requires_grad_(True)
        mask = torch.tensor([[1.0, 1.0, 0.0], [1.0, 0.0, 1.0]]) if use_mask else None
        dy = torch.randn(2, 3, 10, 32, generator=g)
        mod.zero_grad()
        y = mod(x, mask)
        y.backward(dy)
        out.update({f"{case}/x": _np(x), f"{case}/dy": _np(dy), f"{case}/y": _np(y), f"{case}/dx": _np(x.grad)})
        if mask is not None:
            out[f"{case}/mask"] = _np(mask)
        for name, p in mod.named_parameters():
            out[f"{case}/g/{name}"] = _np(p.grad)
    for name, p in mod.named_parameters():
        out[f"l0w/{name}"] = _np(p)
    # the same module and inputs in float64: the exact answer the fp32 results
    # (the reference's and this library's) are both measured against
    mod64 = copy.deepcopy(mod).double()
    for case in ("l0m", "l0"):
        x = torch.from_numpy(out[f"{case}/x"]).double().requires_grad_(True)
        mask = torch.from_numpy(out[f"{case}/mask"]).double() if f"{case}/mask" in out else None
        mod64.zero_grad()
        y = mod64(x, mask)
        y.backward(torch.from_numpy(out[f"{case}/dy"]).double())
        out[f"{case}/y64"] = y.detach().numpy().copy()
        out[f"{case}/dx64"] = x.grad.numpy().copy()
        for name, p in mod64.named_parameters():
            out[f"{case}/g64/{name}"] = p.grad.numpy().copy()
    return out


def dsa_cases():
    """DynamicSlotAttention.forward (hclsm/objects/dynamic_slots.py:133-203)
    under no_grad with fixed initial slots (the module's _init_slots replaced,
    its draw is random), 3 iterations, the existence head, and slot birth.  With
    the softmax over slots every token receives attention 1 up to rounding, so
    the birth energy is rounding noise: birth_threshold -1 forces births (the
    token chosen is arbitrary), 0.7 (the default) never births."""
    from hclsm.config import ObjectConfig
    from hclsm.objects.dynamic_slots import DynamicSlotAttention

    out = {}
    for case, thr, seed0 in (("dsa_birth", -1.0, 700), ("dsa", 0.7, 800)):
        # the first seed whose existence probabilities all sit at least 0.1
        # from the threshold, so bf16 rounding cannot flip a dormant decision
        for seed in range(seed0, seed0 + 100):
            g = torch.Generator().manual_seed(seed)
            cfg = ObjectConfig(d_slot=32, n_max_slots=6, n_iterations=3, existence_threshold=0.5,
                               birth_threshold=thr)
            mod = DynamicSlotAttention(cfg, d_input=24)
            with torch.no_grad():
                for name, p in mod.named_parameters():
                    if "norm" in name:
                        continue
                    p.copy_(torch.randn(p.shape, generator=g) * 0.2)
            slots0 = torch.randn(3, 6, 32, generator=g) * 0.5
            mod._init_slots = lambda B, device, s0=slots0: s0.clone()
            inputs = torch.randn(3, 10, 24, generator=g)
            with torch.no_grad():
                slots, alive, attn = mod(inputs, return_attention=True)
            if float((alive - 0.5).abs().min()) > 0.1 and bool((alive < 0.5).any()):
                break
        out.update({f"{case}/inputs": _np(inputs), f"{case}/slots0": _np(slots0), f"{case}/slots": _np(slots),
                    f"{case}/alive": _np(alive), f"{case}/attn": _np(attn), f"{case}/thr": np.array(thr)})
        for name, p in mod.named_parameters():
            out[f"{case}/w/{name}"] = _np(p)
    return out


def detector_cases():
    """EventDetector.forward (hclsm/dynamics/event_detector.py:133-172): its
    probabilities, the straight-through mask and the gradient of sum(mask * w)
    with respect to the probabilities; "ed0" has a video without an event (the
    t = 0 rule fires), "ed1" does not."""
    from hclsm.dynamics.event_detector import EventDetector

    out = {}
    for case, want_empty, seed0 in (("ed0", True, 900), ("ed1", False, 950)):
        for seed in range(seed0, seed0 + 200):
            g = torch.Generator().manual_seed(seed)
            det = EventDetector(d_input=16, threshold=0.5)
            with torch.no_grad():
                for name, p in det.named_parameters():
                    if name == "threshold_logit" or "norm" in name:
                        continue
                    p.copy_(torch.randn(p.shape, generator=g) * 0.4)
            states = torch.randn(4, 12, 16, generator=g)
            probs, mask = det(states)
            thr = float(det.learned_threshold.detach())
            empty = bool(((probs > thr).sum(dim=1) == 0).any())
            margin = float((probs - thr).abs().min())
            if empty == want_empty and margin > 1e-3:
                break
        probs_leaf = probs.detach().clone().requires_grad_(True)
        hard = (probs_leaf > thr).float()
        m2 = hard - probs_leaf.detach() + probs_leaf
        if hard.sum(dim=1).min() == 0:
            m2 = m2.clone()
            m2[:, 0] = 1.0
        w = torch.randn(4, 12, generator=g)
        (m2 * w).sum().backward()
        out.update({f"{case}/probs": _np(probs), f"{case}/mask": _np(mask), f"{case}/thr": np.array(thr, np.float32),
                    f"{case}/w": _np(w), f"{case}/dprobs": _np(probs_leaf.grad)})
    return out


def slot_cases():
    from hclsm.kernels.slot_attention_kernel import naive_slot_attention
    from hclsm.config import ObjectConfig
    from hclsm.objects.dynamic_slots import DynamicSlotAttention

    out = {}
    for ci, (Bn, N, M, D) in enumerate([(2, 16, 64, 128), (1, 8, 32, 64), (2, 32, 49, 64)]):
        g = torch.Generator().manual_seed(200 + ci)
        Q = torch.randn(Bn, N, D, generator=g)
        K = torch.randn(Bn, M, D, generator=g)
        V = torch.randn(Bn, M, D, generator=g)
        o, a = naive_slot_attention(Q, K, V)
        out.update({f"core{ci}/Q": _np(Q), f"core{ci}/K": _np(K), f"core{ci}/V": _np(V),
                    f"core{ci}/out": _np(o), f"core{ci}/attn": _np(a)})
    # DynamicSlotAttention._iteration_step x 3 (hclsm/objects/dynamic_slots.py:98-131)
    g = torch.Generator().manual_seed(300)
    F_, N, M, D = 3, 8, 49, 64
    cfg = ObjectConfig(d_slot=D, n_max_slots=N, n_iterations=3)
    mod = DynamicSlotAttention(cfg, d_input=D)
    with torch.no_grad():
        for name, p in mod.named_parameters():
            if "norm" in name:
                continue  # LayerNorm affine stays at gamma=1, beta=0
            p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    slots = torch.randn(F_, N, D, generator=g)
    k = torch.randn(F_, M, D, generator=g)
    v = torch.randn(F_, M, D, generator=g)
    out["iter/slots0"] = _np(slots)
    out["iter/k"] = _np(k)
    out["iter/v"] = _np(v)
    for name, p in mod.named_parameters():
        out[f"iter/w/{name}"] = _np(p)
    s = slots
    with torch.no_grad():
        for i in range(3):
            s = mod._iteration_step(s, k, v)
            out[f"iter/slots{i + 1}"] = _np(s)
    return out


def event_cases():
    from hclsm.config import Level1Config
    from hclsm.dynamics.level1_event import Level1EventDynamics
    from hclsm.dynamics.hierarchy_manager import HierarchyManager
    from hclsm.kernels.sparse_event_attn import naive_sparse_event_attention, sparse_event_attention

    out = {}
    g = torch.Generator().manual_seed(400)
    Bn, T, N, D = 3, 10, 6, 64
    cfg = Level1Config(d_model=64, n_layers=2, n_heads=4)
    l1 = Level1EventDynamics(cfg, d_slot=D)
    with torch.no_grad():
        for name, p in l1.named_parameters():
            if "norm" in name:
                continue
            p.copy_(torch.randn(p.shape, generator=g) * 0.02)
    l1.eval()
    states = torch.randn(Bn, T, N, D, generator=g)
    mask = (torch.rand(Bn, T, generator=g) < 0.3).float()
    mask[2] = 0.0
    mask[2, 0] = 1.0  # at least one event per video, as event_detector.py:167-170 forces
    # Level1EventDynamics.forward takes (B, K, N, D) (level1_event.py:101) while
    # sparse_event_attn_fn hands attn_fn a (B*K, N, D) tensor
    # (sparse_event_attn.py:73-74); each event frame is processed on its own, so
    # the adapter runs it as K=1.
    def attn_fn(f):
        return l1(f[:, None])[:, 0]

    with torch.no_grad():
        y_naive = naive_sparse_event_attention(states, mask, attn_fn)
        y_vec = sparse_event_attention(states, mask, attn_fn)
        hm = HierarchyManager(D, 32)
        ev, pad, kmax = hm.gather_events(states, mask)
        alive = torch.ones(Bn, N)
        alive[1, 4:] = 0.0
        upd = l1(ev, pad, alive)
        y_model = hm.scatter_events(states, upd, mask)
    out.update({"ev/states": _np(states), "ev/mask": _np(mask), "ev/y_naive": _np(y_naive),
                "ev/y_vectorized": _np(y_vec), "ev/alive": _np(alive), "ev/y_model": _np(y_model),
                "ev/n_heads": np.array(cfg.n_heads), "ev/n_layers": np.array(cfg.n_layers)})
    for name, p in l1.named_parameters():
        out[f"ev/w/{name}"] = _np(p)
    return out


def train_cases():
    """Training-mode fixtures (fp32, CPU): gradients the reference's autograd
    takes through (a) three DynamicSlotAttention._iteration_step calls
    (hclsm/objects/dynamic_slots.py:98-131) w.r.t. the initial slots, k, v and
    every parameter, with inputs that make the +-30 logit clamp and the +-50
    state clamp bind; (b) DynamicSlotAttention.forward (:133-203) with fixed
    initial slots, loss on slots and existence; (c) the model's event path
    HierarchyManager.gather_events -> Level1EventDynamics(ev, pad, alive) ->
    scatter_events (hierarchy_manager.py:42-118, level1_event.py:85-133).
    Each loss is sum(output * w) with a fixed random w."""
    from hclsm.config import Level1Config, ObjectConfig
    from hclsm.dynamics.hierarchy_manager import HierarchyManager
    from hclsm.dynamics.level1_event import Level1EventDynamics
    from hclsm.objects.dynamic_slots import DynamicSlotAttention

    out = {}
    # (a) iterations
    g = torch.Generator().manual_seed(1100)
    F_, N, M, D = 3, 8, 49, 64
    mod = DynamicSlotAttention(ObjectConfig(d_slot=D, n_max_slots=N, n_iterations=3), d_input=D)
    with torch.no_grad():
        for name, p in mod.named_parameters():
            if "norm" in name:
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g) if name.endswith("weight")
                        else 0.1 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.1)
    slots = torch.randn(F_, N, D, generator=g)
    slots[0, 1, :5] = 70.0  # past the +-50 clamp
    slots[1, 2, 3:9] = -65.0
    k = torch.randn(F_, M, D, generator=g)
    v = torch.randn(F_, M, D, generator=g)
    k[2, 7] *= 40.0  # logits past +-30
    w = torch.randn(F_, N, D, generator=g)
    leaves = [t.clone().requires_grad_(True) for t in (slots, k, v)]
    s = leaves[0]
    for _ in range(3):
        s = mod._iteration_step(s, leaves[1], leaves[2])
    (s * w).sum().backward()
    out.update({"it/slots0": _np(slots), "it/k": _np(k), "it/v": _np(v), "it/w": _np(w), "it/slots3": _np(s),
                "it/dslots": _np(leaves[0].grad), "it/dk": _np(leaves[1].grad), "it/dv": _np(leaves[2].grad)})
    for name, p in mod.named_parameters():
        out[f"it/p/{name}"] = _np(p)
        if p.grad is not None:
            out[f"it/g/{name}"] = _np(p.grad)
    # (b) the whole forward, differentiable
    g = torch.Generator().manual_seed(1200)
    cfg = ObjectConfig(d_slot=32, n_max_slots=6, n_iterations=3, existence_threshold=0.5, birth_threshold=0.7)
    mod = DynamicSlotAttention(cfg, d_input=24)
    with torch.no_grad():
        for name, p in mod.named_parameters():
            if "norm" in name:
                continue
            p.copy_(torch.randn(p.shape, generator=g) * 0.2)
    slots0 = torch.randn(3, 6, 32, generator=g) * 0.5
    mod._init_slots = lambda B, device, s0=slots0: s0.clone()
    inputs = torch.randn(3, 10, 24, generator=g, requires_grad=True)
    ws = torch.randn(3, 6, 32, generator=g)
    wa = torch.randn(3, 6, generator=g)
    sl, alive = mod(inputs)
    ((sl * ws).sum() + (alive * wa).sum()).backward()
    out.update({"dsa/inputs": _np(inputs), "dsa/slots0": _np(slots0), "dsa/ws": _np(ws), "dsa/wa": _np(wa),
                "dsa/slots": _np(sl), "dsa/alive": _np(alive), "dsa/dinputs": _np(inputs.grad)})
    for name, p in mod.named_parameters():
        out[f"dsa/p/{name}"] = _np(p)
        if p.grad is not None:
            out[f"dsa/g/{name}"] = _np(p.grad)
    # (c) the event path of the model
    g = torch.Generator().manual_seed(1300)
    Bn, T, N, D = 3, 10, 6, 64
    l1 = Level1EventDynamics(Level1Config(d_model=64, n_layers=2, n_heads=4), d_slot=D)
    with torch.no_grad():
        for name, p in l1.named_parameters():
            if "norm" in name:
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g) if name.endswith("weight")
                        else 0.1 * torch.randn(p.shape, generator=g))
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.1)
    states = torch.randn(Bn, T, N, D, generator=g, requires_grad=True)
    mask = (torch.rand(Bn, T, generator=g) < 0.3).float()
    mask[2] = 0.0
    mask[2, 0] = 1.0
    alive = torch.ones(Bn, N)
    alive[1, 4:] = 0.0
    wy = torch.randn(Bn, T, N, D, generator=g)
    hm = HierarchyManager(D, 32)
    ev, pad, kmax = hm.gather_events(states, mask)
    upd = l1(ev, pad, alive)
    y = hm.scatter_events(states, upd, mask)
    (y * wy).sum().backward()
    out.update({"ev/states": _np(states), "ev/mask": _np(mask), "ev/alive": _np(alive), "ev/wy": _np(wy),
                "ev/y": _np(y), "ev/dstates": _np(states.grad), "ev/n_heads": np.array(4), "ev/n_layers": np.array(2)})
    for name, p in l1.named_parameters():
        out[f"ev/p/{name}"] = _np(p)
        out[f"ev/g/{name}"] = _np(p.grad)
    return out


def model_cases():
    """The tiny-preset HCLSMWorldModel (hclsm/model.py:200-412) run forward and
    backward on CPU in fp32 (loss = sum(final_prediction * w)).  Recorded at
    every hot-path call site: the inputs, outputs and upstream gradients of
    DynamicSlotAttention (with the initial slots its _init_slots drew),
    Level0SSM, the EventDetector's decision, HierarchyManager.gather_events,
    Level1EventDynamics and HierarchyManager.scatter_events, plus the
    parameter gradients of those modules.  Their weights come from name-seeded
    generators (model_weights.py), so the fixture stores none."""
    from hclsm.config import HCLSMConfig
    from hclsm.model import HCLSMWorldModel

    sys.path.insert(0, HERE)
    from model_weights import grad_sample, load_seeded

    torch.manual_seed(1400)
    model = HCLSMWorldModel(HCLSMConfig.tiny())
    model.eval()
    load_seeded("sa", model.slot_attention)
    load_seeded("l0", model.level0_ssm)
    load_seeded("l1", model.level1_event)
    rec = {}

    def keep(name, t):
        rec[name] = t
        if t.requires_grad:
            t.register_hook(lambda g, n=name: rec.__setitem__(n + "/grad", g))

    sa, l0, ed, l1, hm = (model.slot_attention, model.level0_ssm, model.event_detector, model.level1_event,
                          model.hierarchy_manager)
    f_init, f_sa, f_l0, f_ed, f_l1 = sa._init_slots, sa.forward, l0.forward, ed.forward, l1.forward
    f_g, f_s = hm.gather_events, hm.scatter_events

    def init_slots(B, device):
        s0 = f_init(B, device)
        rec["sa/slots0"] = s0.detach().clone()
        return s0

    def sa_fwd(inputs, return_attention=False):
        keep("sa/inputs", inputs)
        slots, alive = f_sa(inputs)
        keep("sa/slots", slots)
        keep("sa/alive", alive)
        return slots, alive

    def l0_fwd(obj_states, obj_mask=None):
        keep("l0/x", obj_states)
        rec["l0/mask"] = obj_mask
        y = f_l0(obj_states, obj_mask)
        keep("l0/y", y)
        return y

    def ed_fwd(states):
        probs, mask = f_ed(states)
        rec["ed/probs"] = probs.detach()
        rec["ed/mask"] = mask.detach()
        return probs, mask

    def gather(states, event_mask):
        keep("g/states", states)
        rec["g/mask"] = event_mask.detach()
        ev, pad, k = f_g(states, event_mask)
        keep("g/ev", ev)
        rec["g/pad"] = pad
        return ev, pad, k

    def l1_fwd(ev, pad=None, obj_mask=None):
        keep("l1/x", ev)
        rec["l1/pad"] = pad
        rec["l1/obj_mask"] = obj_mask
        y = f_l1(ev, pad, obj_mask)
        keep("l1/y", y)
        return y

    def scatter(base, upd, event_mask):
        keep("s/base", base)
        keep("s/upd", upd)
        y = f_s(base, upd, event_mask)
        keep("s/y", y)
        return y

    sa._init_slots, sa.forward, l0.forward, ed.forward, l1.forward = init_slots, sa_fwd, l0_fwd, ed_fwd, l1_fwd
    hm.gather_events, hm.scatter_events = gather, scatter
    g = torch.Generator().manual_seed(1401)
    video = torch.rand(2, 3, 3, 224, 224, generator=g)
    out = model(video)
    w = torch.randn(out.predicted_states.shape, generator=g)
    (out.predicted_states * w).sum().backward()
    res = {"m/w": _np(w), "m/pred": _np(out.predicted_states)}
    for k, v in rec.items():
        if v is not None:
            res[f"m/{k}"] = _np(v)
    for prefix, mod in (("sa", sa), ("l0", l0), ("l1", l1)):
        for name, p in mod.named_parameters():
            if p.grad is not None:
                res[f"m/{prefix}/g/{name}"] = _np(grad_sample(name, p.grad))
    res["m/ed/thr"] = _np(ed.learned_threshold.reshape(1))
    res["m/n_heads"] = np.array(model.level1_event.blocks[0].attn.num_heads)
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", default=None, help="write only this fixture (level0, dsa, detector, train, model)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.reference))
    torch.set_num_threads(1)
    if args.only == "level0":
        np.savez_compressed(os.path.join(HERE, "level0_golden.npz"), **level0_cases())
        print("wrote level0_golden.npz")
        return
    if args.only == "detector":
        np.savez_compressed(os.path.join(HERE, "detector_golden.npz"), **detector_cases())
        print("wrote detector_golden.npz")
        return
    if args.only == "model":
        np.savez_compressed(os.path.join(HERE, "model_golden.npz"), **model_cases())
        print("wrote model_golden.npz")
        return
    if args.only == "train":
        np.savez_compressed(os.path.join(HERE, "train_golden.npz"), **train_cases())
        print("wrote train_golden.npz")
        return
    if args.only == "dsa":
        np.savez_compressed(os.path.join(HERE, "dsa_golden.npz"), **dsa_cases())
        print("wrote dsa_golden.npz")
        return
    np.savez_compressed(os.path.join(HERE, "scan_golden.npz"), **scan_cases(), **block_cases())
    np.savez_compressed(os.path.join(HERE, "slot_golden.npz"), **slot_cases())
    np.savez_compressed(os.path.join(HERE, "event_golden.npz"), **event_cases())
    np.savez_compressed(os.path.join(HERE, "level0_golden.npz"), **level0_cases())
    np.savez_compressed(os.path.join(HERE, "dsa_golden.npz"), **dsa_cases())
    np.savez_compressed(os.path.join(HERE, "detector_golden.npz"), **detector_cases())
    np.savez_compressed(os.path.join(HERE, "train_golden.npz"), **train_cases())
    np.savez_compressed(os.path.join(HERE, "model_golden.npz"), **model_cases())
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
