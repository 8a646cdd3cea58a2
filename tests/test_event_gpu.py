"""Parity of the sm_100a sparse event attention against the reference's golden
vectors, its known-answer tests and the CPU oracle (1e-5 relative for fp32,
2e-2 relative for bf16)."""
import os

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import event_attn as oev
from hclsm_b200.kernels import EventTransformer, sparse_event_attention_fused, sparse_event_attn_fn
from hclsm_b200.kernels.sparse_event_attn import event_compact
from hclsm_b200.workloads import event_inputs

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "event_golden.npz")


def _np(t):
    return t.detach().float().cpu().numpy()


def _gold():
    g = np.load(GOLD)
    W = {k[len("ev/w/"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("ev/w/")}
    return g, W


def test_golden_fp32_fused_and_callable():
    g, W = _gold()
    tr = EventTransformer.from_state(W, int(g["ev/n_heads"]), "cuda", dtype=torch.float32)
    st, m = torch.from_numpy(g["ev/states"]).cuda(), torch.from_numpy(g["ev/mask"]).cuda()
    assert rel_err(_np(sparse_event_attn_fn(st, m, tr)), g["ev/y_naive"]) < 1e-5
    # a Python attn_fn sees the reference's padded batch
    assert rel_err(_np(sparse_event_attn_fn(st, m, lambda f: tr(f))), g["ev/y_vectorized"]) < 1e-5


def test_golden_model_path_with_dead_slots():
    g, W = _gold()
    tr = EventTransformer.from_state(W, int(g["ev/n_heads"]), "cuda", dtype=torch.float32)
    st, m = torch.from_numpy(g["ev/states"]).cuda(), torch.from_numpy(g["ev/mask"]).cuda()
    alive = torch.from_numpy(g["ev/alive"]).cuda()
    y = sparse_event_attention_fused(st, m, tr, obj_mask=alive)
    assert rel_err(_np(y), g["ev/y_model"]) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_known_answers(dtype):
    """tests/test_kernels.py:182-232 of the reference."""
    st = torch.randn(2, 16, 8, 32).to(dtype).cuda()
    m = torch.zeros(2, 16, device="cuda")
    m[0, [2, 5, 10]] = 1
    m[1, [1, 7]] = 1
    out = sparse_event_attn_fn(st, m, lambda x: x * 2.0)
    assert torch.equal(out[0, 0], st[0, 0]) and torch.equal(out[0, 3], st[0, 3])
    assert torch.equal(out[0, 2], st[0, 2] * 2) and torch.equal(out[1, 7], st[1, 7] * 2)
    assert torch.equal(sparse_event_attn_fn(st, torch.zeros(2, 16, device="cuda"), lambda x: x), st)
    assert torch.all(sparse_event_attn_fn(st, torch.ones(2, 16, device="cuda"), lambda x: x * 0) == 0)
    m2 = torch.zeros(2, 16, device="cuda")
    m2[0, [2, 5, 10]] = 1
    m2[1, [1, 7, 9, 14]] = 1
    ident = sparse_event_attn_fn(st, m2, lambda x: x)
    assert torch.equal(ident, st)


@pytest.mark.parametrize("B,T,p,mdtype", [(7, 300, 0.3, torch.float32), (8, 64, 0.1, torch.float32),
                                          (3, 50, 0.0, torch.float32), (2, 40, 1.0, torch.float32),
                                          (1, 1, 1.0, torch.float32), (3000, 5, 0.4, torch.float32),
                                          (5, 700, 0.5, torch.bfloat16)])
def test_compaction_matches_nonzero_order(B, T, p, mdtype):
    gen = torch.Generator().manual_seed(5)
    m = (torch.rand(B, T, generator=gen) < p).float()
    idx, pos, counts, meta = event_compact(m.to(mdtype).cuda())
    nz = torch.nonzero(m.reshape(-1) > 0.5).flatten()
    n = int(meta[0])
    assert n == len(nz) and torch.equal(idx[:n].cpu().long(), nz)
    assert torch.equal(counts[:B].cpu(), (m > 0.5).sum(1).int())
    assert int(meta[1]) == int((m > 0.5).sum(1).max())
    p = pos.cpu()
    assert torch.equal(p[nz], torch.arange(n, dtype=torch.int32))


def test_max_events_truncates():
    st = torch.randn(2, 10, 4, 16).cuda()
    m = torch.zeros(2, 10, device="cuda")
    m[0, [1, 3, 6]] = 1
    m[1, [0, 9]] = 1
    out = sparse_event_attn_fn(st, m, lambda x: x + 1.0, max_events=2)
    ref = oev.naive_sparse_event_attention(_np(st), _np(m), lambda f: f + 1.0, max_events=2)
    assert np.array_equal(_np(out), ref)


def test_config3_bf16_vs_oracle():
    d = event_inputs(seed=0)
    W = d["weights"]
    Wq = {k: (t.to(torch.bfloat16).float() if t.dim() == 2 else t) for k, t in W.items()}
    tr = EventTransformer.from_state(W, d["heads"], "cuda", dtype=torch.bfloat16)
    st = d["states"].to(torch.bfloat16)
    y = sparse_event_attn_fn(st.cuda(), d["mask"].cuda(), tr)
    Wn = {k: t.numpy() for k, t in Wq.items()}
    ref = oev.naive_sparse_event_attention(st.float().numpy(), d["mask"].numpy(),
                                           lambda f: oev.level1_event(f, Wn, d["heads"], d["layers"]))
    assert rel_err(_np(y), ref) < 2e-2
    # non-event frames are bit-identical copies
    nz = d["mask"] < 0.5
    assert torch.equal(y.cpu()[nz], st[nz])


DET_GOLD = os.path.join(os.path.dirname(__file__), "golden", "detector_golden.npz")


def _ref_detector_tail(probs, thr):
    hard = (probs > thr).float()
    mask = hard - probs.detach() + probs
    if hard.sum(dim=1).min() == 0:
        mask = mask.clone()
        mask[:, 0] = 1.0
    return mask


@pytest.mark.parametrize("case", ["ed0", "ed1"])
def test_detector_tail_matches_reference_golden(case):
    """EventDetector's mask (event_detector.py:162-170) from the reference's
    own probabilities: bit-identical mask, gradient to the probabilities, and
    the attached compaction equals that of the mask."""
    from hclsm_b200.kernels.sparse_event_attn import _cached_compaction, event_detect
    g = np.load(DET_GOLD)
    probs = torch.from_numpy(g[f"{case}/probs"]).cuda().requires_grad_(True)
    thr = torch.tensor([float(g[f"{case}/thr"])], device="cuda")
    mask = event_detect(probs, thr)
    assert torch.equal(mask.detach().cpu(), torch.from_numpy(g[f"{case}/mask"]))
    (mask * torch.from_numpy(g[f"{case}/w"]).cuda()).sum().backward()
    assert torch.equal(probs.grad.cpu(), torch.from_numpy(g[f"{case}/dprobs"]))
    idx, pos, counts, meta = _cached_compaction(mask)
    ref = event_compact(mask.detach())
    n = int(ref[3][0])
    assert int(meta[0]) == n and int(meta[1]) == int(ref[3][1])
    assert torch.equal(idx[:n], ref[0][:n]) and torch.equal(pos, ref[1]) and torch.equal(counts, ref[2])


@pytest.mark.parametrize("B,T,empty_rows", [(8, 64, []), (8, 64, [3]), (5, 300, [0, 4]), (3, 7, [0, 1, 2]),
                                            (1200, 3, [7])])
def test_detector_tail_vs_torch(B, T, empty_rows):
    from hclsm_b200.kernels.sparse_event_attn import _cached_compaction, event_detect
    gen = torch.Generator().manual_seed(B * T)
    probs = torch.rand(B, T, generator=gen)
    for r in empty_rows:
        probs[r] = probs[r] * 0.4  # below the threshold everywhere
    probs = probs.cuda().requires_grad_(True)
    p2 = probs.detach().clone().requires_grad_(True)
    thr = torch.tensor([0.6], device="cuda")
    mask = event_detect(probs, thr)
    ref = _ref_detector_tail(p2, 0.6)
    assert torch.equal(mask, ref)
    w = torch.randn(B, T, generator=gen).cuda()
    (mask * w).sum().backward()
    (ref * w).sum().backward()
    assert torch.equal(probs.grad, p2.grad)
    idx, pos, counts, meta = _cached_compaction(mask)
    assert int(meta[2]) == (1 if empty_rows else 0)
    nz = torch.nonzero(ref.detach().reshape(-1) > 0.5).flatten()
    assert int(meta[0]) == len(nz) and torch.equal(idx[: len(nz)].long(), nz)


def test_gather_scatter_use_the_detector_compaction():
    """The patched HierarchyManager.gather_events / scatter_events give the
    same results from the compaction the detector attached as from their own."""
    from hclsm_b200 import install as inst
    from hclsm_b200.kernels.sparse_event_attn import event_detect
    gen = torch.Generator().manual_seed(9)
    probs = torch.rand(6, 20, generator=gen).cuda()
    probs[2] *= 0.3
    mask = event_detect(probs, torch.tensor([0.7], device="cuda"))
    plain = mask.detach().clone()
    assert getattr(plain, "_hclsm_events", None) is None
    states = torch.randn(6, 20, 4, 16, generator=gen).cuda()
    gather = inst._make_gather(None)
    scatter = inst._make_scatter(None)
    with torch.no_grad():
        e1, p1, k1 = gather(None, states, mask)
        e2, p2, k2 = gather(None, states, plain)
        assert k1 == k2 and torch.equal(e1, e2) and torch.equal(p1, p2)
        upd = torch.randn(e1.shape, generator=gen).cuda()
        s1 = scatter(None, states, upd, mask)
        s2 = scatter(None, states, upd, plain)
        assert torch.equal(s1, s2)
        # an in-place edit of the mask after the detector drops the attached
        # compaction: gather and scatter follow the edited mask
        mask[1, :] = 1.0
        plain[1, :] = 1.0
        e3, p3, k3 = gather(None, states, mask)
        e4, p4, k4 = gather(None, states, plain)
        assert k3 == k4 == 20 and torch.equal(e3, e4) and torch.equal(p3, p4)
        upd = torch.randn(e3.shape, generator=gen).cuda()
        assert torch.equal(scatter(None, states, upd, mask), scatter(None, states, upd, plain))


def _mha_call(qkv, kp, frames, T, H, HD, scale):
    from hclsm_b200 import _lib
    out = torch.empty(frames * T, H * HD, dtype=torch.bfloat16, device="cuda")
    rc = _lib.load().hclsm_event_mha(_lib.ptr(qkv), _lib.ptr(kp), _lib.ptr(out), frames, T, H, HD, scale,
                                     _lib.dtype_code(torch.bfloat16), _lib.stream_ptr(qkv.device))
    _lib.check(rc, "hclsm_event_mha")
    return out


@pytest.mark.parametrize("frames,T", [(58, 32), (7, 16), (9, 64), (1, 32), (33, 16)])
@pytest.mark.parametrize("padded", [False, True])
def test_event_mha_tcgen05_and_mma_vs_torch(frames, T, padded, monkeypatch):
    """Both attention kernels (tcgen05 for head dim 64 and T in {16, 32, 64},
    mma.sync otherwise or when selected) against fp32 torch attention on the
    same bf16 q|k|v, with dead slots ignored as keys (a frame with every key
    ignored gives NaN in both, as torch does)."""
    H, HD = 6, 64
    E = H * HD
    g = torch.Generator().manual_seed(frames * T)
    qkv = torch.randn(frames * T, 3 * E, generator=g).to(torch.bfloat16).cuda()
    kp = None
    if padded:
        kp = (torch.rand(frames, T, generator=g) < 0.3).to(torch.uint8)
        if frames > 1:
            kp[0] = 1  # a frame whose keys are all ignored
        kp = kp.cuda()
    scale = HD ** -0.5
    q, k, v = (qkv.float().reshape(frames, T, 3, H, HD)[:, :, i].transpose(1, 2) for i in range(3))
    logits = (q @ k.transpose(-1, -2)) * scale
    if kp is not None:
        logits = logits.masked_fill(kp.bool()[:, None, None, :], float("-inf"))
    ref = (torch.softmax(logits, dim=-1) @ v).transpose(1, 2).reshape(frames * T, E)
    outs = {}
    for sel in ("tc", "mma"):
        if sel == "mma":
            monkeypatch.setenv("HCLSM_EVENT_MHA", "mma")
        else:
            monkeypatch.delenv("HCLSM_EVENT_MHA", raising=False)
        outs[sel] = _mha_call(qkv, kp, frames, T, H, HD, scale).float()
    for sel, o in outs.items():
        nan_ref = torch.isnan(ref)
        assert torch.equal(torch.isnan(o), nan_ref), sel
        assert rel_err(o[~nan_ref].cpu().numpy(), ref[~nan_ref].cpu().numpy()) < 2e-2, sel


@pytest.mark.parametrize("max_events", [None, 2])
def test_sparse_event_attn_fn_gradients(max_events):
    """sparse_event_attn_fn with a Python attn_fn under autograd: gradients to
    the states and to attn_fn's parameters equal those of the reference's
    clone-and-assign loop (sparse_event_attn.py:35-86) restated in torch."""
    from hclsm_b200.kernels import sparse_event_attn_fn
    gen = torch.Generator().manual_seed(21)
    B, T, N, D = 3, 9, 4, 16
    states = torch.randn(B, T, N, D, generator=gen).cuda()
    mask = (torch.rand(B, T, generator=gen) < 0.4).float().cuda()
    mask[2] = 0.0
    mask[2, 5] = 1.0
    lin = torch.nn.Linear(D, D).cuda()
    w = torch.randn(B, T, N, D, generator=gen).cuda()
    s1 = states.clone().requires_grad_(True)
    out = sparse_event_attn_fn(s1, mask, lambda f: torch.tanh(lin(f)), max_events=max_events)
    (out * w).sum().backward()
    g_lin = [p.grad.clone() for p in lin.parameters()]
    lin.zero_grad()
    s2 = states.clone().requires_grad_(True)
    ref = s2.clone()
    for b in range(B):
        idx = torch.nonzero(mask[b] > 0.5).flatten()
        if max_events is not None:
            idx = idx[:max_events]
        if len(idx):
            ref[b, idx] = torch.tanh(lin(s2[b, idx]))
    (ref * w).sum().backward()
    assert rel_err(out.detach().cpu().numpy(), ref.detach().cpu().numpy()) < 1e-6
    assert rel_err(s1.grad.cpu().numpy(), s2.grad.cpu().numpy()) < 1e-6
    for a, p in zip(g_lin, lin.parameters()):
        assert rel_err(a.cpu().numpy(), p.grad.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("C", [1536, 97])
@pytest.mark.parametrize("udt", [torch.float32, torch.bfloat16])
def test_swiglu_kernel(C, udt):
    """hclsm_swiglu (SwiGLUFFN's silu(a) * b, level1_event.py:28) for fp32 and
    bf16 products, even (column pairs) and odd C, against torch in fp32."""
    from hclsm_b200 import _lib
    gen = torch.Generator().manual_seed(C)
    u = (torch.randn(301, 2 * C, generator=gen) * 3).to(udt).cuda()
    ref = torch.nn.functional.silu(u[:, :C].float()) * u[:, C:].float()
    for odt, tol in ((torch.float32, 1e-6), (torch.bfloat16, 8e-3)):
        y = torch.empty(301, C, dtype=odt, device="cuda")
        rc = _lib.load().hclsm_swiglu(_lib.ptr(u), _lib.dtype_code(udt), _lib.ptr(y), 301, C, _lib.dtype_code(odt),
                                      _lib.stream_ptr(u.device))
        _lib.check(rc, "hclsm_swiglu")
        assert float((y.float() - ref).abs().max() / ref.abs().max()) < tol
