"""Parity of the sm_100a slot attention (core and fused iteration) against the
reference's golden vectors and the CPU oracle.  Tolerances: 1e-5 relative for
fp32 I/O, 2e-2 relative for bf16 with fp32 accumulation."""
import os

import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import slot_attn as osl
from hclsm_b200.kernels import (SlotIterationParams, fold_query_into_keys, key_value_weights, project_keys_values,
                                slot_attention_core, slot_attention_fn, slot_attention_iterations)
from hclsm_b200.workloads import slot_inputs

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "slot_golden.npz")


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.mark.parametrize("ci", [0, 1, 2])
def test_core_golden_fp32(ci):
    g = np.load(GOLD)
    Q, K, V = (torch.from_numpy(g[f"core{ci}/{k}"]).cuda() for k in ("Q", "K", "V"))
    out, attn = slot_attention_fn(Q, K, V, backend="naive")
    assert rel_err(_np(out), g[f"core{ci}/out"]) < 1e-5
    assert rel_err(_np(attn), g[f"core{ci}/attn"]) < 1e-5
    assert torch.allclose(attn.sum(dim=1), torch.ones_like(attn.sum(dim=1)), atol=1e-5)


@pytest.mark.parametrize("shape", [(2, 16, 64, 128), (1, 8, 32, 64), (4, 32, 196, 256), (128, 32, 196, 384),
                                   (3, 5, 33, 64), (2, 64, 130, 512), (1, 17, 1, 16)])
def test_core_bf16_vs_oracle(shape):
    B, N, M, D = shape
    gen = torch.Generator().manual_seed(sum(shape))
    Q, K, V = (torch.randn(B, n, D, generator=gen).to(torch.bfloat16) for n in (N, M, M))
    for clamp, eps in ((0.0, 0.0), (30.0, 0.0), (0.0, 1e-8)):
        out, attn = slot_attention_core(Q.cuda(), K.cuda(), V.cuda(), clamp=clamp, eps=eps, attn_fp32=True)
        Qn, Kn, Vn = (t.float().numpy() for t in (Q, K, V))
        logits = (Qn @ Kn.transpose(0, 2, 1)) * D ** -0.5
        if clamp:
            logits = np.clip(logits, -clamp, clamp)
        e = np.exp(logits - logits.max(1, keepdims=True))
        a = e / (e.sum(1, keepdims=True) + eps)
        assert rel_err(_np(attn), a) < 2e-2
        assert rel_err(_np(out), a @ Vn) < 2e-2


def test_core_backward_matches_autograd():
    gen = torch.Generator().manual_seed(3)
    Q, K, V = (torch.randn(2, n, 64, generator=gen).cuda().requires_grad_(True) for n in (8, 40, 40))
    out, attn = slot_attention_fn(Q, K, V)
    (out.square().sum() + attn.sum()).backward()
    Q2, K2, V2 = (t.detach().clone().requires_grad_(True) for t in (Q, K, V))
    lg = torch.bmm(Q2, K2.transpose(1, 2)) * 64 ** -0.5
    a = torch.softmax(lg, dim=1)
    o = torch.bmm(a, V2)
    (o.square().sum() + a.sum()).backward()
    for x, y in ((Q, Q2), (K, K2), (V, V2)):
        assert rel_err(_np(x.grad), _np(y.grad)) < 1e-4


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
def test_iterations_golden(dtype, tol):
    """fp32: every weight product in fp32 (the reference without autocast);
    bf16: bf16 operands, fp32 accumulation (the reference under autocast)."""
    g = np.load(GOLD)
    W = {k[len("iter/w/"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("iter/w/")}
    p = SlotIterationParams.from_state(W, "cuda", dtype=dtype)
    k, v = (torch.from_numpy(g[f"iter/{n}"]).cuda() for n in ("k", "v"))
    s = torch.from_numpy(g["iter/slots0"]).cuda()
    out = slot_attention_iterations(s, k, v, p, 3)
    assert rel_err(_np(out), g["iter/slots3"]) < tol


def test_config2_three_iterations_vs_oracle():
    d = slot_inputs(seed=0)
    W = d["weights"]
    Wq = {k: t.to(torch.bfloat16).float() if t.dim() == 2 else t for k, t in W.items()}
    # k and v as DynamicSlotAttention.forward builds them (dynamic_slots.py:152-154)
    inp = d["inputs"].to(torch.bfloat16).float()
    k = (inp @ Wq["project_k.weight"].T).to(torch.bfloat16)
    v = (inp @ Wq["project_v.weight"].T).to(torch.bfloat16)
    p = SlotIterationParams.from_state(W, "cuda")
    out = slot_attention_iterations(d["slots"].cuda(), k.cuda(), v.cuda(), p, 3)
    Wn = {kk: t.numpy() for kk, t in Wq.items()}
    s = d["slots"].numpy()
    for _ in range(3):
        s = osl.iteration_step(s, k.float().numpy(), v.float().numpy(), Wn)
    assert rel_err(_np(out), s) < 2e-2


def test_config2_folded_keys_vs_oracle():
    """Keys projected with W_k^T W_q (no per-step W_q product) against the
    oracle's unfolded steps at 2e-2, and against this library's unfolded path."""
    d = slot_inputs(seed=0)
    W = d["weights"]
    Wq = {k: t.to(torch.bfloat16).float() if t.dim() == 2 else t for k, t in W.items()}
    inp = d["inputs"].to(torch.bfloat16)
    k = (inp.float() @ Wq["project_k.weight"].T).to(torch.bfloat16)
    v = (inp.float() @ Wq["project_v.weight"].T).to(torch.bfloat16)
    p = SlotIterationParams.from_state(W, "cuda")
    wkq = fold_query_into_keys(W["project_k.weight"], W["project_q.weight"]).cuda()
    kf = torch.mm(inp.cuda().reshape(-1, inp.shape[-1]), wkq).reshape(k.shape)
    # the stacked k/v product gives the same keys and values
    w_kv = key_value_weights(W["project_k.weight"], W["project_v.weight"], W["project_q.weight"]).cuda()
    kf2, vf2 = project_keys_values(inp.cuda(), w_kv)
    assert torch.equal(kf2, kf)
    assert rel_err(_np(vf2), _np(v)) < 1e-2
    out = slot_attention_iterations(d["slots"].cuda(), kf, v.cuda(), p, 3, keys_folded=True)
    plain = slot_attention_iterations(d["slots"].cuda(), k.cuda(), v.cuda(), p, 3)
    Wn = {kk: t.numpy() for kk, t in Wq.items()}
    s = d["slots"].numpy()
    for _ in range(3):
        s = osl.iteration_step(s, k.float().numpy(), v.float().numpy(), Wn)
    assert rel_err(_np(out), s) < 2e-2
    assert rel_err(_np(out), _np(plain)) < 2e-2


@pytest.mark.parametrize("shape", [(128, 32, 196, 384), (3, 5, 33, 128), (2, 64, 130, 256)])
def test_core_tcgen05_and_mma_agree_with_oracle(shape, monkeypatch):
    """Shapes the tcgen05 core covers, run once on it and once on the
    mma.sync core (HCLSM_SLOT_CORE=mma forces that one): both against the
    oracle at 2e-2 (bf16 operands, fp32 accumulation)."""
    B, N, M, D = shape
    gen = torch.Generator().manual_seed(sum(shape) + 1)
    Q, K, V = (torch.randn(B, n, D, generator=gen).to(torch.bfloat16) for n in (N, M, M))
    ro, ra = osl.naive_slot_attention(Q.float().numpy(), K.float().numpy(), V.float().numpy())
    for sel in ("tc", "mma"):
        if sel == "mma":
            monkeypatch.setenv("HCLSM_SLOT_CORE", "mma")
        else:
            monkeypatch.delenv("HCLSM_SLOT_CORE", raising=False)
        out, attn = slot_attention_core(Q.cuda(), K.cuda(), V.cuda(), attn_fp32=True)
        assert rel_err(_np(out), ro) < 2e-2, sel
        assert rel_err(_np(attn), ra) < 2e-2, sel


@pytest.mark.parametrize("H", [384, 128, 1024])
def test_row_fused_stages_match_separate_kernels(H):
    """hclsm_gru_cell_ln and hclsm_residual_clamp_ln against the separate
    GRU / residual-clamp and LayerNorm kernels they fuse."""
    from hclsm_b200.kernels.slot_attention_kernel import (gru_cell, gru_cell_ln, layernorm, residual_clamp,
                                                          residual_clamp_ln)
    gen = torch.Generator().manual_seed(H)
    R = 77
    gi, gh = (torch.randn(R, 3 * H, generator=gen).cuda() for _ in range(2))
    b_ih, b_hh = (torch.randn(3 * H, generator=gen).cuda() * 0.1 for _ in range(2))
    h0 = torch.randn(R, H, generator=gen).cuda() * 20
    w, b = 1 + 0.1 * torch.randn(H, generator=gen).cuda(), 0.1 * torch.randn(H, generator=gen).cuda()
    for dt in (torch.float32, torch.bfloat16):
        h1, m1 = gru_cell_ln(gi, gh, b_ih, b_hh, h0, w, b, dt)
        h2 = gru_cell(gi, gh, b_ih, b_hh, h0)
        m2 = layernorm(h2, w, b, out_dtype=dt)
        assert rel_err(_np(h1), _np(h2)) < 1e-6  # same formula; the compiler may contract differently
        assert rel_err(_np(m1), _np(m2)) < (1e-6 if dt == torch.float32 else 8e-3)
        mm = torch.randn(R, H, generator=gen).cuda() * 40
        o1b = torch.empty(R, H, dtype=torch.bfloat16, device="cuda")
        o2b = torch.empty_like(o1b)
        o1, n1 = residual_clamp_ln(h1, mm, b, 50.0, w, b, dt, out_bf16=o1b)
        o2 = residual_clamp(h2, mm, b, 50.0, out_bf16=o2b)
        n2 = layernorm(o2, w, b, out_dtype=dt)
        assert rel_err(_np(o1), _np(o2)) < 1e-6 and rel_err(_np(o1b), _np(o2b)) < 8e-3
        assert rel_err(_np(n1), _np(n2)) < (1e-6 if dt == torch.float32 else 8e-3)
    # bf16 gate products: the same as the fp32 kernel on the rounded values
    gib, ghb = gi.to(torch.bfloat16), gh.to(torch.bfloat16)
    h3, m3 = gru_cell_ln(gib, ghb, b_ih, b_hh, h0, w, b, torch.float32)
    h4 = gru_cell(gib.float(), ghb.float(), b_ih, b_hh, h0)
    assert rel_err(_np(h3), _np(h4)) < 1e-6
    assert rel_err(_np(m3), _np(layernorm(h4, w, b, out_dtype=torch.float32))) < 1e-6
    # bf16 MLP output into the residual kernel: the same as fp32 on the rounded values
    mmb = (torch.randn(R, H, generator=gen).cuda() * 40).to(torch.bfloat16)
    o5, n5 = residual_clamp_ln(h3, mmb, b, 50.0, w, b, torch.float32)
    o6 = residual_clamp(h3, mmb.float(), b, 50.0)
    assert rel_err(_np(o5), _np(o6)) < 1e-6
    assert rel_err(_np(n5), _np(layernorm(o6, w, b, out_dtype=torch.float32))) < 1e-6


@pytest.mark.parametrize("F,N,M,D", [(128, 32, 196, 384), (5, 20, 70, 128), (3, 8, 49, 64)])
def test_slot_attn_iter_entry_point(F, N, M, D):
    """hclsm_slot_attn_iter (the whole step behind one C call) against the
    Python path's bf16 step and the oracle's fp32 step, three iterations."""
    from hclsm_b200.kernels.slot_attention_kernel import slot_attn_iter
    d = slot_inputs(F=F, N=N, M=M, D=D, seed=F + D)
    W = d["weights"]
    Wq = {k: t.to(torch.bfloat16).float() if t.dim() == 2 else t for k, t in W.items()}
    inp = d["inputs"].to(torch.bfloat16).float()
    k = (inp @ Wq["project_k.weight"].T).to(torch.bfloat16)
    v = (inp @ Wq["project_v.weight"].T).to(torch.bfloat16)
    p = SlotIterationParams.from_state(W, "cuda")
    s1 = d["slots"].cuda()
    s2 = d["slots"].cuda()
    for _ in range(3):
        s1 = slot_attn_iter(s1, k.cuda(), v.cuda(), p)
        s2 = slot_attention_iterations(s2, k.cuda(), v.cuda(), p, 1)
    assert rel_err(_np(s1), _np(s2)) < 2e-3
    Wn = {kk: t.numpy() for kk, t in Wq.items()}
    s = d["slots"].numpy()
    for _ in range(3):
        s = osl.iteration_step(s, k.float().numpy(), v.float().numpy(), Wn)
    assert rel_err(_np(s1), s) < 2e-2
