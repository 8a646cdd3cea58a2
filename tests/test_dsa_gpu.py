"""The patched DynamicSlotAttention.forward (device-side slot birth, fused
iterations) against the reference's golden vectors, fp32 module and inputs
(fp32 arithmetic, 1e-5 relative): existence probabilities (and the same dormant
decisions), every slot that is not born, the position of each born slot (the
first dormant one), and that a born slot is the birth projection of one of its
video's tokens.  Which token
is arbitrary in the reference itself: with the softmax over slots the birth
energy is rounding noise."""
import os

import numpy as np
import pytest
import torch
import torch.nn as nn

from conftest import rel_err
from hclsm_b200 import install as inst

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "dsa_golden.npz")


class _DSA(nn.Module):
    """DynamicSlotAttention's parameter layout (dynamic_slots.py:35-83)."""

    def __init__(self, d_slot, n_max, n_iter, exist_thr, birth_thr, d_input, slots0):
        super().__init__()
        self.d_slot, self.n_max_slots, self.n_iterations = d_slot, n_max, n_iter
        self.existence_threshold, self.birth_threshold = exist_thr, birth_thr
        self.use_gradient_checkpointing = False
        self.slot_mu = nn.Parameter(torch.zeros(d_slot))
        self.slot_log_sigma = nn.Parameter(torch.zeros(d_slot))
        self.project_k = nn.Linear(d_input, d_slot, bias=False)
        self.project_v = nn.Linear(d_input, d_slot, bias=False)
        self.project_q = nn.Linear(d_slot, d_slot, bias=False)
        self.gru = nn.GRUCell(d_slot, d_slot)
        self.norm_slots = nn.LayerNorm(d_slot)
        self.mlp = nn.Sequential(nn.Linear(d_slot, 4 * d_slot), nn.ReLU(), nn.Linear(4 * d_slot, d_slot))
        self.norm_input = nn.LayerNorm(d_input)
        self.norm_pre_attn = nn.LayerNorm(d_slot)
        self.existence_head = nn.Sequential(nn.Linear(d_slot, d_slot // 4), nn.ReLU(), nn.Linear(d_slot // 4, 1))
        self.birth_proj = nn.Linear(d_input, d_slot)
        self.scale = d_slot ** -0.5
        self._slots0 = slots0

    def _init_slots(self, B, device):
        return self._slots0.clone()

    _iteration_step = inst._make_iteration_step(None)
    forward = inst._make_dsa_forward(None)


@pytest.mark.parametrize("case", ["dsa_birth", "dsa"])
def test_patched_forward_matches_reference_golden(case):
    g = np.load(GOLD)
    slots0 = torch.from_numpy(g[f"{case}/slots0"]).cuda()
    mod = _DSA(32, 6, 3, 0.5, float(g[f"{case}/thr"]), 24, slots0).cuda()
    with torch.no_grad():
        for name, p in mod.named_parameters():
            p.copy_(torch.from_numpy(g[f"{case}/w/{name}"]))
    inputs = torch.from_numpy(g[f"{case}/inputs"]).cuda()
    with torch.no_grad():
        slots, alive, attn = mod(inputs, return_attention=True)
    ref_alive = g[f"{case}/alive"]
    assert rel_err(alive.cpu().numpy(), ref_alive) < 1e-5
    assert np.array_equal(alive.cpu().numpy() < 0.5, ref_alive < 0.5)
    ref_slots = g[f"{case}/slots"]
    dormant = ref_alive < 0.5
    births = float(g[f"{case}/thr"]) < 0 and dormant.any()
    got = slots.cpu().numpy()
    keep = np.ones(ref_slots.shape[:2], dtype=bool)
    if births:
        for b in range(ref_slots.shape[0]):
            if dormant[b].any():
                j = int(np.argmax(dormant[b]))
                keep[b, j] = False
                # the born slot is birth_proj of one of this video's tokens
                with torch.no_grad():
                    cand = mod.birth_proj(inputs[b]).cpu().numpy()  # (M, d_slot)
                err = np.abs(cand - got[b, j][None, :]).max(axis=1).min()
                assert err < 1e-4 * max(1.0, np.abs(cand).max()), (b, err)
    assert rel_err(got[keep], ref_slots[keep]) < 1e-5
    assert rel_err(attn.float().cpu().numpy(), g[f"{case}/attn"]) < 1e-5


def test_no_host_sync_in_birth():
    """The birth step runs under CUDA stream capture, which fails on any host
    read of device data (the reference's needs_birth.any())."""
    g = np.load(GOLD)
    case = "dsa_birth"
    slots0 = torch.from_numpy(g[f"{case}/slots0"]).cuda()
    mod = _DSA(32, 6, 3, 0.5, -1.0, 24, slots0).cuda()
    with torch.no_grad():
        for name, p in mod.named_parameters():
            p.copy_(torch.from_numpy(g[f"{case}/w/{name}"]))
    inputs = torch.from_numpy(g[f"{case}/inputs"]).cuda()
    with torch.no_grad():
        ref, _ = mod(inputs)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            mod(inputs)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out, _ = mod(inputs)
        graph.replay()
        torch.cuda.synchronize()
    assert torch.equal(out, ref)


def test_fused_bf16_inference_forward():
    """Under bf16 autocast without gradients the patched forward runs the
    fused path (W_q folded into the keys, stacked k/v product, fused steps,
    attention map from the core): slots, alive and the attention map against
    the reference's fp32 arithmetic (oracle/torch_ref.iteration_step) at 2e-2;
    no births (threshold above any energy)."""
    from oracle import torch_ref

    torch.manual_seed(5)
    D, N, Din, B, M = 128, 8, 96, 4, 50
    slots0 = torch.randn(B, N, D, device="cuda")
    mod = _DSA(D, N, 3, 0.5, 1e9, Din, slots0).cuda()
    inputs = torch.randn(B, M, Din, device="cuda")
    W = {n: p.detach() for n, p in mod.named_parameters()}
    with torch.no_grad():
        xn = mod.norm_input(inputs)
        k, v = mod.project_k(xn), mod.project_v(xn)
        s = slots0.clone()
        for _ in range(3):
            s = torch_ref.iteration_step(s, k, v, W)
        alive_ref = torch.sigmoid(mod.existence_head(s).squeeze(-1))
        q = mod.project_q(mod.norm_pre_attn(s))
        attn_ref = torch.softmax(torch.bmm(q, k.transpose(1, 2)) * mod.scale, dim=1)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            slots, alive, attn = mod(inputs, return_attention=True)
    assert mod._hclsm_b200_fused is not None  # the fused path ran
    assert rel_err(slots.float().cpu().numpy(), s.cpu().numpy()) < 2e-2
    assert rel_err(alive.float().cpu().numpy(), alive_ref.cpu().numpy()) < 2e-2
    assert rel_err(attn.float().cpu().numpy(), attn_ref.cpu().numpy()) < 2e-2
