"""Seeded synthetic workloads with the shapes and value distributions of the
five benchmark configurations (no datasets are involved).

All generators draw fp32 values from a ``torch.Generator`` seeded per call and
cast afterwards, so a CPU oracle fed the cast tensors sees identical bits.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass(frozen=True)
class ScanConfig:
    name: str
    videos: int
    slots: int
    L: int
    d_inner: int
    d_state: int
    dtype: torch.dtype
    backward: bool
    clamp: bool

    @property
    def nseq(self) -> int:
        return self.videos * self.slots


# Config 0 runs the CPU dispatch in the reference (sequential_ssm_scan, clamped);
# configs 1 and 4 follow the reference's CUDA semantics (unclamped).
SCAN_CONFIGS = {
    0: ScanConfig("tiny scan fwd fp32", 2, 16, 16, 512, 16, torch.float32, False, True),
    1: ScanConfig("small scan fwd+bwd bf16", 8, 32, 64, 768, 16, torch.bfloat16, True, False),
    4: ScanConfig("base scan fwd+bwd bf16", 64, 128, 256, 2048, 16, torch.bfloat16, True, False),
}


def scan_inputs(nseq, L, d_inner, d_state, dtype=torch.float32, seed=0, device="cpu", gated=False,
                grad=True):
    """x, B, C ~ N(0,1); dt = softplus(N(0,1) - 2); A_log ~ U(0, ln 16) so that
    A = -exp(A_log) in [-16, -1]; D, z, dy ~ N(0,1).  A_log and D stay fp32."""
    g = torch.Generator(device=device).manual_seed(seed)

    def randn(*shape):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32)

    out = {}
    out["x"] = randn(nseq, L, d_inner).to(dtype)
    out["dt"] = F.softplus(randn(nseq, L, d_inner) - 2.0).to(dtype)
    out["A_log"] = torch.rand(d_inner, d_state, generator=g, device=device) * math.log(16.0)
    out["B"] = randn(nseq, L, d_state).to(dtype)
    out["C"] = randn(nseq, L, d_state).to(dtype)
    if gated:
        out["D"] = randn(d_inner)
        out["z"] = randn(nseq, L, d_inner).to(dtype)
    if grad:
        out["dy"] = randn(nseq, L, d_inner).to(dtype)
    return out


def scan_inputs_range(start, nseq, L, d_inner, d_state, dtype=torch.bfloat16, seed=0, device="cpu", block=64):
    """Sequences [start, start + nseq) of a global seeded config-4 style job:
    x, dt, B, C, dy with the distributions of ``scan_inputs``, drawn per block
    of ``block`` sequences from a generator seeded by (seed, block index), so
    any shard of the job (start and nseq multiples of ``block``) regenerates
    exactly the sequences a single-GPU run of the whole job sees.  A_log
    depends on the seed only."""
    if start % block or nseq % block:
        raise ValueError("start and nseq must be multiples of the block size")
    g = torch.Generator(device=device).manual_seed(seed)
    A_log = torch.rand(d_inner, d_state, generator=g, device=device) * math.log(16.0)
    out = {k: torch.empty(nseq, L, d_inner if k in ("x", "dt", "dy") else d_state, dtype=dtype, device=device)
           for k in ("x", "dt", "B", "C", "dy")}
    for i in range(nseq // block):
        gb = torch.Generator(device=device).manual_seed(seed * 1000003 + start // block + i)
        sl = slice(i * block, (i + 1) * block)

        def randn(*shape):
            return torch.randn(block, *shape, generator=gb, device=device, dtype=torch.float32)

        out["x"][sl] = randn(L, d_inner)
        out["dt"][sl] = F.softplus(randn(L, d_inner) - 2.0)
        out["B"][sl] = randn(L, d_state)
        out["C"][sl] = randn(L, d_state)
        out["dy"][sl] = randn(L, d_inner)
    out["A_log"] = A_log
    return out


def slot_inputs(F=128, N=32, M=196, D=384, seed=0, device="cpu"):
    """Config 2: inputs (F, M, D) = LayerNorm(N(0,1)); initial slots
    mu + |sigma| * eps with mu, sigma ~ N(0, 0.1) per dim and eps ~ N(0,1);
    every Linear / GRU weight and bias ~ N(0, 0.02); LayerNorm affines at
    gamma=1, beta=0.  Parameter names follow DynamicSlotAttention."""
    g = torch.Generator(device=device).manual_seed(seed)

    def randn(*shape, std=1.0):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std

    inputs = torch.nn.functional.layer_norm(randn(F, M, D), (D,))
    mu, sigma = randn(D, std=0.1), randn(D, std=0.1)
    slots = mu + sigma.abs() * randn(F, N, D)
    w = {}
    for name, shape in (("project_k.weight", (D, D)), ("project_v.weight", (D, D)), ("project_q.weight", (D, D)),
                        ("gru.weight_ih", (3 * D, D)), ("gru.weight_hh", (3 * D, D)), ("gru.bias_ih", (3 * D,)),
                        ("gru.bias_hh", (3 * D,)), ("mlp.0.weight", (4 * D, D)), ("mlp.0.bias", (4 * D,)),
                        ("mlp.2.weight", (D, 4 * D)), ("mlp.2.bias", (D,))):
        w[name] = randn(*shape, std=0.02)
    for name in ("norm_pre_attn", "norm_slots", "norm_input"):
        w[name + ".weight"] = torch.ones(D, device=device)
        w[name + ".bias"] = torch.zeros(D, device=device)
    return {"inputs": inputs, "slots": slots, "weights": w}


def event_inputs(B=8, T=64, N=32, D=384, heads=6, layers=3, p=0.1, seed=0, device="cpu"):
    """Config 3: states (B, T, N, D) ~ N(0,1); event mask ~ Bernoulli(p) per
    (video, t), with t=0 forced on for a video without events (as
    event_detector.py:167-170 guarantees one event); Level1EventDynamics
    weights ~ N(0, 0.02) (d_model = D, SwiGLU hidden 4D), LayerNorm affines at
    gamma=1, beta=0.  Parameter names follow Level1EventDynamics."""
    g = torch.Generator(device=device).manual_seed(seed)

    def randn(*shape, std=1.0):
        return torch.randn(*shape, generator=g, device=device, dtype=torch.float32) * std

    states = randn(B, T, N, D)
    mask = (torch.rand(B, T, generator=g, device=device) < p).float()
    none = mask.sum(1) == 0
    mask[none, 0] = 1.0
    w = {"proj_in.weight": randn(D, D, std=0.02), "proj_out.weight": randn(D, D, std=0.02),
         "norm.weight": torch.ones(D, device=device), "norm.bias": torch.zeros(D, device=device)}
    for i in range(layers):
        q = f"blocks.{i}."
        w[q + "attn.in_proj_weight"] = randn(3 * D, D, std=0.02)
        w[q + "attn.out_proj.weight"] = randn(D, D, std=0.02)
        w[q + "ffn.w1.weight"] = randn(4 * D, D, std=0.02)
        w[q + "ffn.w3.weight"] = randn(4 * D, D, std=0.02)
        w[q + "ffn.w2.weight"] = randn(D, 4 * D, std=0.02)
        for nm in ("norm1", "norm2"):
            w[q + nm + ".weight"] = torch.ones(D, device=device)
            w[q + nm + ".bias"] = torch.zeros(D, device=device)
    return {"states": states, "mask": mask, "weights": w, "heads": heads, "layers": layers}


class SSMBlockModule(torch.nn.Module):
    """Parameters of SimplifiedSSMBlock (hclsm/dynamics/level0_ssm.py:36-56)
    under the same attribute names, so that hclsm_b200.install's patched
    forward runs on it without the reference package: in_proj / gate_proj
    (d_model -> 2 d_model, no bias), dt_proj (with bias), B_proj / C_proj (no
    bias), A_log ~ -U(0, 0.5), out_proj, LayerNorm; nn.Linear's default init."""

    def __init__(self, d_model: int, d_state: int, expand: int = 2):
        super().__init__()
        di = d_model * expand
        self.d_model, self.d_state = d_model, d_state
        self.in_proj = torch.nn.Linear(d_model, di, bias=False)
        self.gate_proj = torch.nn.Linear(d_model, di, bias=False)
        self.dt_proj = torch.nn.Linear(di, di, bias=True)
        self.B_proj = torch.nn.Linear(di, d_state, bias=False)
        self.C_proj = torch.nn.Linear(di, d_state, bias=False)
        self.A_log = torch.nn.Parameter(-torch.rand(di, d_state) * 0.5)
        self.out_proj = torch.nn.Linear(di, d_model, bias=False)
        self.norm = torch.nn.LayerNorm(d_model)


def ssm_block_inputs(nseq=256, T=64, d_model=384, d_state=16, seed=0, device="cpu"):
    """A SimplifiedSSMBlock-shaped module and its input (nseq, T, d_model) ~
    N(0, 1); d_model 384 gives d_inner 768, BASELINE config 1's scan shape."""
    torch.manual_seed(seed)
    blk = SSMBlockModule(d_model, d_state).to(device)
    g = torch.Generator(device="cpu").manual_seed(seed + 1)
    x = torch.randn(nseq, T, d_model, generator=g).to(device)
    return blk, x


class SlotIterModule(torch.nn.Module):
    """The parameters DynamicSlotAttention._iteration_step uses
    (hclsm/objects/dynamic_slots.py:52-83) under the same attribute names, so
    hclsm_b200.kernels.training.slot_iteration_train runs on it without the
    reference package."""

    def __init__(self, d_slot: int):
        super().__init__()
        self.d_slot = d_slot
        self.project_q = torch.nn.Linear(d_slot, d_slot, bias=False)
        self.gru = torch.nn.GRUCell(d_slot, d_slot)
        self.norm_slots = torch.nn.LayerNorm(d_slot)
        self.mlp = torch.nn.Sequential(torch.nn.Linear(d_slot, 4 * d_slot), torch.nn.ReLU(),
                                       torch.nn.Linear(4 * d_slot, d_slot))
        self.norm_pre_attn = torch.nn.LayerNorm(d_slot)
        self.scale = d_slot ** -0.5

    @classmethod
    def from_weights(cls, w: dict, d_slot: int, device="cpu"):
        """Load the names of ``slot_inputs``' weight dict that this module has."""
        mod = cls(d_slot).to(device)
        with torch.no_grad():
            for name, p in mod.named_parameters():
                p.copy_(w[name])
        return mod


class _SwiGLU(torch.nn.Module):
    def __init__(self, d: int):
        super().__init__()
        self.w1 = torch.nn.Linear(d, 4 * d, bias=False)
        self.w3 = torch.nn.Linear(d, 4 * d, bias=False)
        self.w2 = torch.nn.Linear(4 * d, d, bias=False)


class _EventBlock(torch.nn.Module):
    def __init__(self, d: int, heads: int):
        super().__init__()
        self.norm1 = torch.nn.LayerNorm(d)
        self.attn = torch.nn.MultiheadAttention(d, heads, bias=False, batch_first=True)
        self.norm2 = torch.nn.LayerNorm(d)
        self.ffn = _SwiGLU(d)


class Level1Module(torch.nn.Module):
    """The parameters of Level1EventDynamics (hclsm/dynamics/level1_event.py:63-83:
    proj_in, EventTransformerBlocks with a bias-free MultiheadAttention and a
    SwiGLU FFN, final LayerNorm, proj_out) under the same attribute names, so
    hclsm_b200.kernels.training.level1_train runs on it without the reference
    package; d_slot = d_model = D as in ``event_inputs``."""

    def __init__(self, d: int, heads: int, layers: int):
        super().__init__()
        self.proj_in = torch.nn.Linear(d, d, bias=False)
        self.proj_out = torch.nn.Linear(d, d, bias=False)
        self.blocks = torch.nn.ModuleList([_EventBlock(d, heads) for _ in range(layers)])
        self.norm = torch.nn.LayerNorm(d)

    @classmethod
    def from_weights(cls, w: dict, heads: int, layers: int, device="cpu"):
        """Load ``event_inputs``' weight dict."""
        d = w["proj_in.weight"].shape[0]
        mod = cls(d, heads, layers).to(device)
        with torch.no_grad():
            for name, p in mod.named_parameters():
                p.copy_(w[name])
        return mod
