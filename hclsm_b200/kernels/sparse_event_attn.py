"""Sparse event attention on B200 — drop-in for hclsm/kernels/sparse_event_attn.py.

* ``sparse_event_attn_fn(states, event_mask, attn_fn, max_events=None, backend="auto")``
  keeps the reference signature (sparse_event_attn.py:242-263).  Fired frames
  are found by a device-side stream compaction (video-major, ascending time,
  as the reference's ``nonzero`` loop :62-67), gathered, passed to ``attn_fn``
  and merged back by one fused copy+scatter kernel.  A Python ``attn_fn``
  receives the reference's padded (B * K_max, N, D) batch with zero pad frames
  (:58-78); an ``EventTransformer`` (Level1EventDynamics weights) runs the
  fused transformer on the compacted frames only.
* ``EventTransformer`` restates Level1EventDynamics.forward
  (hclsm/dynamics/level1_event.py:85-133) with this library's kernels: per layer
  LayerNorm -> qkv GEMM -> per-frame multi-head attention (tensor cores) ->
  out-proj GEMM + residual; LayerNorm -> [W1 | W3] GEMM -> SwiGLU -> W2 GEMM +
  residual; final LayerNorm and proj_out.  GEMMs are library GEMMs with bf16
  operands and fp32 outputs for bf16 inputs, fp32 throughout for fp32 inputs.
"""
from __future__ import annotations

from collections import OrderedDict
from dataclasses import dataclass, field

import torch

from .. import _lib
from .slot_attention_kernel import layernorm, residual_clamp, residual_clamp_ln

__all__ = ["sparse_event_attn_fn", "EventTransformer", "event_compact", "event_detect", "event_gather", "event_scatter",
           "sparse_event_attention_fused"]


def _c(t):
    t = t.contiguous()
    if t.data_ptr() % 16:
        t = t.clone()
    return t


# ---- compaction / gather / scatter ---------------------------------------------------
def event_compact(event_mask):
    """Device-side compaction of a (B, T) mask.  Returns (idx, pos, counts, meta)
    int32 tensors: idx[k] = b*T + t of the k-th fired frame, pos[b*T+t] = k or
    -1, counts[b] per video, meta = [total, max per video]."""
    m = event_mask
    if m.dtype not in (torch.float32, torch.bfloat16):
        m = m.float()
    m = _c(m)
    B, T = m.shape
    dev = m.device
    idx = torch.empty(max(B * T, 1), dtype=torch.int32, device=dev)
    pos = torch.empty(max(B * T, 1), dtype=torch.int32, device=dev)
    counts = torch.empty(max(B, 1), dtype=torch.int32, device=dev)
    meta = torch.empty(2, dtype=torch.int32, device=dev)
    rc = _lib.load().hclsm_event_compact(_lib.ptr(m), _lib.dtype_code(m.dtype), B, T, _lib.ptr(idx), _lib.ptr(pos),
                                         _lib.ptr(counts), _lib.ptr(meta), _lib.stream_ptr(dev))
    _lib.check(rc, "hclsm_event_compact")
    return idx, pos, counts, meta


def event_detect(event_probs, threshold):
    """EventDetector's mask from its probabilities (event_detector.py:162-170)
    with the decision and the compaction on the device: hard = probs >
    threshold (a tensor, read on the device), the straight-through mask
    hard - probs.detach() + probs, and, when any video has no event, t = 0
    set to 1 in every video (the reference decides that with a host read).
    The compaction (idx, pos, counts, meta) of the final mask is attached to
    the returned mask as ``_hclsm_events`` for the gather and the scatter."""
    _lib.require_cuda(event_probs, threshold)
    B, T = event_probs.shape
    dev = event_probs.device
    p = _c(event_probs.detach().to(torch.float32))
    thr = _c(threshold.detach().to(torch.float32).reshape(-1)[:1])
    hard = torch.empty(B, T, dtype=torch.float32, device=dev)
    idx = torch.empty(B * T, dtype=torch.int32, device=dev)
    pos = torch.empty(B * T, dtype=torch.int32, device=dev)
    counts = torch.empty(B, dtype=torch.int32, device=dev)
    meta = torch.empty(3, dtype=torch.int32, device=dev)
    rc = _lib.load().hclsm_event_detect(_lib.ptr(p), _lib.ptr(thr), B, T, _lib.ptr(hard), _lib.ptr(idx),
                                        _lib.ptr(pos), _lib.ptr(counts), _lib.ptr(meta), _lib.stream_ptr(dev))
    _lib.check(rc, "hclsm_event_detect")
    mask = hard.to(event_probs.dtype) - event_probs.detach() + event_probs
    first = torch.zeros(B, T, dtype=torch.bool, device=dev)
    first[:, 0] = True
    mask = torch.where(first & (meta[2] > 0), torch.ones((), dtype=mask.dtype, device=dev), mask)
    # tagged with the mask's version: an in-place edit of the mask afterwards
    # invalidates the compaction (the gather / scatter then recompact)
    mask._hclsm_events = (mask._version, (idx, pos, counts, meta))
    return mask


def _cached_compaction(event_mask):
    """The compaction event_detect attached to this mask, or None when there is
    none or the mask was modified in place since."""
    ent = getattr(event_mask, "_hclsm_events", None)
    if ent is None or ent[0] != event_mask._version:
        return None
    return ent[1]


def event_gather(states, idx, counts, meta, n_frames, pad_k=0, out=None):
    """(n_frames, N, D) compacted frames (pad_k=0) or the padded (B*pad_k, N, D)
    layout with zero pad frames; written into ``out`` (contiguous, at least
    n_frames frames) when given."""
    B, T, N, D = states.shape
    if out is None:
        out = torch.empty(n_frames, N, D, dtype=states.dtype, device=states.device)
    if n_frames == 0:
        return out
    rc = _lib.load().hclsm_event_gather(_lib.ptr(states), _lib.ptr(idx), _lib.ptr(counts), _lib.ptr(meta),
                                        _lib.ptr(out), N * D, B, pad_k, n_frames, _lib.dtype_code(states.dtype),
                                        _lib.stream_ptr(states.device))
    _lib.check(rc, "hclsm_event_gather")
    return out


def event_scatter(states, upd, pos, counts, pad_k=0):
    """A copy of states with every fired frame replaced by its update."""
    B, T, N, D = states.shape
    out = torch.empty_like(states)
    upd = upd if upd.numel() else states  # no events: plain copy
    rc = _lib.load().hclsm_event_scatter(_lib.ptr(states), _lib.ptr(_c(upd)), _lib.ptr(pos), _lib.ptr(counts),
                                         _lib.ptr(out), B * T, N * D, T, pad_k, _lib.dtype_code(states.dtype),
                                         _lib.stream_ptr(states.device))
    _lib.check(rc, "hclsm_event_scatter")
    return out


# ---- Level-1 event transformer -----------------------------------------------------------
@dataclass
class _Layer:
    ln1_w: torch.Tensor
    ln1_b: torch.Tensor
    w_qkv_t: torch.Tensor
    w_o_t: torch.Tensor
    ln2_w: torch.Tensor
    ln2_b: torch.Tensor
    w13_t: torch.Tensor
    w2_t: torch.Tensor


@dataclass
class EventTransformer:
    """Weights of Level1EventDynamics prepared for the fused path (parameter
    names of hclsm/dynamics/level1_event.py).  Callable on (frames, N, d_slot)."""
    n_heads: int
    w_in_t: torch.Tensor
    w_out_t: torch.Tensor
    norm_w: torch.Tensor
    norm_b: torch.Tensor
    layers: list = field(default_factory=list)
    dtype: torch.dtype = torch.bfloat16
    # CUDA graphs of the whole stack, one per (frame bucket, N, d_slot, key
    # mask, input dtype, device); every op is per row or per frame, so rows of a
    # bucket past the real frame count do not touch the real rows
    _graphs: OrderedDict = field(default_factory=OrderedDict, repr=False, compare=False)
    _pool: object = field(default=None, repr=False, compare=False)
    max_graphs: int = 32

    @classmethod
    def from_state(cls, sd: dict, n_heads: int, device, dtype=torch.bfloat16):
        def w(name):
            return sd[name].detach().to(device=device, dtype=dtype).t().contiguous()

        def f(name):
            return sd[name].detach().to(device=device, dtype=torch.float32).contiguous()

        n_layers = 1 + max(int(k.split(".")[1]) for k in sd if k.startswith("blocks."))
        layers = []
        for i in range(n_layers):
            p = f"blocks.{i}."
            w13 = torch.cat([sd[p + "ffn.w1.weight"], sd[p + "ffn.w3.weight"]], 0)
            layers.append(_Layer(f(p + "norm1.weight"), f(p + "norm1.bias"), w(p + "attn.in_proj_weight"),
                                 w(p + "attn.out_proj.weight"), f(p + "norm2.weight"), f(p + "norm2.bias"),
                                 w13.detach().to(device=device, dtype=dtype).t().contiguous(),
                                 w(p + "ffn.w2.weight")))
        return cls(n_heads, w("proj_in.weight"), w("proj_out.weight"), f("norm.weight"), f("norm.bias"), layers,
                   dtype)

    @classmethod
    def from_module(cls, mod, dtype=torch.bfloat16):
        heads = mod.blocks[0].attn.num_heads
        return cls.from_state(dict(mod.named_parameters()), heads, next(mod.parameters()).device, dtype)

    def _mm(self, a, w_t):
        if self.dtype == torch.float32:
            return torch.mm(a, w_t)
        return torch.mm(a, w_t, out_dtype=torch.float32)

    def _mm_res(self, a, w_t):
        """A product that the fused residual + LayerNorm kernel reads: in the
        work dtype (bf16 under autocast, as the reference's Linear output),
        the residual sum itself stays fp32."""
        return torch.mm(a, w_t)

    def __call__(self, frames, key_padding_mask=None):
        """frames (n, N, d_slot) -> (n, N, d_slot); key_padding_mask (n, N) bool,
        True = dead slot (ignored as a key).  Replays a CUDA graph of the stack
        (captured on first use of a frame-count bucket)."""
        n = frames.shape[0]
        if n == 0:
            return frames.clone()
        if not frames.is_cuda or torch.cuda.is_current_stream_capturing():
            return self.forward(frames, key_padding_mask)
        fin, kin, out, g = self.graph_slot(n, frames.shape[1], frames.shape[2], key_padding_mask is not None,
                                           frames.dtype, frames.device)
        fin[:n].copy_(frames)
        if kin is not None:
            kin[:n].copy_(key_padding_mask)
        g.replay()
        return out[:n].clone()

    def graph_slot(self, n, N, Ds, has_kp, in_dtype, device):
        """(static input, static key mask or None, static output, graph) for
        n frames: the input and output hold a bucket of frames (n rounded up to
        a multiple of 8); fill input[:n], replay, read output[:n] before the
        next replay."""
        nb = (n + 7) // 8 * 8
        key = (nb, N, Ds, has_kp, in_dtype, str(device))
        ent = self._graphs.get(key)
        if ent is not None:
            self._graphs.move_to_end(key)
            return ent
        if self._pool is None:
            self._pool = torch.cuda.graph_pool_handle()
        fin = torch.zeros(nb, N, Ds, dtype=in_dtype, device=device)
        kin = torch.zeros(nb, N, dtype=torch.bool, device=device) if has_kp else None
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            self.forward(fin, kin)  # first run outside the capture (library handles, workspaces)
        torch.cuda.current_stream(device).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self._pool):
            out = self.forward(fin, kin)
        ent = (fin, kin, out, g)
        self._graphs[key] = ent
        while len(self._graphs) > self.max_graphs:
            self._graphs.popitem(last=False)
        return ent

    def forward(self, frames, key_padding_mask=None):
        """The stack launched op by op (no graph)."""
        n, N, Ds = frames.shape
        if n == 0:
            return frames.clone()
        dt = self.dtype
        E = self.w_in_t.shape[1]
        H = self.n_heads
        hd = E // H
        R = n * N
        x = self._mm(_c(frames.to(dt)).reshape(R, Ds), self.w_in_t)  # fp32 residual stream
        kp = None
        if key_padding_mask is not None:
            kp = _c(key_padding_mask.to(torch.uint8))
        lib = _lib.load()
        # each residual add and the LayerNorm after it run as one row kernel
        # where the row fits (E a multiple of 128, at most 1024)
        fuse = E % 128 == 0 and E <= 1024
        nl = len(self.layers)
        h = layernorm(x, self.layers[0].ln1_w, self.layers[0].ln1_b, out_dtype=dt) if nl else None
        for i, ly in enumerate(self.layers):
            qkv = _c(torch.mm(h, ly.w_qkv_t))
            a = torch.empty(R, E, dtype=dt, device=x.device)
            rc = lib.hclsm_event_mha(_lib.ptr(qkv), _lib.ptr(kp), _lib.ptr(a), n, N, H, hd, float(hd ** -0.5),
                                     _lib.dtype_code(dt), _lib.stream_ptr(x.device))
            _lib.check(rc, "hclsm_event_mha")
            if fuse:
                x, h = residual_clamp_ln(x, self._mm_res(a, ly.w_o_t), None, 0.0, ly.ln2_w, ly.ln2_b, dt)
            else:
                x = residual_clamp(x, self._mm(a, ly.w_o_t), None, 0.0)
                h = layernorm(x, ly.ln2_w, ly.ln2_b, out_dtype=dt)
            u = self._mm_res(h, ly.w13_t)  # bf16 under autocast, as the reference's Linear output
            F = u.shape[1] // 2
            s = torch.empty(R, F, dtype=dt, device=x.device)
            rc = lib.hclsm_swiglu(_lib.ptr(u), _lib.dtype_code(u.dtype), _lib.ptr(s), R, F, _lib.dtype_code(dt),
                                  _lib.stream_ptr(x.device))
            _lib.check(rc, "hclsm_swiglu")
            nw, nb = ((self.layers[i + 1].ln1_w, self.layers[i + 1].ln1_b) if i + 1 < nl
                      else (self.norm_w, self.norm_b))
            if fuse:
                x, h = residual_clamp_ln(x, self._mm_res(s, ly.w2_t), None, 0.0, nw, nb, dt)
            else:
                x = residual_clamp(x, self._mm(s, ly.w2_t), None, 0.0)
                h = layernorm(x, nw, nb, out_dtype=dt)
        if not nl:
            h = layernorm(x, self.norm_w, self.norm_b, out_dtype=dt)
        y = self._mm(h, self.w_out_t)
        return y.reshape(n, N, -1).to(frames.dtype)


def sparse_event_attention_fused(states, event_mask, transformer: EventTransformer, obj_mask=None):
    """Events of ``states`` (B, T, N, D) updated by the Level-1 transformer;
    obj_mask (B, N) (alive > 0.5) masks dead slots as keys, as the model does
    (level1_event.py:108-112)."""
    _lib.require_cuda(states, event_mask)
    states = _c(states)
    B, T, N, D = states.shape
    idx, pos, counts, meta = event_compact(event_mask)
    n = int(meta[0].item())  # one host read (the reference syncs for K_max too)
    if n == 0:
        return event_scatter(states, states[:0].reshape(0, N, D), pos, counts)
    kp = None
    if obj_mask is not None:
        dead = ~(obj_mask > 0.5)
        kp = dead[(idx[:n].long() // T)]
    if torch.cuda.is_current_stream_capturing():
        frames = event_gather(states, idx, counts, meta, n)
        upd = transformer.forward(frames, kp)
        return event_scatter(states, upd.to(states.dtype), pos, counts)
    # the frames are gathered straight into the graph's input, the graph runs
    # the stack, and the scatter reads its output
    fin, kin, out, g = transformer.graph_slot(n, N, D, kp is not None, states.dtype, states.device)
    event_gather(states, idx, counts, meta, n, out=fin)
    if kin is not None:
        kin[:n].copy_(kp)
    g.replay()
    return event_scatter(states, out[:n], pos, counts)


def sparse_event_attn_fn(states, event_mask, attn_fn, max_events=None, backend: str = "auto"):
    """Drop-in for ``hclsm.kernels.sparse_event_attn_fn``.  ``attn_fn`` maps
    (B*K, N, D) -> (B*K, N, D); an ``EventTransformer`` takes the fused path."""
    if backend not in ("auto", "b200", "optimized", "naive"):
        raise ValueError(f"unknown backend {backend!r}")
    _lib.require_cuda(states, event_mask)
    grad = torch.is_grad_enabled()
    if isinstance(attn_fn, EventTransformer):
        if grad and states.requires_grad:
            raise RuntimeError("hclsm_b200: an EventTransformer holds inference weights and has no backward; "
                               "train through the Level1EventDynamics module (patched by install())")
        if max_events is None:
            return sparse_event_attention_fused(states, event_mask, attn_fn)
    states = _c(states)
    B, T, N, D = states.shape
    idx, pos, counts, meta = event_compact(event_mask)
    kmax = int(meta[1].item())
    K = max(kmax if max_events is None else max_events, 1)
    if max_events is not None and max_events < kmax:
        # truncation: keep the first max_events events of each video (:64-67)
        m = (event_mask > 0.5)
        rank = torch.cumsum(m.int(), dim=1) - 1
        m = m & (rank < max_events)
        idx, pos, counts, meta = event_compact(m.float())
    if grad:
        # differentiable gather / scatter: gradients reach the states through
        # attn_fn at the events and directly everywhere else, as in the
        # reference's clone-and-assign (:76-86)
        from .training import event_gather_train, event_scatter_train

        if states.requires_grad:
            padded = event_gather_train(states, idx, pos, counts, meta, K)
        else:
            padded = event_gather(states, idx, counts, meta, B * K, pad_k=K)
        upd = attn_fn(padded.reshape(B * K, N, D))
        return event_scatter_train(states, upd.reshape(B, K, N, D), idx, pos, counts, meta, K)
    padded = event_gather(states, idx, counts, meta, B * K, pad_k=K)
    upd = attn_fn(padded.reshape(B * K, N, D))
    return event_scatter(states, upd.reshape(B * K, N, D).to(states.dtype), pos, counts, pad_k=K)
