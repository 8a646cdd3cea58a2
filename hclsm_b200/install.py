"""Patch a loaded ``hclsm`` package so its own call sites run the B200 kernels.

    import hclsm, hclsm_b200
    hclsm_b200.install()          # or install(hclsm) for an explicit module

What is replaced (paths inside RightNow-AI/hclsm):

* ``hclsm.kernels.ssm_scan_fn`` and ``hclsm.kernels.ssm_scan_kernel.ssm_scan_fn``
  (the package re-exports by value, hclsm/kernels/__init__.py:9-35, so both
  names are patched), likewise ``slot_attention_fn`` and ``sparse_event_attn_fn``;
* ``SimplifiedSSMBlock.forward`` (hclsm/dynamics/level0_ssm.py:58-107):
  softplus(dt_proj(z)) with its clamp, the inline clamped scan and the SiLU
  gate run as one differentiable kernel call (clamp=True, dt_softplus=True,
  z = gate_proj(x));
* ``Level0SSM.forward`` (hclsm/dynamics/level0_ssm.py:159-220): the masked
  mean over objects and the nan_to_num / clamp / mask epilogue as kernels;
* ``DynamicSlotAttention._iteration_step`` (hclsm/objects/dynamic_slots.py:98-131);
* ``DynamicSlotAttention.forward`` (hclsm/objects/dynamic_slots.py:133-203):
  slot birth decided and written on the device (no host read of
  ``needs_birth``, no per-video Python loop);
* ``EventDetector.forward`` (hclsm/dynamics/event_detector.py:133-172): the
  hard decision, the "at least one event" rule and the compaction in one
  kernel (no host read), handed to the gather / scatter through the mask;
* ``HierarchyManager.gather_events`` / ``scatter_events``
  (hclsm/dynamics/hierarchy_manager.py:42-118);
* ``Level1EventDynamics.forward`` (hclsm/dynamics/level1_event.py:85-133).

Every replaced call site is differentiable through this library's kernels:
the scan and the Level-0 epilogue have backward kernels, and the slot-attention
step, the event gather / scatter and the Level-1 transformer run as autograd
Functions (hclsm_b200.kernels.training) whenever a gradient is recorded, with
cheaper forward-only kernels otherwise.  The weight products follow the
caller's arithmetic: bf16 operands under bf16 autocast or for bf16 inputs,
fp32 otherwise.  CPU tensors are not accepted by the replaced functions (no CPU
fallback).
"""
from __future__ import annotations

import torch

_ORIG = {}


def _grad_active(*tensors):
    return torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in tensors)


def _module_grad(mod, *tensors):
    """True when autograd records through ``mod``'s call (an input or a
    parameter requires grad)."""
    if not torch.is_grad_enabled():
        return False
    return _grad_active(*tensors) or any(p.requires_grad for p in mod.parameters())


def _work_dtype(*tensors):
    """Arithmetic of the weight products: bf16 under bf16 autocast or for bf16
    inputs (the reference's autocast arithmetic), else fp32."""
    if torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == torch.bfloat16:
        return torch.bfloat16
    return torch.bfloat16 if any(t is not None and t.dtype == torch.bfloat16 for t in tensors) else torch.float32


def _patch(obj, name, new):
    key = (id(obj), name)
    if key not in _ORIG:
        _ORIG[key] = (obj, name, getattr(obj, name))
    setattr(obj, name, new)


def _orig(obj, name):
    """The attribute as it was before install() (so a second install() does not wrap twice)."""
    ent = _ORIG.get((id(obj), name))
    return ent[2] if ent else getattr(obj, name)


def uninstall():
    """Restore every attribute install() replaced."""
    for obj, name, old in list(_ORIG.values()):
        setattr(obj, name, old)
    _ORIG.clear()


def _ssm_block_forward(self, x):
    """SimplifiedSSMBlock.forward with softplus(dt), its clamp, the scan and
    the gate in one kernel (level0_ssm.py:58-107)."""
    from .kernels import ssm_scan
    from .kernels.training import layer_norm

    residual = x
    x = layer_norm(self.norm, x)  # this library's LayerNorm kernels, forward and backward
    z = self.in_proj(x)
    gate_pre = self.gate_proj(x)
    B_param = self.B_proj(z)
    C_param = self.C_proj(z)
    y = ssm_scan(z, self.dt_proj(z), self.A_log, B_param, C_param, clamp=True, z=gate_pre, dt_softplus=True)
    # under autocast out_proj takes bf16 operands, which y already is: the
    # reference's fp32 round trip (level0_ssm.py:101-105) would change no value
    if not (torch.is_autocast_enabled("cuda") and torch.get_autocast_dtype("cuda") == y.dtype):
        y = y.to(residual.dtype)
    y = self.out_proj(y)
    return residual + y


def _make_iteration_step(orig):
    def _iteration_step(self, slots, k, v):
        from .kernels.slot_attention_kernel import SlotIterationParams, slot_attention_iteration

        dt = _work_dtype(slots, k, v)
        if _module_grad(self, slots, k, v):
            from .kernels.training import slot_iteration_train

            return slot_iteration_train(self, slots, k, v, dt).to(slots.dtype)
        key = (tuple(p._version for p in self.parameters()), dt)
        cache = getattr(self, "_hclsm_b200_params", None)
        if cache is None or cache[0] != key:
            cache = (key, SlotIterationParams.from_module(self, dt))
            self._hclsm_b200_params = cache
        kd = k.to(dt).contiguous()
        vd = v.to(dt).contiguous()
        out, _ = slot_attention_iteration(slots.float().contiguous(), kd, vd, cache[1])
        return out.to(slots.dtype)

    return _iteration_step


def _make_dsa_forward(orig):
    def forward(self, inputs, return_attention=False):
        """DynamicSlotAttention.forward (dynamic_slots.py:133-203) with the
        birth step on the device: per video, the token of largest residual
        attention energy and the first dormant slot are found by argmax, the
        birth projection runs for every video, and torch.where keeps it only
        where the reference would write it (energy above the threshold and a
        dormant slot present).  No host synchronisation.  Inference in bf16
        (no gradient recorded, d_slot a multiple of 128) runs the fused
        refinement path with W_q folded into the keys."""
        import torch.nn.functional as F
        import torch.utils.checkpoint

        B, M, _ = inputs.shape
        inputs_norm = self.norm_input(inputs)
        fused = (not _module_grad(self, inputs) and _work_dtype(inputs) == torch.bfloat16
                 and self.d_slot % 128 == 0)
        slots = None
        if fused:
            # inference in bf16: W_q folded into the keys, the k/v products as
            # one GEMM, every refinement step fused (row kernels, bf16
            # products), the final attention map from the attention core
            from .kernels.slot_attention_kernel import (SlotIterationParams, key_value_weights, layernorm,
                                                        project_keys_values, slot_attention_core,
                                                        slot_attention_iterations)

            key = (tuple(p._version for p in self.parameters()), "fused")
            cache = getattr(self, "_hclsm_b200_fused", None)
            if cache is None or cache[0] != key:
                cache = (key, SlotIterationParams.from_module(self, torch.bfloat16),
                         key_value_weights(self.project_k.weight, self.project_v.weight, self.project_q.weight))
                self._hclsm_b200_fused = cache
            p, w_kv = cache[1], cache[2]
            k, v = project_keys_values(inputs_norm.to(torch.bfloat16).contiguous(), w_kv)
            s0 = self._init_slots(B, inputs.device)
            slots = slot_attention_iterations(s0, k, v, p, self.n_iterations, keys_folded=True).to(s0.dtype)
        else:
            k = self.project_k(inputs_norm)
            v = self.project_v(inputs_norm)
            slots = self._init_slots(B, inputs.device)
            for _ in range(self.n_iterations):
                if self.use_gradient_checkpointing and self.training:
                    slots = torch.utils.checkpoint.checkpoint(self._iteration_step, slots, k, v,
                                                              use_reentrant=False)
                else:
                    slots = self._iteration_step(slots, k, v)
        alive = torch.sigmoid(self.existence_head(slots).squeeze(-1))
        with torch.no_grad():
            if fused:
                sn = layernorm(slots.reshape(-1, self.d_slot), p.ln_attn_w, p.ln_attn_b,
                               out_dtype=torch.bfloat16).reshape(slots.shape)
                _, attn = slot_attention_core(sn, k, v, self.scale, clamp=0.0, eps=0.0, return_attn=True,
                                              attn_fp32=True)
            else:
                q = self.project_q(self.norm_pre_attn(slots))
                attn = F.softmax(torch.bmm(q, k.transpose(1, 2)) * self.scale, dim=1)
            final_attn = attn if return_attention else None
            residual = (1.0 - attn.sum(dim=1)).abs()
            max_residual = residual.max(dim=-1).values
            token = residual.argmax(dim=-1)
            dormant = alive < self.existence_threshold
            birth = (max_residual > self.birth_threshold) & dormant.any(dim=1)
            first = dormant.to(torch.int8).argmax(dim=1)  # first dormant slot (argmax returns the first maximum)
            ar = torch.arange(B, device=inputs.device)
            born = self.birth_proj(inputs[ar, token]).to(slots.dtype)
            sel = birth[:, None] & (torch.arange(slots.shape[1], device=inputs.device)[None, :] == first[:, None])
        slots = torch.where(sel[:, :, None], born[:, None, :], slots)
        if return_attention:
            return slots, alive, final_attn
        return slots, alive

    return forward


def _make_gather(orig):
    def gather_events(self, states, event_mask):
        from .kernels.sparse_event_attn import _cached_compaction, event_compact, event_gather

        B, T, N, D = states.shape
        st = states.contiguous()
        cached = _cached_compaction(event_mask)  # from the patched EventDetector
        idx, pos, counts, meta = cached if cached is not None else event_compact(event_mask)
        kmax = max(int(meta[1].item()), 1)
        if cached is not None:
            event_mask._hclsm_kmax = kmax
        if _grad_active(states):
            from .kernels.training import event_gather_train

            ev = event_gather_train(states, idx, pos, counts, meta, kmax)
        else:
            ev = event_gather(st, idx, counts, meta, B * kmax, pad_k=kmax).reshape(B, kmax, N, D)
        pad = (torch.arange(kmax, device=states.device)[None, :] < counts[:B, None]).float()
        return ev, pad, kmax

    return gather_events


def _make_scatter(orig):
    def scatter_events(self, base_states, event_updates, event_mask):
        from .kernels.sparse_event_attn import _cached_compaction, event_compact, event_scatter

        K = event_updates.shape[1]
        cached = _cached_compaction(event_mask)
        if cached is not None and K >= getattr(event_mask, "_hclsm_kmax", K + 1):
            idx, pos, counts, meta = cached  # every event fits: the detector's compaction as is
        else:
            m = (event_mask > 0.5)
            rank = torch.cumsum(m.int(), dim=1) - 1
            idx, pos, counts, meta = event_compact((m & (rank < K)).float())
        if _grad_active(base_states, event_updates):
            from .kernels.training import event_scatter_train

            return event_scatter_train(base_states, event_updates, idx, pos, counts, meta, K)
        upd = event_updates.reshape(-1, *event_updates.shape[2:]).to(base_states.dtype).contiguous()
        return event_scatter(base_states.contiguous(), upd, pos, counts, pad_k=K)

    return scatter_events


def _make_detector_forward(orig):
    def forward(self, states):
        """EventDetector.forward (event_detector.py:133-172): the module's own
        temporal features, causal dilated convolutions and head, then the
        decision and compaction on the device (no host read)."""
        import torch.nn.functional as F
        from .kernels.sparse_event_attn import event_detect

        B, T, D = states.shape
        temporal_feat = self.temporal_features(states)
        x = temporal_feat.transpose(1, 2)
        h = F.relu(self.conv1(x))[:, :, :T]
        h = F.relu(self.conv2(h))[:, :, :T]
        h = F.relu(self.conv3(h))[:, :, :T]
        conv_out = self.norm(h.transpose(1, 2))
        combined = torch.cat([conv_out, temporal_feat], dim=-1)
        event_probs = torch.sigmoid(self.head(combined).squeeze(-1))
        if not event_probs.is_cuda:
            return orig(self, states)
        return event_probs, event_detect(event_probs, self.learned_threshold)

    return forward


def _make_level1_forward(orig):
    def forward(self, event_states, event_pad_mask=None, obj_mask=None):
        from .kernels.sparse_event_attn import EventTransformer

        dtype = _work_dtype(event_states)
        B, K, N, D = event_states.shape
        kp = None
        if obj_mask is not None:
            kp = (~(obj_mask > 0.5)).unsqueeze(1).expand(B, K, N).reshape(B * K, N)
        if _module_grad(self, event_states):
            from .kernels.training import level1_train

            y = level1_train(self, event_states.reshape(B * K, N, D), kp, dtype).reshape(B, K, N, -1)
        else:
            key = tuple(p._version for p in self.parameters())
            cache = getattr(self, "_hclsm_b200_tr", None)
            if cache is None or cache[0] != (key, dtype):
                cache = ((key, dtype), EventTransformer.from_module(self, dtype))
                self._hclsm_b200_tr = cache
            y = cache[1](event_states.reshape(B * K, N, D), kp).reshape(B, K, N, -1)
        if event_pad_mask is not None:
            y = y * event_pad_mask[:, :, None, None]
        return y

    return forward


def install(hclsm_module=None):
    """Patch ``hclsm`` (imported if not given).  Returns the list of patched names."""
    if hclsm_module is None:
        import importlib

        hclsm_module = importlib.import_module("hclsm")
    from . import kernels as k

    done = []
    kern = getattr(hclsm_module, "kernels", None)
    if kern is not None:
        for name, fn in (("ssm_scan_fn", k.ssm_scan_fn), ("slot_attention_fn", k.slot_attention_fn),
                         ("sparse_event_attn_fn", k.sparse_event_attn_fn)):
            if hasattr(kern, name):
                _patch(kern, name, fn)
                done.append(f"kernels.{name}")
        for sub, name, fn in (("ssm_scan_kernel", "ssm_scan_fn", k.ssm_scan_fn),
                              ("slot_attention_kernel", "slot_attention_fn", k.slot_attention_fn),
                              ("sparse_event_attn", "sparse_event_attn_fn", k.sparse_event_attn_fn)):
            mod = getattr(kern, sub, None)
            if mod is not None and hasattr(mod, name):
                _patch(mod, name, fn)
                done.append(f"kernels.{sub}.{name}")
    dyn = getattr(hclsm_module, "dynamics", None)
    obj = getattr(hclsm_module, "objects", None)
    l0 = getattr(dyn, "level0_ssm", None) if dyn is not None else None
    if l0 is not None and hasattr(l0, "SimplifiedSSMBlock"):
        _patch(l0.SimplifiedSSMBlock, "forward", _ssm_block_forward)
        done.append("SimplifiedSSMBlock.forward")
    if l0 is not None and hasattr(l0, "Level0SSM"):
        from .kernels.level0 import level0_forward

        def _level0(self, obj_states, obj_mask=None):
            return level0_forward(self, obj_states, obj_mask)

        _patch(l0.Level0SSM, "forward", _level0)
        done.append("Level0SSM.forward")
    ds = getattr(obj, "dynamic_slots", None) if obj is not None else None
    if ds is not None and hasattr(ds, "DynamicSlotAttention"):
        cls = ds.DynamicSlotAttention
        _patch(cls, "_iteration_step", _make_iteration_step(_orig(cls, "_iteration_step")))
        _patch(cls, "forward", _make_dsa_forward(_orig(cls, "forward")))
        done += ["DynamicSlotAttention._iteration_step", "DynamicSlotAttention.forward"]
    hm = getattr(dyn, "hierarchy_manager", None) if dyn is not None else None
    if hm is not None and hasattr(hm, "HierarchyManager"):
        cls = hm.HierarchyManager
        _patch(cls, "gather_events", _make_gather(_orig(cls, "gather_events")))
        _patch(cls, "scatter_events", _make_scatter(_orig(cls, "scatter_events")))
        done += ["HierarchyManager.gather_events", "HierarchyManager.scatter_events"]
    ed = getattr(dyn, "event_detector", None) if dyn is not None else None
    if ed is not None and hasattr(ed, "EventDetector"):
        cls = ed.EventDetector
        _patch(cls, "forward", _make_detector_forward(_orig(cls, "forward")))
        done.append("EventDetector.forward")
    l1 = getattr(dyn, "level1_event", None) if dyn is not None else None
    if l1 is not None and hasattr(l1, "Level1EventDynamics"):
        cls = l1.Level1EventDynamics
        _patch(cls, "forward", _make_level1_forward(_orig(cls, "forward")))
        done.append("Level1EventDynamics.forward")
    return done
