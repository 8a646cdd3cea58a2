"""Benchmark of the HCLSM hot path on B200.

Headline: the selective-scan forward + backward of BASELINE config 4, strong
scaled: one job of 64 videos x 128 slots = 8192 sequences (L=256, d_inner=2048,
d_state=16, bf16 I/O, fp32 state), rank r of N scanning sequences
[r * 8192 / N, (r + 1) * 8192 / N).  Beside it, legs for configs 0-3 (the
fp32 scan latency, the config-1 scan fwd+bwd, slot attention, sparse event
attention), each with its roofline and a CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N>1 runs under torchrun, one process per GPU over NCCL.  The scan needs no
collective on its data path (sequences are independent); after the timed
region NCCL gathers every rank's outputs to rank 0, which checks them bit for
bit against its own run of the same shards, and all-reduces dA_log.

Output: one JSON line on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L, DI, DS = 256, 2048, 16
GLOBAL_SEQS = 8192
SEED = 4242
# Algorithmic bytes per sequence (bf16 I/O).  Forward reads x, dt, B, C and
# writes y; backward reads x, dt, dy, B, C and writes dx, ddt, dB, dC.  A_log
# (read) and dA_log (written), fp32, are counted once per call.
FWD_BYTES_PER_SEQ = 3 * L * DI * 2 + 2 * L * DS * 2
BWD_BYTES_PER_SEQ = 5 * L * DI * 2 + 4 * L * DS * 2
ALOG_BYTES = DI * DS * 4
# DRAM bytes per sequence of the backward kernel measured by ncu
# (dram__bytes_read.sum + dram__bytes_write.sum on a 148-sequence config-4
# slice of the state-snapshot path); the forward's snapshots that the backward
# reads (3.28 MB per sequence) put it above the algorithmic bytes.
BWD_TRAFFIC_PER_SEQ = 8.33e6
# exponentials per (t, channel, state) element: one in the forward, one in the
# backward's recomputation
EXPS_PER_ELEM_STEP = 2
# config 2: FLOP per frame (QK^T, attn V, GRU, MLP over 3 iterations, plus the
# k/v projections; W_q is folded into the key projection, so its three
# 4096 x 384 x 384 products, 3.62e9 FLOP, are not executed) and config 3: FLOP per event frame (3 layers of qkv,
# attention, out-proj, SwiGLU, plus proj_in / proj_out) at 32 slots, dim 384
SLOT_FLOP_PER_FRAME = (7.29e10 - 3.62e9) / 128
EVENT_FLOP_PER_FRAME = 2 * 32 * (384 * 384 * 2 + 3 * (384 * 3 * 384 + 384 * 384 + 3 * 384 * 1536)) + \
    3 * 2 * 2 * 6 * 32 * 32 * 64


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--seqs", type=int, default=GLOBAL_SEQS, help="global sequences of the config-4 job")
    ap.add_argument("--ref-seqs", type=int, default=4, help="config-4 sequences per CPU-baseline step")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-verify", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the config 0-3 legs")
    ap.add_argument("--only", choices=["config0", "config1", "slot", "event", "block", "slot_train", "event_train"],
                    help="run this one leg alone (no config-4 step) and print its JSON line; for profiling")
    return ap.parse_args()


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def _best_of(fn, reps=3, warm=1):
    for _ in range(warm):
        fn()
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        fn()
        ts.append(time.perf_counter() - t0)
    return min(ts)


# ---- CPU baselines: the reference's own CPU path (PyTorch), restated --------------
def cpu_scan(nseq, L_, d, s, bwd, dtype_name, reps=3, seed=1234, gated=False, clamp_ref=True):
    """sequential_ssm_scan (+ autograd) of the reference, restated op for op in
    PyTorch on the host cores, on ``nseq`` sequences.  Returns seconds per call."""
    import torch
    import torch.nn.functional as F

    from hclsm_b200.workloads import scan_inputs
    from oracle import torch_ref

    torch.set_num_threads(_cpu_threads())
    d_ = scan_inputs(nseq, L_, d, s, dtype=getattr(torch, dtype_name), seed=seed, gated=gated)
    f = {k: v.float() for k, v in d_.items()}

    def run():
        leaves = {k: f[k].clone().requires_grad_(bwd) for k in ("x", "dt", "A_log", "B", "C")}
        y = torch_ref.sequential_ssm_scan(leaves["x"], leaves["dt"], leaves["A_log"], leaves["B"], leaves["C"])
        if gated:
            y = (y + f["D"] * leaves["x"]) * F.silu(f["z"])
        if bwd:
            y.backward(f["dy"])

    return _best_of(run, reps=reps)


def cpu_scan_c(nseq, reps=1):
    """The C restatement of the scan (fwd + bwd), all host cores, on nseq
    config-4 sequences.  Returns (seconds per call, threads)."""
    import torch

    from hclsm_b200.workloads import scan_inputs
    from oracle import scan as oscan

    threads = oscan.default_threads()
    d = scan_inputs(nseq, L, DI, DS, dtype=torch.bfloat16, seed=1234)
    o = {k: v.float().numpy() for k, v in d.items()}

    def run():
        oscan.scan_fwd(o["x"], o["dt"], o["A_log"], o["B"], o["C"], threads=threads)
        oscan.scan_bwd(o["x"], o["dt"], o["A_log"], o["B"], o["C"], o["dy"], threads=threads)

    return _best_of(run, reps=reps), threads


def cpu_slot(reps=3):
    """Config 2 on the host: k/v projections + 3 x _iteration_step, fp32."""
    import torch
    import torch.nn.functional as F

    from hclsm_b200.workloads import slot_inputs
    from oracle import torch_ref

    torch.set_num_threads(_cpu_threads())
    d = slot_inputs(seed=0)
    W = d["weights"]

    def run():
        with torch.no_grad():
            k = F.linear(d["inputs"], W["project_k.weight"])
            v = F.linear(d["inputs"], W["project_v.weight"])
            s = d["slots"]
            for _ in range(3):
                s = torch_ref.iteration_step(s, k, v, W)

    return _best_of(run, reps=reps)


def cpu_event(reps=3):
    """Config 3 on the host: naive_sparse_event_attention with the 3-layer
    Level-1 transformer, fp32.  Returns (seconds per call, event frames)."""
    import torch

    from hclsm_b200.workloads import event_inputs
    from oracle import torch_ref

    torch.set_num_threads(_cpu_threads())
    e = event_inputs(seed=20)
    W = e["weights"]

    def run():
        with torch.no_grad():
            torch_ref.naive_sparse_event_attention(
                e["states"], e["mask"], lambda fr: torch_ref.level1_event(fr, W, e["heads"], e["layers"]))

    return _best_of(run, reps=reps), int(e["mask"].sum().item())


# ---- clocks ----------------------------------------------------------------------
class Clocks:
    """nvidia-smi sampler running during the timed region."""

    NAMES = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]

    def __init__(self, index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                       "-i", str(index), "-lms", "200"], stdout=self.f,
                                      stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.p = None

    def stop(self):
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.p.terminate()
        self.p.wait()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        os.unlink(self.f.name)
        sm, mx, reasons = [], [], set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx.append(float(r[2]))
            except (ValueError, IndexError):
                continue
            for n, v in zip(self.NAMES, r[5:9]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _max_over_ranks(vals, dev, world):
    import torch
    import torch.distributed as dist

    t = torch.tensor(vals, device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def _barrier(world):
    import torch.distributed as dist

    if world > 1:
        dist.barrier()


# ---- config 4: the headline ----------------------------------------------------------
def run_config4(args, rank, world, dev):
    import torch

    import hclsm_b200
    from hclsm_b200.kernels.ssm_scan_kernel import bwd_workspace_bytes, scan_bwd_raw, scan_fwd_raw, states_bytes
    from hclsm_b200.shard import shard_range
    from hclsm_b200.workloads import scan_inputs_range

    s0, s1 = shard_range(args.seqs // 64, rank, world)
    s0, s1 = s0 * 64, s1 * 64
    nseq = s1 - s0
    d = scan_inputs_range(s0, nseq, L, DI, DS, dtype=torch.bfloat16, seed=SEED, device=dev)
    ws = torch.empty(bwd_workspace_bytes(nseq, L, DI, DS), dtype=torch.uint8, device=dev)
    st = torch.empty(states_bytes(nseq, L, DI, DS, torch.bfloat16), dtype=torch.uint8, device=dev)
    y = torch.empty_like(d["x"])
    stream = torch.cuda.current_stream(dev)

    def fwd():
        scan_fwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], out=y, states=st)

    def bwd():
        return scan_bwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], d["dy"], workspace=ws, states=st)

    for _ in range(args.warmup):
        fwd()
        g = bwd()
    del g
    torch.cuda.synchronize(dev)
    _barrier(world)
    clocks = Clocks(dev.index) if rank == 0 else None
    if clocks:
        time.sleep(0.3)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps + 1)]
    torch.cuda.synchronize(dev)
    _barrier(world)
    ev[0].record(stream)
    for i in range(args.steps):
        fwd()
        ev[2 * i + 1].record(stream)
        g = bwd()
        ev[2 * i + 2].record(stream)
        del g
    torch.cuda.synchronize(dev)
    _barrier(world)
    clk = clocks.stop() if clocks else None
    total_ms = ev[0].elapsed_time(ev[2 * args.steps])
    fwd_ms = sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)) / args.steps
    bwd_ms = sum(ev[2 * i + 1].elapsed_time(ev[2 * i + 2]) for i in range(args.steps)) / args.steps
    total_ms, fwd_ms, bwd_ms = _max_over_ranks([total_ms, fwd_ms, bwd_ms], dev, world)
    err = hclsm_b200.device_error()
    if err:
        raise RuntimeError(f"device error {err}")
    res = dict(ms_per_step=total_ms / args.steps, fwd_ms=fwd_ms, bwd_ms=bwd_ms, clocks=clk, seqs_per_rank=nseq)
    if not args.no_verify:
        fwd()
        grads = bwd()
        res["verify"] = verify_config4(args, rank, world, dev, (s0, s1), y, grads, d)
        del grads
    del d, ws, y, st
    torch.cuda.empty_cache()
    return res


def verify_config4(args, rank, world, dev, shard, y, grads, d):
    """Outside the timed region.  N > 1: rank 0 reruns every rank's shard on
    its own GPU (the same regenerated sequences, the same call size and path),
    NCCL gathers each rank's y, dx, ddt, dB, dC to rank 0 in rounds of 64
    sequences, and rank 0 requires bit equality; dA_log is all-reduced and
    compared with rank 0's sum of the rerun shards at 1e-5 (the two sums run
    in different orders).  Every N: the first 16 sequences against the CPU
    oracle at 2e-2 (bf16 I/O)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from hclsm_b200.kernels.ssm_scan_kernel import scan_bwd_raw, scan_fwd_raw
    from hclsm_b200.shard import shard_range
    from hclsm_b200.workloads import scan_inputs_range

    out = {}
    names = ("y", "dx", "ddt", "dB", "dC")
    mine = dict(zip(names, (y, grads[0], grads[1], grads[3], grads[4])))
    dA = grads[2].clone()
    if world > 1:
        from hclsm_b200.kernels.ssm_scan_kernel import bwd_workspace_bytes, states_bytes

        blk = 64
        ranges = [tuple(64 * v for v in shard_range(args.seqs // 64, r, world)) for r in range(world)]
        exact = True
        tot = torch.zeros_like(dA) if rank == 0 else None
        for r, (s, e) in enumerate(ranges):
            n = e - s
            ref = None
            if rank == 0:
                # rank r's shard again on this GPU: same sequences, same call
                # size (the kernels' work split depends on it), same path
                dd = scan_inputs_range(s, n, L, DI, DS, dtype=torch.bfloat16, seed=SEED, device=dev)
                st = torch.empty(states_bytes(n, L, DI, DS, torch.bfloat16), dtype=torch.uint8, device=dev)
                ws = torch.empty(bwd_workspace_bytes(n, L, DI, DS), dtype=torch.uint8, device=dev)
                yr = scan_fwd_raw(dd["x"], dd["dt"], dd["A_log"], dd["B"], dd["C"], states=st)
                gr = scan_bwd_raw(dd["x"], dd["dt"], dd["A_log"], dd["B"], dd["C"], dd["dy"], workspace=ws, states=st)
                ref = dict(zip(names, (yr, gr[0], gr[1], gr[3], gr[4])))
                tot += gr[2]
                del dd, st, ws
            # NCCL carries rank r's outputs to rank 0 in rounds of 64 sequences
            for j in range(n // blk):
                for k in names:
                    if rank == r and r != 0:
                        dist.send(mine[k][j * blk:(j + 1) * blk].contiguous(), dst=0)
                    elif rank == 0:
                        if r == 0:
                            got = mine[k][j * blk:(j + 1) * blk]
                        else:
                            got = torch.empty((blk,) + tuple(mine[k].shape[1:]), dtype=mine[k].dtype, device=dev)
                            dist.recv(got, src=r)
                        exact &= bool(torch.equal(got, ref[k][j * blk:(j + 1) * blk]))
            del ref
        dist.all_reduce(dA)
        if rank == 0:
            rel = float((dA - tot).abs().max() / tot.abs().max())
            out.update({"gathered_bit_identical": exact, "dA_log_rel_err": rel})
    if rank == 0 and shard[0] == 0:
        from oracle import scan as oscan

        n = 16
        o = {k: d[k][:n].float().cpu().numpy() for k in ("x", "dt", "B", "C", "dy")}
        A = d["A_log"].cpu().numpy()
        yr = oscan.scan_fwd(o["x"], o["dt"], A, o["B"], o["C"])
        gr = oscan.scan_bwd(o["x"], o["dt"], A, o["B"], o["C"], o["dy"])

        def rel(a, b):
            return float(np.abs(a - b).max() / np.abs(b).max())

        errs = {"y": rel(y[:n].float().cpu().numpy(), yr)}
        for k, gi in (("dx", 0), ("ddt", 1), ("dB", 3), ("dC", 4)):
            errs[k] = rel(grads[gi][:n].float().cpu().numpy(), gr[k])
        out["oracle_slice"] = {"sequences": n, "max_rel_err": max(errs.values()), "tol": 2e-2}
    if rank == 0:
        ok = out.get("gathered_bit_identical", True) and out.get("dA_log_rel_err", 0.0) < 1e-5 and \
            out.get("oracle_slice", {"max_rel_err": 0.0})["max_rel_err"] < 2e-2
        out["verified"] = bool(ok)
    return out


def run_weak(args, rank, world, dev):
    """Secondary, N > 1 only: weak scaling -- every rank scans a full 8192-
    sequence job of its own (its own seeded sequences), 2 timed steps; whole-
    job rate = world x 8192 / max-over-ranks step time."""
    import torch

    from hclsm_b200.kernels.ssm_scan_kernel import bwd_workspace_bytes, scan_bwd_raw, scan_fwd_raw, states_bytes
    from hclsm_b200.workloads import scan_inputs_range

    n = GLOBAL_SEQS
    d = scan_inputs_range(0, n, L, DI, DS, dtype=torch.bfloat16, seed=SEED + 1 + rank, device=dev)
    ws = torch.empty(bwd_workspace_bytes(n, L, DI, DS), dtype=torch.uint8, device=dev)
    st = torch.empty(states_bytes(n, L, DI, DS, torch.bfloat16), dtype=torch.uint8, device=dev)
    y = torch.empty_like(d["x"])

    def step():
        scan_fwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], out=y, states=st)
        return scan_bwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], d["dy"], workspace=ws, states=st)

    g = step()
    del g
    torch.cuda.synchronize(dev)
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(2):
        g = step()
        del g
    e1.record()
    torch.cuda.synchronize(dev)
    _barrier(world)
    (ms,) = _max_over_ranks([e0.elapsed_time(e1) / 2], dev, world)
    del d, ws, st, y
    torch.cuda.empty_cache()
    return {"value": world * n / (ms * 1e-3), "unit": "sequences/s", "ms_per_step": ms, "sequences_per_gpu": n,
            "note": "secondary: weak scaling, each rank a full 8192-sequence job"}


def run_e2e(args, rank, world, dev):
    """The public API end to end: inputs in pinned host memory; per step the
    H2D copy, ssm_scan_fn forward + autograd backward, and the D2H copy of y
    and every gradient, for this rank's share of the config-4 job.  Chunks of
    sequences are pipelined over an upload stream, the compute stream and a
    download stream, so both PCIe directions run at once."""
    import torch

    from hclsm_b200.kernels import ssm_scan_fn
    from hclsm_b200.shard import shard_range
    from hclsm_b200.workloads import scan_inputs_range

    s0, s1 = shard_range(args.seqs // 64, rank, world)
    s0, s1 = s0 * 64, s1 * 64
    n = s1 - s0
    host = {}
    for k, v in scan_inputs_range(s0, n, L, DI, DS, dtype=torch.bfloat16, seed=SEED, device=dev).items():
        host[k] = torch.empty(v.shape, dtype=v.dtype, pin_memory=True)
        host[k].copy_(v)
    torch.cuda.empty_cache()
    outs = {k: torch.empty(host["x"].shape, dtype=host["x"].dtype, pin_memory=True) for k in ("y", "dx", "ddt")}
    outs.update({k: torch.empty(host["B"].shape, dtype=host["B"].dtype, pin_memory=True) for k in ("dB", "dC")})
    dA_host = torch.empty(DI, DS, dtype=torch.float32, pin_memory=True)
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = sum(v.numel() * v.element_size() for v in outs.values()) + dA_host.numel() * 4
    up = torch.cuda.Stream(dev)    # host -> device
    down = torch.cuda.Stream(dev)  # device -> host (the other PCIe direction)
    comp = torch.cuda.current_stream(dev)
    chunk = 128
    # chunk boundaries: small chunks first and last, so that the pipeline's
    # fill (the first upload before any compute) and drain (the last download
    # after the last compute) are short
    sizes = [32, 64] + [chunk] * max(0, (n - 192) // chunk)
    rest = n - sum(sizes) - 96
    if rest > 0:
        sizes.append(rest)
    sizes += [64, 32]
    bounds, a = [], 0
    for sz in sizes:
        if a >= n:
            break
        bounds.append((a, min(n, a + sz)))
        a += sz
    if a < n:
        bounds.append((a, n))

    def step():
        # every host->device copy goes through the upload stream: the copy
        # engine serves copies of one direction in submission order across
        # streams, so a copy issued on the compute stream would queue behind
        # all uploads already submitted and stall the compute stream
        with torch.cuda.stream(up):
            A = host["A_log"].to(dev, non_blocking=True)
        for c0, c1 in bounds:
            with torch.cuda.stream(up):
                dv = {k: host[k][c0:c1].to(dev, non_blocking=True) for k in ("x", "dt", "B", "C", "dy")}
                ready = torch.cuda.Event()
                ready.record(up)
            comp.wait_event(ready)
            if c0 == 0:
                A.record_stream(comp)
                A.requires_grad_(True)
            for v in dv.values():
                v.record_stream(comp)
            leaves = [dv[k].requires_grad_(True) for k in ("x", "dt", "B", "C")]
            yy = ssm_scan_fn(leaves[0], leaves[1], A, leaves[2], leaves[3])
            torch.autograd.backward(yy, dv["dy"])
            done = torch.cuda.Event()
            done.record(comp)
            with torch.cuda.stream(down):
                down.wait_event(done)
                for k, t in (("y", yy), ("dx", leaves[0].grad), ("ddt", leaves[1].grad),
                             ("dB", leaves[2].grad), ("dC", leaves[3].grad)):
                    outs[k][c0:c1].copy_(t.detach(), non_blocking=True)
                    t.record_stream(down)
        comp.wait_stream(down)
        dA_host.copy_(A.grad, non_blocking=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    _barrier(world)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    for _ in range(args.steps):
        step()
    e1.record(comp)
    torch.cuda.synchronize(dev)
    (ms,) = _max_over_ranks([e0.elapsed_time(e1) / args.steps], dev, world)
    del host, outs
    return {"value": args.seqs / (ms * 1e-3), "unit": "sequences/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms, "sequences_per_rank": n,
            "note": "per-rank bytes; copies from / to pinned host memory inside the timed region"}


# ---- legs for configs 0-3 ------------------------------------------------------------
class L2Flush:
    """Writes a buffer larger than L2 (126 MB) between timed iterations."""

    def __init__(self, dev):
        import torch

        self.buf = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def __call__(self):
        self.buf.zero_()


def _timed(fn, reps, dev, flush):
    """Mean CUDA-event time (ms) of fn over reps calls, L2 flushed between calls
    (outside the events)."""
    import torch

    stream = torch.cuda.current_stream(dev)
    tot = 0.0
    for _ in range(reps):
        flush()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        tot += e0.elapsed_time(e1)
    return tot / reps


def run_config0(args, rank, world, dev, peaks, flush):
    """Config 0: ssm_scan_fn(backend="sequential") forward, fp32, with the D
    skip and the SiLU gate: 32 sequences, L=16, d_inner=512, d_state=16."""
    import torch

    from hclsm_b200.kernels import ssm_scan_fn
    from hclsm_b200.workloads import scan_inputs

    d = scan_inputs(32, 16, 512, 16, dtype=torch.float32, seed=0, device=dev, gated=True, grad=False)

    def call():
        with torch.no_grad():
            ssm_scan_fn(d["x"], d["dt"], d["A_log"], d["B"], d["C"], backend="sequential", D=d["D"], z=d["z"])

    for _ in range(max(args.warmup, 10)):
        call()
    torch.cuda.synchronize(dev)
    ms = _timed(call, 50, dev, flush)
    (ms,) = _max_over_ranks([ms], dev, world)
    nbytes = 4 * 32 * 16 * 512 * 4 + 2 * 32 * 16 * 16 * 4 + 512 * 16 * 4 + 512 * 4
    gbs = nbytes / (ms * 1e-3) / 1e9
    leg = {"metric": "scan_fwd_latency_fp32", "value": ms, "unit": "ms", "higher_is_better": False,
           "gbs_algorithmic": gbs, "algorithmic_bytes": nbytes,
           "config": "BASELINE config 0: 32 sequences x L=16 x d_inner 512 x d_state 16, fp32, clamped "
                     "(backend='sequential'), D skip + SiLU gate; L2 flushed between calls",
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks[0]["hbm_gbs"], "unit": "GB/s",
                        "frac": gbs / peaks[0]["hbm_gbs"], "peak_source": peaks[1],
                        "note": "4.3 MB per call: launch-latency bound (0.7 us at HBM speed)"}}
    if rank == 0 and world == 1 and not args.no_cpu:
        t = cpu_scan(32, 16, 512, 16, bwd=False, dtype_name="float32", gated=True)
        leg["cpu_baseline"] = {"value": t * 1e3, "unit": "ms", "cores": _cpu_threads(), "kind": "port",
                               "sample": "the whole config-0 call: sequential_ssm_scan restated in PyTorch on "
                                         "the host (+ D skip and SiLU gate), best of 3"}
    return leg


def run_config1(args, rank, world, dev, peaks, flush):
    """Config 1: ssm_scan_fn forward + autograd backward, bf16 in / fp32 state,
    256 sequences x L=64 x d_inner 768 x d_state 16 (unclamped: the reference's
    CUDA dispatch)."""
    import torch

    from hclsm_b200.kernels import ssm_scan_fn
    from hclsm_b200.workloads import scan_inputs

    d = scan_inputs(256, 64, 768, 16, dtype=torch.bfloat16, seed=1, device=dev)
    leaves = {k: d[k].clone().requires_grad_(True) for k in ("x", "dt", "A_log", "B", "C")}

    def step():
        for t in leaves.values():
            t.grad = None
        y = ssm_scan_fn(leaves["x"], leaves["dt"], leaves["A_log"], leaves["B"], leaves["C"])
        y.backward(d["dy"])

    for _ in range(max(args.warmup, 5)):
        step()
    torch.cuda.synchronize(dev)
    ms_eager = _timed(step, 20, dev, flush)
    from hclsm_b200.graphs import GraphedStep

    graphed = GraphedStep(step, list(leaves.values()), warmup=max(args.warmup, 3))
    ms = _timed(graphed.replay, 20, dev, flush)
    ms, ms_eager = _max_over_ranks([ms, ms_eager], dev, world)
    nbytes = 204_619_776
    gbs = nbytes / (ms * 1e-3) / 1e9
    leg = {"metric": "scan_fwd_bwd_sequences_per_s", "value": 256 * world / (ms * 1e-3), "unit": "sequences/s",
           "ms_per_step": ms, "eager_ms_per_step": ms_eager, "gbs_algorithmic": gbs, "algorithmic_bytes": nbytes,
           "config": "BASELINE config 1: 256 sequences x L=64 x d_inner 768 x d_state 16, bf16 I/O, fp32 state, "
                     "fwd + bwd through ssm_scan_fn and autograd, the step captured as one CUDA graph "
                     "(hclsm_b200.GraphedStep), eager launch time beside it; L2 flushed between steps; per rank",
           "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks[0]["hbm_gbs"], "unit": "GB/s",
                        "frac": gbs / peaks[0]["hbm_gbs"], "peak_source": peaks[1],
                        "note": "whole step (fwd + bwd kernels + autograd glue); the kernels are SFU/issue bound"}}
    if rank == 0 and world == 1 and not args.no_cpu:
        n = 32
        t = cpu_scan(n, 64, 768, 16, bwd=True, dtype_name="bfloat16", reps=2)
        leg["cpu_baseline"] = {"value": n / t, "unit": "sequences/s", "cores": _cpu_threads(), "kind": "port",
                               "sample": f"{n} of the 256 config-1 sequences, fwd + autograd bwd of "
                                         "sequential_ssm_scan restated in PyTorch on the host, best of 2"}
    return leg


def run_slot(args, rank, world, dev, peaks, flush):
    """Config 2: DynamicSlotAttention k/v projections + 3 fused iterations on
    128 frames (32 slots, 196 tokens, dim 384, bf16), frames sharded over the
    ranks, as one CUDA graph.  Verification: NCCL all-gather of every rank's
    slots to rank 0 against rank 0's run of all 128 frames."""
    import torch
    import torch.distributed as dist

    from hclsm_b200.kernels import (SlotIterationParams, key_value_weights, project_keys_values,
                                    slot_attention_iterations)
    from hclsm_b200.shard import shard_range
    from hclsm_b200.workloads import slot_inputs

    d = slot_inputs(seed=10, device=dev)
    W = d["weights"]
    p = SlotIterationParams.from_state(W, dev)
    # keys projected with W_k^T W_q (prepared once, like the transposed
    # weights): the steps skip their W_q products; k and v in one GEMM
    w_kv = key_value_weights(W["project_k.weight"], W["project_v.weight"], W["project_q.weight"])
    f0, f1 = shard_range(128, rank, world)
    inp_all = d["inputs"].to(torch.bfloat16)
    slots_all = d["slots"]

    def run(inp, slots):
        k, v = project_keys_values(inp, w_kv)
        return slot_attention_iterations(slots, k, v, p, 3, keys_folded=True)

    inp, slots = inp_all[f0:f1].contiguous(), slots_all[f0:f1].contiguous()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            run(inp, slots)
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = run(inp, slots)
    for _ in range(args.warmup):
        g.replay()
    torch.cuda.synchronize(dev)
    _barrier(world)
    ms = _timed(g.replay, 20, dev, flush)
    (ms,) = _max_over_ranks([ms], dev, world)
    frames = f1 - f0
    tflops = SLOT_FLOP_PER_FRAME * 128 / (ms * 1e-3) / 1e12
    peak = peaks[0].get("bf16_tflops_sustained", peaks[0]["bf16_tflops"])
    leg = {"metric": "slot_attention_frames_per_s", "value": 128 / (ms * 1e-3), "unit": "frames/s",
           "ms_per_step": ms, "frames_per_rank": frames, "scaling": "strong",
           "config": "BASELINE config 2: 128 frames x 32 slots x 196 tokens x 384, 3 iterations, bf16, k/v "
                     "projections included (W_q folded into the key projection), frames sharded over ranks, CUDA graph; L2 flushed between replays",
           "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                        "frac": tflops / peak, "peak_source": peaks[1] + " bf16_tflops_sustained",
                        "flop_per_step": SLOT_FLOP_PER_FRAME * 128}}
    if world > 1 and not args.no_verify:
        g.replay()
        full = [torch.empty((shard_range(128, r, world)[1] - shard_range(128, r, world)[0],) + tuple(out.shape[1:]),
                            dtype=out.dtype, device=dev) for r in range(world)]
        dist.all_gather(full, out)
        if rank == 0:
            ref = run(inp_all, slots_all)
            got = torch.cat(full, 0)
            leg["verify"] = {"rel_err_vs_single_gpu": float((got - ref).abs().max() / ref.abs().max()),
                             "tol": 2e-2}
            leg["verify"]["verified"] = leg["verify"]["rel_err_vs_single_gpu"] < 2e-2
    if rank == 0 and world == 1 and not args.no_cpu:
        t = cpu_slot()
        leg["cpu_baseline"] = {"value": 128 / t, "unit": "frames/s", "cores": _cpu_threads(), "kind": "port",
                               "sample": "the whole config-2 step (k/v projections + 3 x _iteration_step restated "
                                         "in PyTorch, fp32) on the host, best of 3"}
    del g
    return leg


def run_slot_train(args, rank, world, dev, peaks, flush):
    """Config 2 in training mode: 3 differentiable _iteration_steps (this
    library's forward and backward kernels, bf16 weight products with fp32
    accumulation) on 128 frames, forward + backward of sum(slots * w) into the
    slots, k, v and every iteration parameter; k and v are given."""
    import torch

    from hclsm_b200.kernels.training import slot_iteration_train
    from hclsm_b200.workloads import SlotIterModule, slot_inputs

    d = slot_inputs(seed=11, device=dev)
    W = d["weights"]
    mod = SlotIterModule.from_weights(W, 384, dev)
    k = torch.nn.functional.linear(d["inputs"], W["project_k.weight"]).to(torch.bfloat16)
    v = torch.nn.functional.linear(d["inputs"], W["project_v.weight"]).to(torch.bfloat16)
    w = torch.randn(d["slots"].shape, device=dev)
    leaves = [t.detach().clone().requires_grad_(True) for t in (d["slots"], k, v)]

    def step():
        for t in leaves + list(mod.parameters()):
            t.grad = None
        s = leaves[0]
        for _ in range(3):
            s = slot_iteration_train(mod, s, leaves[1], leaves[2], torch.bfloat16)
        (s * w).sum().backward()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    ms_eager = _timed(step, 10, dev, flush)
    # the same step captured as one CUDA graph (the host launches one graph
    # instead of a few hundred kernels through autograd)
    from hclsm_b200.graphs import GraphedStep

    graphed = GraphedStep(step, leaves + list(mod.parameters()), warmup=max(args.warmup, 3))
    ms = _timed(graphed.replay, 10, dev, flush)
    ms, ms_eager = _max_over_ranks([ms, ms_eager], dev, world)
    leg = {"metric": "slot_attention_train_frames_per_s", "value": 128 / (ms * 1e-3), "unit": "frames/s",
           "ms_per_step": ms, "eager_ms_per_step": ms_eager,
           "config": "BASELINE config 2 shapes in training mode: 3 x _iteration_step forward + backward "
                     "(autograd through this library's kernels), 128 frames x 32 slots x 196 tokens x 384, bf16 "
                     "weight products; the step captured as one CUDA graph (hclsm_b200.GraphedStep), eager "
                     "launch time beside it; per rank; L2 flushed between steps"}
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import torch_ref

        torch.set_num_threads(_cpu_threads())
        dc = slot_inputs(seed=11)
        Wc = {n: t.clone().requires_grad_(True) for n, t in dc["weights"].items()}
        kc = torch.nn.functional.linear(dc["inputs"], dc["weights"]["project_k.weight"])
        vc = torch.nn.functional.linear(dc["inputs"], dc["weights"]["project_v.weight"])
        wc = torch.randn(dc["slots"].shape)

        def cpu_step():
            lv = [t.detach().clone().requires_grad_(True) for t in (dc["slots"], kc, vc)]
            s = lv[0]
            for _ in range(3):
                s = torch_ref.iteration_step(s, lv[1], lv[2], Wc)
            (s * wc).sum().backward()

        t = _best_of(cpu_step, reps=2)
        leg["cpu_baseline"] = {"value": 128 / t, "unit": "frames/s", "cores": _cpu_threads(), "kind": "port",
                               "sample": "the whole step on the host: 3 x _iteration_step restated in PyTorch, "
                                         "fp32, forward + autograd backward, best of 2"}
    return leg


def run_event_train(args, rank, world, dev, flush):
    """Config 3 in training mode: the event gather, the 3-layer Level-1 stack
    and the scatter (hierarchy_manager.py:42-118, level1_event.py:85-133)
    forward and backward through this library's kernels, bf16 products, into
    the states and every Level-1 parameter.  The event compaction (which reads
    the event count on the host) runs once before the step; the step is
    captured as one CUDA graph, the eager launch time beside it."""
    import torch

    from hclsm_b200.graphs import GraphedStep
    from hclsm_b200.kernels.sparse_event_attn import event_compact
    from hclsm_b200.kernels.training import event_gather_train, event_scatter_train, level1_train
    from hclsm_b200.workloads import Level1Module, event_inputs

    e = event_inputs(seed=20, device=dev)
    mod = Level1Module.from_weights(e["weights"], e["heads"], e["layers"], dev)
    states = e["states"].to(torch.bfloat16).requires_grad_(True)
    B, T, N, D = states.shape
    idx, pos, counts, meta = event_compact(e["mask"])
    K = max(int(meta[1].item()), 1)
    w = torch.randn(B, T, N, D, device=dev)
    params = [states] + list(mod.parameters())

    def step():
        for t in params:
            t.grad = None
        ev = event_gather_train(states, idx, pos, counts, meta, K)
        upd = level1_train(mod, ev.reshape(B * K, N, D), None, torch.bfloat16)
        out = event_scatter_train(states, upd.reshape(B, K, N, D), idx, pos, counts, meta, K)
        (out.float() * w).sum().backward()

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    ms_eager = _timed(step, 10, dev, flush)
    graphed = GraphedStep(step, params, warmup=max(args.warmup, 3))
    ms = _timed(graphed.replay, 10, dev, flush)
    ms, ms_eager = _max_over_ranks([ms, ms_eager], dev, world)
    n_ev = int(e["mask"].sum().item())
    leg = {"metric": "sparse_event_attention_train_events_per_s", "value": n_ev / (ms * 1e-3),
           "unit": "event frames/s", "ms_per_step": ms, "eager_ms_per_step": ms_eager, "event_frames": n_ev,
           "config": "BASELINE config 3 in training mode: 8 videos x 64 steps x 32 slots x 384, Bernoulli(0.1) "
                     "mask, gather -> 3-layer Level-1 stack -> scatter, forward + backward into the states and "
                     "every Level-1 parameter, bf16 products; the step captured as one CUDA graph "
                     "(hclsm_b200.GraphedStep, compaction before it); per rank; L2 flushed between steps"}
    if rank == 0 and world == 1 and not args.no_cpu:
        from oracle import torch_ref

        torch.set_num_threads(_cpu_threads())
        ec = event_inputs(seed=20)
        Wc = {n: t.clone().requires_grad_(True) for n, t in ec["weights"].items()}
        wc = torch.randn(ec["states"].shape)

        def cpu_step():
            sc = ec["states"].clone().requires_grad_(True)
            out = torch_ref.naive_sparse_event_attention(
                sc, ec["mask"], lambda fr: torch_ref.level1_event(fr, Wc, ec["heads"], ec["layers"]))
            (out * wc).sum().backward()

        t = _best_of(cpu_step, reps=2)
        leg["cpu_baseline"] = {"value": n_ev / t, "unit": "event frames/s", "cores": _cpu_threads(), "kind": "port",
                               "sample": "the whole step on the host: naive_sparse_event_attention with the Level-1 "
                                         "stack restated in PyTorch, fp32, forward + autograd backward, best of 2"}
    return leg


def run_event(args, rank, world, dev, peaks, flush):
    """Config 3: sparse event attention with the 3-layer Level-1 transformer
    over 8 videos x 64 steps x 32 slots x 384 (bf16), Bernoulli(0.1) mask;
    videos sharded over the ranks.  Verification as the slot leg."""
    import torch
    import torch.distributed as dist

    from hclsm_b200.kernels import EventTransformer, sparse_event_attn_fn
    from hclsm_b200.shard import shard_range
    from hclsm_b200.workloads import event_inputs

    e = event_inputs(seed=20, device=dev)
    tr = EventTransformer.from_state(e["weights"], e["heads"], dev, dtype=torch.bfloat16)
    st_all = e["states"].to(torch.bfloat16)
    m_all = e["mask"]
    v0, v1 = shard_range(8, rank, world)
    st, m = st_all[v0:v1].contiguous(), m_all[v0:v1].contiguous()
    for _ in range(args.warmup):
        sparse_event_attn_fn(st, m, tr)
    torch.cuda.synchronize(dev)
    _barrier(world)
    ms = _timed(lambda: sparse_event_attn_fn(st, m, tr), 20, dev, flush)
    (ms,) = _max_over_ranks([ms], dev, world)
    n_ev = int(m_all.sum().item())
    tflops = EVENT_FLOP_PER_FRAME * n_ev / (ms * 1e-3) / 1e12
    peak = peaks[0].get("bf16_tflops_sustained", peaks[0]["bf16_tflops"])
    leg = {"metric": "sparse_event_attention_events_per_s", "value": n_ev / (ms * 1e-3),
           "unit": "event frames/s", "ms_per_call": ms, "event_frames": n_ev, "videos_per_rank": v1 - v0,
           "scaling": "strong",
           "config": "BASELINE config 3: 8 videos x 64 steps x 32 slots x 384, 6 heads, 3 layers, p=0.1, bf16, "
                     "videos sharded over ranks; L2 flushed between calls",
           "roofline": {"bound": "tensor", "achieved": tflops, "peak": peak, "unit": "TFLOP/s",
                        "frac": tflops / peak, "peak_source": peaks[1] + " bf16_tflops_sustained",
                        "flop_per_event_frame": EVENT_FLOP_PER_FRAME,
                        "note": "about 4e9 FLOP per call: launch / latency bound"}}
    if world > 1 and not args.no_verify:
        out = sparse_event_attn_fn(st, m, tr)
        full = [torch.empty((shard_range(8, r, world)[1] - shard_range(8, r, world)[0],) + tuple(out.shape[1:]),
                            dtype=out.dtype, device=dev) for r in range(world)]
        dist.all_gather(full, out)
        if rank == 0:
            ref = sparse_event_attn_fn(st_all, m_all, tr)
            got = torch.cat(full, 0).float()
            r = float((got - ref.float()).abs().max() / ref.float().abs().max())
            leg["verify"] = {"rel_err_vs_single_gpu": r, "tol": 2e-2, "verified": r < 2e-2}
    if rank == 0 and world == 1 and not args.no_cpu:
        t, nev = cpu_event()
        leg["cpu_baseline"] = {"value": nev / t, "unit": "event frames/s", "cores": _cpu_threads(), "kind": "port",
                               "sample": "the whole config-3 call (naive_sparse_event_attention + the Level-1 "
                                         "stack restated in PyTorch, fp32) on the host, best of 3"}
    return leg


def run_ssm_block(args, rank, world, dev, flush):
    """SimplifiedSSMBlock forward + backward through install()'s patched
    forward (LayerNorm, the five projections as library GEMMs, softplus(dt) + clamp +
    scan + SiLU gate in one kernel, out_proj, residual) under bf16 autocast, on
    config-1 scan shapes: 256 sequences x T=64, d_model 384 (d_inner 768),
    d_state 16."""
    import torch

    from hclsm_b200.install import _ssm_block_forward
    from hclsm_b200.workloads import ssm_block_inputs

    blk, x = ssm_block_inputs(seed=30, device=dev)
    x.requires_grad_(True)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16, cache_enabled=False):
            y = _ssm_block_forward(blk, x)
        y.float().sum().backward()

    for _ in range(max(args.warmup, 5)):
        step()
    torch.cuda.synchronize(dev)
    ms_eager = _timed(step, 20, dev, flush)
    from hclsm_b200.graphs import GraphedStep

    graphed = GraphedStep(step, [x] + list(blk.parameters()), warmup=max(args.warmup, 3))
    ms = _timed(graphed.replay, 20, dev, flush)
    ms, ms_eager = _max_over_ranks([ms, ms_eager], dev, world)
    return {"metric": "ssm_block_fwd_bwd_sequences_per_s", "value": x.shape[0] / (ms * 1e-3),
            "unit": "sequences/s", "ms_per_step": ms, "eager_ms_per_step": ms_eager,
            "config": "SimplifiedSSMBlock fwd+bwd, 256 sequences x T=64 x d_model 384 (d_inner 768, d_state 16), "
                      "bf16 autocast, softplus(dt) fused into the scan; the step captured as one CUDA graph "
                      "(hclsm_b200.GraphedStep), eager launch time beside it; per rank; L2 flushed between steps"}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    args.warmup = max(args.warmup, 3)
    if args.seqs % (64 * world):
        raise SystemExit("--seqs must be a multiple of 64 x world size")
    metric = "ssm_scan_fwd_bwd_throughput"
    config = {"workload": "BASELINE config 4: selective scan fwd+bwd, 64 videos x 128 slots = 8192 sequences "
                          "in one job, L=256, d_inner=2048, d_state=16, bf16 I/O / fp32 state, sequences sharded "
                          "over the GPUs",
              "global_sequences": args.seqs, "sequences_per_gpu": args.seqs // world, "L": L,
              "d_inner": DI, "d_state": DS, "parallelism": f"sequence-sharded x{world}",
              "l2": "inputs (8.6 GB per tensor at N=1, 1.07 GB at N=8) are larger than L2; no flush needed"}

    if args.impl == "reference":
        if rank != 0:
            return
        n = args.ref_seqs
        sec = cpu_scan(n, L, DI, DS, bwd=True, dtype_name="bfloat16", reps=args.steps, seed=1234)
        val = n / sec
        line = {"metric": metric, "value": val, "unit": "sequences/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": sec * 1e3, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                "impl": "reference",
                "cpu_baseline": {"value": val, "unit": "sequences/s", "cores": _cpu_threads(), "kind": "port",
                                 "sample": f"{n} config-4 sequences per step: sequential_ssm_scan + autograd "
                                           "backward (hclsm/kernels/ssm_scan_kernel.py:42-86, the reference's CPU "
                                           "path) restated op for op in PyTorch, fp32 on bf16-rounded inputs, "
                                           "best step"},
                "e2e": {"value": val, "unit": "sequences/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    peaks = _peaks()
    if args.only:
        flush = L2Flush(dev)
        run = {"config0": lambda: run_config0(args, rank, world, dev, peaks, flush),
               "config1": lambda: run_config1(args, rank, world, dev, peaks, flush),
               "slot": lambda: run_slot(args, rank, world, dev, peaks, flush),
               "event": lambda: run_event(args, rank, world, dev, peaks, flush),
               "block": lambda: run_ssm_block(args, rank, world, dev, flush),
               "slot_train": lambda: run_slot_train(args, rank, world, dev, peaks, flush),
               "event_train": lambda: run_event_train(args, rank, world, dev, flush)}[args.only]
        leg = run()
        if rank == 0:
            print(json.dumps(dict(leg, n_gpus=world, leg=args.only)), flush=True)
        if world > 1:
            dist.destroy_process_group()
        return
    r = run_config4(args, rank, world, dev)
    weak = run_weak(args, rank, world, dev) if world > 1 and not args.no_extra else None
    e2e = None if args.no_e2e else run_e2e(args, rank, world, dev)
    legs = {}
    if not args.no_extra:
        flush = L2Flush(dev)
        legs["config0"] = run_config0(args, rank, world, dev, peaks, flush)
        legs["config1"] = run_config1(args, rank, world, dev, peaks, flush)
        legs["config2_slot_attention"] = run_slot(args, rank, world, dev, peaks, flush)
        legs["config3_event_attention"] = run_event(args, rank, world, dev, peaks, flush)
        legs["ssm_block"] = run_ssm_block(args, rank, world, dev, flush)
        legs["config2_slot_attention_train"] = run_slot_train(args, rank, world, dev, peaks, flush)
        legs["config3_event_attention_train"] = run_event_train(args, rank, world, dev, flush)
        del flush
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        n = args.ref_seqs
        sec = cpu_scan(n, L, DI, DS, bwd=True, dtype_name="bfloat16", reps=1, seed=1234)
        sec_c, thr_c = cpu_scan_c(16)
        cpu = {"value": n / sec, "unit": "sequences/s", "cores": _cpu_threads(), "kind": "port",
               "sample": f"{n} config-4 sequences fwd + autograd bwd of sequential_ssm_scan restated op for op in "
                         f"PyTorch on the host (the reference's CPU path)",
               "c_restatement": {"value": 16 / sec_c, "unit": "sequences/s", "cores": thr_c,
                                 "sample": "16 config-4 sequences fwd + bwd, the C restatement of the scan"}}
    _barrier(world)
    if rank == 0:
        ms = r["ms_per_step"]
        nloc = r["seqs_per_rank"]
        fwd_bytes = nloc * FWD_BYTES_PER_SEQ + ALOG_BYTES
        bwd_bytes = nloc * BWD_BYTES_PER_SEQ + 2 * ALOG_BYTES
        hbm = peaks[0]["hbm_gbs"]
        bw_bwd = bwd_bytes / (r["bwd_ms"] * 1e-3) / 1e9
        bw_fwd = fwd_bytes / (r["fwd_ms"] * 1e-3) / 1e9
        line = {"metric": metric, "value": args.seqs / (ms * 1e-3), "unit": "sequences/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (seeded, BASELINE distributions)", "config": config,
                "hbm_gbs_algorithmic": (fwd_bytes + bwd_bytes) * world / (ms * 1e-3) / 1e9,
                "roofline": {"bound": "hbm", "kernel": "scan_bwd_bf16_kernel (hclsm_ssm_scan_bwd_states)",
                             "achieved": bw_bwd, "peak": hbm, "unit": "GB/s", "frac": bw_bwd / hbm,
                             "peak_source": peaks[1], "traffic": BWD_TRAFFIC_PER_SEQ * nloc,
                             "algorithmic_bytes": bwd_bytes, "ms": r["bwd_ms"],
                             "exp_floor_ms": nloc * L * DI * DS / (16 * 148 * 1.965e9) * 1e3},
                "roofline_fwd": {"kernel": "scan_fwd_bf16x2_kernel (hclsm_ssm_scan_fwd_states)", "achieved": bw_fwd,
                                 "frac": bw_fwd / hbm, "ms": r["fwd_ms"], "algorithmic_bytes": fwd_bytes,
                                 "exp_floor_ms": nloc * L * DI * DS / (16 * 148 * 1.965e9) * 1e3},
                "verify": r.get("verify"), "weak_scaling": weak, "cpu_baseline": cpu, "e2e": e2e, "clocks": r["clocks"],
                "legs": legs, "gpu_launches": 5 * args.steps}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
