"""Benchmark of the HCLSM hot path on B200: selective-scan forward+backward at
BASELINE config 4 (per GPU: 8192 sequences = 64 videos x 128 slots, L=256,
d_inner=2048, d_state=16, bf16 I/O, fp32 state).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N>1 runs under torchrun, one process per GPU; every rank scans its own 8192
sequences (sequences are independent: no collective on the data path) and the
whole-job throughput is total sequences / max-over-ranks device time.

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
SEQS_PER_GPU = 8192
# Algorithmic bytes per sequence (bf16 I/O).  Forward reads x, dt, B, C and
# writes y; backward reads x, dt, dy, B, C and writes dx, ddt, dB, dC.  A_log
# (read) and dA_log (written), fp32, are counted once per call.
FWD_BYTES_PER_SEQ = 3 * L * DI * 2 + 2 * L * DS * 2
BWD_BYTES_PER_SEQ = 5 * L * DI * 2 + 4 * L * DS * 2
ALOG_BYTES = DI * DS * 4
# DRAM bytes per sequence of the backward kernel measured by ncu
# (dram__bytes_read.sum + dram__bytes_write.sum, 148-sequence config-4 slice
# on the state-snapshot path; see profiles/scan_config4_slice_ncu.md).  Above
# the algorithmic bytes by the forward's snapshots that the backward reads
# (3.28 MB per sequence).
BWD_TRAFFIC_PER_SEQ = 8.33e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--seqs", type=int, default=SEQS_PER_GPU, help="sequences per GPU")
    ap.add_argument("--e2e-seqs", type=int, default=1024, help="sequences per rank in the end-to-end leg")
    ap.add_argument("--e2e-chunk", type=int, default=128, help="sequences per pipelined copy/compute chunk")
    ap.add_argument("--ref-seqs", type=int, default=16, help="sequences per CPU-baseline step")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-extra", action="store_true", help="skip the slot / event attention legs")
    return ap.parse_args()


def cpu_reference(nseq, steps, warmup):
    """Time the CPU restatement of the reference scan (fwd + bwd) on a bounded
    sample of the config-4 workload, using every host core."""
    import torch

    from hclsm_b200.workloads import scan_inputs
    from oracle import scan as oscan

    threads = oscan.default_threads()
    d = scan_inputs(nseq, L, DI, DS, dtype=torch.bfloat16, seed=1234)
    o = {k: v.float().numpy() for k, v in d.items()}

    def step():
        oscan.scan_fwd(o["x"], o["dt"], o["A_log"], o["B"], o["C"], threads=threads)
        oscan.scan_bwd(o["x"], o["dt"], o["A_log"], o["B"], o["C"], o["dy"], threads=threads)

    for _ in range(warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(steps):
        step()
    dt = time.perf_counter() - t0
    return nseq * steps / dt, threads, dt / steps


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


def run_b200(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    import hclsm_b200
    from hclsm_b200.kernels.ssm_scan_kernel import bwd_workspace_bytes, scan_bwd_raw, scan_fwd_raw, states_bytes
    from hclsm_b200.workloads import scan_inputs

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    nseq = args.seqs
    d = scan_inputs(nseq, L, DI, DS, dtype=torch.bfloat16, seed=1000 + rank, device=dev)
    ws = torch.empty(bwd_workspace_bytes(nseq, L, DI, DS), dtype=torch.uint8, device=dev)
    # the forward keeps h every 10 steps; the backward starts from those snapshots
    st = torch.empty(states_bytes(nseq, L, DI, DS, torch.bfloat16), dtype=torch.uint8, device=dev)
    y = torch.empty_like(d["x"])
    stream = torch.cuda.current_stream(dev)

    def step():
        scan_fwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], out=y, states=st)
        return scan_bwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], d["dy"], workspace=ws, states=st)

    for _ in range(args.warmup):
        g = step()
    del g
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clocks = Clocks(local_rank) if rank == 0 else None
    if clocks:
        time.sleep(0.3)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps + 1)]
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ev[0].record(stream)
    for i in range(args.steps):
        scan_fwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], out=y, states=st)
        ev[2 * i + 1].record(stream)
        g = scan_bwd_raw(d["x"], d["dt"], d["A_log"], d["B"], d["C"], d["dy"], workspace=ws, states=st)
        ev[2 * i + 2].record(stream)
        del g
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    clk = clocks.stop() if clocks else None
    total_ms = ev[0].elapsed_time(ev[2 * args.steps])
    fwd_ms = sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(args.steps)) / args.steps
    bwd_ms = sum(ev[2 * i + 1].elapsed_time(ev[2 * i + 2]) for i in range(args.steps)) / args.steps
    t = torch.tensor([total_ms, fwd_ms, bwd_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, fwd_ms, bwd_ms = t.tolist()
    err = hclsm_b200.device_error()
    if err:
        raise RuntimeError(f"device error {err}")
    del d, ws, y, st
    torch.cuda.empty_cache()
    e2e = None if args.no_e2e else run_e2e(args, rank, world, dev)
    return dict(ms_per_step=total_ms / args.steps, fwd_ms=fwd_ms, bwd_ms=bwd_ms, clocks=clk, e2e=e2e)


def run_e2e(args, rank, world, dev):
    """Inputs in pinned host memory; per step: H2D copy, forward + backward via
    ``ssm_scan_fn`` and autograd, D2H copy of y and every gradient.  Chunks of
    sequences are pipelined over an upload stream, the compute stream and a
    download stream, so both PCIe directions run at once."""
    import torch
    import torch.distributed as dist

    from hclsm_b200.kernels import ssm_scan_fn
    from hclsm_b200.workloads import scan_inputs

    n = args.e2e_seqs
    chunk = max(1, min(args.e2e_chunk, n))
    host = {k: v.pin_memory() for k, v in scan_inputs(n, L, DI, DS, dtype=torch.bfloat16, seed=77 + rank).items()}
    outs = {k: torch.empty_like(host["x"]).pin_memory() for k in ("y", "dx", "ddt")}
    outs.update({k: torch.empty_like(host["B"]).pin_memory() for k in ("dB", "dC")})
    dA_host = torch.empty(DI, DS, dtype=torch.float32).pin_memory()
    h2d = sum(v.numel() * v.element_size() for v in host.values())
    d2h = sum(v.numel() * v.element_size() for v in outs.values()) + dA_host.numel() * 4
    up = torch.cuda.Stream(dev)    # host -> device
    down = torch.cuda.Stream(dev)  # device -> host (the other PCIe direction)
    comp = torch.cuda.current_stream(dev)

    # chunk boundaries: small chunks first and last, so that the pipeline's
    # fill (the first upload before any compute) and drain (the last download
    # after the last compute) are short
    bounds, s0 = [], 0
    ramp = [max(1, chunk // 4), max(1, chunk // 2)]
    sizes = ramp + [chunk] * max(0, (n - 2 * sum(ramp)) // chunk)
    rest = n - sum(sizes) - sum(ramp)
    if rest > 0:
        sizes.append(rest)
    sizes += ramp[::-1]
    for sz in sizes:
        if s0 >= n:
            break
        bounds.append((s0, min(n, s0 + sz)))
        s0 += sz
    if s0 < n:
        bounds.append((s0, n))

    def step():
        # every host->device copy goes through the upload stream: the copy
        # engine serves copies of one direction in submission order across
        # streams, so a copy issued on the compute stream would queue behind
        # all uploads already submitted and stall the compute stream
        with torch.cuda.stream(up):
            A = host["A_log"].to(dev, non_blocking=True)
        for s0, s1 in bounds:
            with torch.cuda.stream(up):
                dv = {k: host[k][s0:s1].to(dev, non_blocking=True) for k in ("x", "dt", "B", "C", "dy")}
                ready = torch.cuda.Event()
                ready.record(up)
            comp.wait_event(ready)
            if s0 == 0:
                A.record_stream(comp)
                A.requires_grad_(True)
            for v in dv.values():
                v.record_stream(comp)
            leaves = [dv[k].requires_grad_(True) for k in ("x", "dt", "B", "C")]
            y = ssm_scan_fn(leaves[0], leaves[1], A, leaves[2], leaves[3])
            torch.autograd.backward(y, dv["dy"])
            done = torch.cuda.Event()
            done.record(comp)
            with torch.cuda.stream(down):
                down.wait_event(done)
                for k, t in (("y", y), ("dx", leaves[0].grad), ("ddt", leaves[1].grad),
                             ("dB", leaves[2].grad), ("dC", leaves[3].grad)):
                    outs[k][s0:s1].copy_(t.detach(), non_blocking=True)
                    t.record_stream(down)
        comp.wait_stream(down)
        dA_host.copy_(A.grad, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    for _ in range(args.steps):
        step()
    e1.record(comp)
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    t = torch.tensor([ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    return {"value": n * world / (ms * 1e-3), "unit": "sequences/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms, "sequences_per_rank": n}


SLOT_FLOP_PER_FRAME = 7.29e10 / 128  # config 2: QK^T, attn V, W_q, GRU, MLP over 3 iterations + k/v proj


def run_slot(args, rank, world, dev):
    """Config 2: DynamicSlotAttention k/v projections + 3 fused iterations on 128
    frames (32 slots, 196 tokens, dim 384, bf16), captured in a CUDA graph."""
    import torch
    import torch.distributed as dist

    from hclsm_b200.kernels import SlotIterationParams, slot_attention_iterations
    from hclsm_b200.workloads import slot_inputs

    d = slot_inputs(seed=10 + rank, device=dev)
    W = d["weights"]
    p = SlotIterationParams.from_state(W, dev)
    wk = W["project_k.weight"].to(torch.bfloat16).t().contiguous()
    wv = W["project_v.weight"].to(torch.bfloat16).t().contiguous()
    inp = d["inputs"].to(torch.bfloat16)
    F_, M, D = inp.shape

    def step():
        x = inp.reshape(F_ * M, D)
        k = torch.mm(x, wk).reshape(F_, M, D)
        v = torch.mm(x, wv).reshape(F_, M, D)
        return slot_attention_iterations(d["slots"], k, v, p, 3)

    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(args.warmup):
            step()
    torch.cuda.current_stream(dev).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        step()
    for _ in range(args.warmup):
        g.replay()
    reps = 20
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        g.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    return {"metric": "slot_attention_frames_per_s", "value": F_ * world / (ms * 1e-3), "unit": "frames/s",
            "ms_per_step": ms, "config": "BASELINE config 2: 128 frames x 32 slots x 196 tokens x 384, 3 iterations, "
                                         "bf16, k/v projections included, CUDA graph",
            "tflops": SLOT_FLOP_PER_FRAME * F_ / (ms * 1e-3) / 1e12}


def run_event(args, rank, world, dev):
    """Config 3: sparse event attention with the 3-layer Level-1 transformer over
    8 videos x 64 steps x 32 slots x 384 (bf16), Bernoulli(0.1) event mask."""
    import torch
    import torch.distributed as dist

    from hclsm_b200.kernels import EventTransformer, sparse_event_attn_fn
    from hclsm_b200.workloads import event_inputs

    d = event_inputs(seed=20 + rank, device=dev)
    tr = EventTransformer.from_state(d["weights"], d["heads"], dev, dtype=torch.bfloat16)
    st = d["states"].to(torch.bfloat16)
    m = d["mask"]
    for _ in range(args.warmup):
        sparse_event_attn_fn(st, m, tr)
    reps = 20
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        sparse_event_attn_fn(st, m, tr)
    e1.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    n_ev = int(m.sum().item())
    return {"metric": "sparse_event_attention_events_per_s", "value": n_ev * world / (ms * 1e-3),
            "unit": "event frames/s", "ms_per_call": ms, "event_frames": n_ev,
            "config": "BASELINE config 3: 8 videos x 64 steps x 32 slots x 384, 6 heads, 3 layers, p=0.1, bf16"}


def run_ssm_block(args, rank, world, dev):
    """SimplifiedSSMBlock forward + backward (hclsm_b200.install's patched
    forward: LayerNorm, projections, softplus(dt) + clamp + scan + SiLU gate in
    one kernel, out_proj, residual) under bf16 autocast, on config-1 scan
    shapes: 256 sequences x T=64, d_model 384 (d_inner 768), d_state 16."""
    import torch
    import torch.distributed as dist

    from hclsm_b200.install import _ssm_block_forward
    from hclsm_b200.workloads import ssm_block_inputs

    blk, x = ssm_block_inputs(seed=30 + rank, device=dev)
    x.requires_grad_(True)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            y = _ssm_block_forward(blk, x)
        y.float().sum().backward()

    for _ in range(args.warmup):
        step()
    reps = 20
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    t = torch.tensor([e0.elapsed_time(e1) / reps], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = t.item()
    return {"metric": "ssm_block_fwd_bwd_sequences_per_s", "value": x.shape[0] * world / (ms * 1e-3),
            "unit": "sequences/s", "ms_per_step": ms,
            "config": "SimplifiedSSMBlock fwd+bwd, 256 sequences x T=64 x d_model 384 (d_inner 768, d_state 16), "
                      "bf16 autocast, softplus(dt) fused into the scan"}


def main():
    args = parse()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    args.warmup = max(args.warmup, 3)
    metric = "ssm_scan_fwd_bwd_throughput"
    config = {"workload": "BASELINE config 4: selective scan fwd+bwd, 64 videos x 128 slots = 8192 sequences "
                          "per GPU, L=256, d_inner=2048, d_state=16, bf16 I/O / fp32 state",
              "sequences_per_gpu": args.seqs, "global_sequences": args.seqs * world, "L": L,
              "d_inner": DI, "d_state": DS, "parallelism": f"sequence-sharded x{world}",
              "l2": "inputs (8.6 GB per tensor) are larger than L2; no flush needed"}

    if args.impl == "reference":
        if rank != 0:
            return
        val, cores, step_s = cpu_reference(args.ref_seqs, args.steps, 1)
        line = {"metric": metric, "value": val, "unit": "sequences/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": config,
                "impl": "reference",
                "cpu_baseline": {"value": val, "unit": "sequences/s", "cores": cores, "kind": "port",
                                 "sample": f"{args.ref_seqs} config-4 sequences fwd+bwd per step (C restatement "
                                           f"of the reference scan on bf16-rounded inputs, fp32 arithmetic)"},
                "e2e": {"value": val, "unit": "sequences/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist

    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    r = run_b200(args, rank, world, local_rank)
    dev = torch.device("cuda", local_rank)
    slot = None if args.no_extra else run_slot(args, rank, world, dev)
    event = None if args.no_extra else run_event(args, rank, world, dev)
    block = None if args.no_extra else run_ssm_block(args, rank, world, dev)
    cpu = None
    if rank == 0 and not args.no_cpu:
        v, cores, _ = cpu_reference(args.ref_seqs, 1, 1)
        cpu = {"value": v, "unit": "sequences/s", "cores": cores, "kind": "port",
               "sample": f"{args.ref_seqs} config-4 sequences fwd+bwd (C restatement of the reference scan)"}
    if world > 1:
        dist.barrier()
    if rank == 0:
        ms = r["ms_per_step"]
        fwd_bytes = args.seqs * FWD_BYTES_PER_SEQ + ALOG_BYTES
        bwd_bytes = args.seqs * BWD_BYTES_PER_SEQ + 2 * ALOG_BYTES
        peaks = {}
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                peaks = json.load(f)
        except OSError:
            pass
        hbm_peak = peaks.get("hbm_gbs", 6650.0)
        bw_bwd = bwd_bytes / (r["bwd_ms"] * 1e-3) / 1e9
        bw_fwd = fwd_bytes / (r["fwd_ms"] * 1e-3) / 1e9
        line = {"metric": metric, "value": args.seqs * world / (ms * 1e-3), "unit": "sequences/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic", "config": config,
                "hbm_gbs_algorithmic": (fwd_bytes + bwd_bytes) * world / (ms * 1e-3) / 1e9,
                "roofline": {"bound": "hbm", "kernel": "scan_bwd_bf16_kernel (hclsm_ssm_scan_bwd_states)",
                             "achieved": bw_bwd, "peak": hbm_peak, "unit": "GB/s", "frac": bw_bwd / hbm_peak,
                             "peak_source": "measured" if "hbm_gbs" in peaks else "fallback",
                             "traffic": BWD_TRAFFIC_PER_SEQ * args.seqs, "algorithmic_bytes": bwd_bytes,
                             "ms": r["bwd_ms"]},
                "roofline_fwd": {"kernel": "scan_fwd_bf16x2_kernel (hclsm_ssm_scan_fwd_states)", "achieved": bw_fwd,
                                 "frac": bw_fwd / hbm_peak, "ms": r["fwd_ms"], "algorithmic_bytes": fwd_bytes},
                "cpu_baseline": cpu, "e2e": r["e2e"], "clocks": r["clocks"],
                "slot_attention": slot, "event_attention": event, "ssm_block": block,
                "gpu_launches": 5 * args.steps}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
