"""Host-side sharding logic on two gloo ranks (CPU): the sharded scan backward,
with dA_log all-reduced, equals the unsharded one; shards gather back in order."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hclsm_b200.shard import gather_shards, shard_range, sharded_scan_grads


def test_shard_range_covers():
    for n in (0, 1, 7, 8192, 8193):
        for w in (1, 2, 3, 8):
            rs = [shard_range(n, r, w) for r in range(w)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            assert max(e - s for s, e in rs) - min(e - s for s, e in rs) <= 1


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from hclsm_b200.workloads import scan_inputs
    from oracle import scan as oscan

    d = scan_inputs(5, 12, 16, 8, seed=3)
    o = {k: v.numpy() for k, v in d.items()}

    def compute(sh):
        g = oscan.scan_bwd(sh["x"], sh["dt"], sh["A_log"], sh["B"], sh["C"], sh["dy"], threads=1)
        return {k: torch.from_numpy(v) for k, v in g.items()}

    out, (s, e) = sharded_scan_grads(compute, o, 5)
    full_dx = gather_shards(out["dx"], 5)
    if rank == 0:
        q.put((out["dA_log"].numpy(), full_dx.numpy()))
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_backward_equals_unsharded():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    dA, dx = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from hclsm_b200.workloads import scan_inputs
    from oracle import scan as oscan

    d = {k: v.numpy() for k, v in scan_inputs(5, 12, 16, 8, seed=3).items()}
    ref = oscan.scan_bwd(d["x"], d["dt"], d["A_log"], d["B"], d["C"], d["dy"], threads=1)
    assert np.allclose(dA, ref["dA_log"], rtol=1e-5, atol=1e-6)
    assert np.array_equal(dx, ref["dx"])
