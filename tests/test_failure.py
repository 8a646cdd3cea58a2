"""Failure detection without faulting a GPU.

* host: a rank that dies before a collective surfaces as an error on the
  survivor within the process-group timeout (gloo, CPU ranks);
* device: a bounded wait on a barrier that nothing completes returns
  HCLSM_ERR_TIMEOUT, is recorded in the error word, and the context stays usable.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from hclsm_b200 import _lib


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # dies between steps, no collective in flight
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        q.put("no error")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_dead_rank_is_detected():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
    assert res != "no error"
    assert ps[1].exitcode == 3


@pytest.mark.gpu
def test_device_wait_times_out_cleanly():
    import hclsm_b200

    lib = _lib.load()
    hclsm_b200.device_error()  # clear
    st = torch.full((1,), -1, dtype=torch.int32, device="cuda")
    rc = lib.hclsm_selftest_wait_timeout(2000, _lib.ptr(st), _lib.stream_ptr(st.device))
    assert rc == 0
    torch.cuda.synchronize()
    assert int(st.item()) == 6  # HCLSM_ERR_TIMEOUT
    assert hclsm_b200.device_error() == 6
    assert hclsm_b200.device_error() == 0  # cleared
    x = torch.randn(8, device="cuda")
    assert torch.isfinite(x * 2).all()  # context still usable
