"""The dispatcher operators (torch.ops.hclsm_b200.*): shapes under fake
tensors and the CPU-tensor rejection on the host; on the GPU, equality with the
direct calls, the registered autograd formula, torch.library.opcheck and
torch.compile."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import hclsm_b200.torch_ops  # noqa: F401  (registers the ops)
from conftest import rel_err

OPS = torch.ops.hclsm_b200


def test_ops_registered_and_fake_shapes():
    for name in ("ssm_scan_fwd", "ssm_scan_bwd", "slot_attn_core", "event_compact", "event_gather",
                 "event_scatter", "event_mha"):
        assert hasattr(OPS, name), name
    with FakeTensorMode():
        x = torch.empty(4, 32, 256, dtype=torch.bfloat16, device="cuda")
        A = torch.empty(256, 16, device="cuda")
        B = torch.empty(4, 32, 16, dtype=torch.bfloat16, device="cuda")
        y, st = OPS.ssm_scan_fwd(x, x, A, B, B, None, None, 0, True)
        assert y.shape == x.shape and y.dtype == torch.bfloat16 and st.shape == (4 * 3 * 256 * 16 * 4,)
        g = OPS.ssm_scan_bwd(x, x, A, B, B, x, None, None, 0, st)
        assert [t.shape for t in g[:5]] == [x.shape, x.shape, A.shape, B.shape, B.shape]
        Q = torch.empty(2, 32, 128, dtype=torch.bfloat16, device="cuda")
        K = torch.empty(2, 70, 128, dtype=torch.bfloat16, device="cuda")
        out, attn = OPS.slot_attn_core(Q, K, K, 0.1, 0.0, 0.0, True)
        assert out.shape == Q.shape and attn.shape == (2, 32, 70)
        st4 = torch.empty(2, 9, 4, 16, device="cuda")
        idx, pos, counts, meta = OPS.event_compact(torch.empty(2, 9, device="cuda"))
        assert idx.shape == (18,) and counts.shape == (2,) and meta.shape == (2,)
        assert OPS.event_gather(st4, idx, counts, meta, 5, 0).shape == (5, 4, 16)
        assert OPS.event_mha(torch.empty(64, 3 * 128, device="cuda"), None, 2, 32, 2, 64, 0.125).shape == (64, 128)


def test_ops_reject_cpu_tensors():
    x = torch.zeros(2, 4, 8)
    with pytest.raises(ValueError):
        OPS.ssm_scan_fwd(x, x, torch.zeros(8, 16), torch.zeros(2, 4, 16), torch.zeros(2, 4, 16), None, None, 0,
                         False)


@pytest.mark.gpu
def test_ops_match_direct_calls_and_autograd():
    from hclsm_b200.kernels import ssm_scan
    from hclsm_b200.workloads import scan_inputs
    d = scan_inputs(3, 40, 256, 16, dtype=torch.bfloat16, seed=4, device="cuda")
    leaves = {k: d[k].clone().requires_grad_(True) for k in ("x", "dt", "A_log", "B", "C")}
    y, st = OPS.ssm_scan_fwd(leaves["x"], leaves["dt"], leaves["A_log"], leaves["B"], leaves["C"], None, None, 0,
                             True)
    y.backward(d["dy"])
    ref_leaves = {k: d[k].clone().requires_grad_(True) for k in ("x", "dt", "A_log", "B", "C")}
    yr = ssm_scan(ref_leaves["x"], ref_leaves["dt"], ref_leaves["A_log"], ref_leaves["B"], ref_leaves["C"])
    yr.backward(d["dy"])
    assert torch.equal(y, yr)
    for k in leaves:
        assert torch.equal(leaves[k].grad, ref_leaves[k].grad), k


@pytest.mark.gpu
def test_opcheck_and_compile():
    from hclsm_b200.workloads import scan_inputs
    d = scan_inputs(2, 16, 64, 16, dtype=torch.float32, seed=1, device="cuda")
    args = (d["x"], d["dt"], d["A_log"], d["B"], d["C"], None, None, 1, False)
    torch.library.opcheck(torch.ops.hclsm_b200.ssm_scan_fwd.default, args,
                          test_utils=("test_schema", "test_faketensor"))
    Q = torch.randn(2, 32, 128, device="cuda").to(torch.bfloat16)
    K = torch.randn(2, 70, 128, device="cuda").to(torch.bfloat16)
    torch.library.opcheck(torch.ops.hclsm_b200.slot_attn_core.default, (Q, K, K, 0.1, 0.0, 0.0, True),
                          test_utils=("test_schema", "test_faketensor"))

    def f(x, dt, A_log, B, C):
        y, _ = OPS.ssm_scan_fwd(x, dt, A_log, B, C, None, None, 1, False)
        return y * 2.0

    got = torch.compile(f, fullgraph=True)(d["x"], d["dt"], d["A_log"], d["B"], d["C"])
    ref = f(d["x"], d["dt"], d["A_log"], d["B"], d["C"])
    assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) < 1e-6
