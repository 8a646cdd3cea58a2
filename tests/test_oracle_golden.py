"""Pin the CPU oracle to golden vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""
import os

import numpy as np
import pytest

from conftest import rel_err
from oracle import event_attn, scan, slot_attn

HERE = os.path.join(os.path.dirname(__file__), "golden")


def _g(name):
    return np.load(os.path.join(HERE, name))


@pytest.mark.parametrize("case", ["test0", "test1", "test2", "base"])
def test_scan_fwd(case):
    g = _g("scan_golden.npz")
    a = [g[f"{case}/{k}"] for k in ("x", "dt", "A_log", "B", "C")]
    assert rel_err(scan.scan_fwd(*a, clamp=True), g[f"{case}/y_sequential"]) < 1e-6
    assert rel_err(scan.scan_fwd(*a, clamp=False), g[f"{case}/y_parallel"]) < 1e-6


@pytest.mark.parametrize("case", ["test0", "test1", "test2", "base"])
@pytest.mark.parametrize("tag", ["sequential", "parallel", "tritonbwd"])
def test_scan_bwd(case, tag):
    g = _g("scan_golden.npz")
    a = [g[f"{case}/{k}"] for k in ("x", "dt", "A_log", "B", "C")]
    got = scan.scan_bwd(*a, g[f"{case}/dy"], clamp=(tag == "sequential"))
    for k in ("dx", "ddt", "dA_log", "dB", "dC"):
        assert rel_err(got[k], g[f"{case}/{k}_{tag}"]) < 1e-5, k


def test_scan_gated():
    g = _g("scan_golden.npz")
    c = "base"
    a = [g[f"{c}/{k}"] for k in ("x", "dt", "A_log", "B", "C")]
    y = scan.scan_fwd(*a, D=g[f"{c}/D"], z=g[f"{c}/z"])
    assert rel_err(y, g[f"{c}/y_gated"]) < 1e-6
    got = scan.scan_bwd(*a, g[f"{c}/dy"], D=g[f"{c}/D"], z=g[f"{c}/z"])
    for k in ("dx", "ddt", "dA_log", "dB", "dC", "dD", "dz"):
        assert rel_err(got[k], g[f"{c}/{k}_gated"]) < 1e-5, k


def test_scan_threads_split_is_exact():
    g = _g("scan_golden.npz")
    a = [g[f"test2/{k}"] for k in ("x", "dt", "A_log", "B", "C")]
    assert np.array_equal(scan.scan_fwd(*a, threads=1), scan.scan_fwd(*a, threads=3))


@pytest.mark.parametrize("ci", [0, 1, 2])
def test_slot_core(ci):
    g = _g("slot_golden.npz")
    out, attn = slot_attn.naive_slot_attention(g[f"core{ci}/Q"], g[f"core{ci}/K"], g[f"core{ci}/V"])
    assert rel_err(out, g[f"core{ci}/out"]) < 1e-5
    assert rel_err(attn, g[f"core{ci}/attn"]) < 1e-5
    # softmax over slots: every token's column sums to 1 (tests/test_kernels.py:66-71)
    assert np.allclose(attn.sum(axis=1), 1.0, atol=1e-5)


def test_slot_iterations():
    g = _g("slot_golden.npz")
    W = {k[len("iter/w/"):]: g[k] for k in g.files if k.startswith("iter/w/")}
    s = g["iter/slots0"]
    for i in range(3):
        s = slot_attn.iteration_step(s, g["iter/k"], g["iter/v"], W)
        assert rel_err(s, g[f"iter/slots{i + 1}"]) < 1e-5


def test_event_naive_and_model_path():
    g = _g("event_golden.npz")
    W = {k[len("ev/w/"):]: g[k] for k in g.files if k.startswith("ev/w/")}
    H, nl = int(g["ev/n_heads"]), int(g["ev/n_layers"])
    st, mask = g["ev/states"], g["ev/mask"]
    y = event_attn.naive_sparse_event_attention(st, mask, lambda f: event_attn.level1_event(f, W, H, nl))
    assert rel_err(y, g["ev/y_naive"]) < 1e-5
    assert rel_err(y, g["ev/y_vectorized"]) < 1e-5
    # model path: key padding from dead slots (hierarchy_manager.py + level1_event.py:108-112)
    alive = g["ev/alive"]
    def fn_b(b):
        return lambda f: event_attn.level1_event(f, W, H, nl,
                                                 key_padding_mask=np.repeat(~(alive[b:b + 1] > 0.5), len(f), 0))
    ym = st.copy()
    for b in range(st.shape[0]):
        idx = np.nonzero(mask[b] > 0.5)[0]
        ym[b, idx] = fn_b(b)(st[b, idx])
    assert rel_err(ym, g["ev/y_model"]) < 1e-5


def test_event_kats():
    """Known-answer tests of tests/test_kernels.py:182-232."""
    rng = np.random.default_rng(0)
    st = rng.standard_normal((2, 16, 8, 32)).astype(np.float32)
    m = np.zeros((2, 16), np.float32)
    m[0, [2, 5, 10]] = 1
    m[1, [1, 7]] = 1
    out = event_attn.naive_sparse_event_attention(st, m, lambda f: f * 2.0)
    assert np.array_equal(out[0, 0], st[0, 0]) and np.array_equal(out[0, 3], st[0, 3])
    assert np.allclose(out[0, 2], st[0, 2] * 2) and np.allclose(out[0, 5], st[0, 5] * 2)
    assert np.array_equal(event_attn.naive_sparse_event_attention(st, np.zeros((2, 16)), lambda f: f), st)
    assert np.all(event_attn.naive_sparse_event_attention(st, np.ones((2, 16)), lambda f: f * 0) == 0)


# ---- the PyTorch restatement (oracle/torch_ref.py): CPU baseline and bf16 checker ----
def test_torch_ref_scan_and_gradients():
    import torch

    from oracle import torch_ref

    g = _g("scan_golden.npz")
    for case in ("test0", "base"):
        leaves = [torch.from_numpy(g[f"{case}/{k}"]).requires_grad_(True) for k in ("x", "dt", "A_log", "B", "C")]
        y = torch_ref.sequential_ssm_scan(*leaves)
        assert rel_err(y.detach().numpy(), g[f"{case}/y_sequential"]) < 1e-6
        y.backward(torch.from_numpy(g[f"{case}/dy"]))
        for k, t in zip(("dx", "ddt", "dA_log", "dB", "dC"), leaves):
            assert rel_err(t.grad.numpy(), g[f"{case}/{k}_sequential"]) < 1e-5, k


def test_torch_ref_iteration_gradients():
    """Forward and every gradient of three _iteration_step calls (clamps
    binding) against the reference's autograd."""
    import torch

    from oracle import torch_ref

    g = _g("train_golden.npz")
    W = {k[len("it/p/"):]: torch.from_numpy(g[k]).requires_grad_(True) for k in g.files if k.startswith("it/p/")}
    leaves = [torch.from_numpy(g[f"it/{k}"]).requires_grad_(True) for k in ("slots0", "k", "v")]
    s = leaves[0]
    for _ in range(3):
        s = torch_ref.iteration_step(s, leaves[1], leaves[2], W)
    assert rel_err(s.detach().numpy(), g["it/slots3"]) < 1e-6
    (s * torch.from_numpy(g["it/w"])).sum().backward()
    for t, k in zip(leaves, ("dslots", "dk", "dv")):
        assert rel_err(t.grad.numpy(), g[f"it/{k}"]) < 1e-5, k
    for name, t in W.items():
        key = f"it/g/{name}"
        if key in g.files and name != "norm_pre_attn.bias":  # a cancellation residue, see test_train_gpu.py
            assert rel_err(t.grad.numpy(), g[key]) < 1e-5, name


def test_torch_ref_event_model_path():
    """Level-1 stack with dead-slot key masks on the gathered events, against the
    reference's model path (gather_events -> Level1EventDynamics -> scatter_events)."""
    import torch

    from oracle import torch_ref

    g = _g("train_golden.npz")
    W = {k[len("ev/p/"):]: torch.from_numpy(g[k]) for k in g.files if k.startswith("ev/p/")}
    H, nl = int(g["ev/n_heads"]), int(g["ev/n_layers"])
    st, mask, alive = (torch.from_numpy(g[f"ev/{k}"]) for k in ("states", "mask", "alive"))
    out = st.clone()
    for b in range(st.shape[0]):
        idx = torch.nonzero(mask[b] > 0.5).flatten()
        kp = (~(alive[b] > 0.5))[None, :].expand(len(idx), -1)
        out[b, idx] = torch_ref.level1_event(st[b, idx], W, H, nl, kp)
    assert rel_err(out.numpy(), g["ev/y"]) < 1e-5
