"""The registered operators (``torch.ops.wgkv.*``) without a GPU: shape propagation through their
fake implementations, and CPU tensors refused by the dispatcher (there is no CPU kernel)."""
import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import wgkv.ops  # noqa: F401  (registers the operators)


def test_paged_decode_fake_shapes():
    with FakeTensorMode():
        q = torch.empty(3, 1, 32, 128, dtype=torch.bfloat16, device="cuda")
        kc = torch.empty(100, 16, 128, dtype=torch.bfloat16, device="cuda")
        sl = torch.empty(3, 8, dtype=torch.int32, device="cuda")
        bt = torch.empty(3, 8, 7, dtype=torch.int32, device="cuda")
        out = torch.ops.wgkv.paged_decode(q, kc, kc, sl, bt, 0.1)
        assert out.shape == q.shape and out.dtype == torch.bfloat16 and out.device.type == "cuda"


def test_sparse_attn_fake_shapes():
    B, L, Hq, Hk, D = 2, 300, 8, 2, 64
    R = (L + 63) // 64
    with FakeTensorMode():
        q = torch.empty(B, L, Hq, D, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(B, L, Hk, D, dtype=torch.bfloat16, device="cuda")
        bc = torch.empty(1, 1, R, dtype=torch.int32, device="cuda")
        bo = torch.empty(1, 1, R, 5, dtype=torch.int32, device="cuda")
        cc = torch.empty(B, Hk, R, dtype=torch.int32, device="cuda")
        ci = torch.empty(B, Hk, 1, 40, dtype=torch.int32, device="cuda")
        out = torch.ops.wgkv.sparse_attn(q, k, k, bc, bo, cc, ci, D ** -0.5)
        assert out.shape == q.shape and out.dtype == torch.bfloat16


def test_fake_checks_refuse_bad_shapes():
    with FakeTensorMode():
        q = torch.empty(1, 1, 6, 64, dtype=torch.bfloat16, device="cuda")
        kc = torch.empty(4, 16, 64, dtype=torch.bfloat16, device="cuda")
        sl = torch.empty(1, 4, dtype=torch.int32, device="cuda")  # 6 query heads over 4 KV heads
        bt = torch.empty(1, 4, 2, dtype=torch.int32, device="cuda")
        with pytest.raises(RuntimeError):
            torch.ops.wgkv.paged_decode(q, kc, kc, sl, bt, 0.1)


def test_cpu_tensors_have_no_kernel():
    q = torch.zeros(1, 1, 8, 64, dtype=torch.bfloat16)
    kc = torch.zeros(4, 16, 64, dtype=torch.bfloat16)
    sl = torch.ones(1, 2, dtype=torch.int32)
    bt = torch.zeros(1, 2, 1, dtype=torch.int32)
    with pytest.raises(NotImplementedError):
        torch.ops.wgkv.paged_decode(q, kc, kc, sl, bt, 0.1)


def test_traced_graph_holds_the_operator():
    """A function around the decode op traces (fake tensors, no GPU) into a graph with one wgkv node."""
    from torch.fx.experimental.proxy_tensor import make_fx

    def step(q, kc, vc, sl, bt):
        return torch.ops.wgkv.paged_decode(q * 2, kc, vc, sl, bt, 0.125).float().sum()

    with FakeTensorMode() as mode:
        args = (torch.empty(2, 1, 8, 64, dtype=torch.bfloat16, device="cuda"),
                torch.empty(10, 16, 64, dtype=torch.bfloat16, device="cuda"),
                torch.empty(10, 16, 64, dtype=torch.bfloat16, device="cuda"),
                torch.empty(2, 2, dtype=torch.int32, device="cuda"),
                torch.empty(2, 2, 5, dtype=torch.int32, device="cuda"))
    gm = make_fx(step, tracing_mode="fake")(*args)
    targets = [str(n.target) for n in gm.graph.nodes if n.op == "call_function"]
    assert sum("wgkv.paged_decode" in t for t in targets) == 1
