"""KV-head tensor parallelism (wgkv.tp) on CPU: head sharding of the gate, the row-parallel o_proj
slice, and the all-reduce over ranks (gloo, world size 2).  The attention itself is the CUDA path
on a GPU; here a plain torch attention stands in for it so the host logic runs without one."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from golden_cases import O


def _gate_params(gp):
    Hk, inner, I = gp.num_kv_heads, gp.inner_dim, gp.input_dim
    f = lambda t: t.detach().float().numpy()  # noqa: E731
    return O.GateParams(w1=f(gp.conv1.weight).reshape(Hk, inner, I), b1=f(gp.conv1.bias).reshape(Hk, inner),
                        w2=f(gp.conv2.weight).reshape(Hk, inner), b2=f(gp.conv2.bias))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_gate_scores_equal_full_slice(world):
    import wgkv
    from wgkv.dist import kv_head_shard
    from wgkv.tp import shard_gate
    torch.manual_seed(0)
    Hk, D = 8, 64
    gp = wgkv.GatingPredictor(D, Hk, ["pre_k"], "gelu", 1.0, 1e-3, False, True).bfloat16()
    x = O.randn_bf16(np.random.default_rng(1), (1, Hk, 50, D))
    full = O.gate_scores(_gate_params(gp), pre_key=x)
    for r in range(world):
        (h0, h1), _ = kv_head_shard(Hk, 32, r, world)
        sg = shard_gate(gp, h0, h1)
        assert sg.num_kv_heads == h1 - h0 and sg.g_fast_path == gp.g_fast_path
        part = O.gate_scores(_gate_params(sg), pre_key=x[:, h0:h1])
        assert np.array_equal(O.bf16_bits(part), O.bf16_bits(full[:, h0:h1]))


class _TorchAttention:
    """Stand-in for the CUDA path: causal attention of (B, H, T, D) fp32 inputs, GQA by repetition."""

    @staticmethod
    def self_attn_forward_patch(self, mode, mask, cache, shape, q, pk, k, v):
        G = q.shape[1] // k.shape[1]
        o = torch.nn.functional.scaled_dot_product_attention(q, k.repeat_interleave(G, 1),
                                                             v.repeat_interleave(G, 1), is_causal=True)
        B, H, T, D = o.shape
        return o.transpose(1, 2).reshape(B, T, H * D), None, None


def _inputs(B=2, T=12, Hq=8, Hk=4, D=16, hidden=48):
    g = torch.Generator().manual_seed(5)
    q = torch.randn(B, Hq, T, D, generator=g)
    k, v = torch.randn(B, Hk, T, D, generator=g), torch.randn(B, Hk, T, D, generator=g)
    w = torch.randn(hidden, Hq * D, generator=g) * 0.1
    return q, k, v, w


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_q):
    import torch.distributed as dist
    from wgkv.dist import kv_head_shard
    from wgkv.tp import KVHeadParallelAttention, shard_o_proj
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, w = _inputs()
        (h0, h1), (q0, q1) = kv_head_shard(k.shape[1], q.shape[1], rank, world)
        layer = KVHeadParallelAttention(_TorchAttention(), shard_o_proj(w, q0, q1, q.shape[-1]))
        y = layer(None, (q.shape[0], q.shape[2]), q[:, q0:q1], k[:, h0:h1], k[:, h0:h1], v[:, h0:h1])
        out_q.put((rank, y.numpy()))
    finally:
        dist.destroy_process_group()


def test_gloo_world2_sum_of_shards_equals_unsharded():
    world = 2
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out_q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(out_q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    q, k, v, w = _inputs()
    o, _, _ = _TorchAttention.self_attn_forward_patch(None, 3, None, None, None, q, k, k, v)
    ref = (o.reshape(-1, o.shape[-1]) @ w.t()).numpy()
    for r in range(world):
        np.testing.assert_allclose(res[r], ref, rtol=1e-5, atol=1e-5)


def test_unreduced_partials_sum_to_unsharded():
    from wgkv.dist import kv_head_shard
    from wgkv.tp import KVHeadParallelAttention, shard_o_proj
    q, k, v, w = _inputs()
    o, _, _ = _TorchAttention.self_attn_forward_patch(None, 3, None, None, None, q, k, k, v)
    ref = o.reshape(-1, o.shape[-1]) @ w.t()
    for world in (1, 2, 4):
        acc = torch.zeros_like(ref)
        for r in range(world):
            (h0, h1), (q0, q1) = kv_head_shard(k.shape[1], q.shape[1], r, world)
            layer = KVHeadParallelAttention(_TorchAttention(), shard_o_proj(w, q0, q1, q.shape[-1]), reduce=False)
            acc += layer(None, (q.shape[0], q.shape[2]), q[:, q0:q1], k[:, h0:h1], k[:, h0:h1], v[:, h0:h1])
        torch.testing.assert_close(acc, ref, rtol=1e-5, atol=1e-5)
    with pytest.raises(ValueError):
        KVHeadParallelAttention(_TorchAttention(), w[:, :16])(None, (2, 12), q, k, k, v)
