"""KV-head tensor parallelism (wgkv.tp) on one GPU: every rank of a world of 2, 4 or 8 is run in
turn with its own pool, its gate shard and its o_proj slice, and the partial products are summed here
(the all-reduce's job).  The sum must equal the unsharded layer (all 8 KV heads in one pool, full
o_proj) within 2e-2 abs / 1e-2 rel, through a prefill and decode steps with promotions; each head's
admission bits and global lengths must be identical in both."""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from golden_cases import O
from gpu_util import to_bf16

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _bhld(x):
    return to_bf16(np.ascontiguousarray(np.transpose(x, (0, 2, 1, 3)))).transpose(1, 2)


def _make_attn(wgkv, gp, Hq, B, W, T, L, n_dec):
    Hk, D = gp.num_kv_heads, gp.head_dim
    cfg = SimpleNamespace(num_hidden_layers=1, num_key_value_heads=Hk, num_attention_heads=Hq, head_dim=D,
                          block_size=T, max_total_tokens=B * Hk * (W + L + n_dec) + 64 * T,
                          max_tokens_per_head=W + L + n_dec + T, local_window_size=W, g_defer=False, g_threshold=0.5)
    return wgkv.attach(SimpleNamespace(layer_idx=0, head_dim=D, scaling=D ** -0.5, g_predictors=gp), cfg)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_kv_head_shards_sum_to_unsharded(world):
    import wgkv
    from wgkv.dist import kv_head_shard
    from wgkv.tp import KVHeadParallelAttention, shard_gate, shard_o_proj
    B, Hq, Hk, D, L, W, T, n_dec, hidden = 2, 32, 8, 128, 700, 128, 16, 150, 1024
    rng = np.random.default_rng(world)
    torch.manual_seed(world)
    gp = wgkv.GatingPredictor(D, Hk, ["pre_k"], "gelu", 0.5, 1e-3, False, True).cuda().bfloat16()
    wo = (torch.randn(hidden, Hq * D, device="cuda") * (Hq * D) ** -0.5).bfloat16()
    full = KVHeadParallelAttention(_make_attn(wgkv, gp, Hq, B, W, T, L, n_dec), wo, reduce=False)
    shards, caches = [], []
    for r in range(world):
        (h0, h1), (q0, q1) = kv_head_shard(Hk, Hq, r, world)
        attn = _make_attn(wgkv, shard_gate(gp, h0, h1), q1 - q0, B, W, T, L, n_dec)
        shards.append(((h0, h1), (q0, q1), KVHeadParallelAttention(attn, shard_o_proj(wo, q0, q1, D), reduce=False)))
        caches.append(SimpleNamespace())
    c_full = SimpleNamespace()

    def run(T_, q, pk, k, v):
        y_full = full(c_full, (B, T_), q, pk, k, v).float()
        y_sum = torch.zeros_like(y_full)
        for ((h0, h1), (q0, q1), layer), c in zip(shards, caches):
            y_sum += layer(c, (B, T_), q[:, q0:q1], pk[:, h0:h1], k[:, h0:h1], v[:, h0:h1]).float()
        return y_full, y_sum

    q, k, v, pk = (O.randn_bf16(rng, (B, h, L, D)) for h in (Hq, Hk, Hk, Hk))
    y_full, y_sum = run(L, _bhld(q), _bhld(pk), _bhld(k), _bhld(v))
    torch.testing.assert_close(y_sum, y_full, atol=ATOL, rtol=RTOL)
    for s in range(n_dec):
        q, k, v, pk = (O.randn_bf16(rng, (B, h, 1, D)) for h in (Hq, Hk, Hk, Hk))
        y_full, y_sum = run(1, _bhld(q), _bhld(pk), _bhld(k), _bhld(v))
        torch.testing.assert_close(y_sum, y_full, atol=ATOL, rtol=RTOL, msg=lambda m: f"step {s}: {m}")
    torch.cuda.synchronize()
    wgkv.check_errors()
    for ((h0, h1), _, _), c in zip(shards, caches):
        assert torch.equal(c.global_lengths, c_full.global_lengths[:, :, h0:h1])
        assert torch.equal(c.local_is_global, c_full.local_is_global[:, :, h0:h1])
    assert int(c_full.global_lengths.min()) > 0  # prefill admitted some tokens to every head


@pytest.mark.parametrize("rows,k", [(64, 512), (5, 4096), (130, 1024)])
def test_fused_oproj_group_of_one_is_the_gemm(rows, k):
    """``wgkv_oproj_allreduce`` in a group of one GPU is the row-parallel GEMM itself: compared with an
    fp32 torch matmul of the same bf16 operands (the kernel rounds its fp32 accumulator once)."""
    from wgkv.tp import PeerGroup
    g = torch.Generator(device="cuda").manual_seed(rows + k)
    n_out = 4096
    a = torch.randn(rows, k, generator=g, device="cuda").bfloat16()
    w = (torch.randn(n_out, k, generator=g, device="cuda") * k ** -0.5).bfloat16()
    peers = PeerGroup(max_rows=256, max_cols=n_out)
    y = torch.empty(rows, n_out, dtype=torch.bfloat16, device="cuda")
    for _ in range(3):  # repeated calls advance the device epoch
        peers.oproj_allreduce(a, w, y, kernel=True)
    torch.cuda.synchronize()
    import wgkv
    wgkv.check_errors()
    torch.testing.assert_close(y.float(), a.float() @ w.float().t(), atol=ATOL, rtol=RTOL)
