"""Decode steps replayed as CUDA graphs (device ring position) equal eager decode steps exactly.

Two caches get the same prefill; one then decodes eagerly through the reference-named patch
(host ring position, src/modeling_layers.py:1452-1509, :1534-1629), the other through
``wgkv.DecodeGraph`` (one capture, then replays).  Every step's attention output and, at the
end, the page tables, lengths, ring bits, allocator, ring position and pool bytes must be
identical.  The steps cross the ring-fill phase, the first full ring, wrap-around of local_ptr,
promotions and (with g_defer) the whole-ring rescoring at insert position window - 1.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from golden_cases import O
from gpu_util import bits, to_bf16

pytestmark = pytest.mark.gpu


def _layers(wgkv, Ly, Hk, G, D, T, W, max_total, max_head, defer, seed):
    cfg = SimpleNamespace(num_hidden_layers=Ly, num_key_value_heads=Hk, num_attention_heads=Hk * G, head_dim=D,
                          block_size=T, max_total_tokens=max_total, max_tokens_per_head=max_head,
                          local_window_size=W, g_defer=defer, g_threshold=0.5)
    torch.manual_seed(seed)
    out = []
    for l in range(Ly):
        gp = wgkv.GatingPredictor(D, Hk, ["pre_k"], "gelu", 64 / D, 1e-3, False, True).cuda().bfloat16()
        with torch.no_grad():
            gp.conv2.bias.fill_(0.3)
        out.append(wgkv.attach(SimpleNamespace(layer_idx=l, head_dim=D, scaling=D ** -0.5, g_predictors=gp), cfg))
    return out


@pytest.mark.parametrize("defer", [False, True])
@pytest.mark.parametrize("B,Ly,Hk,G,D,L,W,T,n_dec", [(1, 3, 2, 4, 128, 300, 64, 16, 150),
                                                     (2, 2, 4, 2, 64, 40, 64, 16, 100)])
def test_graph_decode_equals_eager(defer, B, Ly, Hk, G, D, L, W, T, n_dec):
    import wgkv
    Hq = Hk * G
    max_head = W + L + n_dec + T
    max_total = Ly * B * Hk * max_head + 64 * T
    layers = _layers(wgkv, Ly, Hk, G, D, T, W, max_total, max_head, defer, seed=B + 10 * L)
    rng = np.random.default_rng(L)
    caches = [SimpleNamespace(), SimpleNamespace()]
    for l in range(Ly):
        q, k, v, pk = (to_bf16(O.randn_bf16(rng, (B, h, L, D))) for h in (Hq, Hk, Hk, Hk))
        for c in caches:
            layers[l].self_attn_forward_patch(layers[l], 3, None, c, (B, L), q, pk, k, v)
    torch.cuda.synchronize()
    wgkv.check_errors()
    ce, cg = caches

    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    steps = torch.randn(n_dec, Ly, 4, B, Hq, 1, D, generator=g, device="cuda").to(torch.bfloat16)
    # static inputs of the graph, refilled before each replay
    s_in = torch.empty_like(steps[0])
    s_out = torch.empty(Ly, B, 1, Hq, D, dtype=torch.bfloat16, device="cuda")

    def run_step(cache, x, out):
        for l in range(Ly):
            q, k, v, pk = x[l, 0], x[l, 1, :, :Hk], x[l, 2, :, :Hk], x[l, 3, :, :Hk]
            o, _, _ = layers[l].self_attn_forward_patch(layers[l], 3, None, cache, (B, 1), q, pk, k, v)
            out[l].copy_(o.reshape(B, 1, Hq, D))
        return out

    e_out = torch.empty_like(s_out)
    dg = wgkv.DecodeGraph(cg, W, defer=defer)
    for s in range(n_dec):
        run_step(ce, steps[s], e_out)
        if s == 0:
            s_in.copy_(steps[0])
            dg.capture(lambda: run_step(cg, s_in, s_out))
            got = s_out
        else:
            s_in.copy_(steps[s])
            got = dg.replay()
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int16), e_out.view(torch.int16)), f"step {s}"
    wgkv.check_errors()

    assert (cg.local_length, cg.local_ptr) == (ce.local_length, ce.local_ptr)
    assert cg.ring_state.tolist() == [ce.local_length, ce.local_ptr]
    for name in ("block_table", "global_lengths", "local_is_global", "next_free_block", "cache_seqlens"):
        assert torch.equal(getattr(cg, name), getattr(ce, name)), name
    dge = O.pool_digest(ce.block_table.cpu().numpy(), ce.global_lengths.cpu().numpy(), ce.local_length,
                        bits(ce.block_pool_k), bits(ce.block_pool_v), T, W)
    dgg = O.pool_digest(cg.block_table.cpu().numpy(), cg.global_lengths.cpu().numpy(), cg.local_length,
                        bits(cg.block_pool_k), bits(cg.block_pool_v), T, W)
    assert np.array_equal(dge, dgg)
    # after the graph steps, eager steps continue from the same position
    run_step(ce, steps[0], e_out)
    run_step(cg, steps[0], s_out)
    torch.cuda.synchronize()
    assert torch.equal(s_out.view(torch.int16), e_out.view(torch.int16))
