"""Batch > 1 through the whole patch (prefill, then decode steps with promotions) against the oracle.

The reference asserts batch 1 (src/modeling_layers.py:1614); the batch axis is this build's
generalisation, so its oracle is the batched restatement in oracle/wgkv_oracle.py (which equals the
reference for batch 1, see test_oracle_golden.py).  Tables, lengths, ring bits, the allocator and the
pool bytes must match exactly; attention within 2e-2 abs / 1e-2 rel.  Masks come from the GPU gate and
are fed to the oracle, so the comparison isolates the state machine and the attention.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from golden_cases import O
from gpu_util import bits, to_bf16, to_np

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _bhld(x):
    return to_bf16(np.ascontiguousarray(np.transpose(x, (0, 2, 1, 3)))).transpose(1, 2)


@pytest.mark.parametrize("B,Ly,Hk,G,L,W,T,n_dec", [(3, 2, 2, 4, 300, 64, 16, 70), (2, 3, 4, 2, 180, 64, 32, 40)])
def test_batched_prefill_and_decode(B, Ly, Hk, G, L, W, T, n_dec):
    import wgkv
    rng = np.random.default_rng(B * 1000 + L)
    D, inner, Hq = 128, 64, Hk * G
    max_total, max_head = Ly * B * Hk * (W + L + n_dec) + 64 * T, W + L + n_dec + T
    cfg = SimpleNamespace(num_hidden_layers=Ly, num_key_value_heads=Hk, num_attention_heads=Hq, head_dim=D,
                          block_size=T, max_total_tokens=max_total, max_tokens_per_head=max_head,
                          local_window_size=W, g_defer=False, g_threshold=0.5)
    layers = []
    torch.manual_seed(B)
    for l in range(Ly):
        gp = wgkv.GatingPredictor(D, Hk, ["pre_k"], "gelu", inner / D, 1e-3, False, True).cuda().bfloat16()
        with torch.no_grad():
            gp.conv2.bias.fill_(0.3)  # admit a healthy fraction
        layers.append(wgkv.attach(SimpleNamespace(layer_idx=l, head_dim=D, scaling=D ** -0.5, g_predictors=gp), cfg))
    st = O.PoolState(layers=Ly, batch=B, kv_heads=Hk, head_dim=D, window=W, page=T, max_total_tokens=max_total,
                     max_tokens_per_head=max_head)
    cache = SimpleNamespace()
    for l in range(Ly):
        q, k, v, pk = (O.randn_bf16(rng, (B, h, L, D)) for h in (Hq, Hk, Hk, Hk))
        o, _, _ = layers[l].self_attn_forward_patch(layers[l], 3, None, cache, (B, L), _bhld(q), _bhld(pk), _bhld(k),
                                                    _bhld(v))
        g = torch.empty(B, Hk, L, dtype=torch.uint8, device="cuda")
        layers[l].g_predictors.admit(_bhld(pk), _bhld(k), _bhld(v), 0.5, g)
        gm = to_np(g).astype(bool)
        st.prefill_layer(l, k, v, gm)
        rows = np.arange(L - 16, L)
        idx = O.generate_sparse_indices(gm, W, L)
        mk = O.sparse_mask_from_indices(*idx, L, G, rows=rows)
        ref = O.masked_attention(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3), mk, rows=rows)
        np.testing.assert_allclose(to_np(o)[:, rows], ref, atol=ATOL, rtol=RTOL)
    torch.cuda.synchronize()
    wgkv.check_errors()

    def check_state():
        assert np.array_equal(cache.block_table.cpu().numpy(), st.block_table)
        assert np.array_equal(cache.global_lengths.cpu().numpy(), st.global_lengths)
        assert np.array_equal(cache.local_is_global.cpu().numpy().astype(bool), st.local_is_global)
        assert int(cache.next_free_block.item()) == st.next_free_block
        assert cache.local_ptr == st.local_ptr and cache.local_length == st.local_length
        dg = O.pool_digest(cache.block_table.cpu().numpy(), cache.global_lengths.cpu().numpy(), cache.local_length,
                           bits(cache.block_pool_k), bits(cache.block_pool_v), T, W)
        ds = O.pool_digest(st.block_table, st.global_lengths, st.local_length, O.bf16_bits(st.k), O.bf16_bits(st.v),
                           T, W)
        assert np.array_equal(dg, ds)

    check_state()
    for s in range(n_dec):
        for l in range(Ly):
            q, k, v, pk = (O.randn_bf16(rng, (B, h, 1, D)) for h in (Hq, Hk, Hk, Hk))
            if l == 0 and st.local_length == W:
                st.promote()
            ins = st.local_ptr if st.local_length == W else st.local_length
            o, _, _ = layers[l].self_attn_forward_patch(layers[l], 3, None, cache, (B, 1), _bhld(q), _bhld(pk),
                                                        _bhld(k), _bhld(v))
            gbit = cache.local_is_global[l, :, :, ins].cpu().numpy().astype(bool)  # the GPU gate's decision
            cur = st.append_layer(l, k[:, :, 0], v[:, :, 0], gbit)
            sl, bt = st.decode_tables(l, cur)
            kc, vc = st.paged_views()
            ref = O.paged_decode(q.transpose(0, 2, 1, 3), kc, vc, sl, bt, D ** -0.5)
            np.testing.assert_allclose(to_np(o), ref, atol=ATOL, rtol=RTOL)
        if s % 10 == 9 or s == n_dec - 1:
            torch.cuda.synchronize()
            wgkv.check_errors()
            check_state()
