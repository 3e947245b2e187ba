"""SnapKV eviction on the GPU (snapkv_enabled; reference snapkv_record_queries / snapkv_evict,
src/modeling_layers.py:579-671, free-list reuse :694-709).

The oracle (pinned to the reference's own run in test_oracle_golden.py, where evicted sets agree
with torch.topk's up to the order of tied scores) and the CUDA path use the same tie rule, so after
every eviction the page tables, lengths, free list and pool bytes must be identical.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from golden_cases import O, PipelineCase
from gpu_util import bits, to_bf16, to_np
from pipeline_util import bhld, make_config, make_layers

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _check_state(cache, st):
    assert np.array_equal(cache.block_table.cpu().numpy(), st.block_table)
    assert np.array_equal(cache.global_lengths.cpu().numpy(), st.global_lengths)
    assert int(cache.next_free_block.item()) == st.next_free_block
    n = int(cache.free_block_count.item())
    assert cache.free_block_ids[:n].cpu().tolist() == st.free
    dg = O.pool_digest(cache.block_table.cpu().numpy(), cache.global_lengths.cpu().numpy(), cache.local_length,
                       bits(cache.block_pool_k), bits(cache.block_pool_v), st.page, st.window)
    ds = O.pool_digest(st.block_table, st.global_lengths, st.local_length, O.bf16_bits(st.k), O.bf16_bits(st.v),
                       st.page, st.window)
    assert np.array_equal(dg, ds)


def test_snapkv_golden_pipeline():
    import wgkv
    case = PipelineCase("snapkv_small")
    W, scale = case.W, case.D ** -0.5
    cfg = make_config(case)
    cfg.snapkv_enabled = True
    cfg.snapkv_max_cached_tokens, cfg.snapkv_evict_ratio, cfg.snapkv_window_size, cfg.snapkv_kernel_size = case.snapkv
    layers = make_layers(wgkv, case)
    for a in layers:
        a.config = cfg
    st = case.new_state()
    cache = SimpleNamespace()
    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        layers[l].self_attn_forward_patch(layers[l], 3, None, cache, (1, case.L), bhld(q), bhld(pk), bhld(k), bhld(v))
        st.prefill_layer(l, k, v, case.ref_mask(l), pre_key=pk)
        st.snap_record(l, q)
        if l == case.Ly - 1 and st.snap_should_evict():
            st.snap_evict(scale)
    torch.cuda.synchronize()
    wgkv.check_errors()
    assert cache.snapkv_evict_count == st.evict_count == 1
    _check_state(cache, st)
    for s in range(case.n_decode):
        for l in range(case.Ly):
            q, k, v, pk = case.decode[s][l]
            if l == 0 and st.local_length == st.window:
                st.promote()
            ins = st.local_length if st.local_length < W else st.local_ptr
            o, _, _ = layers[l].self_attn_forward_patch(layers[l], 3, None, cache, (1, 1), bhld(q), bhld(pk), bhld(k),
                                                        bhld(v))
            gbit = cache.local_is_global[l, 0, :, ins].cpu().numpy().astype(bool)
            cur = st.append_layer(l, k[:, :, 0], v[:, :, 0], gbit[None])
            sl, bt = st.decode_tables(l, cur)
            kc, vc = st.paged_views()
            ref = O.paged_decode(q.transpose(0, 2, 1, 3), kc, vc, sl, bt, scale)
            np.testing.assert_allclose(to_np(o)[0, 0], ref[0, 0], atol=ATOL, rtol=RTOL)
            st.snap_record(l, q)
            if l == case.Ly - 1 and st.snap_should_evict():
                st.snap_evict(scale)
        torch.cuda.synchronize()
        wgkv.check_errors()
        assert cache.snapkv_evict_count == st.evict_count, s
        _check_state(cache, st)
    assert st.evict_count == 2


@pytest.mark.parametrize("B,Hk,G,D,win,ks,ratio", [(2, 2, 4, 128, 32, 5, 0.3), (1, 4, 2, 64, 64, 3, 0.55),
                                                   (1, 2, 8, 128, 16, 7, 1.0),
                                                   # several 256-row chunks / a 16-row last chunk / a
                                                   # half-filled 32-row piece / G = 16 (tensor-core passes)
                                                   (1, 2, 4, 128, 256, 5, 0.3), (1, 1, 4, 128, 260, 5, 0.3),
                                                   (2, 2, 2, 64, 40, 3, 0.4), (1, 1, 16, 128, 16, 5, 0.3)])
def test_snapkv_evict_matches_oracle(B, Hk, G, D, win, ks, ratio):
    import wgkv
    W, T, L = 64, 16, 2500
    Hq = Hk * G
    tot = 2 * B * Hk * (L + 64) + 64
    cache = SimpleNamespace()
    wgkv.init_pool(cache, layers=2, batch=B, kv_heads=Hk, head_dim=D, window=W, page=T, max_total_tokens=tot,
                   max_tokens_per_head=L + 64, device="cuda", snapkv_window=win, q_heads=Hq)
    st = O.PoolState(layers=2, batch=B, kv_heads=Hk, head_dim=D, window=W, page=T, max_total_tokens=tot,
                     max_tokens_per_head=L + 64, snapkv=(0, ratio, win, ks), q_heads=Hq)
    rng = np.random.default_rng(win + ks)
    ws = torch.empty(int(wgkv.lib.wgkv_prefill_admit_workspace_size(B, Hk, L)), dtype=torch.uint8, device="cuda")
    for l in range(2):
        k = O.randn_bf16(rng, (B, Hk, L, D))
        v = O.randn_bf16(rng, (B, Hk, L, D))
        g = (rng.random((B, Hk, L)) < rng.uniform(0.05, 0.8, (B, Hk))[..., None]).astype(np.uint8)
        kt, vt, gm = to_bf16(k), to_bf16(v), torch.from_numpy(g).cuda()
        assert wgkv.lib.wgkv_prefill_admit(wgkv.pool.pool_ref(cache), l, L, kt.data_ptr(), *kt.stride()[:3],
                                           vt.data_ptr(), *vt.stride()[:3], None, 0, 0, 0, gm.data_ptr(), *gm.stride(),
                                           ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream) == 0
        st.prefill_layer(l, k, v, g.astype(bool))
    qb = O.randn_bf16(rng, (2, B, win, Hq, D))
    st.snap_q[:] = qb
    cache.snapkv_query_buffer.copy_(to_bf16(qb))
    cache.local_length = W
    st.local_length = W
    scale = D ** -0.5
    wsb = torch.empty(int(wgkv.lib.wgkv_snapkv_workspace_size(wgkv.pool.pool_ref(cache), win, Hq)), dtype=torch.uint8,
                      device="cuda")
    for rep in range(2):  # a second eviction frees more pages behind the first ones
        assert wgkv.lib.wgkv_snapkv_evict(wgkv.pool.pool_ref(cache), cache.snapkv_query_buffer.data_ptr(), win, Hq,
                                          scale, ratio, ks, wsb.data_ptr(), wsb.numel(),
                                          torch.cuda.current_stream().cuda_stream) == 0
        st.snap_evict(scale)
        torch.cuda.synchronize()
        wgkv.check_errors()
        _check_state(cache, st)
