"""QUEST block selection on the GPU (use_quest; reference quest_select_blocks,
src/modeling_layers.py:452-576, page bounds :744-761 and :1333-1347).

* golden replay: the quest_small fixture (reference run on CPU) through the patched layers; page key
  bounds bit-exact, selected pages equal to the oracle's (same tie rule) and to the reference's up to
  the order of tied scores, attention within 2e-2 / 1e-2;
* a batched case with many pages: the kernel's selection equals the oracle's on the same pool state;
* the device ring position (graph capture) gives the same selection as the host one.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from golden_cases import O, PipelineCase, quest_sets_agree
from gpu_util import bits, to_bf16, to_np
from pipeline_util import bhld, make_config, make_layers

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _live_bounds(cache, T, W):
    bt = cache.block_table.cpu().numpy()
    gl = cache.global_lengths.cpu().numpy()
    Ly, B, Hk, _ = bt.shape
    pages = []
    for l in range(Ly):
        for b in range(B):
            for h in range(Hk):
                n = (int(gl[l, b, h]) + T - 1) // T
                pages += list(bt[l, b, h, W // T:W // T + n])
    idx = torch.tensor(pages, dtype=torch.long, device="cuda")
    return bits(cache.quest_block_key_min[idx]), bits(cache.quest_block_key_max[idx])


def test_quest_golden_pipeline():
    import wgkv
    case = PipelineCase("quest_small")
    T, W, z = case.T, case.W, case.z
    cfg = make_config(case)
    cfg.use_quest, cfg.quest_token_budget = True, case.quest_budget
    layers = make_layers(wgkv, case)
    for a in layers:
        a.config = cfg
    st = case.new_state()
    cache = SimpleNamespace()
    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        layers[l].self_attn_forward_patch(layers[l], 3, None, cache, (1, case.L), bhld(q), bhld(pk), bhld(k), bhld(v))
        st.prefill_layer(l, k, v, case.ref_mask(l), pre_key=pk)
    torch.cuda.synchronize()
    wgkv.check_errors()
    mn, mx = _live_bounds(cache, T, W)
    assert np.array_equal(mn, z["prefill_quest_min"]) and np.array_equal(mx, z["prefill_quest_max"])
    exact_ref = 0
    for s in range(case.n_decode):
        for l in range(case.Ly):
            q, k, v, pk = case.decode[s][l]
            if l == 0 and st.local_length == st.window:
                st.promote()
            cur = cache.local_length + 1 if cache.local_length < W else W
            ins = st.local_length if st.local_length < W else st.local_ptr
            o, _, _ = layers[l].self_attn_forward_patch(layers[l], 3, None, cache, (1, 1), bhld(q), bhld(pk), bhld(k),
                                                        bhld(v))
            gbit = cache.local_is_global[l, 0, :, ins].cpu().numpy()
            cur_o = st.append_layer(l, k[:, :, 0], v[:, :, 0], gbit.astype(bool)[None])
            assert cur_o == cur
            sl_o, tabs_o = st.quest_select(l, cur, q[:, :, 0], case.quest_budget)
            sl, bt = wgkv.quest_select_blocks(layers[l], bhld(q), cache, W // T, "cuda", cur)
            sl, bt = sl.cpu().numpy(), bt.cpu().numpy()
            assert np.array_equal(sl, sl_o) and np.array_equal(sl[0], z[f"d{s}_l{l}_qsl"]), (s, l)
            for h in range(case.Hk):
                n = len(tabs_o[h])
                assert np.array_equal(bt[0, h, :n], tabs_o[h]), (s, l, h)
                ref = z[f"d{s}_l{l}_qbt"][h, :n]
                assert quest_sets_agree(st, l, 0, h, q[0, h * case.G:(h + 1) * case.G, 0], tabs_o[h], ref)
                exact_ref += set(ref.tolist()) == set(tabs_o[h].tolist())
            kc, vc = st.paged_views()
            maxn = max(len(t) for t in tabs_o)
            tb = np.full((1, case.Hk, maxn), 0, np.int32)
            for h, t in enumerate(tabs_o):
                tb[0, h, :len(t)] = t
            ref_o = O.paged_decode(q.transpose(0, 2, 1, 3), kc, vc, sl_o, tb, case.D ** -0.5)
            np.testing.assert_allclose(to_np(o)[0, 0], ref_o[0, 0], atol=ATOL, rtol=RTOL)
        torch.cuda.synchronize()
        wgkv.check_errors()
    assert exact_ref > 0
    mn, mx = _live_bounds(cache, T, W)
    assert np.array_equal(mn, z["final_quest_min"]) and np.array_equal(mx, z["final_quest_max"])


@pytest.mark.parametrize("G,D", [(4, 128), (2, 64), (3, 128)])
@pytest.mark.parametrize("budget", [64 + 400, 64 + 17, 64 + 16 * 500, 32])
def test_quest_select_batched_matches_oracle(budget, G, D):
    import wgkv
    B, Hk, W, T, L = 2, 4, 64, 16, 3000
    Hq = Hk * G
    cache = SimpleNamespace()
    wgkv.init_pool(cache, layers=1, batch=B, kv_heads=Hk, head_dim=D, window=W, page=T,
                   max_total_tokens=B * Hk * (L + 64) + 64, max_tokens_per_head=L + 64, device="cuda", quest=True)
    rng = np.random.default_rng(budget)
    k = O.randn_bf16(rng, (B, Hk, L, D))
    v = O.randn_bf16(rng, (B, Hk, L, D))
    rates = rng.uniform(0.1, 0.9, (B, Hk))
    g = (rng.random((B, Hk, L)) < rates[..., None]).astype(np.uint8)
    kt, vt = to_bf16(k), to_bf16(v)
    gm = torch.from_numpy(g).cuda()
    ws = torch.empty(int(wgkv.lib.wgkv_prefill_admit_workspace_size(B, Hk, L)), dtype=torch.uint8, device="cuda")
    st_ = wgkv.lib.wgkv_prefill_admit(wgkv.pool.pool_ref(cache), 0, L, kt.data_ptr(), *kt.stride()[:3],
                                      vt.data_ptr(), *vt.stride()[:3], None, 0, 0, 0, gm.data_ptr(), *gm.stride(),
                                      ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    assert st_ == 0
    cache.local_length = W
    torch.cuda.synchronize()
    wgkv.check_errors()
    st = O.PoolState(layers=1, batch=B, kv_heads=Hk, head_dim=D, window=W, page=T,
                     max_total_tokens=B * Hk * (L + 64) + 64, max_tokens_per_head=L + 64, quest=True)
    st.prefill_layer(0, k, v, g.astype(bool))
    assert np.array_equal(bits(cache.quest_block_key_min), O.bf16_bits(st.qmin))  # bounds of every page
    assert np.array_equal(bits(cache.quest_block_key_max), O.bf16_bits(st.qmax))
    a = SimpleNamespace(layer_idx=0, head_dim=D, scaling=D ** -0.5,
                        config=SimpleNamespace(quest_token_budget=budget))
    for trial in range(3):
        q = O.randn_bf16(rng, (B, Hq, 1, D)) * (trial + 1)
        q = O.bf16(q)
        sl, bt = wgkv.quest_select_blocks(a, to_bf16(q), cache, W // T, "cuda", W)
        sl_o, tabs = st.quest_select(0, W, q[:, :, 0], budget)
        assert np.array_equal(sl.cpu().numpy(), sl_o)
        btn = bt.cpu().numpy()
        for i, t in enumerate(tabs):
            assert np.array_equal(btn[i // Hk, i % Hk, :len(t)], t), (trial, i)
    # graph-capture form: the ring length read from the device copy gives the same selection
    cache.local_length, cache.local_ptr = W, 5
    wgkv.ring_to_device(cache)
    sl2, bt2 = wgkv.quest_select_blocks(a, to_bf16(q), cache, W // T, "cuda", wgkv.RING_ON_DEVICE)
    assert torch.equal(sl2, sl)
    b2n, sln = bt2.cpu().numpy(), sl.cpu().numpy()
    for i in range(B * Hk):
        n = (int(sln[i // Hk, i % Hk]) + T - 1) // T  # entries past a head's pages are not written
        assert np.array_equal(b2n[i // Hk, i % Hk, :n], btn[i // Hk, i % Hk, :n])
