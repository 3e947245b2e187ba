"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

These run on CPU only.  They check that ``oracle/wgkv_oracle.py`` reproduces
what the reference code produced in ``tests/golden/make_golden.py``:
admission scores/masks, page tables, global lengths, pool contents, sparse
indices, sparse-prefill rows and decode outputs.
"""
import numpy as np
import pytest

from golden_cases import O, PipelineCase, indices_case, load, regen_decode_inputs

PIPELINES = ["c1_prefill", "promote_small", "defer_small"]


@pytest.fixture(scope="module", params=PIPELINES)
def case(request):
    return PipelineCase(request.param)


def test_sparse_indices_match_reference():
    z = load("sparse_indices")
    for i in range(int(z["n_cases"])):
        (B, Hk, L, W, gs), g, fast, ref = indices_case(z, i)
        mine = O.generate_sparse_indices(g, W, L)
        for a, b in zip(mine, fast):
            assert a.shape == b.shape and np.array_equal(a, b), f"case {i}"
        mine_ref = O.generate_sparse_indices_ref(g, W, L)
        for a, b in zip(mine_ref, ref):
            assert a.shape == b.shape and np.array_equal(a, b), f"case {i}"
        # the reference's own acceptance rule (utils/test_sparse_indices.py:30-46)
        assert O.indices_equal(mine, ref)


def test_paged_decode_matches_reference_oracle():
    z = load("paged_decode")
    for i in range(int(z["n_cases"])):
        p = z[f"c{i}_params"]
        q, kc, vc, sl, tbl = regen_decode_inputs(p)
        o = O.paged_decode(q, kc, vc, sl, tbl, int(p[2]) ** -0.5)
        # the reference oracle computes in bf16 (torch CPU); 2e-2 covers its rounding
        np.testing.assert_allclose(o, z[f"c{i}_out"], atol=2e-2, rtol=1e-2)


def test_gate_scores_match_reference(case):
    total = mism = 0
    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        s = O.gate_scores(case.params[l], pre_key=pk, post_key=k, value=v)
        ref = case.ref_scores(l)
        diff = O.bf16_bits(s) != O.bf16_bits(ref)
        total += s.size
        mism += int(diff.sum())
        # masks: bit-exact required
        assert np.array_equal(O.admission_mask(s, case.threshold), case.ref_mask(l))
    # scores: identical bf16 except for rare 1-ulp accumulation-order differences
    assert mism <= max(2, total // 2000), (mism, total)


def test_prefill_state_matches_reference(case):
    st = case.new_state()
    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        st.prefill_layer(l, k, v, case.ref_mask(l), pre_key=pk)
    z = case.z
    assert np.array_equal(st.block_table[:, 0], z["prefill_block_table"])
    assert np.array_equal(st.global_lengths[:, 0], z["prefill_global_lengths"])
    assert np.array_equal(st.local_is_global[:, 0], z["prefill_local_is_global"])
    assert st.next_free_block == int(z["prefill_next_free_block"])
    dig = O.pool_digest(st.block_table, st.global_lengths, st.local_length,
                        O.bf16_bits(st.k), O.bf16_bits(st.v), st.page, st.window)
    assert np.array_equal(dig, z["prefill_pool_sha"])


def test_prefill_indices_and_attention_rows(case):
    L = case.L
    rows = np.arange(L - case.rows_out, L)
    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        g = case.ref_mask(l)
        idx = O.generate_sparse_indices(g, case.W, L)
        for a, n in zip(idx, ("bc", "bo", "cc", "ci")):
            assert np.array_equal(a, case.z[f"l{l}_{n}"])
        m1 = O.sparse_mask_from_indices(*idx, L, case.G, rows=rows)
        m2 = O.ideal_mask(g, case.W, L, rows=rows)
        assert np.array_equal(m1, m2)
        o = O.masked_attention(q.transpose(0, 2, 1, 3), k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3), m1, rows=rows)
        np.testing.assert_allclose(o[0], case.z[f"l{l}_attn_rows"], atol=1e-5, rtol=1e-5)


def test_decode_steps_match_reference(case):
    st = case.new_state()
    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        st.prefill_layer(l, k, v, case.ref_mask(l), pre_key=pk)
    z = case.z
    gate = lambda l: (lambda pre, post, val: O.gate_scores(case.params[l], pre_key=pre, post_key=post, value=val))
    for s in range(case.n_decode):
        for l in range(case.Ly):
            q, k, v, pk = case.decode[s][l]
            if l == 0 and st.local_length == st.window:
                st.promote()
            gm = case.ref_decode_mask(s, l)
            cur = st.append_layer(l, k[:, :, 0], v[:, :, 0], None if gm is None else gm[:, :, 0],
                                  pre_key_new=pk[:, :, 0], gate_fn=gate(l), threshold=case.threshold)
            sl, bt = st.decode_tables(l, cur)
            kc, vc = st.paged_views()
            o = O.paged_decode(q.transpose(0, 2, 1, 3), kc, vc, sl, bt, case.D ** -0.5)
            np.testing.assert_allclose(o[0, 0], z[f"d{s}_l{l}_out"], atol=2e-2, rtol=1e-2)
        assert np.array_equal(st.block_table[:, 0], z[f"d{s}_block_table"]), s
        assert np.array_equal(st.global_lengths[:, 0], z[f"d{s}_global_lengths"]), s
        assert np.array_equal(st.local_is_global[:, 0], z[f"d{s}_local_is_global"]), s
        assert st.next_free_block == int(z[f"d{s}_next_free_block"])
        assert st.local_ptr == int(z[f"d{s}_local_ptr"]) and st.local_length == int(z[f"d{s}_local_length"])
        dig = O.pool_digest(st.block_table, st.global_lengths, st.local_length,
                            O.bf16_bits(st.k), O.bf16_bits(st.v), st.page, st.window)
        assert np.array_equal(dig, z[f"d{s}_pool_sha"]), s


def test_quest_selection_matches_reference():
    """QUEST (use_quest): page key bounds after prefill and promotion, the selected pages and lengths
    of quest_select_blocks, and the attention over them, against the reference run on CPU."""
    from golden_cases import PipelineCase, quest_sets_agree
    case = PipelineCase("quest_small")
    st = case.new_state()
    z = case.z
    T, W = case.T, case.W

    def live_bounds():
        pages = []
        for l in range(case.Ly):
            for h in range(case.Hk):
                n = (int(st.global_lengths[l, 0, h]) + T - 1) // T
                pages += list(st.block_table[l, 0, h, W // T:W // T + n])
        return O.bf16_bits(st.qmin[pages]), O.bf16_bits(st.qmax[pages])

    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        st.prefill_layer(l, k, v, case.ref_mask(l), pre_key=pk)
    mn, mx = live_bounds()
    assert np.array_equal(mn, z["prefill_quest_min"]) and np.array_equal(mx, z["prefill_quest_max"])
    partial = 0
    for s in range(case.n_decode):
        for l in range(case.Ly):
            q, k, v, pk = case.decode[s][l]
            if l == 0 and st.local_length == st.window:
                st.promote()
            gm = case.ref_decode_mask(s, l)
            cur = st.append_layer(l, k[:, :, 0], v[:, :, 0], gm[:, :, 0])
            sl, tables = st.quest_select(l, cur, q[:, :, 0], case.quest_budget)
            assert np.array_equal(sl[0], z[f"d{s}_l{l}_qsl"]), (s, l)
            for h in range(case.Hk):
                n = (int(sl[0, h]) - cur + T - 1) // T + (cur + T - 1) // T
                ref_pages = z[f"d{s}_l{l}_qbt"][h, :n]
                assert quest_sets_agree(st, l, 0, h, q[0, h * case.G:(h + 1) * case.G, 0], tables[h], ref_pages), (s, l, h)
                partial += n < (cur + T - 1) // T + (int(st.global_lengths[l, 0, h]) + T - 1) // T
            # attention over the reference's choice (equal to ours up to tie order, checked above)
            bt = z[f"d{s}_l{l}_qbt"][None].astype(np.int32)
            kc, vc = st.paged_views()
            o = O.paged_decode(q.transpose(0, 2, 1, 3), kc, vc, sl, bt, case.D ** -0.5)
            np.testing.assert_allclose(o[0, 0], z[f"d{s}_l{l}_out"], atol=2e-2, rtol=1e-2)
    assert partial > 0  # the budget left pages out
    mn, mx = live_bounds()
    assert np.array_equal(mn, z["final_quest_min"]) and np.array_equal(mx, z["final_quest_max"])


def test_snapkv_eviction_matches_reference():
    """SnapKV (snapkv_enabled): query window, head scores, evicted sets (up to tied scores), front
    compaction, freed pages and their reuse by promotion, against the reference run on CPU."""
    from golden_cases import PipelineCase, snap_evicted_agree
    case = PipelineCase("snapkv_small")
    st = case.new_state()
    z = case.z
    scale = case.D ** -0.5
    n_ev = [0]

    def evict():
        e = n_ev[0]
        n_ev[0] += 1
        override, j = {}, 0
        for l in range(case.Ly):
            for h in range(case.Hk):
                glen = int(st.global_lengths[l, 0, h])
                if int(glen * case.snapkv[1]) == 0:
                    continue
                ref_sc = z[f"snap_e{e}_{j}_scores"]
                ref_ev = z[f"snap_e{e}_{j}_evict"]
                sc = st.snap_scores(l, 0, h, scale)
                np.testing.assert_allclose(sc, ref_sc, rtol=1e-5, atol=1e-8)
                mine = np.lexsort((np.arange(glen), sc.astype(np.float64)))[:len(ref_ev)]
                assert snap_evicted_agree(ref_sc, mine, ref_ev), (e, l, h)
                override[(l, 0, h)] = ref_ev
                j += 1
        st.snap_evict(scale, override=override)

    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        st.prefill_layer(l, k, v, case.ref_mask(l), pre_key=pk)
        st.snap_record(l, q)
        if l == case.Ly - 1 and st.snap_should_evict():
            evict()
    assert np.array_equal(st.block_table[:, 0], z["prefill_block_table"])
    assert np.array_equal(st.global_lengths[:, 0], z["prefill_global_lengths"])
    for s in range(case.n_decode):
        for l in range(case.Ly):
            q, k, v, pk = case.decode[s][l]
            if l == 0 and st.local_length == st.window:
                st.promote()
            cur = st.append_layer(l, k[:, :, 0], v[:, :, 0], case.ref_decode_mask(s, l)[:, :, 0])
            sl, bt = st.decode_tables(l, cur)
            kc, vc = st.paged_views()
            o = O.paged_decode(q.transpose(0, 2, 1, 3), kc, vc, sl, bt, scale)
            np.testing.assert_allclose(o[0, 0], z[f"d{s}_l{l}_out"], atol=2e-2, rtol=1e-2)
            st.snap_record(l, q)
            if l == case.Ly - 1 and st.snap_should_evict():
                evict()
        assert np.array_equal(st.block_table[:, 0], z[f"d{s}_block_table"]), s
        assert np.array_equal(st.global_lengths[:, 0], z[f"d{s}_global_lengths"]), s
        assert st.next_free_block == int(z[f"d{s}_next_free_block"]), s
        assert st.free == [int(x) for x in z[f"d{s}_free_ids"]], s
        assert st.evict_count == int(z[f"d{s}_evict_count"]), s
        dig = O.pool_digest(st.block_table, st.global_lengths, st.local_length,
                            O.bf16_bits(st.k), O.bf16_bits(st.v), st.page, st.window)
        assert np.array_equal(dig, z[f"d{s}_pool_sha"]), s
    assert n_ev[0] == int(z["snap_n_evictions"]) == 2


@pytest.mark.parametrize("name", ["a", "b"])
def test_gate_conv_path_matches_reference(name):
    """g_fast_path=False (the reference's default): the oracle's conv-path scores equal the reference's
    (rare 1-ulp accumulation-order differences allowed) and the masks at two thresholds, one below the
    clamp floor, are identical."""
    from gate_conv_util import conv_case
    p, ins, ref, _, eps, *_ = conv_case(name)
    s = O.gate_scores(p, **ins)
    mism = int((O.bf16_bits(s) != O.bf16_bits(ref)).sum())
    assert mism <= max(1, s.size // 2000), (mism, s.size)
    assert (ref >= O.bf16(np.float32(eps))).all()
    for thr in (0.5, 0.1):
        assert np.array_equal(O.admission_mask(s, thr), O.admission_mask(ref, thr))
