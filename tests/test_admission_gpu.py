"""GPU parity of the admission path against the reference's golden outputs.

* gate scores / admission masks (bit-exact masks)
* sparse indices (bit-exact, full arrays)
* prefill: page tables, global lengths, ring bits, allocator, pool bytes (bit-exact)
  and the sparse-prefill attention rows (2e-2 abs / 1e-2 rel)
* decode steps through the full patch: lazy promotion, ring append, deferred
  gating, per-step state (bit-exact) and decode outputs (2e-2 abs / 1e-2 rel)
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from golden_cases import O, PipelineCase, indices_case, load
from gpu_util import bits, to_bf16, to_np
from pipeline_util import bhld, make_config, make_layers

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2
PIPELINES = ["c1_prefill", "promote_small", "defer_small"]


@pytest.fixture(scope="module")
def wgkv():
    import wgkv as m
    return m


@pytest.fixture(scope="module", params=PIPELINES)
def case(request):
    return PipelineCase(request.param)


def test_gate_scores_bits(wgkv, case):
    layers = make_layers(wgkv, case)
    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        s = layers[l].g_predictors(bhld(pk), bhld(k), bhld(v))
        torch.cuda.synchronize()
        got = bits(s)
        ref = case.z[f"l{l}_scores"][None]
        mism = int((got != ref).sum())
        assert mism <= max(2, got.size // 2000), mism
        mask = torch.empty(s.shape, dtype=torch.uint8, device="cuda")
        layers[l].g_predictors.admit(bhld(pk), bhld(k), bhld(v), case.threshold, mask)
        assert np.array_equal(to_np(mask).astype(bool), case.ref_mask(l)), f"layer {l}"


def test_gate_rms_vs_oracle(wgkv):
    """RMS-normed pre_k + post_k inputs (the reference's default gate config)."""
    rng = np.random.default_rng(9)
    B, Hk, L, D, inner = 2, 4, 300, 128, 512
    pk, k = O.randn_bf16(rng, (B, Hk, L, D)), O.randn_bf16(rng, (B, Hk, L, D))
    gp = wgkv.GatingPredictor(D, Hk, ["pre_k", "post_k"], "gelu", inner / D, 1e-3, True, True).cuda().bfloat16()
    with torch.no_grad():
        gp.pre_key_norm.weight.copy_(to_bf16(O.bf16(1 + 0.1 * rng.standard_normal(D, dtype=np.float32))))
        gp.post_key_norm.weight.copy_(to_bf16(O.bf16(1 + 0.1 * rng.standard_normal(D, dtype=np.float32))))
    p = O.GateParams(w1=to_np(gp.conv1.weight).reshape(Hk, inner, 2 * D), b1=to_np(gp.conv1.bias).reshape(Hk, inner),
                     w2=to_np(gp.conv2.weight).reshape(Hk, inner), b2=to_np(gp.conv2.bias), inputs=("pre_k", "post_k"),
                     rms=True, norms={"pre_k": to_np(gp.pre_key_norm.weight), "post_k": to_np(gp.post_key_norm.weight)})
    ref = O.gate_scores(p, pre_key=pk, post_key=k)
    got = to_np(gp(to_bf16(pk), to_bf16(k), None))
    diff = np.abs(got - ref)
    # 1-ulp disagreements from accumulation order only
    assert (diff > 0).mean() < 0.01 and diff.max() <= 2 ** -7


def test_sparse_indices_exact(wgkv):
    z = load("sparse_indices")
    for i in range(int(z["n_cases"])):
        (B, Hk, L, W, gs), g, fast, ref = indices_case(z, i)
        gm = torch.from_numpy(g).cuda()
        got = wgkv.generate_sparse_indices(gm, W, B, Hk, L, gm.device, 64)
        torch.cuda.synchronize()
        for a, b, n in zip(got, fast, ("bc", "bo", "cc", "ci")):
            a = a.cpu().numpy()
            assert a.shape == b.shape and np.array_equal(a, b), (i, n)
        assert O.indices_equal(tuple(x.cpu().numpy() for x in got), ref)


def _prefill(wgkv, case, layers, pkv, use_ref_mask):
    outs = []
    for l in range(case.Ly):
        q, k, v, pk = case.prefill[l]
        a = layers[l]
        if use_ref_mask:
            gm = torch.from_numpy(case.ref_mask(l).astype(np.uint8)).cuda()
            o = wgkv.self_attn_forward_patch_inference(a, pkv, (1, case.L), bhld(q), bhld(pk), bhld(k), bhld(v), None,
                                                       g_mask=gm)
        else:
            o, _, _ = a.self_attn_forward_patch(a, 3, None, pkv, (1, case.L), bhld(q), bhld(pk), bhld(k), bhld(v))
        outs.append(o)
    torch.cuda.synchronize()
    wgkv.check_errors()
    return outs


def _digest(pkv, case, local_length):
    kb = bits(pkv.block_pool_k)
    vb = bits(pkv.block_pool_v)
    return O.pool_digest(pkv.block_table.cpu().numpy(), pkv.global_lengths.cpu().numpy(), local_length, kb, vb,
                         case.T, case.W)


@pytest.mark.parametrize("use_ref_mask", [True, False])
def test_prefill_state_and_rows(wgkv, case, use_ref_mask):
    layers = make_layers(wgkv, case)
    pkv = SimpleNamespace()
    outs = _prefill(wgkv, case, layers, pkv, use_ref_mask)
    z = case.z
    assert np.array_equal(pkv.block_table[:, 0].cpu().numpy(), z["prefill_block_table"])
    assert np.array_equal(pkv.global_lengths[:, 0].cpu().numpy(), z["prefill_global_lengths"])
    assert np.array_equal(pkv.local_is_global[:, 0].cpu().numpy().astype(bool), z["prefill_local_is_global"])
    assert int(pkv.next_free_block.item()) == int(z["prefill_next_free_block"])
    assert pkv.local_length == min(case.L, case.W) and pkv.local_ptr == 0
    assert np.array_equal(_digest(pkv, case, pkv.local_length), z["prefill_pool_sha"])
    for l in range(case.Ly):
        rows = to_np(outs[l])[0, case.L - case.rows_out:]
        np.testing.assert_allclose(rows, z[f"l{l}_attn_rows"], atol=ATOL, rtol=RTOL)


def test_decode_steps(wgkv, case):
    layers = make_layers(wgkv, case)
    pkv = SimpleNamespace()
    _prefill(wgkv, case, layers, pkv, use_ref_mask=False)
    z = case.z
    for s in range(case.n_decode):
        for l in range(case.Ly):
            q, k, v, pk = case.decode[s][l]
            a = layers[l]
            o, _, _ = a.self_attn_forward_patch(a, 3, None, pkv, (1, 1), bhld(q), bhld(pk), bhld(k), bhld(v))
            np.testing.assert_allclose(to_np(o)[0, 0], z[f"d{s}_l{l}_out"], atol=ATOL, rtol=RTOL)
        torch.cuda.synchronize()
        wgkv.check_errors()
        assert np.array_equal(pkv.block_table[:, 0].cpu().numpy(), z[f"d{s}_block_table"]), s
        assert np.array_equal(pkv.global_lengths[:, 0].cpu().numpy(), z[f"d{s}_global_lengths"]), s
        assert np.array_equal(pkv.local_is_global[:, 0].cpu().numpy().astype(bool), z[f"d{s}_local_is_global"]), s
        assert int(pkv.next_free_block.item()) == int(z[f"d{s}_next_free_block"]), s
        assert pkv.local_ptr == int(z[f"d{s}_local_ptr"]) and pkv.local_length == int(z[f"d{s}_local_length"])
        assert np.array_equal(_digest(pkv, case, pkv.local_length), z[f"d{s}_pool_sha"]), s


def _rand_mask(rng, B, Hk, L, gs):
    g = np.zeros((B, Hk, L), bool)
    for b in range(B):
        for h in range(Hk):
            g[b, h, rng.permutation(L)[:gs]] = True
    return g


@pytest.mark.parametrize("B,Hk,G", [(1, 8, 4), (2, 3, 2), (1, 1, 1), (2, 2, 3)])
@pytest.mark.parametrize("L", [2, 63, 64, 65, 129, 257, 1000])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("W", [64, 256])
def test_sparse_prefill_vs_oracle(wgkv, B, Hk, G, L, D, W):
    """Sweep in the spirit of utils/test_sparse_attn.py (global_size 0 / 123 / L/3)."""
    rng = np.random.default_rng(L * 7 + D + W + Hk)
    for gs in sorted({0, min(123, L), L // 3}):
        g = _rand_mask(rng, B, Hk, L, gs)
        q = O.randn_bf16(rng, (B, L, Hk * G, D))
        k = O.randn_bf16(rng, (B, L, Hk, D))
        v = O.randn_bf16(rng, (B, L, Hk, D))
        gm = torch.from_numpy(g).cuda()
        idx = wgkv.generate_sparse_indices(gm, W, B, Hk, L, gm.device)
        o = wgkv.sparse_attn_func(to_bf16(q), to_bf16(k), to_bf16(v), *idx, softmax_scale=D ** -0.5, causal=True)
        torch.cuda.synchronize()
        nidx = tuple(x.cpu().numpy() for x in idx)
        rows = np.arange(L) if L <= 300 else np.concatenate([np.arange(70), np.arange(L - 200, L)])
        mk = O.sparse_mask_from_indices(*nidx, L, G, rows=rows)
        assert np.array_equal(mk, O.ideal_mask(g, W, L, rows=rows))
        ref = O.masked_attention(q, k, v, mk, rows=rows)
        np.testing.assert_allclose(to_np(o)[:, rows], ref, atol=ATOL, rtol=RTOL)


def test_pool_exhaustion_reports_and_writes_nothing(wgkv):
    """Capacity violations set the device error word (AssertionError on check) and leave the tables alone."""
    case = PipelineCase("promote_small")
    cfg = make_config(case)
    cfg.max_total_tokens = case.Ly * case.Hk * case.W + 16  # ring pages + one global page
    layers = make_layers(wgkv, case)
    for a in layers:
        a.config = cfg
    pkv = SimpleNamespace()
    q, k, v, pk = case.prefill[0]
    gm = torch.from_numpy(case.ref_mask(0).astype(np.uint8)).cuda()
    wgkv.self_attn_forward_patch_inference(layers[0], pkv, (1, case.L), bhld(q), bhld(pk), bhld(k), bhld(v), None,
                                           g_mask=gm)
    torch.cuda.synchronize()
    with pytest.raises(AssertionError, match="pool exhausted"):
        wgkv.check_errors()
    assert int(pkv.global_lengths.sum().item()) == 0
    assert int(pkv.next_free_block.item()) == case.Ly * case.Hk * case.W // case.T
    wgkv.check_errors()  # the word was reset


def test_head_capacity_reports(wgkv):
    case = PipelineCase("promote_small")
    cfg = make_config(case)
    cfg.max_tokens_per_head = case.W + 16
    layers = make_layers(wgkv, case)
    for a in layers:
        a.config = cfg
    pkv = SimpleNamespace()
    q, k, v, pk = case.prefill[0]
    gm = torch.from_numpy(case.ref_mask(0).astype(np.uint8)).cuda()
    wgkv.self_attn_forward_patch_inference(layers[0], pkv, (1, case.L), bhld(q), bhld(pk), bhld(k), bhld(v), None,
                                           g_mask=gm)
    torch.cuda.synchronize()
    with pytest.raises(AssertionError, match="max_tokens_per_head"):
        wgkv.check_errors()


@pytest.mark.parametrize("B,Hk,G,D", [(2, 4, 4, 128), (1, 2, 2, 64), (2, 2, 3, 128)])
def test_pooled_prefill_matches_gather(wgkv, B, Hk, G, D):
    """Reading admitted columns from the compacted pool gives the gathered result (same bits)."""
    from types import SimpleNamespace
    rng = np.random.default_rng(B * 100 + Hk * 10 + G + D)
    L, W, T = 3000, 256, 16
    Hq = Hk * G
    q = O.randn_bf16(rng, (B, L, Hq, D))
    k = O.randn_bf16(rng, (B, L, Hk, D))
    v = O.randn_bf16(rng, (B, L, Hk, D))
    g = rng.random((B, Hk, L)) < 0.3
    cache = SimpleNamespace()
    a = SimpleNamespace(layer_idx=0, head_dim=D, scaling=D ** -0.5,
                        config=SimpleNamespace(num_hidden_layers=1, num_key_value_heads=Hk, local_window_size=W,
                                               block_size=T, max_total_tokens=B * Hk * (L + W) + 64 * T,
                                               max_tokens_per_head=L + W))
    wgkv.attach(a, a.config)
    tq, tk, tv = to_bf16(q), to_bf16(k), to_bf16(v)
    gm = torch.from_numpy(g.astype(np.uint8)).cuda()
    pooled = wgkv.prefill_wrapper(a, cache, tq.transpose(1, 2), None, tk.transpose(1, 2), tv.transpose(1, 2), B, L,
                                  tq.device, gm, W // T)
    idx = wgkv.generate_sparse_indices(gm, W, B, Hk, L, gm.device)
    gathered = wgkv.sparse_attn_func(tq, tk, tv, *idx, softmax_scale=D ** -0.5)
    torch.cuda.synchronize()
    wgkv.check_errors()
    assert torch.equal(pooled, gathered)


@pytest.mark.parametrize("fast", [True, False])
@pytest.mark.parametrize("inputs,rms,act,inner", [(["pre_k"], False, "gelu", 64), (["pre_k", "post_k"], True, "gelu", 512),
                                                   (["post_k", "v"], False, "silu", 192)])
def test_fused_decode_gate_matches_gate_kernel(wgkv, inputs, rms, act, inner, fast):
    """wgkv_decode_gate_append writes the same admission bits / ring rows as the gate kernel + append
    (both gate numerics: the einsum fast path and the conv path with its clamp floor)."""
    from types import SimpleNamespace
    B, Hk, D, W, T = 6, 4, 128, 64, 16
    torch.manual_seed(0)
    gp = wgkv.GatingPredictor(D, Hk, inputs, act, inner / D, 0.45, rms, fast).cuda().bfloat16()
    if rms:
        with torch.no_grad():
            gp.pre_key_norm.weight.add_(0.1 * torch.randn_like(gp.pre_key_norm.weight))
    cache = SimpleNamespace()
    wgkv.init_pool(cache, layers=2, batch=B, kv_heads=Hk, head_dim=D, window=W, page=T, max_total_tokens=8192,
                   max_tokens_per_head=1024, device="cuda")
    mism = 0
    for step in range(20):
        pk, k, v = (torch.randn(B, 1, Hk, D, device="cuda").bfloat16().transpose(1, 2) for _ in range(3))
        ref = torch.empty(B, Hk, 1, dtype=torch.uint8, device="cuda")
        gp.admit(pk, k, v, 0.5, ref)
        ins = step % W
        gp.decode_admit_append(cache, 1, ins, 7, pk, k, v, 0.5)
        torch.cuda.synchronize()
        mism += int((cache.local_is_global[1, :, :, ins] != ref[:, :, 0]).sum())
        rows = cache.block_pool_k[:2 * B * Hk * W].view(2, B, Hk, W, D)[1, :, :, ins]
        assert torch.equal(rows, k[:, :, 0])
        assert torch.equal(cache.cache_seqlens, torch.full((B, Hk), 7, dtype=torch.int32, device="cuda"))
    assert mism <= 1, mism  # accumulation order differs; a bit may flip only at an exact bf16 tie


@pytest.mark.parametrize("name", ["a", "b"])
def test_gate_conv_path_matches_reference(wgkv, name):
    """g_fast_path=False (the reference's default, src/configuration_llama.py:207): the CUDA gate
    reproduces the reference GatingPredictor's conv-path scores (:198-205, clamp floor included) and
    its masks bit-exactly, at a threshold above and one below the floor."""
    from gate_conv_util import conv_case
    p, ins, ref, (D, Hk, L, inner), eps, z, inputs, act, rms = conv_case(name)
    gp = wgkv.GatingPredictor(D, Hk, inputs, act, inner / D, eps, rms, False).cuda().bfloat16()
    with torch.no_grad():
        for k_, v_ in gp.state_dict().items():
            v_.copy_(torch.from_numpy(O.from_bf16_bits(z[f"{name}_{k_}"])).reshape(v_.shape))
    x = [bhld(ins[k]) for k in ("pre_key", "post_key", "value")]
    s = gp(*x)
    torch.cuda.synchronize()
    got = bits(s)
    assert int((got != O.bf16_bits(ref)).sum()) <= max(1, got.size // 2000)
    for thr in (0.5, 0.1):
        mask = torch.empty(s.shape, dtype=torch.uint8, device="cuda")
        gp.admit(*x, thr, mask)
        assert np.array_equal(to_np(mask).astype(bool), O.admission_mask(ref, thr)), thr
    # the fast-path numerics really differ here (the flag reaches the kernel)
    gp.g_fast_path = True
    assert (bits(gp(*x)) != got).sum() > got.size // 20

