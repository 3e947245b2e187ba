"""Parity at the sizes the benchmark times (BASELINE configurations 3 and 2), against the oracle.

* C3: one Llama-3.1-8B-shaped prefill layer of 400,000 tokens (32 query / 8 KV heads, d=128, window
  4096, page 16, ~30 % admitted) through ``self_attn_forward_patch``: admission bits on sampled tokens,
  the four sparse-index tensors (full arrays, bit-exact), the page tables, global lengths, ring bits,
  allocator and pool rows (bit-exact), and sampled attention rows -- the first band rows, a middle
  row block and the last 64 rows, two query heads of different KV heads -- within 2e-2 abs / 1e-2 rel
  (the checks of utils/test_sparse_indices.py and utils/test_sparse_attn.py:34-93 at full size).
* C2: one decode layer of the 128K workload (batch 16, 8 KV heads, ring 4096 + Beta(2,8) global
  lengths, pages randomly permuted over a ~2 GB pool as utils/benchmark_decode.py:72-77 lays them
  out): ``paged_decode`` for the longest, the shortest and random (b, h) against the oracle
  (utils/test_flash_attn_with_kvcache.py:116-146 semantics), within 2e-2 abs / 1e-2 rel.

Inputs are generated on the GPU from seeds; the oracle sees host copies of exactly what the
kernels read.  Both cases fit in ~12 GB of device memory and run in seconds.
"""
from types import SimpleNamespace

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from golden_cases import O

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _host(t):
    return t.float().cpu().numpy()


def _calibrated_gate(wgkv, D, Hk, rates, dev):
    """pre_k -> 64 -> 1 GELU gate whose per-head output bias admits ~rates[h] of N(0,1) keys."""
    gp = wgkv.GatingPredictor(D, Hk, ["pre_k"], "gelu", 0.5, 1e-3, False, True).to(dev, torch.bfloat16)
    x = torch.randn(8192, D, device=dev, generator=torch.Generator(device=dev).manual_seed(1)).bfloat16().float()
    with torch.no_grad():
        w1 = gp.conv1.weight.float().view(Hk, -1, D)
        b1 = gp.conv1.bias.float().view(Hk, -1)
        w2 = gp.conv2.weight.float().view(Hk, -1)
        logit = torch.einsum("htj,hj->ht", F.gelu(torch.einsum("td,hjd->htj", x, w1) + b1[:, None, :]), w2)
        b2 = -torch.stack([torch.quantile(logit[h], 1 - float(rates[h])) for h in range(Hk)])
        gp.conv2.bias.copy_(b2.to(torch.bfloat16))
    return gp


def _gate_params(gp):
    Hk, inner, I = gp.num_kv_heads, gp.inner_dim, gp.input_dim
    f = lambda t: t.detach().float().cpu().numpy()  # noqa: E731
    return O.GateParams(w1=f(gp.conv1.weight).reshape(Hk, inner, I), b1=f(gp.conv1.bias).reshape(Hk, inner),
                        w2=f(gp.conv2.weight).reshape(Hk, inner), b2=f(gp.conv2.bias))


def test_c3_prefill_layer_400k():
    import wgkv
    dev = torch.device("cuda")
    L, Hq, Hk, D, W, T, thr = 400_000, 32, 8, 128, 4096, 16, 0.5
    G = Hq // Hk
    torch.manual_seed(3)
    rates = np.clip(np.random.default_rng(3).beta(3, 7, Hk), 0.05, 0.9)  # mean ~0.3
    gp = _calibrated_gate(wgkv, D, Hk, rates, dev)
    g = torch.Generator(device=dev).manual_seed(11)
    q = torch.randn(1, L, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    kvp = torch.randn(1, L, 3 * Hk, D, generator=g, device=dev).to(torch.bfloat16)
    k, v, pk = (kvp[:, :, i * Hk:(i + 1) * Hk].transpose(1, 2) for i in range(3))  # (1, Hk, L, D) views
    max_head = L + 64
    total = int(Hk * (W + 1.1 * rates.max() * L)) + Hk * 64
    cfg = SimpleNamespace(num_hidden_layers=1, num_key_value_heads=Hk, num_attention_heads=Hq, head_dim=D,
                          block_size=T, max_total_tokens=total, max_tokens_per_head=max_head, local_window_size=W,
                          g_defer=False, g_threshold=thr)
    attn = wgkv.attach(SimpleNamespace(layer_idx=0, head_dim=D, scaling=D ** -0.5, g_predictors=gp), cfg)
    cache = SimpleNamespace()
    o, _, _ = attn.self_attn_forward_patch(attn, 3, None, cache, (1, L), q.transpose(1, 2), pk, k, v)
    gm = torch.empty(1, Hk, L, dtype=torch.uint8, device=dev)
    gp.admit(pk, k, v, thr, gm)
    idx = wgkv.generate_sparse_indices(gm, W, 1, Hk, L, dev)
    torch.cuda.synchronize()
    wgkv.check_errors()
    gm_np = gm.cpu().numpy().astype(bool)
    frac = gm_np[:, :, :L - W].mean()
    assert 0.15 < frac < 0.5, frac

    # admission bits on 4096 sampled tokens per head against the oracle gate
    rng = np.random.default_rng(0)
    pos = np.sort(rng.choice(L, 4096, replace=False))
    pk_s = _host(pk[:, :, torch.from_numpy(pos).to(dev)])
    s_ref = O.gate_scores(_gate_params(gp), pre_key=pk_s)
    differ = O.admission_mask(s_ref, thr) != gm_np[:, :, pos]
    near = np.abs(s_ref - thr) <= 2.0 ** -8  # a last-bit score difference can only flip these
    assert not (differ & ~near).any(), int(differ.sum())

    # sparse indices: full arrays, bit-exact
    ref_idx = O.generate_sparse_indices(gm_np, W, L)
    for got, want in zip(idx, ref_idx):
        got = got.cpu().numpy()
        assert got.shape == want.shape and np.array_equal(got, want)

    # pool state: tables, lengths, ring bits, allocator bit-exact; pool rows through their first 8 columns
    # against the oracle pool (its layout does not depend on the head width), and whole rows on the device
    st = O.PoolState(layers=1, batch=1, kv_heads=Hk, head_dim=8, window=W, page=T, max_total_tokens=total,
                     max_tokens_per_head=max_head)
    st.prefill_layer(0, _host(k[..., :8]), _host(v[..., :8]), gm_np)
    assert np.array_equal(cache.block_table.cpu().numpy(), st.block_table)
    assert np.array_equal(cache.global_lengths.cpu().numpy(), st.global_lengths)
    assert np.array_equal(cache.local_is_global.cpu().numpy().astype(bool), st.local_is_global)
    assert int(cache.next_free_block.item()) == st.next_free_block
    # rows the prefill writes: every ring row, and each head's admitted rows (a head's last page is
    # written only up to its length; the rest of that page is unwritten in both)
    lp = W // T
    written = np.zeros(st.next_free_block * T, bool)
    written[:Hk * W] = True
    for h in range(Hk):
        first = int(st.block_table[0, 0, h, lp]) if st.global_lengths[0, 0, h] else 0
        written[first * T:first * T + int(st.global_lengths[0, 0, h])] = True
    rows_w = torch.from_numpy(np.flatnonzero(written)).to(dev)
    nw = written.size
    assert np.array_equal(_host(cache.block_pool_k[rows_w, :8]), st.k[:nw][written])
    assert np.array_equal(_host(cache.block_pool_v[rows_w, :8]), st.v[:nw][written])
    for h in range(Hk):
        n = int(st.global_lengths[0, 0, h])
        pages = cache.block_table[0, 0, h, lp:lp + (n + T - 1) // T].long()
        rows = (pages[:, None] * T + torch.arange(T, device=dev)[None]).reshape(-1)[:n]
        adm = torch.from_numpy(np.flatnonzero(gm_np[0, h, :L - W])).to(dev)
        assert torch.equal(cache.block_pool_k[rows], k[0, h, adm]) and torch.equal(cache.block_pool_v[rows], v[0, h, adm])

    # attention rows: first band rows, a middle row block, the last 64 rows; query heads 0 and 29
    rows = np.concatenate([np.arange(64), np.arange(200_000, 200_064), np.arange(L - 64, L)])
    o = o.view(1, L, Hq, D)
    for hq in (0, 29):
        h = hq // G
        sl = slice(h, h + 1)
        mask = O.sparse_mask_from_indices(ref_idx[0], ref_idx[1], ref_idx[2][:, sl], ref_idx[3][:, sl], L, G,
                                          rows=rows)
        # one query head against its KV head's mask: a group of one
        q_1 = _host(q[:, torch.from_numpy(rows).to(dev), hq:hq + 1])
        ref = O.masked_attention(q_1, _host(k[:, h:h + 1].transpose(1, 2)), _host(v[:, h:h + 1].transpose(1, 2)),
                                 mask, rows=np.arange(rows.size))
        got = _host(o[0, torch.from_numpy(rows).to(dev), hq])
        np.testing.assert_allclose(got, ref[0, :, 0], atol=ATOL, rtol=RTOL, err_msg=f"query head {hq}")


def test_c2_decode_layer_128k():
    import wgkv
    dev = torch.device("cuda")
    B, Hq, Hk, D, W, T, ctx = 16, 32, 8, 128, 4096, 16, 131072
    G = Hq // Hk
    rng = np.random.default_rng(2)
    rate = rng.beta(2, 8, (B, Hk))
    seqlens = (W + np.round(rate * (ctx - W))).astype(np.int32)
    pages = (seqlens + T - 1) // T
    maxb = int(pages.max())
    n_pages = int(pages.sum()) + 7
    perm = rng.permutation(n_pages).astype(np.int32)
    table = np.full((B, Hk, maxb), n_pages - 1, np.int32)
    off = 0
    for b in range(B):
        for h in range(Hk):
            table[b, h, :pages[b, h]] = perm[off:off + pages[b, h]]
            off += pages[b, h]
    g = torch.Generator(device=dev).manual_seed(5)
    kc = torch.randn(n_pages, T, D, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(n_pages, T, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(B, 1, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    tt, sl = torch.from_numpy(table).to(dev), torch.from_numpy(seqlens).to(dev)
    out = wgkv.paged_decode(q, kc, vc, sl, tt, D ** -0.5)
    torch.cuda.synchronize()
    wgkv.check_errors()
    flat = seqlens.reshape(-1)
    picks = {int(flat.argmax()), int(flat.argmin())} | set(int(i) for i in rng.choice(B * Hk, 6, replace=False))
    for i in sorted(picks):
        b, h = divmod(i, Hk)
        pg = torch.from_numpy(table[b, h, :pages[b, h]].astype(np.int64)).to(dev)
        kk, vv = _host(kc[pg]), _host(vc[pg])
        ref = O.paged_decode(_host(q[b:b + 1, :, h * G:(h + 1) * G]), kk, vv, seqlens[b:b + 1, h:h + 1],
                             np.arange(pages[b, h], dtype=np.int32)[None, None], D ** -0.5)
        np.testing.assert_allclose(_host(out[b, 0, h * G:(h + 1) * G]), ref[0, 0], atol=ATOL, rtol=RTOL,
                                   err_msg=f"(b, h) = ({b}, {h}), length {seqlens[b, h]}")
