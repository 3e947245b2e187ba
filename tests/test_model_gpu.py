"""End-to-end decoder driver (wgkv.model) on the WG-KV path.

* With every token admitted, WG-KV attention is dense causal attention, so the driver's prefill
  and decode logits must match a dense torch SDPA forward of the same weights (the integration of
  RoPE, pre-RoPE gate keys and layouts, src/modeling_llama.py:265-287).
* Graph-replayed decode steps (device token, position and ring state) equal eager steps exactly,
  with and without deferred gating.
"""
from types import SimpleNamespace

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _tiny(qk_norm=False, D=64):
    from wgkv.model import DecoderShape
    return DecoderShape("tiny", 256, 2, 4, 2, D, 512, 1000, 10000.0, qk_norm, 1e-5)


def _dense_logits(m, ids):
    """Dense causal forward of the same weights (no WG-KV); logits of every position."""
    B, T = ids.shape
    cos, sin = m._rope_table(T)
    h = F.embedding(ids, m.embed)
    for L in m.layers:
        q, k, v = m._qkv(L, h)
        q, k = m._apply_rope(q, k, cos[:T], sin[:T])
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                           enable_gqa=True)
        h = m._after_attn(L, h, o.transpose(1, 2).reshape(B, T, -1))
    from wgkv.model import _rms
    return (_rms(h, m.final_norm, m.s.rms_eps) @ m.lm_head.t()).float()


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("qk_norm,D", [(False, 64), (True, 128)])
def test_all_admitted_matches_dense(qk_norm, D, fused):
    from wgkv.model import WgkvDecoder
    torch.manual_seed(0)
    B, P, n = 2, 200, 20
    m = WgkvDecoder(_tiny(qk_norm, D), batch=B, window=64, max_tokens_per_head=P + n + 64, g_defer=False,
                    max_positions=P + n + 1, device="cuda", seed=3, fused=fused)
    for L in m.layers:
        with torch.no_grad():
            L.attn.g_predictors.conv2.bias.fill_(30.0)  # admit everything
    ids = torch.randint(0, 1000, (B, P + n), device="cuda")
    ref = _dense_logits(m, ids)
    cache = SimpleNamespace()
    lg = m.prefill(ids[:, :P], cache)

    def close(a, b):
        cos = F.cosine_similarity(a.flatten(1), b.flatten(1), dim=1)
        return bool((cos > 0.999).all()), cos.min().item()

    ok, c = close(lg, ref[:, P - 1])
    assert ok, c
    for s in range(n):
        m.token.copy_(ids[:, P + s:P + s + 1])  # teacher forcing
        lg = m.decode_step(cache)
        ok, c = close(lg, ref[:, P + s])
        assert ok, (s, c)
    import wgkv
    torch.cuda.synchronize()
    wgkv.check_errors()


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("defer", [False, True])
def test_graph_steps_equal_eager(defer, fused):
    import wgkv
    from wgkv.model import WgkvDecoder
    B, P, n = 2, 150, 90
    m = WgkvDecoder(_tiny(), batch=B, window=64, max_tokens_per_head=P + n + 128, g_defer=defer,
                    max_positions=P + n + 8, device="cuda", seed=5, fused=fused)
    m.calibrate_gates(n_tokens=256)
    ids = torch.randint(0, 1000, (B, P), device="cuda", generator=torch.Generator(device="cuda").manual_seed(2))
    ca = SimpleNamespace()
    m.prefill(ids, ca)
    eager = []
    for _ in range(n):
        eager.append((m.decode_step(ca).clone(), m.token.clone()))
    cb = SimpleNamespace()
    m.prefill(ids, cb)
    dg = m.decode_graph(cb)  # step 0, eager
    got = [(dg.first.clone(), m.token.clone())]
    for _ in range(n - 1):
        lg = dg.replay()
        got.append((lg.clone(), m.token.clone()))
    torch.cuda.synchronize()
    wgkv.check_errors()
    for s, ((le, te), (lg, tg)) in enumerate(zip(eager, got)):
        assert torch.equal(te, tg), s
        assert torch.equal(le, lg), s
    for name in ("block_table", "global_lengths", "local_is_global", "next_free_block"):
        assert torch.equal(getattr(ca, name), getattr(cb, name)), name
    assert (ca.local_length, ca.local_ptr) == (cb.local_length, cb.local_ptr)


def test_position_bound_is_checked_on_the_host():
    from wgkv.model import WgkvDecoder
    B, P = 1, 70
    m = WgkvDecoder(_tiny(), batch=B, window=64, max_tokens_per_head=P + 64, g_defer=False, max_positions=P + 2,
                    device="cuda", seed=1)
    ids = torch.randint(0, 1000, (B, P), device="cuda")
    cache = SimpleNamespace()
    m.prefill(ids, cache)
    m.decode_step(cache)  # position P
    dg = m.decode_graph(cache)  # position P + 1, eager, then captured
    with pytest.raises(ValueError):
        dg.replay()  # position P + 2 is past the table
    torch.cuda.synchronize()
