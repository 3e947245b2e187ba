"""End-to-end decoder driver (wgkv.model) on the WG-KV path.

* With every token admitted, WG-KV attention is dense causal attention, so every layer's attention
  output must match fp32 dense attention computed with plain torch from the same layer input, and
  the projections / MLP / logits fp32 matmuls of the same weights (the integration of RoPE, pre-RoPE
  gate keys and layouts, src/modeling_llama.py:265-287), at 2e-2 abs / 1e-2 rel.
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


ATOL, RTOL = 2e-2, 1e-2


def _f32_rms(x, w, eps):
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def _f32_attention(m, L, h_in):
    """fp32 dense causal attention of one layer from its bf16 input residual stream h_in (B, T, Hd):
    plain torch matmuls on the layer's weights, fp32 RoPE tables, fp32 SDPA."""
    s = m.s
    B, T, _ = h_in.shape
    D, Hq, Hk = s.head_dim, s.q_heads, s.kv_heads
    qkv = _f32_rms(h_in, L.in_norm, s.rms_eps) @ L.qkv.float().t()
    q = qkv[..., :Hq * D].view(B, T, Hq, D)
    k = qkv[..., Hq * D:(Hq + Hk) * D].view(B, T, Hk, D)
    v = qkv[..., (Hq + Hk) * D:].view(B, T, Hk, D)
    if s.qk_norm:
        q, k = _f32_rms(q, L.q_norm, s.rms_eps), _f32_rms(k, L.k_norm, s.rms_eps)
    inv = 1.0 / (s.rope_theta ** (torch.arange(0, D, 2, dtype=torch.float64, device=h_in.device) / D))
    f = torch.outer(torch.arange(T, dtype=torch.float64, device=h_in.device), inv)
    e = torch.cat((f, f), -1)
    c, n = e.cos().float()[None, :, None], e.sin().float()[None, :, None]
    rot = lambda x: torch.cat((-x[..., D // 2:], x[..., :D // 2]), -1)  # noqa: E731
    q, k = q * c + rot(q) * n, k * c + rot(k) * n
    o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), is_causal=True,
                                       enable_gqa=True)
    return o.transpose(1, 2).reshape(B, T, Hq * D)


def _f32_after_attn(m, L, h_in, a):
    """fp32 o_proj + residual + post-norm + SiLU MLP + residual from the bf16 inputs."""
    s = m.s
    h = h_in.float() + a.float() @ L.o.float().t()
    gu = _f32_rms(h, L.post_norm, s.rms_eps) @ L.gate_up.float().t()
    I = s.intermediate
    return h + (F.silu(gu[..., :I]) * gu[..., I:]) @ L.down.float().t()


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("qk_norm,D", [(False, 64), (True, 128)])
def test_all_admitted_matches_dense(qk_norm, D, fused):
    """Every token admitted: WG-KV attention is dense causal attention.  Each layer's attention output
    (prefill positions and every decode step) is compared with fp32 attention computed by plain torch
    from the same layer input, and each layer's projections + MLP and the final logits with fp32
    matmuls from their recorded bf16 inputs, all within 2e-2 abs / 1e-2 rel."""
    from wgkv.model import WgkvDecoder
    torch.manual_seed(0)
    B, P, n = 2, 200, 20
    m = WgkvDecoder(_tiny(qk_norm, D), batch=B, window=64, max_tokens_per_head=P + n + 64, g_defer=False,
                    max_positions=P + n + 1, device="cuda", seed=3, fused=fused)
    for L in m.layers:
        with torch.no_grad():
            L.attn.g_predictors.conv2.bias.fill_(30.0)  # admit everything
    rec = {id(L): [] for L in m.layers}
    inner = m._after_attn

    def recording(L, h, a):
        h_in, a_in = h.clone(), a.clone()
        out = inner(L, h, a)
        rec[id(L)].append((h_in, a_in, out.clone()))
        return out
    m._after_attn = recording
    ids = torch.randint(0, 1000, (B, P + n), device="cuda")
    cache = SimpleNamespace()
    logits = [m.prefill(ids[:, :P], cache)]
    for s in range(n):
        m.token.copy_(ids[:, P + s:P + s + 1])  # teacher forcing
        logits.append(m.decode_step(cache).clone())
    import wgkv
    torch.cuda.synchronize()
    wgkv.check_errors()
    for l, L in enumerate(m.layers):
        h_in = torch.cat([r[0] for r in rec[id(L)]], 1)  # (B, P + n, Hd) layer input, every position
        a = torch.cat([r[1] for r in rec[id(L)]], 1)
        h_out = torch.cat([r[2] for r in rec[id(L)]], 1)
        assert h_in.shape[1] == P + n
        torch.testing.assert_close(a.float(), _f32_attention(m, L, h_in), atol=ATOL, rtol=RTOL)
        torch.testing.assert_close(h_out.float(), _f32_after_attn(m, L, h_in, a), atol=ATOL, rtol=RTOL)
    last = torch.cat([r[2] for r in rec[id(m.layers[-1])]], 1)
    ref_logits = _f32_rms(last, m.final_norm, m.s.rms_eps) @ m.lm_head.float().t()
    got = torch.stack([lg.float() for lg in logits], 1)  # (B, 1 + n, vocab): positions P-1 .. P+n-1
    torch.testing.assert_close(got, ref_logits[:, P - 1:], atol=ATOL, rtol=RTOL)


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
