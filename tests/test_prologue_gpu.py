"""Fused decode prologue (wgkv_decode_prologue) and the decoder plumbing kernels.

The prologue replaces, on a decode step, the patched layers' q/k norm + RoPE
(src/modeling_llama.py:265-271, src/modeling_qwen3.py:236-239) followed by the gate + ring append.
Its reference here is that unfused sequence: torch bf16 RoPE, then wgkv_decode_gate_append (itself
pinned to the oracle in test_admission_gpu.py).  Without q/k norm every rounding is the same, so
q, the ring rows, the admission bits and the lengths must be identical; with the Qwen3 norms the
mean-square reduction order differs from torch's, so values are compared within bf16 tolerance.
"""
from types import SimpleNamespace

import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup(B, Hk, G, D, W, defer, seed):
    import wgkv
    Ly = 2
    cache = SimpleNamespace()
    wgkv.init_pool(cache, layers=Ly, batch=B, kv_heads=Hk, head_dim=D, window=W, page=16,
                   max_total_tokens=Ly * B * Hk * (W + 64) + 64, max_tokens_per_head=W + 64, device="cuda",
                   defer=defer)
    cache.local_length = W // 2
    torch.manual_seed(seed)
    gp = wgkv.GatingPredictor(D, Hk, ["pre_k"], "gelu", 64 / D, 1e-3, False, True).cuda().bfloat16()
    return cache, gp


def _rope_tables(n, D):
    inv = 1.0 / (10000.0 ** (torch.arange(0, D, 2, dtype=torch.float32, device="cuda") / D))
    f = torch.outer(torch.arange(n, dtype=torch.float32, device="cuda"), inv)
    e = torch.cat((f, f), -1)
    return e.cos().to(torch.bfloat16), e.sin().to(torch.bfloat16)


def _rms(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def _torch_prologue(qkv, Hq, Hk, D, cos_row, sin_row, qn, kn, eps):
    B = qkv.shape[0]
    q = qkv[:, :Hq * D].view(B, Hq, D)
    k = qkv[:, Hq * D:(Hq + Hk) * D].view(B, Hk, D)
    v = qkv[:, (Hq + Hk) * D:].view(B, Hk, D)
    if qn is not None:
        q, k = _rms(q, qn, eps), _rms(k, kn, eps)

    def rot(x):
        h = D // 2
        return torch.cat((-x[..., h:], x[..., :h]), -1)
    qr = q * cos_row + rot(q) * sin_row
    kr = k * cos_row + rot(k) * sin_row
    return qr, k, kr, v


@pytest.mark.parametrize("qk_norm", [False, True])
@pytest.mark.parametrize("B,Hk,G,D", [(3, 8, 4, 128), (2, 4, 2, 64)])
def test_prologue_matches_unfused(qk_norm, B, Hk, G, D):
    import wgkv
    W, Hq, layer, eps = 64, Hk * G, 1, 1e-6
    ca, gp = _setup(B, Hk, G, D, W, False, 1)
    cb, _ = _setup(B, Hk, G, D, W, False, 1)
    cos, sin = _rope_tables(4096, D)
    pos = torch.tensor([1234], dtype=torch.int64, device="cuda")
    qkv = (torch.randn(B, (Hq + 2 * Hk) * D, device="cuda") * 2).to(torch.bfloat16)
    qn = (torch.rand(D, device="cuda") + 0.5).to(torch.bfloat16) if qk_norm else None
    kn = (torch.rand(D, device="cuda") + 0.5).to(torch.bfloat16) if qk_norm else None
    ins, cur = W // 2, W // 2 + 1
    q_out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    gp.decode_prologue(ca, layer, ins, cur, qkv, Hq, pos, cos, sin, q_out, 0.5, q_norm=qn, k_norm=kn, qk_eps=eps)
    qr, pk, kr, v = _torch_prologue(qkv, Hq, Hk, D, cos[1234], sin[1234], qn, kn, eps)
    gp.decode_admit_append(cb, layer, ins, cur, pk, kr, v, 0.5)
    torch.cuda.synchronize()
    wgkv.check_errors()
    ring = lambda c, t: t[:Ly_rows(c)].view(2, B, Hk, W, D)[layer, :, :, ins]  # noqa: E731
    if not qk_norm:
        assert torch.equal(q_out, qr)
        assert torch.equal(ring(ca, ca.block_pool_k), ring(cb, cb.block_pool_k))
        assert torch.equal(ring(ca, ca.block_pool_v), ring(cb, cb.block_pool_v))
        assert torch.equal(ca.local_is_global, cb.local_is_global)
    else:
        torch.testing.assert_close(q_out.float(), qr.float(), atol=2e-2, rtol=1e-2)
        torch.testing.assert_close(ring(ca, ca.block_pool_k).float(), ring(cb, cb.block_pool_k).float(), atol=2e-2,
                                   rtol=1e-2)
        assert torch.equal(ring(ca, ca.block_pool_v), ring(cb, cb.block_pool_v))
        # Admission bits may differ only where the normalised key's last-bit differences can move the
        # score across the threshold: the unfused score within one bf16 ulp at 0.5 (2^-8) of it.
        s_ref = gp(pk[:, :, None], kr[:, :, None], v[:, :, None])[:, :, 0].float()
        differ = (ca.local_is_global[layer, :, :, ins] != cb.local_is_global[layer, :, :, ins])
        near = (s_ref - 0.5).abs() <= 2.0 ** -8
        assert int((differ & ~near).sum()) == 0, (int(differ.sum()), int((differ & ~near).sum()))
        assert int(differ.sum()) <= max(1, differ.numel() // 8)
    assert torch.equal(ca.cache_seqlens, cb.cache_seqlens)


def Ly_rows(c):
    return c.local_is_global.numel()  # layers * B * Hk * W ring rows


def test_prologue_deferred_stores_pre_key():
    import wgkv
    B, Hk, G, D, W, layer = 2, 4, 4, 128, 64, 0
    Hq = Hk * G
    c, gp = _setup(B, Hk, G, D, W, True, 2)
    cos, sin = _rope_tables(256, D)
    pos = torch.tensor([17], dtype=torch.int64, device="cuda")
    qkv = torch.randn(B, (Hq + 2 * Hk) * D, device="cuda").to(torch.bfloat16)
    q_out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    before = c.local_is_global.clone()
    ins = W // 2
    gp.decode_prologue(c, layer, ins, ins + 1, qkv, Hq, pos, cos, sin, q_out, 0.5, gate=False)
    torch.cuda.synchronize()
    wgkv.check_errors()
    qr, pk, kr, v = _torch_prologue(qkv, Hq, Hk, D, cos[17], sin[17], None, None, 0)
    assert torch.equal(c.local_pre_key[layer, :, :, ins], pk)
    assert torch.equal(c.block_pool_k[:Ly_rows(c)].view(2, B, Hk, W, D)[layer, :, :, ins], kr)
    assert torch.equal(q_out, qr)
    assert torch.equal(c.local_is_global, before)  # no gate on a deferred step


def test_prologue_position_out_of_range_flags_error():
    import wgkv
    B, Hk, G, D, W = 1, 2, 2, 64, 64
    c, gp = _setup(B, Hk, G, D, W, False, 3)
    cos, sin = _rope_tables(32, D)
    pos = torch.tensor([32], dtype=torch.int64, device="cuda")  # one past the tables: clamped
    qkv = torch.randn(B, (Hk * G + 2 * Hk) * D, device="cuda").to(torch.bfloat16)
    q_out = torch.empty(B, Hk * G, D, dtype=torch.bfloat16, device="cuda")
    gp.decode_prologue(c, 0, 0, 1, qkv, Hk * G, pos, cos, sin, q_out, 0.5)
    torch.cuda.synchronize()
    with pytest.raises(AssertionError, match="RoPE position"):
        wgkv.check_errors()


@pytest.mark.parametrize("rows,cols", [(1, 2048), (37, 4096), (5, 2560), (3, 128)])
def test_rms_norm_matches_torch(rows, cols):
    from wgkv.model import rms_norm
    x = (torch.randn(rows, cols, device="cuda") * 3).to(torch.bfloat16)
    w = (torch.rand(cols, device="cuda") + 0.5).to(torch.bfloat16)
    got = rms_norm(x, w, 1e-5)
    ref = _rms(x, w, 1e-5)
    diff = (got.float() - ref.float()).abs()
    # equal up to the last bit of the mean-square (summation order)
    assert (diff <= ref.float().abs() * 2 ** -7 + 1e-6).all()
    assert (got == ref).float().mean().item() > 0.99


@pytest.mark.parametrize("rows,inter", [(1, 8192), (70000, 64), (9, 14336)])
def test_silu_mul_matches_torch(rows, inter):
    import torch.nn.functional as F
    from wgkv.model import silu_mul
    gu = (torch.randn(rows, 2 * inter, device="cuda") * 3).to(torch.bfloat16)
    got = silu_mul(gu)
    ref = F.silu(gu[:, :inter]) * gu[:, inter:]
    torch.testing.assert_close(got.float(), ref.float(), atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize("m,n,k", [(1, 2048, 8192), (1, 3072, 2048), (2, 16384, 2048), (3, 1000, 72), (8, 517, 4096),
                                   (5, 128256, 256), (7, 9, 8)])
def test_skinny_gemm_matches_fp32(m, n, k):
    from wgkv.model import skinny_linear
    x = torch.randn(m, k, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda") * 0.05).to(torch.bfloat16)
    ref = x.float() @ w.float().t()
    tol = dict(atol=1e-2 * (k / 64) ** 0.5 * 0.05 + 1e-3, rtol=1e-2)
    got32 = skinny_linear(x, w, out_f32=True)
    torch.testing.assert_close(got32, ref, atol=1e-3 * (k ** 0.5) * 0.05 + 1e-4, rtol=1e-4)
    got = skinny_linear(x, w)
    torch.testing.assert_close(got.float(), ref, **tol)
    r = torch.randn(m, n, device="cuda").to(torch.bfloat16)
    r0 = r.float().clone()
    skinny_linear(x, w, residual=r)  # in place
    torch.testing.assert_close(r.float(), r0 + ref, **tol)


@pytest.mark.parametrize("rows,n", [(1, 128256), (3, 151936), (8, 100), (2, 4096)])
def test_argmax_matches_torch(rows, n):
    from wgkv.model import argmax_into
    x = torch.randn(rows, n, device="cuda")
    x[0, n // 3] = 50.0
    x[0, n // 2] = 50.0  # a tie: the first index wins, as torch.argmax
    out = torch.empty(rows, 1, dtype=torch.int64, device="cuda")
    for _ in range(3):  # the ticket counters reset themselves between calls
        argmax_into(x, out)
        assert torch.equal(out, x.argmax(-1, keepdim=True))



@pytest.mark.parametrize("m,n,k", [(1, 2048, 2048), (2, 16384, 2048), (3, 3072, 4096)])
def test_skinny_gemm_fused_norm_and_activation(m, n, k):
    """rms_weight / paired reproduce rms_norm -> GEMM and GEMM -> silu_mul (same roundings)."""
    from wgkv.model import rms_norm, silu_mul, skinny_linear
    x = (torch.randn(m, k, device="cuda") * 2).to(torch.bfloat16)
    nw = (torch.rand(k, device="cuda") + 0.5).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda") * 0.05).to(torch.bfloat16)
    ref = skinny_linear(rms_norm(x, nw, 1e-5), w)
    got = skinny_linear(x, w, rms_weight=nw, rms_eps=1e-5)
    # the mean square may differ in its last bit (summation order): compare within bf16 rounding
    torch.testing.assert_close(got.float(), ref.float(), atol=1e-2, rtol=1e-2)
    assert (got == ref).float().mean().item() > 0.95
    ref2 = silu_mul(skinny_linear(x, w))
    got2 = skinny_linear(x, w, paired=True)
    # same roundings; the projection's fp32 sum may take another order (K split across warps)
    torch.testing.assert_close(got2.float(), ref2.float(), atol=1e-2, rtol=1e-2)
    assert (got2 == ref2).float().mean().item() > 0.95
    got3 = skinny_linear(x, w, paired=True, rms_weight=nw, rms_eps=1e-5)
    torch.testing.assert_close(got3.float(), silu_mul(ref).float(), atol=2e-2, rtol=2e-2)
