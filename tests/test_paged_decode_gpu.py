"""GPU parity of the ragged paged decode kernel against the CPU oracle.

Tolerance: 2e-2 absolute / 1e-2 relative on bf16 outputs (fp32 accumulate),
the bound stated for attention outputs of this path."""
import numpy as np
import pytest
import torch

from golden_cases import O, load, regen_decode_inputs
from gpu_util import to_bf16, to_np

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def wgkv():
    import wgkv as m
    return m


def run(wgkv, q, kc, vc, sl, tbl, scale):
    out = wgkv.paged_decode(to_bf16(q), to_bf16(kc), to_bf16(vc), torch.from_numpy(sl).cuda(),
                            torch.from_numpy(tbl).cuda(), scale)
    torch.cuda.synchronize()
    wgkv.check_errors()
    return to_np(out)


def test_golden_cases(wgkv):
    z = load("paged_decode")
    for i in range(int(z["n_cases"])):
        p = z[f"c{i}_params"]
        q, kc, vc, sl, tbl = regen_decode_inputs(p)
        scale = int(p[2]) ** -0.5
        o = run(wgkv, q, kc, vc, sl, tbl, scale)
        np.testing.assert_allclose(o, O.paged_decode(q, kc, vc, sl, tbl, scale), atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(o, z[f"c{i}_out"], atol=ATOL, rtol=RTOL)


def make_case(seed, B, Hq, Hk, D, T, maxs, zero_heads=False, garbage=True):
    rng = np.random.default_rng(seed)
    sl = rng.integers(1, maxs + 1, (B, Hk)).astype(np.int32)
    if zero_heads:
        sl[rng.random((B, Hk)) < 0.3] = 0
    maxb = (maxs + T - 1) // T
    need = int(sum((s + T - 1) // T for s in sl.ravel()))
    nb = max(need + 3, 8)
    perm = rng.permutation(nb).astype(np.int32)
    tbl = np.full((B, Hk, maxb), -1, np.int32)
    off = 0
    for b in range(B):
        for h in range(Hk):
            n = (int(sl[b, h]) + T - 1) // T
            tbl[b, h, :n] = perm[off:off + n]
            off += n
    q = O.randn_bf16(rng, (B, 1, Hq, D))
    kc = O.randn_bf16(rng, (nb, T, D))
    vc = O.randn_bf16(rng, (nb, T, D))
    if garbage:
        # rows past each head's length: NaN / huge values must not leak into the output
        for b in range(B):
            for h in range(Hk):
                n = int(sl[b, h])
                if n % T:
                    pg = tbl[b, h, n // T]
                    kc[pg, n % T:] = np.nan
                    vc[pg, n % T:] = np.nan
    return q, kc, vc, sl, tbl


@pytest.mark.parametrize("heads", [(4, 4), (8, 2), (8, 4), (32, 8), (16, 1), (12, 4)])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("T", [16, 32, 64])
@pytest.mark.parametrize("B,maxs", [(1, 123), (3, 789), (2, 4000)])
def test_sweep(wgkv, heads, D, T, B, maxs):
    Hq, Hk = heads
    q, kc, vc, sl, tbl = make_case(hash((Hq, Hk, D, T, B, maxs)) % 2**31, B, Hq, Hk, D, T, maxs)
    o = run(wgkv, q, kc, vc, sl, tbl, D ** -0.5)
    np.testing.assert_allclose(o, O.paged_decode(q, kc, vc, sl, tbl, D ** -0.5), atol=ATOL, rtol=RTOL)


def test_zero_length_heads(wgkv):
    q, kc, vc, sl, tbl = make_case(7, 3, 16, 4, 128, 16, 300, zero_heads=True)
    o = run(wgkv, q, kc, vc, sl, tbl, 128 ** -0.5)
    np.testing.assert_allclose(o, O.paged_decode(q, kc, vc, sl, tbl, 128 ** -0.5), atol=ATOL, rtol=RTOL)
    assert np.all(o[sl.repeat(4, axis=1)[:, None, :] == 0] == 0)


def test_large_ragged(wgkv):
    """Llama-8B-shaped heads (G=4, D=128, T=16), ragged lengths up to 40K."""
    q, kc, vc, sl, tbl = make_case(11, 4, 32, 8, 128, 16, 40000, garbage=False)
    o = run(wgkv, q, kc, vc, sl, tbl, 128 ** -0.5)
    np.testing.assert_allclose(o, O.paged_decode(q, kc, vc, sl, tbl, 128 ** -0.5), atol=ATOL, rtol=RTOL)


def test_repeat_calls_stable(wgkv):
    """The per-head counters reset themselves: repeated calls give identical bits."""
    q, kc, vc, sl, tbl = make_case(5, 2, 32, 8, 128, 16, 20000, garbage=False)
    args = (to_bf16(q), to_bf16(kc), to_bf16(vc), torch.from_numpy(sl).cuda(), torch.from_numpy(tbl).cuda(), 128 ** -0.5)
    a = wgkv.paged_decode(*args).clone()
    for _ in range(5):
        b = wgkv.paged_decode(*args)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_triton_handle_signature(wgkv):
    q, kc, vc, sl, tbl = make_case(3, 1, 32, 8, 128, 16, 3000, garbage=False)
    h = wgkv.flash_attn_with_kvcache_wrapper_triton_handle(to_bf16(q), to_bf16(kc), to_bf16(vc),
                                                           torch.from_numpy(sl).cuda(), torch.from_numpy(tbl).cuda(),
                                                           128 ** -0.5)
    o = to_np(h())
    np.testing.assert_allclose(o, O.paged_decode(q, kc, vc, sl, tbl, 128 ** -0.5), atol=ATOL, rtol=RTOL)
    with pytest.raises(TypeError):
        wgkv.flash_attn_with_kvcache_wrapper_triton_handle(to_bf16(q).half(), to_bf16(kc), to_bf16(vc),
                                                           torch.from_numpy(sl).cuda(), torch.from_numpy(tbl).cuda(), 1.0)


def test_workspace_counter_prefix_grows(wgkv):
    """A second call with more (batch, kv-head) counters than the first reuses the cached workspace:
    the counter bytes it adds held the first call's partial results and must be cleared."""
    small = make_case(31, 1, 32, 2, 128, 16, 30000, garbage=False)   # few counters, large partials
    large = make_case(32, 20, 8, 8, 64, 16, 700, garbage=False)      # 160 counters, small partials
    for q, kc, vc, sl, tbl in (small, large, small, large):
        D = q.shape[-1]
        o = run(wgkv, q, kc, vc, sl, tbl, D ** -0.5)
        np.testing.assert_allclose(o, O.paged_decode(q, kc, vc, sl, tbl, D ** -0.5), atol=ATOL, rtol=RTOL)


def test_argmax_ticket_prefix_grows():
    """Same rule for the argmax tickets: one long row, then many short rows, on one stream."""
    from wgkv.model import argmax_into
    g = torch.Generator(device="cuda").manual_seed(3)
    for rows, n in ((1, 128256), (100, 1000), (1, 128256), (100, 1000)):
        x = torch.randn(rows, n, device="cuda", generator=g)
        out = torch.empty(rows, 1, dtype=torch.int64, device="cuda")
        argmax_into(x, out)
        assert torch.equal(out, x.argmax(-1, keepdim=True))
