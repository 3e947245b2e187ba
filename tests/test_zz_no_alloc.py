"""The allocation-free decode entry point, called through the C ABI.

``wgkv_paged_decode_noalloc`` serves callers that cannot allocate device
memory while they decode (an engine that owns the whole memory budget, or a
plugin running while its framework captures a stream): its split-K scratch is
a static device array inside libwgkv.so.  These checks compare it with the
workspace-taking ``wgkv_paged_decode`` on the same inputs, for two calls in a
row (the array keeps the previous call's contents, so the second call checks
that the per-call clearing works), and check that oversize problems are
refused.  This file is collected last so that a stop-at-first-failure run has
already run every other test.
"""
import numpy as np
import pytest
import torch

from golden_cases import O
from gpu_util import to_bf16, to_np

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _case(seed, B, Hq, Hk, D, T, maxs):
    rng = np.random.default_rng(seed)
    sl = rng.integers(1, maxs + 1, (B, Hk)).astype(np.int32)
    maxb = (maxs + T - 1) // T
    nb = int(sum((s + T - 1) // T for s in sl.ravel())) + 4
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
    return q, kc, vc, sl, tbl


def _call_noalloc(lib, q, kc, vc, sl, tbl, out, err, scale):
    B, _, Hq, D = q.shape
    Hk = sl.shape[1]
    return lib.wgkv_paged_decode_noalloc(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), kc.shape[0], kc.shape[1],
                                         sl.data_ptr(), tbl.data_ptr(), tbl.stride(1), B, Hq, Hk, D, scale,
                                         out.data_ptr(), err.data_ptr(), torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("shape", [(4, 32, 8, 128, 16, 20000), (3, 8, 2, 64, 32, 789)])
def test_noalloc_matches_workspace_entry_twice(shape):
    import wgkv
    from wgkv._lib import lib
    B, Hq, Hk, D, T, maxs = shape
    scale = D ** -0.5
    outs = []
    for seed in (21, 22):  # two calls in a row, different inputs
        q, kc, vc, sl, tbl = _case(seed + D, B, Hq, Hk, D, T, maxs)
        tq, tk, tv = to_bf16(q), to_bf16(kc), to_bf16(vc)
        ts, tt = torch.from_numpy(sl).cuda(), torch.from_numpy(tbl).cuda()
        ref = wgkv.paged_decode(tq, tk, tv, ts, tt, scale)
        out = torch.empty_like(tq)
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        st = _call_noalloc(lib, tq, tk, tv, ts, tt, out, err, scale)
        assert st == 0, st
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        np.testing.assert_allclose(to_np(out), to_np(ref), atol=ATOL, rtol=RTOL)
        np.testing.assert_allclose(to_np(out), O.paged_decode(q, kc, vc, sl, tbl, scale), atol=ATOL, rtol=RTOL)
        outs.append(out)
    assert not torch.equal(outs[0], outs[1])


def test_noalloc_rejects_oversize():
    from wgkv._lib import lib
    B, Hq, Hk, D = 512, 128, 8, 128  # scratch need far above the static array
    q = torch.zeros(B, 1, Hq, D, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(4, 16, D, dtype=torch.bfloat16, device="cuda")
    sl = torch.ones(B, Hk, dtype=torch.int32, device="cuda")
    tbl = torch.zeros(B, Hk, 1, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _call_noalloc(lib, q, kc, kc, sl, tbl, out, err, 1.0) == -3  # WGKV_ENOSPC


def test_noalloc_refuses_bad_head_dim_before_touching_the_array():
    from wgkv._lib import lib
    q = torch.zeros(1, 1, 8, 96, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(4, 16, 96, dtype=torch.bfloat16, device="cuda")
    sl = torch.ones(1, 2, dtype=torch.int32, device="cuda")
    tbl = torch.zeros(1, 2, 1, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert _call_noalloc(lib, q, kc, kc, sl, tbl, out, err, 1.0) == -1  # WGKV_EINVAL, not ENOSPC
