"""The registered operators on the GPU: ``torch.ops.wgkv.*`` give the same bits as the direct
calls they wrap, and the decode operator matches the CPU oracle (2e-2 absolute / 1e-2 relative
on bf16 outputs, the attention tolerance of this path)."""
import numpy as np
import pytest
import torch

from golden_cases import O
from gpu_util import to_bf16, to_np
from test_paged_decode_gpu import make_case

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


@pytest.fixture(scope="module")
def wgkv():
    import wgkv as m
    import wgkv.ops  # noqa: F401
    return m


def test_paged_decode_op(wgkv):
    q, kc, vc, sl, tbl = make_case(11, 3, 16, 4, 128, 16, 700, zero_heads=True)[:5]
    args = (to_bf16(q), to_bf16(kc), to_bf16(vc), torch.from_numpy(sl).cuda(), torch.from_numpy(tbl).cuda(),
            128 ** -0.5)
    got = torch.ops.wgkv.paged_decode(*args)
    direct = wgkv.paged_decode(*args)
    torch.cuda.synchronize()
    wgkv.check_errors()
    assert torch.equal(got.view(torch.int16), direct.view(torch.int16))
    np.testing.assert_allclose(to_np(got), O.paged_decode(q, kc, vc, sl, tbl, 128 ** -0.5), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("G,D", [(4, 128), (3, 64)])
def test_sparse_attn_op(wgkv, G, D):
    rng = np.random.default_rng(5 + G)
    B, Hk, L, W = 1, 2, 500, 64
    g = (rng.random((B, Hk, L)) < 0.3).astype(np.uint8)
    q = to_bf16(O.randn_bf16(rng, (B, L, Hk * G, D)))
    k = to_bf16(O.randn_bf16(rng, (B, L, Hk, D)))
    v = to_bf16(O.randn_bf16(rng, (B, L, Hk, D)))
    gm = torch.from_numpy(g).cuda()
    idx = wgkv.generate_sparse_indices(gm, W, B, Hk, L, gm.device)
    got = torch.ops.wgkv.sparse_attn(q, k, v, *idx, D ** -0.5)
    direct = wgkv.sparse_attn_func(q, k, v, *idx, softmax_scale=D ** -0.5)
    torch.cuda.synchronize()
    wgkv.check_errors()
    assert torch.equal(got.view(torch.int16), direct.view(torch.int16))
