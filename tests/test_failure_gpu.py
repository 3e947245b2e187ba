"""The device error path without a GPU fault: a bounded wait that runs out reports
WGKV_ERR_TIMEOUT through the error word (as the capacity checks report theirs), the host raises
the reference's AssertionError on the next check, and the context keeps working."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_wait_limit_reports_and_context_survives():
    import wgkv
    from wgkv.runtime import err_word, stream_ptr
    dev = torch.device("cuda", 0)
    wgkv.check_errors()  # clean start
    assert wgkv.lib.wgkv_selftest_wait_limit(err_word(dev).data_ptr(), stream_ptr(dev)) == 0
    torch.cuda.synchronize()
    with pytest.raises(AssertionError, match="timed out"):
        wgkv.check_errors()
    wgkv.check_errors()  # the word was reset by the check above
    # the context still runs kernels: a small paged decode against a dense softmax reference
    B, Hq, Hk, D, T, pages = 1, 4, 1, 64, 16, 8
    g = torch.Generator(device=dev).manual_seed(0)
    k = torch.randn(pages, T, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(pages, T, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(B, 1, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    sl = torch.tensor([[pages * T]], dtype=torch.int32, device=dev)
    bt = torch.arange(pages, dtype=torch.int32, device=dev).view(1, 1, pages)
    out = wgkv.paged_decode(q, k, v, sl, bt, D ** -0.5)
    s = (q[0, 0].float() @ k.view(-1, D).float().t()) * D ** -0.5
    ref = torch.softmax(s, -1) @ v.view(-1, D).float()
    np.testing.assert_allclose(out[0, 0].float().cpu().numpy(), ref.cpu().numpy(), atol=2e-2, rtol=1e-2)
    wgkv.check_errors()
