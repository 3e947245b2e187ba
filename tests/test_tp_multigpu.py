"""The fused row-parallel o_proj + sum over GPUs (``wgkv_oproj_allreduce``) on 2..8 GPUs.

Each rank runs in its own process on its own GPU (NCCL process group for the host-side handle
exchange and the comparison).  Every call's output must equal the unfused path -- the same GEMM
rounded to bf16 on each rank, then an NCCL all-reduce -- within 2e-2 abs / 1e-2 rel, and be
bit-identical on every rank; consecutive calls (alternating buffer parities, several row counts)
must not interfere.  A last call made by rank 0 alone must end with WGKV_ERR_TIMEOUT (its peers
never publish) and leave the GPU usable.  Skipped when fewer than 2 GPUs are visible."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-2, 1e-2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        import wgkv
        from wgkv.tp import PeerGroup
        n_out, k = 4096, 512
        peers = PeerGroup(max_rows=128, max_cols=n_out)
        worst = 0.0
        same = True
        for call, rows in enumerate([64, 64, 7, 128, 64, 33, 64, 64]):
            g = torch.Generator(device="cuda").manual_seed(1000 * call + rank)
            a = torch.randn(rows, k, generator=g, device="cuda").bfloat16()
            w = (torch.randn(n_out, k, generator=g, device="cuda") * (k * world) ** -0.5).bfloat16()
            y = torch.empty(rows, n_out, dtype=torch.bfloat16, device="cuda")
            peers.oproj_allreduce(a, w, y)
            ref = a @ w.t()
            dist.all_reduce(ref)
            torch.cuda.synchronize()
            wgkv.check_errors()
            torch.testing.assert_close(y.float(), ref.float(), atol=ATOL, rtol=RTOL)
            worst = max(worst, float((y.float() - ref.float()).abs().max()))
            gathered = [torch.empty_like(y) for _ in range(world)]
            dist.all_gather(gathered, y)
            same = same and all(torch.equal(gathered[0], t) for t in gathered)
        dist.barrier()
        torch.cuda.synchronize()
        # a call that only rank 0 makes: its peers never publish, so its bounded waits run out and
        # it reports WGKV_ERR_TIMEOUT instead of hanging (no GPU fault involved)
        timed_out = None
        if rank == 0:
            a = torch.randn(8, k, device="cuda").bfloat16()
            w = torch.randn(n_out, k, device="cuda").bfloat16()
            y = torch.empty(8, n_out, dtype=torch.bfloat16, device="cuda")
            peers.oproj_allreduce(a, w, y)
            torch.cuda.synchronize()
            try:
                wgkv.check_errors()
                timed_out = False
            except AssertionError:
                timed_out = True
            torch.zeros(1, device="cuda").add_(1)  # the context is still usable
            torch.cuda.synchronize()
        dist.barrier()
        peers.close()
        out_q.put((rank, True, same, worst if rank else (worst, timed_out)))
    except Exception as e:  # reported to the parent
        out_q.put((rank, False, False, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 or more GPUs")
def test_fused_oproj_allreduce_matches_gemm_plus_nccl():
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] for r in res), res
    assert all(r[2] for r in res), "ranks disagree"
    assert res[0][3][1] is True, "the unmatched call did not report a timeout"
    assert all(p.exitcode == 0 for p in procs)
