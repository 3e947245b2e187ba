"""Benchmark of the WG-KV admission hot path on B200.

Default workload (C2): Llama-3.1-8B-shaped decode, 32 layers,
batch 16, 128K-token context per sequence, 32 query / 8 KV heads, d=128,
bf16, a 4096-token local ring, page size 16, per-(layer, sequence, head)
global lengths from admit rates ~ Beta(2, 8).  One step = one decode token
for every sequence through all 32 layers of the hot path: write gate on the
new key, lazy promotion (layer 0), ring append, ragged paged attention --
called through the reference-named patch ``self_attn_forward_patch``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Under torchrun (N > 1) every rank runs its own batch-16 workload on its own
GPU (weak scaling: sequences are independent, no collective on the data
path); the step time is the max over ranks.  ``--impl reference`` times the
reference algorithm's CPU restatement (the test oracle) on the host cores.
Inputs are synthetic (seeded N(0,1) bf16, random-init gate weights); the
cache (~62 GB) is far larger than L2, so no L2 flush is needed.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import tempfile
import threading
import time
from types import SimpleNamespace

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "wg-kv_b200"))

CFG = dict(model="Llama-3.1-8B-shaped", layers=32, batch=16, ctx=131072, q_heads=32, kv_heads=8, head_dim=128,
           window=4096, page=16, admit="Beta(2,8)", gate="pre_k->64->1 GELU sigmoid", threshold=0.5)
METRIC = "decode tok/s @128K ragged cache (Llama-8B shape, B=16, 32 layers)"
# C4: Qwen3-4B-shaped decode, batch 64, per-sequence context uniform in 8K..32K,
# ring 2048, aggressive gating (per-head admit ~ Beta(1,10))
QWEN3_CFG = dict(model="Qwen3-4B-shaped", layers=36, batch=64, ctx=32768, ctx_min=8192, q_heads=32, kv_heads=8,
                 head_dim=128, window=2048, page=16, admit="Beta(1,10)", gate="pre_k->64->1 GELU sigmoid",
                 threshold=0.5)
WORKLOAD_NAME = "C2 decode: Llama-3.1-8B shape, B=16/GPU, 128K ctx, W=4096, T=16, Beta(2,8) admit"
QWEN3_METRIC = "decode tok/s @8-32K mixed ragged cache (Qwen3-4B shape, B=64, 36 layers)"
QWEN3_NAME = "C4 decode: Qwen3-4B shape, B=64/GPU, ctx U[8K,32K] per sequence, W=2048, T=16, Beta(1,10) admit"


def _admit_params():
    a = CFG["admit"]
    return tuple(float(x) for x in a[a.index("(") + 1:a.index(")")].split(","))


def peaks():
    p = os.path.join(HERE, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ----------------------------------------------------------------------------
# synthetic decode state
# ----------------------------------------------------------------------------

def draw_lengths(seed, Ly, B, Hk, ctx, W):
    """Per-(layer, sequence, head) admit rates and global lengths; per-sequence contexts are uniform in
    [ctx_min, ctx] when the workload sets ctx_min."""
    rng = np.random.default_rng(seed)
    a, b = _admit_params()
    rate = rng.beta(a, b, (Ly, B, Hk))
    ctx_b = rng.integers(CFG["ctx_min"], ctx + 1, B) if "ctx_min" in CFG else np.full(B, ctx)
    glen = np.round(rate * (ctx_b[None, :, None] - W)).astype(np.int64)
    return rate, glen


def build_state(dev, steps_total, seed=2):
    import torch
    import wgkv
    Ly, B, Hk, Hq, D = CFG["layers"], CFG["batch"], CFG["kv_heads"], CFG["q_heads"], CFG["head_dim"]
    W, T, ctx = CFG["window"], CFG["page"], CFG["ctx"]
    rate, glen = draw_lengths(seed, Ly, B, Hk, ctx, W)
    gpages = (glen + T - 1) // T
    ring_pages = Ly * B * Hk * (W // T)
    grow = (steps_total + T - 1) // T + 1  # pages a head may gain during the run
    total_blocks = int(ring_pages + gpages.sum() + Ly * B * Hk * grow + 1)
    max_tokens_per_head = int(W + glen.max() + steps_total + T)
    cache = SimpleNamespace()
    wgkv.init_pool(cache, layers=Ly, batch=B, kv_heads=Hk, head_dim=D, window=W, page=T,
                   max_total_tokens=total_blocks * T, max_tokens_per_head=max_tokens_per_head, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    rows = cache.block_pool_k.shape[0]
    step = 1 << 26
    for t in (cache.block_pool_k, cache.block_pool_v):
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            t[r0:r1].normal_(generator=g)
    # global pages: a random permutation of the pool after the ring pages (as utils/benchmark_decode.py:72-77)
    n_g = int(gpages.sum())
    perm = torch.randperm(n_g, generator=torch.Generator().manual_seed(seed), dtype=torch.int64).to(torch.int32)
    perm += ring_pages
    table = cache.block_table.view(Ly * B * Hk, -1)
    lp = W // T
    flat_pages = gpages.reshape(-1)
    off = 0
    host_rows = table[:, lp:].cpu()
    for i, n in enumerate(flat_pages):
        n = int(n)
        host_rows[i, :n] = perm[off:off + n]
        off += n
    table[:, lp:].copy_(host_rows.to(dev))
    cache.global_lengths.copy_(torch.from_numpy(glen.astype(np.int32)).to(dev))
    lig = torch.from_numpy((np.random.default_rng(seed + 1).random((Ly, B, Hk, W)) < rate[..., None]).astype(np.uint8))
    cache.local_is_global.copy_(lig.to(dev))
    cache.next_free_block.fill_(ring_pages + n_g)
    cache.local_length = W
    cache.local_ptr = 0
    return cache, rate, glen


def build_layers(dev, rate, seed=3):
    import torch
    import torch.nn.functional as F
    import wgkv
    Ly, Hk, D = CFG["layers"], CFG["kv_heads"], CFG["head_dim"]
    cfg = SimpleNamespace(num_hidden_layers=Ly, num_key_value_heads=Hk, num_attention_heads=CFG["q_heads"],
                          head_dim=D, block_size=CFG["page"], local_window_size=CFG["window"], g_defer=False,
                          g_threshold=CFG["threshold"], max_total_tokens=None, max_tokens_per_head=None)
    torch.manual_seed(seed)
    layers = []
    x = torch.randn(4096, D, device=dev)
    for l in range(Ly):
        gp = wgkv.GatingPredictor(D, Hk, ["pre_k"], "gelu", 0.5, 1e-3, False, True).to(dev, torch.bfloat16)
        # bias per head so that P(score > 0.5) ~ the head's admit rate (calibrated on N(0,1) keys)
        with torch.no_grad():
            w1 = gp.conv1.weight.float().view(Hk, -1, D)
            b1 = gp.conv1.bias.float().view(Hk, -1)
            w2 = gp.conv2.weight.float().view(Hk, -1)
            hdn = F.gelu(torch.einsum("td,hjd->htj", x, w1) + b1[:, None, :])
            logit = torch.einsum("htj,hj->ht", hdn, w2)
            r = torch.from_numpy(rate[l].mean(axis=0)).to(dev).float()
            b2 = -torch.stack([torch.quantile(logit[h], 1 - r[h]) for h in range(Hk)])
            gp.conv2.bias.copy_(b2.to(torch.bfloat16))
        a = SimpleNamespace(layer_idx=l, head_dim=D, scaling=D ** -0.5, g_predictors=gp)
        wgkv.attach(a, cfg)
        layers.append(a)
    return layers


def algorithmic_bytes(cache, glen_now):
    """Bytes one decode step must move (K/V of every live token, q/o, page ids, append, gate input)."""
    Ly, B, Hk, Hq, D, W, T = (CFG[k] for k in ("layers", "batch", "kv_heads", "q_heads", "head_dim", "window", "page"))
    seqlen = W + glen_now
    attn = int(seqlen.sum()) * D * 2 * 2
    pages = int(((seqlen + T - 1) // T).sum()) * 4
    qo = Ly * B * Hq * D * 2 * 2
    append = Ly * B * Hk * D * 2 * 2 * 2  # read new k/v, write ring
    gate = Ly * B * Hk * D * 2
    return attn + pages + qo + append + gate, attn + pages + qo


# ----------------------------------------------------------------------------
# clocks
# ----------------------------------------------------------------------------

class ClockSampler:
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--id={gpu_index}", f"--query-gpu={self.Q}", "--format=csv,noheader",
                                       "-lms", "50"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self):
        if self.p is None:
            return None
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.flush()
        lines = open(self.f.name).read().strip().splitlines()
        os.unlink(self.f.name)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in lines:
            c = [x.strip() for x in ln.split(",")]
            if len(c) < 9:
                continue
            try:
                sm.append(float(c[1].split()[0]))
                mx = float(c[2].split()[0])
            except ValueError:
                continue
            for n, v in zip(names, c[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# CPU arms: the reference's PyTorch decode step on the host cores (oracle/torch_cpu_step.py)
# ----------------------------------------------------------------------------

def cpu_threads():
    """Use every host core: torchrun sets OMP_NUM_THREADS=1 for its ranks."""
    import torch
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return torch.get_num_threads()


def cpu_sample_step(layers_in_sample=2, seed=5):
    """A bounded CPU sample of the workload's decode step: all ``batch`` sequences x
    ``layers_in_sample`` layers at the GPU run's length distribution (rank 0's draw), with the
    reference's operations in bf16 torch on the host.  Returns (callable, description, layers)."""
    import torch
    from oracle.torch_cpu_step import TorchCpuDecode
    Ly, B, Hk, Hq, D, W, T, ctx = (CFG[k] for k in ("layers", "batch", "kv_heads", "q_heads", "head_dim", "window",
                                                    "page", "ctx"))
    S = min(layers_in_sample, Ly)
    _, glen = draw_lengths(2, Ly, B, Hk, ctx, W)
    st = TorchCpuDecode(S, B, Hk, Hq, D, W, T, glen[:S], steps=4096, seed=seed, threshold=CFG["threshold"])
    g = torch.Generator().manual_seed(seed + 1)
    q = torch.randn(S, B, Hq, D, generator=g).to(torch.bfloat16)
    kn, vn, pk = (torch.randn(S, B, Hk, D, generator=g).to(torch.bfloat16) for _ in range(3))

    def run():
        st.step(q, kn, vn, pk)
    tokens = int((W + glen[:S]).sum())
    desc = (f"{B} sequences x {S} of {Ly} layers of the decode step ({tokens} cached tokens: gate, promotion, "
            f"ring append, paged attention), the reference's torch operations in bf16 on the host "
            f"(oracle/torch_cpu_step.py); tok/s = {B} / (t_sample x {Ly}/{S})")
    return run, desc, S


def time_cpu(budget_s=15.0, min_reps=2, max_reps=50):
    cores = cpu_threads()
    run, desc, S = cpu_sample_step()
    run()  # warm
    t0 = time.perf_counter()
    reps = 0
    while reps < min_reps or (time.perf_counter() - t0 < budget_s and reps < max_reps):
        run()
        reps += 1
    t = (time.perf_counter() - t0) / reps
    return CFG["batch"] / (t * CFG["layers"] / S), desc + f"; {reps} samples of {t * 1e3:.1f} ms", cores


def reference_arm(args, rank, world):
    """The reference's kind of computation on the host cores: each step is one bounded sample (all
    sequences x 1 layer of the decode step), run by rank 0 alone."""
    if rank != 0:
        return
    cores = cpu_threads()
    run, desc, S = cpu_sample_step(layers_in_sample=1)
    for _ in range(args.warmup):
        run()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        run()
    t = (time.perf_counter() - t0) / args.steps
    val = CFG["batch"] / (t * CFG["layers"] / S)
    line = {"metric": METRIC, "value": val, "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": t * 1e3 * CFG["layers"] / S, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD_NAME + " (each step: one bounded sample, all sequences x 1 layer)",
                       **CFG},
            "cpu_baseline": {"value": val, "unit": "tok/s", "cores": cores, "kind": "port", "sample": desc},
            "e2e": {"value": val, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------

def gpu_arm(args, rank, world, local_rank, emit=True, steps=None, extras=True):
    """The decode workload of CFG (C2 by default, C4 with --workload qwen3_decode).  The default run
    (``extras``) adds the other BASELINE workloads as sub-records of its line: the 400K prefill (C3)
    and the Qwen3-4B decode (C4) on one GPU, and the KV-head-sharded decode (C5) at every N."""
    import torch
    import torch.distributed as dist
    import wgkv
    from wgkv.dist import max_over_ranks
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    Ly, B, Hk, Hq, D = CFG["layers"], CFG["batch"], CFG["kv_heads"], CFG["q_heads"], CFG["head_dim"]
    K = steps if steps is not None else args.steps
    steps_total = args.warmup + 2 * K + 8
    cache, rate, glen0 = build_state(dev, steps_total, seed=2 + 1000 * rank)
    layers = build_layers(dev, rate, seed=3 + 1000 * rank)
    NI = 4
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    # per-step inputs laid out as the q/k/v projections produce them, (B, 1, H, D), viewed (B, H, 1, D)
    per_layer = Hq + 3 * Hk
    inputs = torch.randn(NI, Ly, B, 1, per_layer, D, generator=g, device=dev).to(torch.bfloat16)
    qbuf = inputs[:, :, :, :, :Hq].contiguous()

    outbuf = torch.empty(Ly, B, 1, Hq, D, dtype=torch.bfloat16, device=dev)
    outs = [None] * Ly

    def step(s, inp=None, qin=None):
        for l in range(Ly):
            if inp is None:
                x = inputs[s % NI, l]
                q = qbuf[s % NI, l].transpose(1, 2)
            else:
                x = inp[l]
                q = qin[l].transpose(1, 2)
            k = x[:, :, Hq:Hq + Hk].transpose(1, 2)
            v = x[:, :, Hq + Hk:Hq + 2 * Hk].transpose(1, 2)
            pk = x[:, :, Hq + 2 * Hk:].transpose(1, 2)
            a = layers[l]
            o, _, _ = a.self_attn_forward_patch(a, 3, None, cache, (B, 1), q, pk, k, v)
            outs[l] = o

    def barrier():
        if world > 1:
            dist.barrier()

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    wgkv.check_errors()
    glen_start = cache.global_lengths.cpu().numpy().astype(np.int64)

    # ---- device-resident timed region ----
    clk = ClockSampler(local_rank) if (rank == 0 and emit) else None
    barrier()
    torch.cuda.synchronize()
    l0 = wgkv.lib.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("wgkv_timed")
    e0.record()
    for s in range(K):
        step(s)
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    launches = wgkv.lib.launches - l0
    ms = e0.elapsed_time(e1)
    clocks = clk.stop() if clk else None
    wgkv.check_errors()
    glen_end = cache.global_lengths.cpu().numpy().astype(np.int64)
    ms = max_over_ranks(ms, dev)
    ms_step = ms / K
    value = world * B * K / (ms / 1e3)
    bytes_step, _ = algorithmic_bytes(cache, (glen_start + glen_end) / 2.0)

    # ---- end-to-end through the public API with host buffers ----
    host_in = torch.empty(NI, *inputs.shape[1:], dtype=torch.bfloat16, pin_memory=True)
    host_in.copy_(inputs)
    host_q = torch.empty(NI, *qbuf.shape[1:], dtype=torch.bfloat16, pin_memory=True)
    host_q.copy_(qbuf)
    # double-buffered: step s+1's inputs go up and step s-1's outputs come back on a copy stream while
    # step s computes; every copy is inside the timed region
    dev_in = [torch.empty_like(inputs[0]) for _ in range(2)]
    dev_q = [torch.empty_like(qbuf[0]) for _ in range(2)]
    dev_out = [torch.empty_like(outbuf) for _ in range(2)]
    host_out = [torch.empty(outbuf.shape, dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
    e_steps = max(1, min(K, 64))
    main = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()  # noqa: E731
    in_ready, in_free, out_ready, out_free = ([ev(), ev()] for _ in range(4))
    barrier()
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    cs.wait_stream(main)

    def upload(s_, j):
        with torch.cuda.stream(cs):
            dev_in[j].copy_(host_in[s_ % NI], non_blocking=True)
            dev_q[j].copy_(host_q[s_ % NI], non_blocking=True)
            in_ready[j].record(cs)

    upload(0, 0)
    for s in range(e_steps):
        i = s % 2
        if s + 1 < e_steps:
            if s >= 1:
                cs.wait_event(in_free[1 - i])  # step s-1 has read that buffer
            upload(s + 1, 1 - i)
        main.wait_event(in_ready[i])
        if s >= 2:
            main.wait_event(out_free[i])  # step s-2's outputs are on the host
        step(s, dev_in[i], dev_q[i])
        in_free[i].record(main)
        for l in range(Ly):
            dev_out[i][l].copy_(outs[l])
        out_ready[i].record(main)
        with torch.cuda.stream(cs):
            cs.wait_event(out_ready[i])
            host_out[i].copy_(dev_out[i], non_blocking=True)
            out_free[i].record(cs)
    main.wait_stream(cs)
    e3.record()
    torch.cuda.synchronize()
    barrier()
    e2e = world * B * e_steps / (max_over_ranks(e2.elapsed_time(e3), dev) / 1e3)
    wgkv.check_errors()

    # ---- roofline of the dominant kernel (paged decode), timed alone ----
    T = CFG["page"]
    W = CFG["window"]
    kc = cache.block_pool_k.view(cache.total_blocks, T, D)
    vc = cache.block_pool_v.view(cache.total_blocks, T, D)
    gl = cache.global_lengths
    seq_l = [(gl[l] + W).to(torch.int32).contiguous() for l in range(Ly)]
    qd = qbuf[0]  # (Ly, B, 1, Hq, D)
    od = torch.empty(B, 1, Hq, D, dtype=torch.bfloat16, device=dev)
    reps = 3
    for l in range(Ly):
        wgkv.paged_decode(qd[l].contiguous(), kc, vc, seq_l[l], cache.block_table[l], D ** -0.5, out=od)
    qs = [qd[l].contiguous() for l in range(Ly)]
    torch.cuda.synchronize()
    e4, e5 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e4.record()
    for _ in range(reps):
        for l in range(Ly):
            wgkv.paged_decode(qs[l], kc, vc, seq_l[l], cache.block_table[l], D ** -0.5, out=od)
    e5.record()
    torch.cuda.synchronize()
    per_launch_ms = e4.elapsed_time(e5) / (reps * Ly)
    glen_now = cache.global_lengths.cpu().numpy().astype(np.int64)
    sl = W + glen_now
    kbytes = (int(sl.sum()) * D * 2 * 2 + int(((sl + T - 1) // T).sum()) * 4 + Ly * B * Hq * D * 2 * 2) / Ly
    achieved = kbytes / (per_launch_ms / 1e3) / 1e9
    peak, peak_kind = peaks()
    traffic = None
    prof = os.path.join(HERE, "profiles", "paged_decode_traffic.json")
    if os.path.exists(prof):
        try:
            traffic = float(json.load(open(prof))["dram_bytes_per_algorithmic_byte"]) * kbytes
        except Exception:
            traffic = None

    cache_gb = cache.block_pool_k.numel() * 4 / 1e9
    h2d_step = int((inputs[0].numel() + qbuf[0].numel()) * 2)  # the bytes the e2e loop uploads per step
    d2h_step = int(outbuf.numel() * 2)
    prefill = c4 = c5 = None
    extras = extras and args.workload == "decode" and not args.small and not args.no_extras
    if extras:
        # release the decode state (the pool views of the roofline timing included) before the next workload
        del cache, layers, inputs, qbuf, outbuf, outs, host_in, host_q, dev_in, dev_q, host_out
        del kc, vc, gl, seq_l, qd, qs, od
        torch.cuda.empty_cache()
    if extras and world == 1 and not args.no_prefill:
        # the 400K sparse prefill (C3) on the same GPU, decode cache released first
        pl = prefill_arm(args, rank, world, local_rank, emit=False)
        prefill = {k: pl[k] for k in ("metric", "value", "unit", "admitted_frac", "tflops_step", "roofline",
                                      "sparse_attn_func_gather_ms", "kernels", "gpu_launches", "clocks")}
        prefill["workload"] = pl["config"]["workload"]
        torch.cuda.empty_cache()
    if extras and world == 1:
        # C4: Qwen3-4B-shaped decode, batch 64, mixed 8-32K contexts
        c4 = run_workload(QWEN3_CFG, lambda: gpu_arm(args, rank, world, local_rank, emit=False,
                                                     steps=min(K, 64), extras=False))
        c4 = {k: c4[k] for k in ("value", "unit", "ms_per_step", "hbm_gbs_step", "e2e", "roofline", "gpu_launches")}
        c4.update(metric=QWEN3_METRIC, workload=QWEN3_NAME, steps=min(K, 64))
        torch.cuda.empty_cache()
    if extras:
        # C5: KV heads sharded over the N GPUs of this run, o_proj all-reduce per layer
        c5 = c5_arm(args, rank, world, local_rank, emit=False, steps=min(K, 16))
        c5 = {k: c5[k] for k in ("metric", "value", "unit", "n_gpus", "steps", "ms_per_step", "scaling",
                                 "per_gpu_tok_s", "fused_projection", "per_layer_us", "per_layer_us_note",
                                 "nccl_baseline", "e2e",
                                 "attn_hbm_gbs_per_gpu", "attn_hbm_frac_per_gpu", "roofline", "gpu_launches")}
        c5["config"] = {"workload": "C5 decode: B=64, 256K ctx, KV heads 8/N per GPU, o_proj + sum over GPUs fused",
                        "parallelism": f"tp{world} (KV heads)", "note": "resident layer pools cycled when the "
                        "cache does not fit (N < 4)"}
    line = None
    if rank == 0:
        cpu_val, cpu_desc, cpu_cores = (None, None, None)
        if world == 1 and emit:
            cpu_val, cpu_desc, cpu_cores = time_cpu()
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD_NAME,
                       "l2": f"inputs larger than L2 ({cache_gb:.0f} GB cache), no flush", "parallelism": f"dp{world} (sequences)",
                       **CFG},
            "hbm_gbs_step": bytes_step / (ms_step / 1e3) / 1e9,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": h2d_step,
                    "d2h_bytes_per_step": d2h_step},
            "roofline": {"bound": "hbm", "kernel": "paged_decode_kernel<128>", "achieved": achieved, "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                         "bytes_per_launch": kbytes, "ms_per_launch": per_launch_ms},
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if prefill is not None:
            line["prefill_400k"] = prefill
        if c4 is not None:
            line["c4_qwen3_decode"] = c4
        if c5 is not None:
            line["c5_decode"] = c5
        if cpu_val is not None:
            line["cpu_baseline"] = {"value": cpu_val, "unit": "tok/s", "cores": cpu_cores, "kind": "port",
                                    "sample": cpu_desc}
        if emit:
            print(json.dumps(line), flush=True)
    return line


def run_workload(cfg, fn):
    """Run ``fn`` with the decode globals (CFG) switched to ``cfg``, then restore them."""
    saved = dict(CFG)
    CFG.clear()
    CFG.update(cfg)
    try:
        return fn()
    finally:
        CFG.clear()
        CFG.update(saved)


# ----------------------------------------------------------------------------
# prefill workload (C3): 400K tokens, 32 layers, ~30 % admitted
# ----------------------------------------------------------------------------
PCFG = dict(model="Llama-3.1-8B-shaped", layers=32, seq_len=400000, q_heads=32, kv_heads=8, head_dim=128,
            window=4096, page=16, admit="~30% mean per head", max_tokens_per_head=401000,
            gate="pre_k->64->1 GELU sigmoid", threshold=0.5)


def useful_flops(cc, L, W, D, G, blk=64):
    """4*D FLOPs per unmasked (q, k) pair of the vertical-slash mask, summed over query heads."""
    B, Hk, R = cc.shape
    q = np.arange(L)
    s = (q // blk) * blk
    band = q - np.maximum(0, s - W + 1) + 1  # causal band keys of each query
    rows_per_block = np.bincount(q // blk, minlength=R)
    pairs = cc.astype(np.int64) * rows_per_block[None, None, :]
    return 4.0 * D * G * (float(pairs.sum()) + B * Hk * float(band.sum()))


def prefill_arm(args, rank, world, local_rank, emit=True):
    import torch
    import wgkv
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    Ly, L, Hq, Hk, D, W, T = (PCFG[k] for k in ("layers", "seq_len", "q_heads", "kv_heads", "head_dim", "window", "page"))
    if args.small:
        Ly, L = 2, 65536
    G = Hq // Hk
    rng = np.random.default_rng(3 + rank)
    rates = np.clip(rng.beta(3, 7, (Ly, Hk)), 0.05, 0.9)  # mean 0.3
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)
    q = torch.randn(1, L, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    kvp = torch.randn(1, L, 3 * Hk, D, generator=g, device=dev).to(torch.bfloat16)
    k, v, pk = (kvp[:, :, i * Hk:(i + 1) * Hk].transpose(1, 2) for i in range(3))
    # gates calibrated per (layer, head) to the drawn rates
    CFG_save = dict(CFG)
    CFG["layers"] = Ly
    layers = build_layers(dev, np.repeat(rates[:, None, :], 1, axis=1), seed=5 + rank)
    CFG.update(CFG_save)
    total = int(Ly * Hk * (W + 1.1 * rates.mean() * L + L * 0.05)) + Ly * Hk * 64
    for a in layers:
        a.config.max_total_tokens = total
        a.config.max_tokens_per_head = PCFG["max_tokens_per_head"] if not args.small else L + 64

    def run(n_layers):
        cache = SimpleNamespace()
        for l in range(n_layers):
            a = layers[l]
            a.g_predictors  # noqa
            o, _, _ = a.self_attn_forward_patch(a, 3, None, cache, (1, L), q.transpose(1, 2), pk, k, v)
        return cache

    c = run(1)  # warm-up: one layer
    torch.cuda.synchronize()
    wgkv.check_errors()
    del c
    torch.cuda.empty_cache()
    clk = ClockSampler(local_rank) if rank == 0 else None
    l0 = wgkv.lib.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    cache = run(Ly)
    e1.record()
    torch.cuda.synchronize()
    launches = wgkv.lib.launches - l0
    ms = e0.elapsed_time(e1)
    clocks = clk.stop() if clk else None
    wgkv.check_errors()
    admitted = int(cache.global_lengths.sum().item())
    # useful FLOPs from each layer's indices, and the sparse attention kernel timed alone (layer 0's mask)
    flops = 0.0
    idx0 = None
    for l in range(Ly):
        gm = torch.empty(1, Hk, L, dtype=torch.uint8, device=dev)
        layers[l].g_predictors.admit(pk, k, v, PCFG["threshold"], gm)
        idx = wgkv.sparse_indices_into(gm, W, L, 64)
        flops += useful_flops(idx[2].cpu().numpy(), L, W, D, G)
        if l == 0:
            idx0 = idx
    torch.cuda.synchronize()
    out = torch.empty_like(q)
    kk, vv = kvp[:, :, :Hk], kvp[:, :, Hk:2 * Hk]

    def timed(fn, reps=3):
        """Mean CUDA-event time of ``reps`` back-to-back calls after one warm-up call (ms)."""
        fn()
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for _ in range(reps):
            fn()
        a1.record()
        torch.cuda.synchronize()
        return a0.elapsed_time(a1) / reps

    # the product path: admitted columns from layer 0's compacted pool (same mask as idx0)
    attn_ms = timed(lambda: wgkv.sparse_attn_func_pooled(q, kk, vv, *idx0, cache.block_pool_k, cache.block_pool_v,
                                                         cache.block_table[0], W // T, T, softmax_scale=D ** -0.5,
                                                         out=out))
    # the generic sparse_attn_func (columns gathered by index from k / v)
    gather_ms = timed(lambda: wgkv.sparse_attn_func(q, kk, vv, *idx0, softmax_scale=D ** -0.5, out=out))
    f0 = useful_flops(idx0[2].cpu().numpy(), L, W, D, G)
    tf = f0 / (attn_ms / 1e3) / 1e12
    kernels = admission_kernel_rates(cache, layers[0], q, pk, k, v, L, W, T, D, Hk, timed)
    try:
        pk_tf = float(json.load(open(os.path.join(HERE, "MEASURED_PEAKS.json")))["bf16_tflops"]), "measured"
    except Exception:
        pk_tf = 1590.0, "fallback"
    line = {"metric": f"{L // 1000}K sparse-prefill ms ({Ly} layers)", "value": ms, "unit": "ms", "n_gpus": 1,
            "steps": 1, "warmup": 1, "ms_per_step": ms, "higher_is_better": False, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C3 prefill" + (" (small)" if args.small else ""), **PCFG, "layers": Ly,
                       "seq_len": L},
            "admitted_frac": admitted / (Ly * Hk * max(L - W, 1)),
            "useful_tflops_total": flops / 1e12, "tflops_step": flops / (ms / 1e3) / 1e12,
            "sparse_attn_func_gather_ms": gather_ms,
            "kernels": kernels,
            "roofline": {"bound": "tensor", "kernel": "sparse_prefill_tc_kernel (pooled)", "achieved": tf, "peak": pk_tf[0],
                         "peak_kind": pk_tf[1], "unit": "TFLOP/s", "frac": tf / pk_tf[0], "traffic": None,
                         "ms_per_launch": attn_ms, "flops_per_launch": f0},
            "gpu_launches": launches, "clocks": clocks}
    if rank == 0 and emit:
        print(json.dumps(line), flush=True)
    return line


def admission_kernel_rates(cache, a0, q, pk, k, v, L, W, T, D, Hk, timed):
    """CUDA-event time and HBM rate of the admission kernels of one C3 layer (layer 0 of the run):
    the gate (gate_kernel), the ring fill + compaction (chunk_count, prefill_alloc, prefill_scatter)
    and the sparse-index builder, each against its algorithmic bytes:

    * gate: pre_k read (2 B per element) + one mask byte per (head, token);
    * compaction: mask read + K/V rows of the ring and of the admitted tokens read and written;
    * indices: mask read + 4 B per admitted column index + the per-row-block counts and offsets.

    The compaction is re-run on layer 0 of the finished cache with the allocator rewound to the
    ring pages, so it rewrites the same pages with the same rows."""
    import torch
    import wgkv
    from wgkv._lib import lib
    from wgkv.pool import pool_ref
    from wgkv.runtime import stream_ptr, workspace
    peak, kind = peaks()
    dev = q.device
    thr = a0.config.g_threshold
    gm = torch.empty(1, Hk, L, dtype=torch.uint8, device=dev)
    g_ms = timed(lambda: a0.g_predictors.admit(pk, k, v, thr, gm))
    n_adm = cache.global_lengths[0].to(torch.int64).sum().item()
    g_bytes = Hk * L * (D * 2 + 1)
    total_local = int(cache.block_table[..., :W // T].numel())
    saved = cache.next_free_block.clone()
    nbytes = int(lib.wgkv_prefill_admit_workspace_size(1, Hk, L - W))
    ws = workspace(dev, "prefill_admit", nbytes)

    def s4(t):
        return t.data_ptr(), t.stride(0), t.stride(1), t.stride(2)

    def compact():
        cache.next_free_block.fill_(total_local)
        lib.wgkv_prefill_admit(pool_ref(cache), 0, L, *s4(k), *s4(v), None, 0, 0, 0, *s4(gm), ws.data_ptr(),
                               ws.numel(), stream_ptr(dev))

    c_ms = timed(compact)
    cache.next_free_block.copy_(saved)
    c_bytes = Hk * L + (Hk * min(L, W) + n_adm) * D * 2 * 2 * 2
    ci = torch.zeros(1, Hk, 1, L, dtype=torch.int32, device=dev)
    mc = torch.zeros(1, dtype=torch.int32, device=dev)
    i_ms = timed(lambda: wgkv.sparse_indices_into(gm, W, L, 64, column_index=ci, max_count=mc))
    R = (L + 63) // 64
    i_bytes = Hk * L + 4 * n_adm + 4 * Hk * R + 4 * R * (min(W // 64, R) + 2)
    wgkv.check_errors()
    out = {}
    for name, ms, by, kern in (("gate", g_ms, g_bytes, "gate_kernel"),
                               ("compaction", c_ms, c_bytes, "chunk_count + prefill_alloc + prefill_scatter"),
                               ("sparse_indices", i_ms, i_bytes, "idx_count + idx_scan + idx_scatter (+ block offsets)")):
        gbs = by / (ms / 1e3) / 1e9
        out[name] = {"kernels": kern, "ms": ms, "algorithmic_bytes": by, "achieved_gbs": gbs, "peak_gbs": peak,
                     "peak_kind": kind, "frac": gbs / peak}
    return out


# ----------------------------------------------------------------------------
# C5: Llama-8B decode, batch 64 at 256K context, KV heads sharded across GPUs
# (8 -> 8/N per GPU, each GPU its own paged pool), row-parallel o_proj + NCCL all-reduce per layer.
# ----------------------------------------------------------------------------
C5_CFG = dict(model="Llama-3.1-8B-shaped", layers=32, batch=64, ctx=262144, q_heads=32, kv_heads=8, head_dim=128,
              window=4096, page=16, admit="Beta(2,8)", gate="pre_k->64->1 GELU sigmoid", threshold=0.5, hidden=4096)


def c5_arm(args, rank, world, local_rank, emit=True, steps=None):
    """BASELINE config 5 through ``wgkv.tp.KVHeadParallelAttention``: this rank's KV heads and their
    query heads, its own pool, the row-parallel o_proj slice of every layer and one all-reduce per
    layer.  Returns the JSON record (printed by rank 0 when ``emit``)."""
    import torch
    import torch.distributed as dist
    import wgkv
    from wgkv.dist import kv_head_shard, max_over_ranks
    from wgkv.tp import KVHeadParallelAttention, PeerGroup, shard_o_proj
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    K = steps if steps is not None else args.steps
    Ly, B, D, W, T = C5_CFG["layers"], C5_CFG["batch"], C5_CFG["head_dim"], C5_CFG["window"], C5_CFG["page"]
    Hq_all, Hk_all, hidden = C5_CFG["q_heads"], C5_CFG["kv_heads"], C5_CFG["hidden"]
    (h0, h1), (q0, q1) = kv_head_shard(Hk_all, Hq_all, rank, world)
    Hk, Hq = h1 - h0, q1 - q0
    # resident layer pools: all 32 when they fit in ~150 GB, else as many as fit, cycled over the 32 layers
    saved = dict(CFG)
    CFG.clear()
    CFG.update(C5_CFG)
    CFG["kv_heads"], CFG["q_heads"] = Hk, Hq
    _, glen = draw_lengths(2 + 1000 * rank, 1, B, Hk, C5_CFG["ctx"], W)
    per_layer = float(((W + glen) * D * 2 * 2).sum()) * 1.02
    resident = int(max(1, min(Ly, 150e9 // per_layer)))
    CFG["layers"] = resident
    steps_total = args.warmup + K + 40  # + the NCCL comparison, end-to-end and instrumented steps
    cache, rate, glen0 = build_state(dev, steps_total * ((Ly + resident - 1) // resident), seed=2 + 1000 * rank)
    layers = build_layers(dev, rate, seed=3 + 1000 * rank)
    CFG.clear()
    CFG.update(saved)
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    NI = 4
    inputs = torch.randn(NI, Ly, B, 1, Hq + 3 * Hk, D, generator=g, device=dev).to(torch.bfloat16)
    qbuf = inputs[..., :Hq, :].contiguous()
    # every layer its own W_o (hidden, 32 * 128); this rank keeps the columns of its query heads
    gw = torch.Generator(device=dev)
    gw.manual_seed(99)  # same full weights on every rank
    # o_proj + sum over GPUs as one kernel over NVLink peer memory (the NCCL path is timed beside it)
    try:
        peers = PeerGroup(max_rows=B, max_cols=hidden, device=dev)
    except RuntimeError as e:  # raised on every rank alike: the step then uses GEMM + NCCL
        print(f"rank {rank}: fused projection unavailable ({e}); using NCCL", file=sys.stderr)
        peers = None
    tp_layers = []
    for l in range(Ly):
        w_full = (torch.randn(hidden, Hq_all * D, generator=gw, device=dev) * (Hq_all * D) ** -0.5).to(torch.bfloat16)
        tp_layers.append(KVHeadParallelAttention(layers[l % resident], shard_o_proj(w_full, q0, q1, D), peers=peers))
        del w_full
    y = torch.empty(B, hidden, dtype=torch.bfloat16, device=dev)

    def step(s, xin=None, qin=None):
        for l in range(Ly):
            x = inputs[s % NI, l] if xin is None else xin[l]
            q = (qbuf[s % NI, l] if qin is None else qin[l]).transpose(1, 2)
            k = x[:, :, Hq:Hq + Hk].transpose(1, 2)
            v = x[:, :, Hq + Hk:Hq + 2 * Hk].transpose(1, 2)
            pk = x[:, :, Hq + 2 * Hk:].transpose(1, 2)
            tp_layers[l](cache, (B, 1), q, pk, k, v, out=y)

    def barrier():
        if world > 1:
            dist.barrier()

    for s in range(args.warmup):
        step(s)
    torch.cuda.synchronize()
    wgkv.check_errors()
    glen_start = cache.global_lengths.cpu().numpy().astype(np.int64)
    barrier()
    torch.cuda.synchronize()
    clk = ClockSampler(local_rank) if (rank == 0 and emit) else None
    l0 = wgkv.lib.launches
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for s in range(K):
        step(s)
    e1.record()
    torch.cuda.synchronize()
    launches = wgkv.lib.launches - l0
    barrier()
    clocks = clk.stop() if clk else None
    ms = max_over_ranks(e0.elapsed_time(e1), dev) / K
    wgkv.check_errors()
    glen_end = cache.global_lengths.cpu().numpy().astype(np.int64)

    def phases():
        """Per-layer phase times (CUDA events around attention and the projection / sum) on 2 extra steps."""
        for t in tp_layers:
            t.timers = {}
        barrier()
        for s in range(2):
            step(s)
        torch.cuda.synchronize()
        out = {}
        for key in ("attn", "o_proj_allreduce", "o_proj", "all_reduce"):
            vals = [x for t in tp_layers for x in t.breakdown().get(key, [])]
            if vals:
                out[key] = max_over_ranks(1e3 * float(np.median(vals)), dev)
        for t in tp_layers:
            t.timers = None
        return out

    phase = phases()

    # the same step with the unfused projection: torch GEMM + NCCL all-reduce (the baseline)
    for t in tp_layers:
        t.peers = None
    nccl_steps = max(1, min(K, 8))
    for s in range(2):  # warm-up: cuBLAS heuristics and the first NCCL all-reduce on this stream
        step(s)
    barrier()
    torch.cuda.synchronize()
    e8, e9 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e8.record()
    for s in range(nccl_steps):
        step(s)
    e9.record()
    torch.cuda.synchronize()
    nccl_ms = max_over_ranks(e8.elapsed_time(e9), dev) / nccl_steps
    nccl_phase = phases()
    for t in tp_layers:
        t.peers = peers
    wgkv.check_errors()
    fused = peers is not None

    # end to end: each step's q/k/v/pre-k rows come from pinned host memory and the step's output
    # (the last layer's all-reduced o_proj rows) goes back, double-buffered on a copy stream
    host_in = torch.empty(NI, *inputs.shape[1:], dtype=torch.bfloat16, pin_memory=True)
    host_in.copy_(inputs)
    host_q = torch.empty(NI, *qbuf.shape[1:], dtype=torch.bfloat16, pin_memory=True)
    host_q.copy_(qbuf)
    dev_in = [torch.empty_like(inputs[0]) for _ in range(2)]
    dev_q = [torch.empty_like(qbuf[0]) for _ in range(2)]
    dev_y = [torch.empty_like(y) for _ in range(2)]
    host_y = [torch.empty(y.shape, dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
    e_steps = max(1, min(K, 16))
    main = torch.cuda.current_stream(dev)
    cs = torch.cuda.Stream(dev)
    in_ready, in_free, out_ready, out_free = ([torch.cuda.Event(), torch.cuda.Event()] for _ in range(4))
    barrier()
    torch.cuda.synchronize()
    e6, e7 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e6.record()
    cs.wait_stream(main)

    def upload(s_, j):
        with torch.cuda.stream(cs):
            dev_in[j].copy_(host_in[s_ % NI], non_blocking=True)
            dev_q[j].copy_(host_q[s_ % NI], non_blocking=True)
            in_ready[j].record(cs)

    upload(0, 0)
    for s in range(e_steps):
        i = s % 2
        if s + 1 < e_steps:
            if s >= 1:
                cs.wait_event(in_free[1 - i])
            upload(s + 1, 1 - i)
        main.wait_event(in_ready[i])
        if s >= 2:
            main.wait_event(out_free[i])
        step(s, dev_in[i], dev_q[i])
        in_free[i].record(main)
        dev_y[i].copy_(y)
        out_ready[i].record(main)
        with torch.cuda.stream(cs):
            cs.wait_event(out_ready[i])
            host_y[i].copy_(dev_y[i], non_blocking=True)
            out_free[i].record(cs)
    main.wait_stream(cs)
    e7.record()
    torch.cuda.synchronize()
    barrier()
    e2e = B * e_steps / (max_over_ranks(e6.elapsed_time(e7), dev) / 1e3)
    wgkv.check_errors()
    # per-GPU attention bytes per step (32 layer visits over the resident pools)
    sl = W + (glen_start + glen_end) / 2.0
    visits = np.bincount(np.arange(Ly) % resident, minlength=resident)
    attn_bytes = float((sl.sum(axis=(1, 2)) * visits).sum()) * D * 2 * 2
    kc = cache.block_pool_k.view(cache.total_blocks, T, D)
    vc = cache.block_pool_v.view(cache.total_blocks, T, D)
    seq0 = (cache.global_lengths[0] + W).to(torch.int32).contiguous()
    od = torch.empty(B, 1, Hq, D, dtype=torch.bfloat16, device=dev)
    qd = qbuf[0, 0].contiguous()
    wgkv.paged_decode(qd, kc, vc, seq0, cache.block_table[0], D ** -0.5, out=od)
    torch.cuda.synchronize()
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record()
    for _ in range(5):
        wgkv.paged_decode(qd, kc, vc, seq0, cache.block_table[0], D ** -0.5, out=od)
    e3.record()
    torch.cuda.synchronize()
    kms = e2.elapsed_time(e3) / 5
    kbytes = float(seq0.sum().item()) * D * 2 * 2
    peak, peak_kind = peaks()
    ach = kbytes / (kms / 1e3) / 1e9
    barrier()
    torch.cuda.synchronize()
    if peers is not None:
        peers.close()
    del cache, layers, tp_layers, inputs, qbuf, host_in, host_q, peers
    torch.cuda.empty_cache()
    line = {"metric": "decode tok/s @256K ragged cache, KV heads sharded (Llama-8B shape, B=64, 32 layers)",
            "value": B / (ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "C5 decode: B=64, 256K ctx, KV heads 8/N per GPU, o_proj + sum over GPUs fused "
                                   "(one kernel over NVLink peer memory)",
                       "resident_layer_pools": resident,
                       "note": ("all 32 layer pools resident" if resident == Ly else
                                f"cache does not fit: {resident} resident layer pools cycled over 32 layers"),
                       "parallelism": f"tp{world} (KV heads)", **C5_CFG},
            "per_gpu_tok_s": B / (ms / 1e3) / world,
            "fused_projection": fused,
            "per_layer_us": phase,
            "per_layer_us_note": ("median over 2 instrumented steps x 32 layers, max over ranks; the sum over "
                                  "GPUs includes waiting for the slowest rank"),
            "nccl_baseline": {"what": "same step with torch GEMM + NCCL all-reduce for o_proj", "steps": nccl_steps,
                              "ms_per_step": nccl_ms, "value": B / (nccl_ms / 1e3), "per_layer_us": nccl_phase},
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": int(host_in_bytes(NI, Ly, B, Hq, Hk, D)),
                    "d2h_bytes_per_step": int(B * hidden * 2)},
            "gpu_launches": launches,
            "attn_hbm_gbs_per_gpu": attn_bytes / (ms / 1e3) / 1e9,
            "attn_hbm_frac_per_gpu": attn_bytes / (ms / 1e3) / 1e9 / peak,
            "roofline": {"bound": "hbm", "kernel": "paged_decode_kernel<128>", "achieved": ach, "peak": peak,
                         "peak_kind": peak_kind, "unit": "GB/s", "frac": ach / peak, "ms_per_launch": kms,
                         "bytes_per_launch": kbytes},
            "clocks": clocks}
    if rank == 0 and emit:
        print(json.dumps(line), flush=True)
    return line


def host_in_bytes(NI, Ly, B, Hq, Hk, D):
    """Bytes the C5 end-to-end loop uploads per step: q/k/v/pre-k rows of every layer + the q copy."""
    return Ly * B * (Hq + 3 * Hk) * D * 2 + Ly * B * Hq * D * 2


def quest_arm(args, rank, world, local_rank):
    """C2 decode with QUEST page selection (use_quest, modeling_layers.py:452-576) under a token budget,
    and one SnapKV eviction (snapkv_evict, :595-671) timed over the same pool."""
    import torch
    import wgkv
    from wgkv.dist import max_over_ranks
    from wgkv.pool import pool_ref
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    Ly, B, Hk, Hq, D = CFG["layers"], CFG["batch"], CFG["kv_heads"], CFG["q_heads"], CFG["head_dim"]
    W, T = CFG["window"], CFG["page"]
    budget = args.quest_budget
    cache, rate, glen0 = build_state(dev, args.warmup + args.steps + 8, seed=2 + 1000 * rank)
    NB = cache.total_blocks
    kp = cache.block_pool_k.view(NB, T, D)
    cache.quest_block_key_min = torch.empty(NB, D, dtype=torch.bfloat16, device=dev)
    cache.quest_block_key_max = torch.empty(NB, D, dtype=torch.bfloat16, device=dev)
    for p0 in range(0, NB, 1 << 20):  # page key bounds of the synthetic pool (all 16 rows of each page)
        p1 = min(NB, p0 + (1 << 20))
        torch.amin(kp[p0:p1], dim=1, out=cache.quest_block_key_min[p0:p1])
        torch.amax(kp[p0:p1], dim=1, out=cache.quest_block_key_max[p0:p1])
    cache.wgkv_pool.quest_min = cache.quest_block_key_min.data_ptr()
    cache.wgkv_pool.quest_max = cache.quest_block_key_max.data_ptr()
    layers = build_layers(dev, rate, seed=3 + 1000 * rank)
    for a in layers:
        a.config.use_quest, a.config.quest_token_budget = True, budget
    g = torch.Generator(device=dev)
    g.manual_seed(7 + rank)
    NI = 4
    inputs = torch.randn(NI, Ly, B, 1, Hq + 3 * Hk, D, generator=g, device=dev).to(torch.bfloat16)

    qbuf = inputs[:, :, :, :, :Hq].contiguous()  # q as the projection writes it, (B, 1, Hq, D) per layer
    static_in = torch.empty_like(inputs[0])  # the captured step reads its inputs from here
    static_q = torch.empty_like(qbuf[0])

    def step(xs, qs):
        for l in range(Ly):
            x = xs[l]
            q = qs[l].transpose(1, 2)
            k, v, pk = (x[:, :, Hq + i * Hk:Hq + (i + 1) * Hk].transpose(1, 2) for i in range(3))
            layers[l].self_attn_forward_patch(layers[l], 3, None, cache, (B, 1), q, pk, k, v)

    for s in range(args.warmup):
        l0 = wgkv.lib.launches
        step(inputs[s % NI], qbuf[s % NI])
        per_step_launches = wgkv.lib.launches - l0
    torch.cuda.synchronize()
    wgkv.check_errors()
    # replayed as a CUDA graph (one capture; each replay one more step)
    static_in.copy_(inputs[0])
    static_q.copy_(qbuf[0])
    dg = wgkv.DecodeGraph(cache, W)
    dg.capture(lambda: step(static_in, static_q))
    torch.cuda.synchronize()
    wgkv.check_errors()
    clk = ClockSampler(local_rank) if rank == 0 else None
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("wgkv_timed")
    e0.record()
    for s in range(args.steps):
        static_in.copy_(inputs[s % NI])
        static_q.copy_(qbuf[s % NI])
        dg.replay()
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    launches = per_step_launches * args.steps
    clocks = clk.stop() if clk else None
    wgkv.check_errors()
    ms = max_over_ranks(e0.elapsed_time(e1), dev) / args.steps
    glen = cache.global_lengths.cpu().numpy().astype(np.int64)
    full = W + glen
    kept = np.minimum(full, W + ((budget - W + T - 1) // T) * T)  # tokens attended per head (upper bound)
    attn_bytes = float(kept.sum()) * D * 2 * 2 + float((glen // T).sum()) * 2 * D * 2  # K/V read + page bounds
    # ---- one SnapKV eviction over the whole pool ----
    snap = None
    if world == 1:
        win, ratio, ks = 256, 0.3, 5
        gq = torch.Generator(device=dev)
        gq.manual_seed(9)
        qbuf = torch.randn(Ly, B, win, Hq, D, generator=gq, device=dev).to(torch.bfloat16)
        free_ids = torch.zeros(NB, dtype=torch.int32, device=dev)
        free_n = torch.zeros(1, dtype=torch.int32, device=dev)
        cache.wgkv_pool.free_ids, cache.wgkv_pool.free_count = free_ids.data_ptr(), free_n.data_ptr()
        nbytes = int(wgkv.lib.wgkv_snapkv_workspace_size(pool_ref(cache), win, Hq))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        before = int(cache.global_lengths.sum().item())
        torch.cuda.synchronize()
        e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2.record()
        st = wgkv.lib.wgkv_snapkv_evict(pool_ref(cache), qbuf.data_ptr(), win, Hq, D ** -0.5, ratio, ks,
                                        ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
        e3.record()
        torch.cuda.synchronize()
        assert st == 0
        wgkv.check_errors()
        after = int(cache.global_lengths.sum().item())
        evict_ms = e2.elapsed_time(e3)
        flops = 2.0 * 2 * win * (Hq // Hk) * D * before  # two passes of window-queries x keys (2 M N K each)
        snap = {"metric": "SnapKV eviction ms (all layers, whole pool)", "value": evict_ms, "unit": "ms",
                "window": win, "evict_ratio": ratio, "kernel_size": ks, "tokens_before": before,
                "tokens_after": after, "pages_freed": int(free_n.item()),
                "score_tflops": flops / (evict_ms / 1e3) / 1e12,
                "kernels": ("snap_rowstats / snap_scores (mma.sync)" if os.environ.get("WGKV_SNAPKV_MMA_SYNC") == "1"
                            else "snap_rowstats_tc / snap_scores_tc (tcgen05)")
                + " + snap_select_compact + snap_free"}
    peak, kind = peaks()
    if rank == 0:
        line = {
            "metric": f"decode tok/s @128K ragged cache with QUEST (budget {budget} tokens / head)",
            "value": world * B / (ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (page bounds over all rows of each page)",
            "config": {"workload": "C2 decode + QUEST selection (use_quest), steps replayed as a CUDA graph",
                       "quest_token_budget": budget,
                       "l2": "inputs larger than L2, no flush", **CFG},
            "attended_tokens_per_head": float(kept.mean()), "cached_tokens_per_head": float(full.mean()),
            "roofline": {"bound": "hbm", "kernel": "quest_select + paged_decode (whole step)",
                         "achieved": attn_bytes / (ms / 1e3) / 1e9, "peak": peak, "peak_kind": kind, "unit": "GB/s",
                         "frac": attn_bytes / (ms / 1e3) / 1e9 / peak, "traffic": None},
            "gpu_launches": launches, "clocks": clocks,
        }
        if snap is not None:
            line["snapkv_evict"] = snap
        print(json.dumps(line), flush=True)


def model_arm(args, rank, world, local_rank):
    """TTFT / TPOT of a whole random-init decoder on the WG-KV path (scripts/profiling.py:346-418)."""
    import torch
    import wgkv
    from wgkv.dist import max_over_ranks
    from wgkv.model import SHAPES, WgkvDecoder
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    shape = SHAPES[args.model]
    B, P, K, Wu = args.batch, args.prompt, args.steps, args.warmup
    n_eager = min(K, 32)
    total = P + Wu + n_eager + 2 * K + 24
    m = WgkvDecoder(shape, batch=B, window=args.window, max_tokens_per_head=total + args.window + 64,
                    g_defer=not args.no_defer, max_positions=total, device=dev, seed=rank)
    m.calibrate_gates()
    g = torch.Generator(device=dev)
    g.manual_seed(11 + rank)
    ids = torch.randint(0, shape.vocab, (B, P), generator=g, device=dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def sync_ms(fn):
        torch.cuda.synchronize()
        a, b = ev(), ev()
        a.record()
        r = fn()
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b), r

    # warm-up: a prefill and decode steps on a throw-away cache (profiling.py:351-362)
    c = SimpleNamespace()
    m.prefill(ids, c)
    for _ in range(Wu):
        m.decode_step(c)
    torch.cuda.synchronize()
    wgkv.check_errors()
    del c
    # attention / MLP / lm_head breakdown (profiling.py:251-344), eager, on its own cache
    c = SimpleNamespace()
    m.timers = {}
    m.prefill(ids, c)
    torch.cuda.synchronize()
    bd_prefill = m.breakdown()
    m.timers = {}
    for _ in range(8):
        m.decode_step(c)
    torch.cuda.synchronize()
    bd_decode = {k: v / 8 for k, v in m.breakdown().items()}
    m.timers = None
    del c
    torch.cuda.empty_cache()

    clk = ClockSampler(local_rank) if rank == 0 else None
    cache = SimpleNamespace()
    ttft, _ = sync_ms(lambda: m.prefill(ids, cache))
    for _ in range(2):  # steady state: first-use costs (allocator segments, module loads) stay untimed
        m.decode_step(cache)
    l0 = wgkv.lib.launches
    eager_ms, _ = sync_ms(lambda: [m.decode_step(cache) for _ in range(n_eager)])
    per_step_launches = (wgkv.lib.launches - l0) // n_eager
    dg = m.decode_graph(cache)  # one more real step, eager, then captured
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("wgkv_timed")
    graph_ms, _ = sync_ms(lambda: [dg.replay() for _ in range(K)])
    torch.cuda.nvtx.range_pop()
    clocks = clk.stop() if clk else None
    wgkv.check_errors()
    glen = cache.global_lengths.double().mean().item()
    D, Hk, Ly = shape.head_dim, shape.kv_heads, shape.layers
    kv_bytes = B * Ly * Hk * (glen + min(args.window, P)) * 2 * D * 2
    w_bytes = m.weight_bytes() - m.embed.numel() * 2
    tpot = max_over_ranks(graph_ms, dev) / K
    tpot_eager = max_over_ranks(eager_ms, dev) / n_eager
    ttft = max_over_ranks(ttft, dev)

    # end to end through the public API: each step's token ids come from pinned host memory (teacher
    # forcing) and each step's greedy token is read back to the host
    host_tok = torch.randint(0, shape.vocab, (K, B, 1), dtype=torch.int64).pin_memory()
    out_host = torch.empty(K, B, dtype=torch.int64, pin_memory=True)

    def e2e_run():
        for s in range(K):
            m.token.copy_(host_tok[s], non_blocking=True)
            dg.replay()
            out_host[s].copy_(m.token[:, 0], non_blocking=True)
    e2e_ms, _ = sync_ms(e2e_run)
    e2e_ms = max_over_ranks(e2e_ms, dev)
    wgkv.check_errors()
    peak, kind = peaks()
    achieved = (w_bytes + kv_bytes) / (tpot / 1e3) / 1e9
    if rank == 0:
        line = {
            "metric": f"decode tok/s, graph-replayed steps after a {P}-token prefill ({shape.name}, B={B})",
            "value": world * B / (tpot / 1e3), "unit": "tok/s", "n_gpus": world, "steps": K, "warmup": Wu,
            "ms_per_step": tpot, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic token ids; random-init weights",
            "config": {"workload": f"end-to-end decoder ({args.model}), TTFT + TPOT as scripts/profiling.py",
                       "model": shape.name, "batch": B, "prompt": P, "window": args.window, "page": 16,
                       "g_defer": not args.no_defer, "admit": "Beta(2,8) per head (calibrated gate bias)",
                       "l2": "weights + KV larger than L2 each step, no flush"},
            "ttft_ms": ttft, "prefill_tok_s": B * P / (ttft / 1e3), "tpot_ms_graph": tpot, "tpot_ms_eager": tpot_eager,
            "breakdown_ms": {"prefill": bd_prefill, "decode_step": bd_decode},
            "e2e": {"value": world * B * K / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": B * 8,
                    "d2h_bytes_per_step": B * 8},
            "roofline": {"bound": "hbm", "kernel": "whole decode step (weights + KV read)", "achieved": achieved,
                         "peak": peak, "peak_kind": kind, "unit": "GB/s", "frac": achieved / peak, "traffic": None,
                         "bytes_per_step": w_bytes + kv_bytes},
            "gpu_launches": per_step_launches * K, "clocks": clocks,
        }
        print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="wgkv", choices=["wgkv", "reference"])
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "qwen3_decode", "c5_decode", "model", "quest_decode"])
    ap.add_argument("--quest-budget", type=int, default=8192, help="quest_decode workload: tokens kept per head")
    ap.add_argument("--model", default="llama-3.2-1b", help="model workload: llama-3.2-1b | llama-3.1-8b | qwen3-4b")
    ap.add_argument("--prompt", type=int, default=32000, help="model workload: prompt length")
    ap.add_argument("--batch", type=int, default=1, help="model workload: sequences")
    ap.add_argument("--window", type=int, default=4096, help="model workload: local window")
    ap.add_argument("--no-defer", action="store_true", help="model workload: gate each token at decode")
    ap.add_argument("--small", action="store_true", help="reduced layer count for profiling captures")
    ap.add_argument("--no-prefill", action="store_true", help="skip the 400K prefill measurement of the default run")
    ap.add_argument("--no-extras", action="store_true", help="the default run without its C3/C4/C5 sub-records")
    args = ap.parse_args()
    global METRIC, WORKLOAD_NAME
    if args.workload == "qwen3_decode":
        CFG.clear()
        CFG.update(QWEN3_CFG)
        METRIC = QWEN3_METRIC
        WORKLOAD_NAME = QWEN3_NAME
    if args.small and args.workload != "prefill":
        CFG["layers"] = 2
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        reference_arm(args, rank, world)
        return
    if world > 1:
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "prefill":
            prefill_arm(args, rank, world, local_rank)
        elif args.workload == "c5_decode":
            c5_arm(args, rank, world, local_rank)
        elif args.workload == "model":
            model_arm(args, rank, world, local_rank)
        elif args.workload == "quest_decode":
            quest_arm(args, rank, world, local_rank)
        else:
            gpu_arm(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
