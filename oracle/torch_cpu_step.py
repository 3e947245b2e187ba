"""CPU baseline of the decode step: the reference's PyTorch operations, run on the host cores.

TEST / MEASUREMENT INFRASTRUCTURE ONLY.  Nothing in the product (``wg-kv_b200/``) imports
this file; ``bench.py`` times it as the CPU baseline and its ``--impl reference`` arm.

The reference (src/modeling_layers.py) is PyTorch; its decode step on a GPU runs Triton, but every
other statement is plain torch that runs unchanged on a CPU, and its own CPU stand-in for the
attention kernel is ``flash_attn_with_kvcache_ref`` (utils/test_flash_attn_with_kvcache.py:16-71:
per (sequence, KV head) the head's pages are gathered, then bf16 ``q @ k.T * scale``, softmax,
``@ v``).  This module restates that step with torch on the CPU, in the reference's dtype (bf16),
with a batch axis and the page gathers vectorised (one ``index_select`` per head instead of a Python
loop per page, so the baseline is not slowed by interpreter overhead the reference's GPU path does
not have):

* gate fast path, ``GatingPredictor.forward`` :185-196 (bf16 einsums, GELU, sigmoid) and
  ``g_scores > g_threshold`` :1465;
* lazy promotion at layer 0, ``migrate_local_kv_to_global`` :674-763 (nonzero over the ring slot,
  page allocation when a head's length is a multiple of the page size, K/V row copy, lengths);
* ring append and lengths, ``decode_wrapper`` :1390-1413, :1429-1436;
* paged attention with the semantics of ``flash_attn_with_kvcache_ref``.

Parity of these semantics is pinned elsewhere (``oracle/wgkv_oracle.py`` against reference-run
fixtures); this file exists to time the reference's kind of computation, not to check results.
"""
from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


class TorchCpuDecode:
    """``layers`` layers x ``batch`` sequences of the decode state, in host memory.

    ``glen`` (layers, batch, kv_heads) are the global lengths; the ring holds ``window`` tokens
    (full), page ids are a random permutation after the ring pages (as the GPU benchmark lays
    them out).  Pool contents are random bf16."""

    def __init__(self, layers, batch, kv_heads, q_heads, head_dim, window, page, glen, steps=8, seed=5,
                 inner=64, threshold=0.5, admit=0.2):
        self.Ly, self.B, self.Hk, self.Hq, self.D, self.W, self.T = layers, batch, kv_heads, q_heads, head_dim, window, page
        self.G = q_heads // kv_heads
        self.thr = threshold
        g = torch.Generator().manual_seed(seed)
        Ly, B, Hk, D, W, T = self.Ly, self.B, self.Hk, self.D, self.W, self.T
        glen = torch.as_tensor(np.asarray(glen), dtype=torch.int64)
        gpages = (glen + T - 1) // T
        self.lp = W // T
        ring_pages = Ly * B * Hk * self.lp
        spare = Ly * B * Hk * ((steps + T - 1) // T + 1)
        self.total_blocks = int(ring_pages + gpages.sum() + spare + 1)
        self.maxb = self.lp + int(gpages.max()) + (steps + T - 1) // T + 1
        rows = self.total_blocks * T
        # random bf16 pool: one random chunk tiled over the rows (the values do not change the cost)
        chunk = torch.randn(min(rows, 1 << 20), D, generator=g).to(torch.bfloat16)
        self.k = torch.empty(rows, D, dtype=torch.bfloat16)
        self.v = torch.empty(rows, D, dtype=torch.bfloat16)
        for r0 in range(0, rows, chunk.shape[0]):
            n = min(chunk.shape[0], rows - r0)
            self.k[r0:r0 + n] = chunk[:n]
            self.v[r0:r0 + n] = chunk.flip(0)[:n]
        self.block_table = torch.full((Ly, B, Hk, self.maxb), self.total_blocks - 1, dtype=torch.int32)
        self.block_table[..., :self.lp] = torch.arange(ring_pages, dtype=torch.int32).view(Ly, B, Hk, self.lp)
        n_g = int(gpages.sum())
        perm = torch.randperm(n_g, generator=g).to(torch.int32) + ring_pages
        off = 0
        flat = self.block_table.view(-1, self.maxb)
        for i, n in enumerate(gpages.view(-1).tolist()):
            flat[i, self.lp:self.lp + n] = perm[off:off + n]
            off += n
        self.global_lengths = glen.to(torch.int32).clone()
        self.local_is_global = torch.rand(Ly, B, Hk, W, generator=g) < admit
        self.next_free_block = ring_pages + n_g
        self.local_ptr = 0
        # ring rows of (layer, b, h) start here (the reference's local_region_starts, :1264-1284)
        self.ring_start = (torch.arange(Ly * B * Hk, dtype=torch.int64) * W).view(Ly, B, Hk)
        # gate: pre_k -> inner -> 1, GELU, random weights on the bf16 grid
        bound1, bound2 = 1 / math.sqrt(D), 1 / math.sqrt(inner)
        self.w1 = ((torch.rand(Ly, Hk, inner, D, generator=g) * 2 - 1) * bound1).to(torch.bfloat16)
        self.b1 = ((torch.rand(Ly, Hk, inner, generator=g) * 2 - 1) * bound1).to(torch.bfloat16)
        self.w2 = ((torch.rand(Ly, Hk, inner, generator=g) * 2 - 1) * bound2).to(torch.bfloat16)
        self.b2 = torch.zeros(Ly, Hk, dtype=torch.bfloat16)
        self.scale = D ** -0.5

    # -- one decode step ----------------------------------------------------------------------
    def _gate(self, l, pre_k):
        """pre_k (B, Hk, D) bf16 -> admission bits (B, Hk): the fast path's bf16 einsums."""
        h = torch.einsum("bhi,hji->bhj", pre_k, self.w1[l]) + self.b1[l]
        h = F.gelu(h)
        o = torch.einsum("bhj,hj->bh", h, self.w2[l]) + self.b2[l]
        return torch.sigmoid(o) > self.thr

    def _promote(self):
        """Every (layer, b, h) whose ring slot at local_ptr is admitted moves that token to its pages."""
        p = self.local_ptr
        lidx, bidx, hidx = torch.nonzero(self.local_is_global[:, :, :, p], as_tuple=True)
        if lidx.numel() == 0:
            return
        gl = self.global_lengths[lidx, bidx, hidx].to(torch.int64)
        blk = self.lp + gl // self.T
        off = gl % self.T
        new = off == 0
        n_new = int(new.sum())
        if n_new:
            ids = torch.arange(self.next_free_block, self.next_free_block + n_new, dtype=torch.int32)
            self.block_table[lidx[new], bidx[new], hidx[new], blk[new]] = ids
            self.next_free_block += n_new
        phys = self.block_table[lidx, bidx, hidx, blk].to(torch.int64)
        dst = phys * self.T + off
        src = self.ring_start[lidx, bidx, hidx] + p
        self.k[dst] = self.k[src]
        self.v[dst] = self.v[src]
        self.global_lengths[lidx, bidx, hidx] += 1

    def _attention(self, l, q):
        """q (B, Hq, D) bf16 -> (B, Hq, D): per (b, h) gather of the ring + global pages, then the
        bf16 matmul / softmax / matmul of flash_attn_with_kvcache_ref."""
        out = torch.empty_like(q)
        T, G = self.T, self.G
        ar = torch.arange(T, dtype=torch.int64)
        for b in range(self.B):
            for h in range(self.Hk):
                n = self.W + int(self.global_lengths[l, b, h])
                pages = self.block_table[l, b, h, :(n + T - 1) // T].to(torch.int64)
                rows = (pages[:, None] * T + ar[None]).reshape(-1)[:n]
                kk = self.k.index_select(0, rows)
                vv = self.v.index_select(0, rows)
                s = (q[b, h * G:(h + 1) * G] @ kk.T) * self.scale
                out[b, h * G:(h + 1) * G] = F.softmax(s, dim=-1) @ vv
        return out

    def step(self, q, k_new, v_new, pre_k):
        """q (Ly, B, Hq, D), k_new / v_new / pre_k (Ly, B, Hk, D) bf16.  The ring is full, so the new
        token goes to slot local_ptr after that slot's old token was promoted (or dropped)."""
        self._promote()
        p = self.local_ptr
        outs = []
        for l in range(self.Ly):
            admit = self._gate(l, pre_k[l])
            rows = self.ring_start[l] + p
            self.k[rows.view(-1)] = k_new[l].reshape(-1, self.D)
            self.v[rows.view(-1)] = v_new[l].reshape(-1, self.D)
            self.local_is_global[l, :, :, p] = admit
            outs.append(self._attention(l, q[l]))
        self.local_ptr = (p + 1) % self.W
        return outs
