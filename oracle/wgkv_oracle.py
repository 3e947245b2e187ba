"""CPU oracle for the WG-KV admission hot path -- TEST INFRASTRUCTURE ONLY.

This module restates, in numpy, the algorithm of the reference's hot path
(EMCLab-Sinica/WG-KV, ``src/modeling_layers.py``) so that the CUDA kernels of
``wg-kv_b200`` can be checked against it.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import it; the product path never does.

Parity pin: the restatement is checked against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference's own Python
code (``src/modeling_layers.py`` imported unmodified, on CPU) and the
reference's own test oracles (``utils/test_flash_attn_with_kvcache.py:16-71``,
``utils/test_sparse_attn.py:34-93``).  ``tests/test_oracle_golden.py`` does the
check -- including QUEST page selection (``quest_select_blocks`` :452-576) and
SnapKV eviction (``snapkv_evict`` :595-671), whose fixtures record what the
reference selected / evicted (equal up to the order of tied scores, which
``torch.topk`` leaves unspecified; the restatement takes the lower positions).

Layout conventions (batch generalisation of the reference, identical to it
for batch 1):

* pool ``k/v``: ``(total_blocks * T, D)`` bf16 rows; page ``p`` = rows
  ``[p*T, (p+1)*T)`` (reference ``:1209-1216``).
* ring region of (layer l, batch b, kv head h): rows
  ``((l*B + b)*Hk + h) * W + slot`` (reference ``:1282-1284`` with B=1).
* ``block_table``: ``(Lyr, B, Hk, maxb)`` int32; entries ``[0, W/T)`` are the
  ring pages, entries from ``W/T`` on are global pages, unused entries hold
  the sentinel ``total_blocks - 1`` (reference ``:1204-1208``, ``:1264-1271``).
* ``global_lengths``: ``(Lyr, B, Hk)``; ``local_is_global``: ``(Lyr, B, Hk, W)``.

bf16 arithmetic is emulated by rounding float32 values to nearest-even
bfloat16 at the same operation boundaries the reference's bf16 tensors round
at.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

try:  # scipy is in the image; the pure-python fallback keeps the oracle usable without it
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    _erf = np.vectorize(math.erf)


# ----------------------------------------------------------------------------
# bf16 helpers
# ----------------------------------------------------------------------------

def bf16(x) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even); returns float32."""
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    u = a.view(np.uint32)
    r = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    out = ((u + r) & np.uint32(0xFFFF0000)).astype(np.uint32)
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.uint32(0x7FC00000)
    return out.view(np.float32)


def bf16_bits(x) -> np.ndarray:
    """bfloat16 bit patterns (uint16) of float32 values already on the bf16 grid."""
    return (bf16(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def from_bf16_bits(bits) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def randn_bf16(rng: np.random.Generator, shape) -> np.ndarray:
    """Seeded N(0,1) values rounded to bf16 (float32 array on the bf16 grid)."""
    return bf16(rng.standard_normal(shape, dtype=np.float32))


# ----------------------------------------------------------------------------
# (a1, a2) write gate -- GatingPredictor fast path, modeling_layers.py:170-196
# ----------------------------------------------------------------------------

@dataclass
class GateParams:
    """Per-layer gate parameters, float32 arrays on the bf16 grid.

    w1 ``(Hk, inner, input_dim)`` = ``conv1.weight.view(Hk, -1, input_dim)``
    (``:185``); b1 ``(Hk, inner)``; w2 ``(Hk, inner)`` = ``conv2.weight``
    (``:190``); b2 ``(Hk,)``; norms ``{name: (D,)}`` for the RMS-normed inputs
    (``:144-146``).
    """
    w1: np.ndarray
    b1: np.ndarray
    w2: np.ndarray
    b2: np.ndarray
    inputs: tuple = ("pre_k",)
    act: str = "gelu"
    rms: bool = False
    rms_eps: float = 1e-6
    norms: dict = field(default_factory=dict)
    fast_path: bool = True   # g_fast_path (configuration_llama.py:207 defaults to False)
    epsilon: float = 0.0     # g_epsilon: score floor of the conv path (:205)


def _rms_norm_bf16(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """GatingRMSNorm.forward (modeling_layers.py:123-128) on bf16 input."""
    x32 = x.astype(np.float32)
    var = np.mean(x32 * x32, axis=-1, keepdims=True, dtype=np.float32)
    y = bf16(x32 * (1.0 / np.sqrt(var + np.float32(eps))).astype(np.float32))
    return bf16(weight.astype(np.float32) * y)


def _act(x: np.ndarray, kind: str) -> np.ndarray:
    x64 = x.astype(np.float64)
    if kind == "silu":
        y = x64 / (1.0 + np.exp(-x64))
    else:  # nn.GELU() default: exact erf form
        y = 0.5 * x64 * (1.0 + _erf(x64 / math.sqrt(2.0)))
    return bf16(y.astype(np.float32))


def _gate_states(p: GateParams, pre_key, post_key, value) -> np.ndarray:
    """Concatenation of the selected (optionally RMS-normed) inputs, modeling_layers.py:172-183."""
    src = {"pre_k": pre_key, "post_k": post_key, "v": value}
    parts = []
    for name in p.inputs:
        x = src[name].astype(np.float32)
        if p.rms:
            x = _rms_norm_bf16(x, p.norms[name], p.rms_eps)
        parts.append(x)
    return np.concatenate(parts, axis=-1)  # (B, Hk, L, I)


def gate_logits_nobias(p: GateParams, pre_key=None, post_key=None, value=None) -> np.ndarray:
    """``einsum(act(einsum(x, w1) + b1), w2)`` rounded to bf16, before ``+ b2``.

    Follows modeling_layers.py:172-190 (fast path): concat of the selected
    inputs (``:173-183``), einsum ``'bhli,hji->bhlj'`` with fp32 accumulation
    rounded to bf16, ``+ b1`` (bf16), activation (bf16), einsum with w2
    (bf16).  Inputs are ``(B, Hk, L, D)``; returns ``(B, Hk, L)``.
    """
    states = _gate_states(p, pre_key, post_key, value)
    h = np.matmul(states, np.swapaxes(p.w1.astype(np.float32), -1, -2)[None])
    h = bf16(h)
    h = bf16(h + p.b1[None, :, None, :])
    h = _act(h, p.act)
    return bf16(np.matmul(h, p.w2.astype(np.float32)[None, :, :, None])[..., 0])


def gate_finish(o: np.ndarray, b2: np.ndarray) -> np.ndarray:
    """``sigmoid(o + b2)`` with bf16 rounding after the add and the sigmoid
    (modeling_layers.py:190-193)."""
    o = bf16(o + b2[None, :, None])
    s = 1.0 / (1.0 + np.exp(-o.astype(np.float64)))
    return bf16(s.astype(np.float32))


def gate_scores_conv(p: GateParams, pre_key=None, post_key=None, value=None) -> np.ndarray:
    """The reference's default gate path (``g_fast_path=False``, modeling_layers.py:198-205):
    grouped 1x1 ``conv1`` (fp32 accumulation with the bias, one bf16 rounding), activation (bf16),
    ``conv2`` (fp32 accumulation with the bias, one rounding), sigmoid (bf16), then
    ``torch.clamp(min=g_epsilon)``, whose floor is ``g_epsilon`` rounded to bf16."""
    states = _gate_states(p, pre_key, post_key, value)
    h = np.matmul(states, np.swapaxes(p.w1.astype(np.float32), -1, -2)[None])
    h = bf16((h + p.b1[None, :, None, :]).astype(np.float32))
    h = _act(h, p.act)
    o = np.matmul(h, p.w2.astype(np.float32)[None, :, :, None])[..., 0]
    o = bf16((o + p.b2[None, :, None]).astype(np.float32))
    s = bf16((1.0 / (1.0 + np.exp(-o.astype(np.float64)))).astype(np.float32))
    floor = bf16(np.float32(p.epsilon))
    return np.where(s < floor, floor, s).astype(np.float32)


def gate_scores(p: GateParams, pre_key=None, post_key=None, value=None) -> np.ndarray:
    """g = sigmoid(w2 . act(w1 . x + b1) + b2) per (b, h, t), bf16 at op boundaries
    (GatingPredictor.forward, modeling_layers.py:170-205: the einsum fast path, or the conv
    path when ``p.fast_path`` is False).  Returns ``(B, Hk, L)`` float32 on the bf16 grid."""
    if not p.fast_path:
        return gate_scores_conv(p, pre_key, post_key, value)
    return gate_finish(gate_logits_nobias(p, pre_key, post_key, value), p.b2)


def admission_mask(scores: np.ndarray, threshold: float) -> np.ndarray:
    """``g_mask = g_scores > g_threshold`` (modeling_layers.py:1465).

    The comparison is done as torch does it for a bf16 tensor against a
    Python float: in float32 after widening the bf16 score.
    """
    return scores.astype(np.float32) > np.float32(threshold)


# ----------------------------------------------------------------------------
# (a9-a11) vertical-slash sparse indices
# ----------------------------------------------------------------------------

def generate_block_offset(W: int, L: int, block: int = 64):
    """modeling_layers.py:321-349 (local band, shared by all heads)."""
    R = (L + block - 1) // block
    P = min(W // block, R)
    maxb = P + 1
    bc = np.zeros((1, 1, R), np.int32)
    bo = np.zeros((1, 1, R, maxb), np.int32)
    bc[0, 0, :P] = np.arange(1, P + 1)
    bc[0, 0, P:] = P + 1
    if P:
        bo[0, 0, :P, :P] = np.arange(0, block * P, block)[None, :]
    rows = np.arange(R - P)[:, None]
    cols = np.arange(maxb)[None, :]
    bo[0, 0, P:] = 1 + (rows + cols) * block
    s_last = (R - 1) * block
    start = max(0, s_last - W + 1)
    bc[0, 0, -1] = len(range(start, L, block))
    return bc, bo


def generate_column_index(g_mask: np.ndarray, W: int, L: int, block: int = 64):
    """modeling_layers.py:352-381.  Returns column_count (B,Hk,R) and
    column_index (B,Hk,1,Gmax) where Gmax = max admitted count (``:369``)."""
    B, Hk, _ = g_mask.shape
    R = (L + block - 1) // block
    P = min(W // block, R)
    nch = (L - 1) // block
    trimmed = g_mask[:, :, 1:1 + nch * block].reshape(B, Hk, nch, block).sum(axis=3)
    sums = np.concatenate([g_mask[:, :, :1].astype(np.int64), trimmed], axis=2)
    cums = np.cumsum(sums, axis=2)
    gmax = int(cums[:, :, -1].max()) if cums.size else 0
    cc = np.zeros((B, Hk, R), np.int32)
    cc[:, :, P:] = cums[:, :, :R - P]
    ci = np.zeros((B, Hk, 1, gmax), np.int32)
    for b in range(B):
        for h in range(Hk):
            nz = np.flatnonzero(g_mask[b, h])[:gmax]
            ci[b, h, 0, :nz.size] = nz
    return cc, ci


def generate_sparse_indices(g_mask: np.ndarray, W: int, L: int, block: int = 64):
    """modeling_layers.py:385-409 (asserts W % block == 0, ``:394``)."""
    assert W % block == 0
    bc, bo = generate_block_offset(W, L, block)
    cc, ci = generate_column_index(g_mask, W, L, block)
    return bc, bo, cc, ci


def generate_sparse_indices_ref(g_mask: np.ndarray, W: int, L: int, block: int = 64):
    """Loop reference, modeling_layers.py:274-318."""
    B, Hk, _ = g_mask.shape
    R = (L + block - 1) // block
    maxb = (W + block - 1 + block - 1) // block
    gmax = int(g_mask.sum(axis=2).max()) if g_mask.size else 0
    bc = np.zeros((1, 1, R), np.int32)
    bo = np.zeros((1, 1, R, maxb), np.int32)
    cc = np.zeros((B, Hk, R), np.int32)
    ci = np.zeros((B, Hk, 1, gmax), np.int32)
    for i in range(R):
        s = i * block
        st = max(0, s - W + 1)
        en = min(s + block, L)
        idx = np.arange(st, en, block, dtype=np.int32)
        bc[0, 0, i] = idx.size
        bo[0, 0, i, :idx.size] = idx
    for b in range(B):
        for h in range(Hk):
            nz = np.flatnonzero(g_mask[b, h])
            ci[b, h, 0, :nz.size] = nz
            for i in range(R):
                st = max(0, i * block - W + 1)
                cc[b, h, i] = int((nz < st).sum())
    return bc, bo, cc, ci


def indices_equal(a, b) -> bool:
    """Comparison rules of utils/test_sparse_indices.py:30-46 (prefix-exact)."""
    bc, bo, cc, ci = a
    bcr, bor, ccr, cir = b
    if not np.array_equal(bc, bcr) or not np.array_equal(cc, ccr):
        return False
    R = bcr.shape[2]
    for i in range(R):
        n = int(bcr[0, 0, i])
        if not np.array_equal(bo[0, 0, i, :n], bor[0, 0, i, :n]):
            return False
    B, Hk = ccr.shape[:2]
    for b in range(B):
        for h in range(Hk):
            n = int(ccr[b, h].max()) if R else 0
            if not np.array_equal(ci[b, h, 0, :n], cir[b, h, 0, :n]):
                return False
    return True


def sparse_mask_from_indices(bc, bo, cc, ci, L: int, G: int, rows=None, block: int = 64):
    """Dense boolean mask implied by the indices, per KV head (B, Hk, |rows|, L).

    utils/test_sparse_attn.py:34-58 (band blocks + admitted columns, then the
    causal mask).  ``rows`` selects query rows (default all)."""
    B, Hk, _ = cc.shape
    rows = np.arange(L) if rows is None else np.asarray(rows)
    m = np.zeros((B, Hk, rows.size, L), bool)
    for r_i, q in enumerate(rows):
        i = q // block
        for c in range(int(bc[0, 0, i])):
            st = int(bo[0, 0, i, c])
            m[:, :, r_i, st:min(st + block, L)] = True
        for b in range(B):
            for h in range(Hk):
                n = int(cc[b, h, i])
                m[b, h, r_i, ci[b, h, 0, :n]] = True
        m[:, :, r_i, q + 1:] = False
    return m


def ideal_mask(g_mask: np.ndarray, W: int, L: int, rows=None, block: int = 64):
    """utils/test_sparse_attn.py:78-88: admitted columns or per-row-block band
    ``[start_row - W + 1, end_row)``, intersected with causal."""
    B, Hk, _ = g_mask.shape
    rows = np.arange(L) if rows is None else np.asarray(rows)
    m = np.repeat(g_mask[:, :, None, :], rows.size, axis=2).copy()
    for r_i, q in enumerate(rows):
        s = (q // block) * block
        e = min(s + block, L)
        m[:, :, r_i, max(0, s - W + 1):e] = True
        m[:, :, r_i, q + 1:] = False
    return m


def masked_attention(q, k, v, mask, scale=None, rows=None):
    """Reference value of the sparse prefill output: fp64 softmax attention
    under ``mask`` (utils/test_sparse_attn.py:60-62).

    q ``(B, L, Hq, D)``, k/v ``(B, L, Hk, D)``, mask ``(B, Hk, |rows|, L)``.
    Returns ``(B, |rows|, Hq, D)`` float64.  Rows with an empty mask give 0.
    """
    B, L, Hq, D = q.shape
    Hk = k.shape[2]
    G = Hq // Hk
    scale = D ** -0.5 if scale is None else scale
    rows = np.arange(L) if rows is None else np.asarray(rows)
    out = np.zeros((B, rows.size, Hq, D), np.float64)
    for b in range(B):
        for hq in range(Hq):
            h = hq // G
            qq = q[b, rows, hq].astype(np.float64)
            s = qq @ k[b, :, h].astype(np.float64).T * scale
            mk = mask[b, h]
            s = np.where(mk, s, -np.inf)
            mx = s.max(axis=1, keepdims=True)
            mx = np.where(np.isfinite(mx), mx, 0.0)
            e = np.where(mk, np.exp(s - mx), 0.0)
            den = e.sum(axis=1, keepdims=True)
            den = np.where(den > 0, den, 1.0)
            out[b, :, hq] = (e / den) @ v[b, :, h].astype(np.float64)
    return out


# ----------------------------------------------------------------------------
# (a7, a8) ragged paged decode attention
# ----------------------------------------------------------------------------

def paged_decode(q, k_cache, v_cache, cache_seqlens, block_table, scale):
    """Decode attention over per-(b, kv-head) page tables.

    Semantics of ``flash_attn_with_kvcache_ref`` (utils/test_flash_attn_with_kvcache.py:16-71)
    computed in float64: q ``(B, 1, Hq, D)``, caches ``(NB, T, D)``,
    cache_seqlens ``(B, Hk)``, block_table ``(B, Hk, maxb)``; GQA maps query
    head ``hq`` to kv head ``hq // G``.  A head with length 0 yields 0 (the
    guard of modeling_layers.py:997-999).  Returns ``(B, 1, Hq, D)`` float64.
    """
    B, _, Hq, D = q.shape
    T = k_cache.shape[1]
    Hk = cache_seqlens.shape[1]
    G = Hq // Hk
    out = np.zeros((B, 1, Hq, D), np.float64)
    for b in range(B):
        for h in range(Hk):
            n = int(cache_seqlens[b, h])
            if n <= 0:
                continue
            nb = (n + T - 1) // T
            pages = block_table[b, h, :nb].astype(np.int64)
            kk = k_cache[pages].reshape(-1, D)[:n].astype(np.float64)
            vv = v_cache[pages].reshape(-1, D)[:n].astype(np.float64)
            qq = q[b, 0, h * G:(h + 1) * G].astype(np.float64)
            s = qq @ kk.T * scale
            s -= s.max(axis=1, keepdims=True)
            e = np.exp(s)
            out[b, 0, h * G:(h + 1) * G] = (e / e.sum(axis=1, keepdims=True)) @ vv
    return out


# ----------------------------------------------------------------------------
# (a3-a6) paged pool state: prefill admission, lazy promotion, ring append
# ----------------------------------------------------------------------------

class PoolError(AssertionError):
    """Capacity violation (the reference's asserts at :1313-1321, :683-686, :702-704)."""


@dataclass
class PoolState:
    """Mirror of the attributes prefill_wrapper attaches to the cache
    (modeling_layers.py:1196-1288), with a batch axis."""
    layers: int
    batch: int
    kv_heads: int
    head_dim: int
    window: int
    page: int
    max_total_tokens: int
    max_tokens_per_head: int
    defer: bool = False
    quest: bool = False
    snapkv: tuple | None = None  # (max_cached_tokens, evict_ratio, window, kernel_size)
    q_heads: int = 0             # needed with snapkv (query buffer)

    def __post_init__(self):
        assert self.window % self.page == 0
        self.local_pages = self.window // self.page
        self.total_blocks = (self.max_total_tokens + self.page - 1) // self.page
        self.max_blocks_per_head = (self.max_tokens_per_head + self.page - 1) // self.page
        Ly, B, Hk = self.layers, self.batch, self.kv_heads
        self.block_table = np.full((Ly, B, Hk, self.max_blocks_per_head), self.total_blocks - 1, np.int32)
        lp = np.arange(Ly * B * Hk * self.local_pages, dtype=np.int32).reshape(Ly, B, Hk, self.local_pages)
        self.block_table[..., :self.local_pages] = lp
        self.k = np.zeros((self.total_blocks * self.page, self.head_dim), np.float32)
        self.v = np.zeros_like(self.k)
        self.local_is_global = np.zeros((Ly, B, Hk, self.window), bool)
        self.global_lengths = np.zeros((Ly, B, Hk), np.int32)
        self.local_pre_key = np.zeros((Ly, B, Hk, self.window, self.head_dim), np.float32) if self.defer else None
        self.local_ptr = 0
        self.local_length = 0
        self.next_free_block = Ly * B * Hk * self.local_pages
        if self.snapkv is not None:  # modeling_layers.py:1249-1262, with a batch axis
            win = self.snapkv[2]
            self.snap_q = np.zeros((Ly, B, win, self.q_heads, self.head_dim), np.float32)
            self.snap_len = 0
            self.snap_ptr = 0
            self.evict_count = 0
            self.free = []
        if self.quest:  # per-page key bounds (quest_block_key_min / _max, modeling_layers.py:1232-1240)
            self.qmin = np.zeros((self.total_blocks, self.head_dim), np.float32)
            self.qmax = np.zeros((self.total_blocks, self.head_dim), np.float32)

    def ring_row(self, l, b, h, slot):
        return ((l * self.batch + b) * self.kv_heads + h) * self.window + slot

    # -- prefill_wrapper parts 1-2 (modeling_layers.py:1290-1331) -------------
    def prefill_layer(self, l, k, v, g_mask, pre_key=None):
        """k/v ``(B, Hk, L, D)``, g_mask ``(B, Hk, L)`` bool."""
        B, Hk, L, _ = k.shape
        W, T = self.window, self.page
        n_loc = min(L, W)
        for b in range(B):
            for h in range(Hk):
                r0 = self.ring_row(l, b, h, 0)
                self.k[r0:r0 + n_loc] = k[b, h, L - n_loc:]
                self.v[r0:r0 + n_loc] = v[b, h, L - n_loc:]
                self.local_is_global[l, b, h, :n_loc] = g_mask[b, h, L - n_loc:]
                if self.defer and pre_key is not None:
                    self.local_pre_key[l, b, h, :n_loc] = pre_key[b, h, L - n_loc:]
        self.local_length = n_loc
        n_early = L - W
        if n_early <= 0:
            return
        for b in range(B):
            for h in range(Hk):
                idx = np.flatnonzero(g_mask[b, h, :n_early])
                n = idx.size
                if n == 0:
                    continue
                if n_loc + n > self.max_tokens_per_head:
                    raise PoolError(f"layer {l} head {h}: {n_loc + n} tokens exceed max_tokens_per_head")
                need = (n + T - 1) // T
                first = self.next_free_block
                if first + need > self.total_blocks:
                    raise PoolError(f"layer {l} head {h}: pool exhausted")
                self.block_table[l, b, h, self.local_pages:self.local_pages + need] = np.arange(first, first + need)
                self.k[first * T:first * T + n] = k[b, h, idx]
                self.v[first * T:first * T + n] = v[b, h, idx]
                self.global_lengths[l, b, h] = n
                self.next_free_block += need
                if self.quest:  # key bounds of every new page (:1333-1347)
                    for pg in range(need):
                        rows = self.k[(first + pg) * T:(first + pg) * T + min(T, n - pg * T)]
                        self.qmin[first + pg] = rows.min(axis=0)
                        self.qmax[first + pg] = rows.max(axis=0)

    # -- migrate_local_kv_to_global (modeling_layers.py:674-763) --------------
    def promote(self):
        ptr = self.local_ptr
        flat = np.argwhere(self.local_is_global[:, :, :, ptr])  # (l, b, h) row-major
        if flat.size == 0:
            return
        T = self.page
        glen = self.global_lengths[flat[:, 0], flat[:, 1], flat[:, 2]]
        if np.any(self.window + glen + 1 > self.max_tokens_per_head):
            raise PoolError("Tokens exceed max_tokens_per_head")
        gblk = self.local_pages + glen // T
        off = glen % T
        need = off == 0
        nnew = int(need.sum())
        if nnew:
            nff = min(nnew, len(self.free)) if self.snapkv is not None else 0
            ids = self.free[len(self.free) - nff:] if nff else []  # :694-709: the free list's tail first
            if nff:
                self.free = self.free[:len(self.free) - nff]
            if self.next_free_block + nnew - nff > self.total_blocks:
                raise PoolError("Allocation exceeds total_blocks")
            ids = list(ids) + list(range(self.next_free_block, self.next_free_block + nnew - nff))
            sel = flat[need]
            self.block_table[sel[:, 0], sel[:, 1], sel[:, 2], gblk[need]] = np.array(ids, np.int32)
            self.next_free_block += nnew - nff
        src = np.array([self.ring_row(l, b, h, ptr) for l, b, h in flat])
        phys = self.block_table[flat[:, 0], flat[:, 1], flat[:, 2], gblk].astype(np.int64)
        dst = phys * T + off
        self.k[dst] = self.k[src]
        self.v[dst] = self.v[src]
        if self.quest:  # :744-761: a new page starts at the key, else min / max with it
            kk = self.k[src]
            self.qmin[phys] = np.where(need[:, None], kk, np.minimum(self.qmin[phys], kk))
            self.qmax[phys] = np.where(need[:, None], kk, np.maximum(self.qmax[phys], kk))
        self.global_lengths[flat[:, 0], flat[:, 1], flat[:, 2]] = glen + 1

    # -- decode_wrapper state part (modeling_layers.py:1390-1413) -------------
    def append_layer(self, l, k_new, v_new, g_mask_new=None, pre_key_new=None, gate_fn=None, threshold=None):
        """k_new/v_new ``(B, Hk, D)``; g_mask_new ``(B, Hk)`` or None (deferred
        gating: ``gate_fn(pre_k, post_k, v) -> scores`` re-scores the ring when
        the last slot is written, ``refresh_local_is_global`` :1169-1180)."""
        W = self.window
        if self.local_length < W:
            ins = self.local_length
            cur = self.local_length + 1
        else:
            ins = self.local_ptr
            cur = W
        B, Hk = self.batch, self.kv_heads
        for b in range(B):
            for h in range(Hk):
                r = self.ring_row(l, b, h, ins)
                self.k[r] = k_new[b, h]
                self.v[r] = v_new[b, h]
        if g_mask_new is None:
            self.local_pre_key[l, :, :, ins] = pre_key_new
            if ins == W - 1:
                rows = np.array([[self.ring_row(l, b, h, 0) for h in range(Hk)] for b in range(B)])
                ring_k = np.stack([[self.k[rows[b, h]:rows[b, h] + W] for h in range(Hk)] for b in range(B)])
                ring_v = np.stack([[self.v[rows[b, h]:rows[b, h] + W] for h in range(Hk)] for b in range(B)])
                scores = gate_fn(self.local_pre_key[l], ring_k, ring_v)
                self.local_is_global[l] = admission_mask(scores, threshold)
        else:
            self.local_is_global[l, :, :, ins] = g_mask_new
        if l == self.layers - 1:
            if self.local_length < W:
                self.local_length = cur
            else:
                self.local_ptr = (self.local_ptr + 1) % W
        return cur

    def decode_tables(self, l, cur_local_len):
        """``cache_seqlens``/``block_table`` views of modeling_layers.py:1429-1436."""
        return (cur_local_len + self.global_lengths[l]).astype(np.int32), self.block_table[l]

    # -- SnapKV (modeling_layers.py:579-671) ------------------------------------------------------
    def snap_record(self, l, q):
        """snapkv_record_queries (:579-592): q ``(B, Hq, Lq, D)`` (post-RoPE queries of layer l)."""
        win = self.snapkv[2]
        Lq = q.shape[2]
        if Lq > 1:
            take = min(win, Lq)
            self.snap_q[l, :, :take] = np.transpose(q[:, :, Lq - take:], (0, 2, 1, 3))
            if l == self.layers - 1:
                self.snap_len = take
                self.snap_ptr = take % win
        else:
            self.snap_q[l, :, self.snap_ptr] = q[:, :, 0]
            if l == self.layers - 1:
                self.snap_len = min(win, self.snap_len + 1)
                self.snap_ptr = (self.snap_ptr + 1) % win

    def snap_should_evict(self):
        """The trigger of :1500-1507 (checked after the last layer)."""
        return int(self.global_lengths.sum()) > self.snapkv[0]

    def snap_scores(self, l, b, h, scale):
        """head_scores of snapkv_evict (:611-625): softmax over the head's global keys of each window
        query (scores rounded to bf16, then scaled in bf16), max over the group, mean over the
        window, max-pooled with the odd kernel (padding kernel // 2)."""
        T, win, ks = self.page, self.snapkv[2], self.snapkv[3]
        glen = int(self.global_lengths[l, b, h])
        G = self.q_heads // self.kv_heads
        q = self.snap_q[l, b][:, h * G:(h + 1) * G]                         # (win, G, D)
        pos = np.arange(glen)
        rows = self.block_table[l, b, h, self.local_pages + pos // T].astype(np.int64) * T + pos % T
        keys = self.k[rows]                                                   # (glen, D)
        att = bf16(bf16((np.transpose(q, (1, 0, 2)).astype(np.float64) @ keys.T.astype(np.float64)).astype(np.float32))
                   * np.float32(scale))                                       # (G, win, glen)
        att = att - att.max(-1, keepdims=True)
        e = np.exp(att.astype(np.float64))
        p = (e / e.sum(-1, keepdims=True)).astype(np.float32)
        sc = p.max(0).astype(np.float64).mean(0).astype(np.float32)          # (glen,)
        pad = ks // 2
        padded = np.concatenate([np.full(pad, -np.inf, np.float32), sc, np.full(pad, -np.inf, np.float32)])
        return np.lib.stride_tricks.sliding_window_view(padded, ks).max(-1).astype(np.float32)

    def snap_evict(self, scale, override=None):
        """snapkv_evict (:595-671) for every (layer, b, h).  The num_evict lowest-scored global tokens
        go, ties to the lower positions (the reference's torch.topk leaves their order open);
        ``override[(l, b, h)]`` = positions to evict instead.  Kept tokens are packed to the front of
        the head's pages, freed pages go to the free list in (layer, b, h) order."""
        T, ratio = self.page, self.snapkv[1]
        self.evict_count += 1
        for l in range(self.layers):
            for b in range(self.batch):
                for h in range(self.kv_heads):
                    glen = int(self.global_lengths[l, b, h])
                    n_ev = int(glen * ratio)
                    if n_ev == 0:
                        continue
                    if override is not None:
                        ev = np.asarray(override[(l, b, h)])
                    else:
                        sc = self.snap_scores(l, b, h, scale)
                        ev = np.lexsort((np.arange(glen), sc.astype(np.float64)))[:n_ev]
                    keep = np.setdiff1d(np.arange(glen), ev)
                    nb_old = (glen + T - 1) // T
                    nb_new = (len(keep) + T - 1) // T
                    tab = self.block_table[l, b, h, self.local_pages:self.local_pages + nb_old].astype(np.int64)
                    rows = tab[np.arange(glen) // T] * T + np.arange(glen) % T
                    if len(keep):
                        kk, vv = self.k[rows[keep]].copy(), self.v[rows[keep]].copy()
                        self.k[rows[:len(keep)]] = kk
                        self.v[rows[:len(keep)]] = vv
                    if nb_new < nb_old:
                        self.free.extend(int(x) for x in tab[nb_new:])
                        self.block_table[l, b, h, self.local_pages + nb_new:self.local_pages + nb_old] = \
                            self.total_blocks - 1
                    self.global_lengths[l, b, h] = len(keep)

    def quest_scores(self, l, b, h, q):
        """Block scores of quest_select_blocks (:495-504) for the head's full and partial global pages:
        max over the G query heads of bf16(sum_d bf16(q_d * (q_d >= 0 ? kmax_d : kmin_d))).
        q ``(G, D)`` (bf16 values); returns float32 scores (bf16 values), one per global page."""
        T = self.page
        glen = int(self.global_lengths[l, b, h])
        nb = (glen + T - 1) // T
        pages = self.block_table[l, b, h, self.local_pages:self.local_pages + nb].astype(np.int64)
        sel = np.where(q[:, None, :] >= 0, self.qmax[pages][None], self.qmin[pages][None])  # (G, nb, D)
        prod = bf16(q[:, None, :].astype(np.float32) * sel)
        sc = bf16(prod.astype(np.float64).sum(-1).astype(np.float32))
        return sc.max(axis=0) if nb else np.zeros(0, np.float32)

    def quest_select(self, l, cur_local_len, q, token_budget):
        """quest_select_blocks (modeling_layers.py:452-576) for every (b, h) of layer l.

        q ``(B, Hq, D)``.  Returns (cache_seqlens ``(B, Hk)`` int32, list over (b, h) of the selected
        page ids: ring pages, then the chosen full global pages in ascending position, then the
        trailing partial page).  The reference lists the full pages in torch.topk order; the set is
        what attention depends on.  Ties at the k-th score go to the lowest position (torch.topk
        leaves their order unspecified)."""
        T = self.page
        B, Hk = self.batch, self.kv_heads
        G = q.shape[1] // Hk
        local_blocks = (cur_local_len + T - 1) // T
        budget_blocks = (max(token_budget - cur_local_len, 0) + T - 1) // T
        seqlens = np.zeros((B, Hk), np.int32)
        tables = []
        for b in range(B):
            for h in range(Hk):
                glen = int(self.global_lengths[l, b, h])
                full, rem = divmod(glen, T)
                nb = full + (rem > 0)
                cap = min(budget_blocks, nb)
                chosen = np.zeros(0, np.int64)
                partial = False
                if cap > 0:
                    full_cap = cap - (1 if rem > 0 else 0)
                    if full_cap > 0 and full > 0:
                        if full_cap >= full:
                            chosen = np.arange(full)
                        else:
                            sc = self.quest_scores(l, b, h, q[b, h * G:(h + 1) * G])[:full]
                            order = np.lexsort((np.arange(full), -sc.astype(np.float64)))
                            chosen = np.sort(order[:full_cap])
                    if rem > 0:
                        chosen = np.concatenate([chosen, [full]])
                        partial = True
                row = self.block_table[l, b, h]
                pages = np.concatenate([row[:local_blocks], row[self.local_pages + chosen]]).astype(np.int32)
                n_tok = len(chosen) * T + (rem - T if partial else 0)
                seqlens[b, h] = cur_local_len + n_tok
                tables.append(pages)
        return seqlens, tables

    def paged_views(self):
        T, D = self.page, self.head_dim
        return self.k.reshape(-1, T, D), self.v.reshape(-1, T, D)


def pool_digest(block_table, global_lengths, local_length, k_bits, v_bits, page, window):
    """sha256 over the live rows of the pool, in logical order per (layer, head):
    ring slots ``[0, local_length)`` then global tokens ``[0, global_length)``.

    ``block_table`` ``(Lyr, [B,] Hk, maxb)``; ``k_bits``/``v_bits`` uint16
    bf16 bit patterns of the pool rows ``(NB*T, D)``.  Matches
    ``tests/golden/make_golden.py:pool_digest`` for batch 1."""
    import hashlib
    bt = np.asarray(block_table)
    gl = np.asarray(global_lengths)
    if bt.ndim == 4:  # (Lyr, B, Hk, maxb): fold batch into heads in (b, h) order
        bt = bt.reshape(bt.shape[0], -1, bt.shape[-1])
        gl = gl.reshape(gl.shape[0], -1)
    T = page
    hsh = hashlib.sha256()
    k_bits = np.asarray(k_bits, np.uint16)
    v_bits = np.asarray(v_bits, np.uint16)
    for l in range(bt.shape[0]):
        for h in range(bt.shape[1]):
            j = np.arange(local_length)
            rows = bt[l, h, j // T].astype(np.int64) * T + j % T
            j = np.arange(int(gl[l, h]))
            rows = np.concatenate([rows, bt[l, h, window // T + j // T].astype(np.int64) * T + j % T])
            inter = np.stack([k_bits[rows], v_bits[rows]], axis=1)  # k row, v row alternating
            hsh.update(inter.astype('<u2').tobytes())
    return np.frombuffer(hsh.digest(), np.uint8)
