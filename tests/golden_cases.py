"""Loaders for the committed golden fixtures (tests/golden/*.npz).

The fixtures hold seeds, gate parameters and the reference's outputs; the
inputs are re-created here with the same numpy streams that
``tests/golden/make_golden.py`` used.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
if REPO not in sys.path:
    sys.path.insert(0, REPO)
from oracle import wgkv_oracle as O  # noqa: E402

GOLDEN = os.path.join(HERE, "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name + ".npz")))


class PipelineCase:
    """One prefill + decode fixture written by make_golden.run_pipeline_case."""

    def __init__(self, name):
        self.name = name
        z = load(name)
        self.z = z
        g = lambda k: int(z[f"meta_{k}"])
        self.Ly, self.L, self.Hq, self.Hk, self.D = g("Ly"), g("L"), g("Hq"), g("Hk"), g("D")
        self.W, self.T, self.inner, self.n_decode = g("W"), g("T"), g("inner"), g("n_decode")
        self.defer = bool(g("defer"))
        self.seed = g("seed")
        self.max_total_tokens, self.max_tokens_per_head = g("max_total_tokens"), g("max_tokens_per_head")
        self.rows_out = g("rows_out")
        self.quest_budget = g("quest_budget") if "meta_quest_budget" in z else -1
        self.snapkv = ((g("snap_max"), float(z["meta_snap_ratio"]), g("snap_window"), g("snap_kernel"))
                       if "meta_snap_max" in z else None)
        self.threshold = float(z["meta_threshold"])
        self.inputs = tuple(str(x) for x in z["meta_inputs"])
        self.act = str(z["meta_act"])
        self.G = self.Hq // self.Hk
        rng = np.random.default_rng(self.seed)
        self.params, self.prefill = [], []
        for l in range(self.Ly):
            q = O.randn_bf16(rng, (1, self.Hq, self.L, self.D))
            k = O.randn_bf16(rng, (1, self.Hk, self.L, self.D))
            v = O.randn_bf16(rng, (1, self.Hk, self.L, self.D))
            pk = O.randn_bf16(rng, (1, self.Hk, self.L, self.D))
            # consume the same draws make_gate_params made
            n_in = len(self.inputs)
            I = self.D * n_in
            rng.uniform(size=(self.Hk, self.inner, I))
            rng.uniform(size=(self.Hk, self.inner))
            rng.uniform(size=(self.Hk, self.inner))
            p = O.GateParams(w1=O.from_bf16_bits(z[f"l{l}_w1"]), b1=O.from_bf16_bits(z[f"l{l}_b1"]),
                             w2=O.from_bf16_bits(z[f"l{l}_w2"]), b2=O.from_bf16_bits(z[f"l{l}_b2"]),
                             inputs=self.inputs, act=self.act)
            self.params.append(p)
            self.prefill.append((q, k, v, pk))
        self.decode = []
        for _ in range(self.n_decode):
            step = []
            for l in range(self.Ly):
                step.append(tuple(O.randn_bf16(rng, sh) for sh in [(1, self.Hq, 1, self.D), (1, self.Hk, 1, self.D),
                                                                  (1, self.Hk, 1, self.D), (1, self.Hk, 1, self.D)]))
            self.decode.append(step)

    def ref_scores(self, l):
        return O.from_bf16_bits(self.z[f"l{l}_scores"])[None]

    def ref_mask(self, l):
        return O.admission_mask(self.ref_scores(l), self.threshold)

    def ref_decode_mask(self, s, l):
        key = f"d{s}_l{l}_scores"
        if key not in self.z:
            return None
        return O.admission_mask(O.from_bf16_bits(self.z[key])[None], self.threshold)

    def new_state(self):
        return O.PoolState(layers=self.Ly, batch=1, kv_heads=self.Hk, head_dim=self.D, window=self.W, page=self.T,
                           max_total_tokens=self.max_total_tokens, max_tokens_per_head=self.max_tokens_per_head,
                           defer=self.defer, quest=self.quest_budget >= 0, snapkv=self.snapkv, q_heads=self.Hq)


def quest_sets_agree(st, l, b, h, q_group, got_pages, ref_pages):
    """Selected page sets of one (layer, b, h) agree up to pages whose score ties the lowest chosen
    full-page score (their order is torch.topk's to choose).  Pages are physical ids, ring pages and
    the trailing partial page included."""
    got, ref = set(int(x) for x in got_pages), set(int(x) for x in ref_pages)
    if got == ref:
        return True
    if len(got) != len(ref):
        return False
    T = st.page
    full = int(st.global_lengths[l, b, h]) // T
    row = st.block_table[l, b, h, st.local_pages:st.local_pages + full]
    pos = {int(p): i for i, p in enumerate(row)}  # full global pages only
    diff = got ^ ref
    if not all(p in pos for p in diff):
        return False
    sc = st.quest_scores(l, b, h, q_group)
    kth_got = min(sc[pos[p]] for p in got if p in pos)
    kth_ref = min(sc[pos[p]] for p in ref if p in pos)
    return kth_got == kth_ref and all(sc[pos[p]] == kth_got for p in diff)


def snap_evicted_agree(scores, got, ref):
    """Evicted position sets agree up to positions whose (pooled) score ties the highest evicted
    score in both: torch.topk(largest=False) leaves the order of equal scores open."""
    got, ref = set(int(x) for x in got), set(int(x) for x in ref)
    if got == ref:
        return True
    if len(got) != len(ref):
        return False
    thr_g = max(scores[list(got)])
    thr_r = max(scores[list(ref)])
    return thr_g == thr_r and all(scores[p] == thr_g for p in got ^ ref)


def regen_decode_inputs(params):
    """Re-create the inputs of a make_golden.decode_cases() entry."""
    Hq, Hk, D, T, B, maxs, pool_nb, seed = (int(x) for x in params)
    rng = np.random.default_rng(seed)
    maxb = (maxs + T - 1) // T
    seqlens = rng.integers(1, maxs + 1, (B, Hk)).astype(np.int32)
    perm = rng.permutation(pool_nb).astype(np.int32)
    table = np.full((B, Hk, maxb), -1, np.int32)
    off = 0
    for b in range(B):
        for h in range(Hk):
            n = (int(seqlens[b, h]) + T - 1) // T
            table[b, h, :n] = perm[off:off + n]
            off += n
    q = O.randn_bf16(rng, (B, 1, Hq, D))
    kc = O.randn_bf16(rng, (pool_nb, T, D))
    vc = O.randn_bf16(rng, (pool_nb, T, D))
    return q, kc, vc, seqlens, table


def indices_case(z, i):
    B, Hk, L, W, gs = (int(x) for x in z[f"c{i}_params"])
    g = np.unpackbits(z[f"c{i}_mask"], axis=-1, count=L).astype(bool)
    fast = tuple(z[f"c{i}_{n}"] for n in ("bc", "bo", "cc", "ci"))
    ref = tuple(z[f"c{i}_ref_{n}"] for n in ("bc", "bo", "cc", "ci"))
    return (B, Hk, L, W, gs), g, fast, ref
