"""End-to-end decoder driver: time-to-first-token and time-per-output-token on the WG-KV path.

Stands in for the reference's profiling loop (scripts/profiling.py:346-418: one prefill of the
prompt with ``logits_to_keep=1``, then greedy decode steps, CUDA-event timed, with an optional
attention / MLP / lm_head breakdown, :251-344) on a Llama- or Qwen3-shaped decoder whose weights
are random-initialised (no checkpoints are available offline).  Around the attention path this
is plain PyTorch: the q/k/v/o, MLP and lm_head GEMMs are cuBLAS calls, RMSNorm, RoPE and SiLU are
torch element-wise ops.  The attention of every layer is this library's
``self_attn_forward_patch`` (gate, admission compaction, sparse prefill; gate, append, promotion,
paged decode), called with the arguments the patched attention layers pass
(src/modeling_llama.py:265-287: q/k/v after RoPE, ``pre_key`` before it; src/modeling_qwen3.py:
236-239: ``pre_key`` after k_norm).

A decode step keeps its changing inputs on the device -- the token ids, the RoPE position and
(with ``cache.wgkv_device_ring``) the ring position -- and writes the next greedy token back into
its input buffer, so a whole step, argmax included, replays as one CUDA graph
(:class:`wgkv.graph.DecodeGraph`).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from types import SimpleNamespace

import numpy as np
import torch
import torch.nn.functional as F

from ._lib import check, lib
from .gate import GatingPredictor
from .graph import DecodeGraph
from .runtime import stream_ptr


@dataclass(frozen=True)
class DecoderShape:
    name: str
    hidden: int
    layers: int
    q_heads: int
    kv_heads: int
    head_dim: int
    intermediate: int
    vocab: int
    rope_theta: float
    qk_norm: bool
    rms_eps: float


# public architecture shapes of the models the reference patches (weights are random here)
SHAPES = {
    "llama-3.2-1b": DecoderShape("Llama-3.2-1B-shaped", 2048, 16, 32, 8, 64, 8192, 128256, 500000.0, False, 1e-5),
    "llama-3.1-8b": DecoderShape("Llama-3.1-8B-shaped", 4096, 32, 32, 8, 128, 14336, 128256, 500000.0, False, 1e-5),
    "qwen3-4b": DecoderShape("Qwen3-4B-shaped", 2560, 36, 32, 8, 128, 9728, 151936, 1000000.0, True, 1e-6),
}


def _rms(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * w


def rms_norm(x, w, eps):
    """``wgkv_rms_norm`` over the last axis of a bf16 tensor (rows contiguous)."""
    cols = x.shape[-1]
    x2 = x.reshape(-1, cols)
    out = torch.empty(x2.shape, dtype=x.dtype, device=x.device)
    check(lib.wgkv_rms_norm(x2.data_ptr(), x2.stride(0), w.data_ptr(), x2.shape[0], cols, float(eps), out.data_ptr(),
                            out.stride(0), stream_ptr(x.device)), "wgkv_rms_norm")
    return out.view(x.shape)


def silu_mul(gu):
    """``wgkv_silu_mul``: (rows, 2 I) [gate | up] -> (rows, I)."""
    inter = gu.shape[-1] // 2
    out = torch.empty(gu.shape[0], inter, dtype=gu.dtype, device=gu.device)
    check(lib.wgkv_silu_mul(gu.data_ptr(), gu.stride(0), gu.shape[0], inter, out.data_ptr(), out.stride(0),
                            stream_ptr(gu.device)), "wgkv_silu_mul")
    return out


def skinny_linear(x, w, residual=None, out_f32=False, rms_weight=None, rms_eps=1e-6, paired=False):
    """``wgkv_skinny_gemm``: x (m <= 8, k) bf16 @ w (n, k)^T, fp32 accumulate; ``residual`` (m, n)
    bf16 is added and receives the result in place; ``out_f32`` returns fp32 (no residual);
    ``rms_weight`` RMS-normalises x first (as :func:`rms_norm`); ``paired`` treats w as
    [gate | up] and returns silu(x gate^T) * (x up^T) (as :func:`silu_mul` on the projection)."""
    m, k = x.shape
    n = w.shape[0]
    assert x.stride(1) == 1 and w.is_contiguous() and m <= 8
    if residual is not None:
        y = residual
        assert y.stride(1) == 1 and y.shape == (m, n)
    else:
        y = torch.empty(m, n // 2 if paired else n, dtype=torch.float32 if out_f32 else x.dtype, device=x.device)
    check(lib.wgkv_skinny_gemm(x.data_ptr(), x.stride(0), m, w.data_ptr(), n, k, y.data_ptr(), y.stride(0),
                               int(out_f32), residual.data_ptr() if residual is not None else None,
                               residual.stride(0) if residual is not None else 0,
                               rms_weight.data_ptr() if rms_weight is not None else None, float(rms_eps), int(paired),
                               stream_ptr(x.device)), "wgkv_skinny_gemm")
    return y


def argmax_into(logits, out):
    """``wgkv_argmax``: out (rows, 1) int64 = first index of each fp32 row's maximum."""
    from .runtime import workspace
    rows, n = logits.shape
    assert logits.stride(1) == 1 and logits.dtype == torch.float32
    nbytes = int(lib.wgkv_argmax_workspace_size(rows, n))
    ws = workspace(logits.device, "argmax", nbytes, zero_prefix=((rows * 4 + 255) // 256) * 256)
    check(lib.wgkv_argmax(logits.data_ptr(), logits.stride(0), rows, n, out.data_ptr(), out.stride(0), ws.data_ptr(),
                          ws.numel(), stream_ptr(logits.device)), "wgkv_argmax")
    return out


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class WgkvDecoder:
    """Random-init decoder over the WG-KV attention path (batch ``batch``, greedy decoding)."""

    def __init__(self, shape: DecoderShape, *, batch=1, window=4096, page=16, max_tokens_per_head=33000,
                 avg_tokens_per_head=None, g_defer=True, threshold=0.5, gate_inner=64, admit=(2.0, 8.0),
                 max_positions=None, device="cuda", seed=0, fused=True):
        self.s = s = shape
        self.fused = fused
        self.B = batch
        self.dev = torch.device(device)
        self.W = window
        self.defer = g_defer
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)
        bf = torch.bfloat16

        def rnd(*shape, std=0.02):
            return (torch.randn(*shape, generator=g, device=self.dev) * std).to(bf)

        D, Hq, Hk, Hd = s.head_dim, s.q_heads, s.kv_heads, s.hidden
        self.embed = rnd(s.vocab, Hd, std=1.0)
        self.lm_head = rnd(s.vocab, Hd)
        self.final_norm = torch.ones(Hd, dtype=bf, device=self.dev)
        # profiling.py:85-91 sizes the pool per (layer, head); one pool row set per sequence here
        per_head = avg_tokens_per_head if avg_tokens_per_head else max_tokens_per_head
        self.config = SimpleNamespace(
            num_hidden_layers=s.layers, num_key_value_heads=Hk, num_attention_heads=Hq, head_dim=D,
            hidden_size=Hd, block_size=page, local_window_size=window, g_defer=g_defer, g_threshold=threshold,
            max_tokens_per_head=max_tokens_per_head, max_total_tokens=per_head * s.layers * Hk * batch + 2 * page)
        from . import attach
        rng = np.random.default_rng(seed + 1)
        self.admit_rates = rng.beta(admit[0], admit[1], (s.layers, Hk))
        self.layers = []
        for l in range(s.layers):
            L = SimpleNamespace()
            L.in_norm = torch.ones(Hd, dtype=bf, device=self.dev)
            L.post_norm = torch.ones(Hd, dtype=bf, device=self.dev)
            L.qkv = rnd((Hq + 2 * Hk) * D, Hd)
            L.o = rnd(Hd, Hq * D)
            L.gate_up = rnd(2 * s.intermediate, Hd)
            L.down = rnd(Hd, s.intermediate)
            if s.qk_norm:
                L.q_norm = torch.ones(D, dtype=bf, device=self.dev)
                L.k_norm = torch.ones(D, dtype=bf, device=self.dev)
            torch.manual_seed(seed * 1000 + l)
            gp = GatingPredictor(D, Hk, ["pre_k"], "gelu", gate_inner / D, 1e-3, False, True).to(self.dev, bf)
            L.attn = attach(SimpleNamespace(layer_idx=l, head_dim=D, scaling=D ** -0.5, g_predictors=gp),
                            self.config)
            self.layers.append(L)
        self.max_pos = max_positions or 1 << 17
        self.host_pos = 0  # host copy of self.pos (bounds the RoPE table lookups without a sync)
        inv = 1.0 / (s.rope_theta ** (torch.arange(0, D, 2, dtype=torch.float32, device=self.dev) / D))
        self._inv_freq = inv
        self._cos = self._sin = None
        self.pos = torch.zeros(1, dtype=torch.int64, device=self.dev)  # position of the next decode token
        self.token = torch.zeros(batch, 1, dtype=torch.int64, device=self.dev)  # next decode input
        self.logits = None
        self.timers = None

    # ------------------------------------------------------------------ helpers
    def _rope_table(self, n):
        n = max(n, self.max_pos)
        if self._cos is None or self._cos.shape[0] < n:
            t = torch.arange(n, dtype=torch.float32, device=self.dev)
            f = torch.outer(t, self._inv_freq)
            emb = torch.cat((f, f), dim=-1)
            self._cos, self._sin = emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)
        return self._cos, self._sin

    def _time(self, key):
        if self.timers is None:
            return None
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
        return key, e0

    def _stop(self, t):
        if t is None:
            return
        key, e0 = t
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record()
        self.timers.setdefault(key, []).append((e0, e1))

    def calibrate_gates(self, n_tokens=1024, seed=7):
        """Set each gate's per-head output bias so that P(score > threshold) ~ the head's admit rate,
        measured on the pre-RoPE keys of a dense causal pass over ``n_tokens`` random tokens."""
        s = self.s
        g = torch.Generator(device=self.dev)
        g.manual_seed(seed)
        ids = torch.randint(0, s.vocab, (1, n_tokens), generator=g, device=self.dev)
        h = F.embedding(ids, self.embed)
        cos, sin = self._rope_table(n_tokens)
        thr = self.config.g_threshold
        with torch.no_grad():
            for l, L in enumerate(self.layers):
                q, k, v = self._qkv(L, h)
                pk = k
                q, k = self._apply_rope(q, k, cos[:n_tokens], sin[:n_tokens])
                gp = L.attn.g_predictors
                D, Hk = s.head_dim, s.kv_heads
                x = pk[0].float()  # (L, Hk, D)
                w1 = gp.conv1.weight.float().view(Hk, -1, D)
                b1 = gp.conv1.bias.float().view(Hk, -1)
                w2 = gp.conv2.weight.float().view(Hk, -1)
                hdn = F.gelu(torch.einsum("thd,hjd->htj", x, w1) + b1[:, None, :])
                logit = torch.einsum("htj,hj->ht", hdn, w2)
                r = torch.from_numpy(self.admit_rates[l]).to(self.dev).float()
                b2 = torch.stack([torch.quantile(logit[i], 1 - r[i]) for i in range(Hk)])
                gp.conv2.bias.copy_((math.log(thr / (1 - thr)) - b2).to(torch.bfloat16))
                o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                                   is_causal=True, enable_gqa=True)
                h = self._after_attn(L, h, o.transpose(1, 2).reshape(1, n_tokens, -1))

    def _norm(self, x, w):
        return rms_norm(x, w, self.s.rms_eps) if self.fused else _rms(x, w, self.s.rms_eps)

    def _skinny(self, rows):
        return self.fused and rows <= 8

    def _qkv_rows(self, L, x_in):
        x = self._norm(x_in, L.in_norm)
        if self._skinny(x.numel() // x.shape[-1]):
            return skinny_linear(x.reshape(-1, x.shape[-1]), L.qkv).view(*x.shape[:-1], -1)
        return x @ L.qkv.t()

    def _qkv(self, L, x_in):
        s = self.s
        B, T, _ = x_in.shape
        qkv = self._qkv_rows(L, x_in)
        D, Hq, Hk = s.head_dim, s.q_heads, s.kv_heads
        q = qkv[..., :Hq * D].view(B, T, Hq, D)
        k = qkv[..., Hq * D:(Hq + Hk) * D].view(B, T, Hk, D)
        v = qkv[..., (Hq + Hk) * D:].view(B, T, Hk, D)
        if s.qk_norm:
            q = _rms(q, L.q_norm, s.rms_eps)
            k = _rms(k, L.k_norm, s.rms_eps)
        return q, k, v

    @staticmethod
    def _apply_rope(q, k, cos, sin):
        c, n = cos[None, :, None, :], sin[None, :, None, :]
        return q * c + _rotate_half(q) * n, k * c + _rotate_half(k) * n

    def _after_attn(self, L, h, a):
        if not self.fused:
            h = h + a @ L.o.t()
            t = self._time("mlp")
            x = _rms(h, L.post_norm, self.s.rms_eps)
            gu = x @ L.gate_up.t()
            I = self.s.intermediate
            h = h + (F.silu(gu[..., :I]) * gu[..., I:]) @ L.down.t()
            self._stop(t)
            return h
        # residual adds fused into the projections; norm and activation one launch each
        h2 = h.view(-1, h.shape[-1])
        a2 = a.reshape(h2.shape[0], -1)
        if self._skinny(h2.shape[0]):
            skinny_linear(a2, L.o, residual=h2)
            t = self._time("mlp")
            # separate one-launch norm and activation: folding them into the projections (the
            # kernel's rms_weight / paired modes) measured slower at batch 1 (1.15 -> 1.36 ms/step)
            x = rms_norm(h2, L.post_norm, self.s.rms_eps)
            skinny_linear(silu_mul(skinny_linear(x, L.gate_up)), L.down, residual=h2)
        else:
            h2.addmm_(a2, L.o.t())
            t = self._time("mlp")
            x = rms_norm(h2, L.post_norm, self.s.rms_eps)
            h2.addmm_(silu_mul(x @ L.gate_up.t()), L.down.t())
        self._stop(t)
        return h

    # ------------------------------------------------------------------ forward
    def forward(self, ids, cache, cos, sin):
        """ids (B, T) int64 -> logits of the last position (B, vocab), float32."""
        B, T = ids.shape
        h = F.embedding(ids, self.embed)
        s = self.s
        for L in self.layers:
            if self.fused and T == 1:
                qkv = self._qkv_rows(L, h.view(B, -1))
                t = self._time("attn")
                o = L.attn.self_attn_decode_fused(L.attn, cache, qkv, s.q_heads, self.pos, self._cos, self._sin,
                                                  q_norm=getattr(L, "q_norm", None),
                                                  k_norm=getattr(L, "k_norm", None), qk_eps=s.rms_eps)
                self._stop(t)
                h = self._after_attn(L, h, o.reshape(B, T, -1))
                continue
            q, k, v = self._qkv(L, h)
            pre_k = k
            q, k = self._apply_rope(q, k, cos, sin)
            t = self._time("attn")
            o, _, _ = L.attn.self_attn_forward_patch(L.attn, 3, None, cache, (B, T), q.transpose(1, 2),
                                                     pre_k.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
            self._stop(t)
            h = self._after_attn(L, h, o.reshape(B, T, -1))
        t = self._time("lm_head")
        x = self._norm(h[:, -1:].contiguous(), self.final_norm)
        if self._skinny(B):
            logits = skinny_linear(x.view(B, -1), self.lm_head, out_f32=True)
        else:
            logits = (x @ self.lm_head.t()).float()[:, 0]
        self._stop(t)
        return logits

    def prefill(self, ids, cache):
        """Prompt (B, L) -> next token into ``self.token``; returns the last-position logits."""
        B, T = ids.shape
        cos, sin = self._rope_table(T + 1)
        logits = self.forward(ids, cache, cos[:T], sin[:T])
        self.token.copy_(logits.argmax(-1, keepdim=True))
        self.pos.fill_(T)
        self.host_pos = T
        return logits

    def _check_pos(self):
        if self.host_pos >= self._rope_table(0)[0].shape[0]:
            raise ValueError(f"position {self.host_pos} is past max_positions={self.max_pos}")

    def decode_step(self, cache):
        """One greedy step from ``self.token`` at position ``self.pos`` (both on the device)."""
        cos, sin = self._rope_table(self.max_pos)
        if not torch.cuda.is_current_stream_capturing():
            self._check_pos()
            self.host_pos += 1
        if self.fused:  # the prologue kernel reads the tables at self.pos itself
            c = n = None
        else:
            c = cos.index_select(0, self.pos)
            n = sin.index_select(0, self.pos)
        logits = self.forward(self.token, cache, c, n)
        if self.fused:
            argmax_into(logits, self.token)
        else:
            self.token.copy_(logits.argmax(-1, keepdim=True))
        self.pos.add_(1)
        self.logits = logits
        return logits

    def decode_graph(self, cache):
        """Run one real decode step eagerly and capture it; ``.replay()`` is then one more step."""
        self._rope_table(self.max_pos)
        dg = DecodeGraph(cache, self.W, defer=self.defer, device=self.dev)
        dg.capture(lambda: self.decode_step(cache))
        model = self
        replay = dg.replay

        def checked_replay():
            model._check_pos()
            model.host_pos += 1
            return replay()
        dg.replay = checked_replay
        return dg

    def breakdown(self):
        """{phase: ms} of the events recorded since ``timers`` was set to {} (after a sync)."""
        return {k: sum(a.elapsed_time(b) for a, b in v) for k, v in (self.timers or {}).items()}

    def weight_bytes(self):
        n = self.embed.numel() + self.lm_head.numel()
        for L in self.layers:
            n += L.qkv.numel() + L.o.numel() + L.gate_up.numel() + L.down.numel()
        return 2 * n
