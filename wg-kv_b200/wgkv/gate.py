"""Write gate: GatingPredictor with the reference's parameters, CUDA forward.

The module keeps the reference's sub-module names and shapes
(src/modeling_layers.py:134-160: ``pre_key_norm`` / ``post_key_norm`` /
``value_norm`` RMS norms, grouped 1x1 ``conv1`` and ``conv2``), so the
published gate checkpoints (``model.layers.{i}.self_attn.g_predictors.*``)
load with ``load_state_dict``.  ``forward`` runs as one sm_100a kernel
(``wgkv_gate_scores``) with the numerics ``g_fast_path`` selects -- the einsum
fast path (``:185-196``) or the grouped-conv path with its ``g_epsilon`` clamp
(``:198-205``, the reference's default) -- and returns bf16 scores of shape
(B, Hk, L); :meth:`admit` writes the admission mask
``scores > threshold`` straight into any uint8 tensor view (e.g. the
cache's ``local_is_global`` slots) without materialising the scores.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ._lib import check, lib
from .runtime import require_cuda, stream_ptr
from .pool import pool_ref

_SLOTS = ("pre_k", "post_k", "v")


class GatingRMSNorm(nn.Module):
    """Parameter holder with the reference's layout (``weight`` (D,), eps);
    the normalisation itself runs inside the gate kernel."""

    def __init__(self, hidden_size, eps=1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(hidden_size))
        self.variance_epsilon = eps

    def forward(self, hidden_states):  # pragma: no cover - the fused kernel is the product path
        raise RuntimeError("GatingRMSNorm is applied inside wgkv_gate_scores")


def _bf16(t):
    return t.detach().to(torch.bfloat16).contiguous()


def _strides4(t):
    if t is None:
        return 0, 0, 0, 0
    assert t.dim() == 4 and t.stride(3) == 1, "gate inputs must be (B, Hk, L, D) with a contiguous last axis"
    return t.data_ptr(), t.stride(0), t.stride(1), t.stride(2)


class GatingPredictor(nn.Module):
    def __init__(self, head_dim, num_kv_heads, g_inputs, g_act_fn, g_expand, g_epsilon, g_rms, g_fast_path=True):
        super().__init__()
        self.g_inputs = list(g_inputs)
        self.g_epsilon = g_epsilon
        self.g_fast_path = g_fast_path
        self.head_dim = head_dim
        self.num_kv_heads = num_kv_heads
        self.input_dim = head_dim * len(self.g_inputs)
        self.inner_dim = int(head_dim * g_expand)
        self.g_rms = g_rms
        # WGKV_GATE_SILU (0x1) / WGKV_GATE_CONV (0x2) bits of the entry points' `act` argument
        self.act = 1 if g_act_fn == "silu" else 0
        self.pre_key_norm = GatingRMSNorm(head_dim) if g_rms and "pre_k" in self.g_inputs else nn.Identity()
        self.post_key_norm = GatingRMSNorm(head_dim) if g_rms and "post_k" in self.g_inputs else nn.Identity()
        self.value_norm = GatingRMSNorm(head_dim) if g_rms and "v" in self.g_inputs else nn.Identity()
        self.conv1 = nn.Conv1d(num_kv_heads * self.input_dim, num_kv_heads * self.inner_dim, kernel_size=1,
                               groups=num_kv_heads)
        self.conv2 = nn.Conv1d(num_kv_heads * self.inner_dim, num_kv_heads, kernel_size=1, groups=num_kv_heads)
        self.input_mask = sum(1 << i for i, s in enumerate(_SLOTS) if s in self.g_inputs)
        # the kernel concatenates inputs in slot order; the reference concatenates in that order too (:173-183)

    def reset_parameters(self):
        for norm in (self.pre_key_norm, self.post_key_norm, self.value_norm):
            if isinstance(norm, GatingRMSNorm):
                nn.init.ones_(norm.weight)
        self.conv1.reset_parameters()
        self.conv2.reset_parameters()

    def _norm_weights(self, device):
        if not self.g_rms:
            return None
        rows = []
        for mod in (self.pre_key_norm, self.post_key_norm, self.value_norm):
            rows.append(mod.weight if isinstance(mod, GatingRMSNorm) else torch.ones(self.head_dim, device=device))
        return _bf16(torch.stack([r.to(device) for r in rows]))

    def _eps(self):
        for mod in (self.pre_key_norm, self.post_key_norm, self.value_norm):
            if isinstance(mod, GatingRMSNorm):
                return float(mod.variance_epsilon)
        return 1e-6

    def _act_flags(self):
        return self.act | (0 if self.g_fast_path else 2)

    def _launch(self, pre_key, post_key, value, threshold, scores, mask):
        ref = next(t for t in (pre_key, post_key, value) if t is not None)
        require_cuda(ref, "gate input")
        B, Hk, L, D = ref.shape
        assert Hk == self.num_kv_heads and D == self.head_dim
        ins = {"pre_k": pre_key, "post_k": post_key, "v": value}
        for s in self.g_inputs:
            assert ins[s] is not None and ins[s].dtype == torch.bfloat16, f"gate input {s} must be bf16"
        w1 = _bf16(self.conv1.weight)  # (Hk*inner, I, 1) == (Hk, inner, I)
        b1 = _bf16(self.conv1.bias)
        w2 = _bf16(self.conv2.weight)  # (Hk, inner, 1)
        b2 = _bf16(self.conv2.bias)
        nw = self._norm_weights(ref.device)
        pk = _strides4(pre_key if "pre_k" in self.g_inputs else None)
        kk = _strides4(post_key if "post_k" in self.g_inputs else None)
        vv = _strides4(value if "v" in self.g_inputs else None)
        sp = (scores.data_ptr(), scores.stride(0), scores.stride(1), scores.stride(2)) if scores is not None else (0, 0, 0, 0)
        mp = (mask.data_ptr(), mask.stride(0), mask.stride(1), mask.stride(2)) if mask is not None else (0, 0, 0, 0)
        st = lib.wgkv_gate_scores(*pk, *kk, *vv, B, Hk, L, D, self.input_mask, w1.data_ptr(), b1.data_ptr(),
                                  w2.data_ptr(), b2.data_ptr(), nw.data_ptr() if nw is not None else None,
                                  self._eps(), self.inner_dim, self._act_flags(), float(self.g_epsilon), float(threshold), *sp, *mp,
                                  stream_ptr(ref.device))
        check(st, "wgkv_gate_scores")

    def forward(self, pre_key, post_key, value):
        """g_scores (B, Hk, L) bf16 (GatingPredictor.forward, :170-205)."""
        ref = post_key if post_key is not None else (pre_key if pre_key is not None else value)
        B, Hk, L, _ = ref.shape
        scores = torch.empty(B, Hk, L, dtype=torch.bfloat16, device=ref.device)
        self._launch(pre_key, post_key, value, 0.0, scores, None)
        return scores

    def admit(self, pre_key, post_key, value, threshold, mask, scores=None):
        """Write ``gate(x) > threshold`` (uint8) into ``mask`` (any (B, Hk, L) view); optionally the scores."""
        self._launch(pre_key, post_key, value, threshold, scores, mask)
        return mask

    def decode_admit_append(self, cache, layer, insert_pos, cur_local_len, pre_key, post_key, value, threshold):
        """Fused decode prologue (``wgkv_decode_gate_append``): gate the new token of every (b, h),
        write its admission bit and its K/V into ring slot ``insert_pos`` of ``layer``, and fill
        ``cache.cache_seqlens``.  Inputs are (B, Hk, 1, D) (or (B, Hk, D)) bf16 views."""
        def rows(t):
            if t is None:
                return None, 0, 0
            t = t[:, :, 0] if t.dim() == 4 else t
            assert t.stride(2) == 1
            return t.data_ptr(), t.stride(0), t.stride(1)
        pk = rows(pre_key if "pre_k" in self.g_inputs else None)
        kk = rows(post_key)
        vv = rows(value)
        w1, b1, w2, b2 = (_bf16(x) for x in (self.conv1.weight, self.conv1.bias, self.conv2.weight, self.conv2.bias))
        nw = self._norm_weights(post_key.device)
        st = lib.wgkv_decode_gate_append(pool_ref(cache), layer, insert_pos, cur_local_len, *pk, *kk, *vv,
                                         self.input_mask, w1.data_ptr(), b1.data_ptr(), w2.data_ptr(), b2.data_ptr(),
                                         nw.data_ptr() if nw is not None else None, self._eps(), self.inner_dim,
                                         self._act_flags(), float(self.g_epsilon), float(threshold),
                                         cache.cache_seqlens.data_ptr(),
                                         stream_ptr(post_key.device))
        check(st, "wgkv_decode_gate_append")


    def decode_prologue(self, cache, layer, insert_pos, cur_local_len, qkv, q_heads, position, rope_cos, rope_sin,
                        q_out, threshold, q_norm=None, k_norm=None, qk_eps=1e-6, gate=True):
        """``wgkv_decode_prologue``: q/k norm + RoPE of the raw projection rows ``qkv`` (B, (Hq + 2 Hk) D),
        then the fused gate + ring append of :meth:`decode_admit_append` (``gate=False``: deferred
        gating, pre_k into the ring's pre-key store).  Rotated queries go to ``q_out`` (B, Hq, D)."""
        assert qkv.dim() == 2 and qkv.stride(1) == 1 and qkv.dtype == torch.bfloat16
        assert q_out.is_contiguous() and rope_cos.is_contiguous() and rope_sin.is_contiguous()
        if gate:
            w1, b1, w2, b2 = (_bf16(x) for x in (self.conv1.weight, self.conv1.bias, self.conv2.weight,
                                                  self.conv2.bias))
            nw = self._norm_weights(qkv.device)
            gp = (self.input_mask, w1.data_ptr(), b1.data_ptr(), w2.data_ptr(), b2.data_ptr(),
                  nw.data_ptr() if nw is not None else None, self._eps(), self.inner_dim, self._act_flags(),
                  float(self.g_epsilon))
        else:
            gp = (0, None, None, None, None, None, 0.0, 0, 0, 0.0)
        st = lib.wgkv_decode_prologue(pool_ref(cache), layer, insert_pos, cur_local_len, qkv.data_ptr(),
                                      qkv.stride(0), q_heads, q_norm.data_ptr() if q_norm is not None else None,
                                      k_norm.data_ptr() if k_norm is not None else None, float(qk_eps),
                                      rope_cos.data_ptr(), rope_sin.data_ptr(), position.data_ptr(),
                                      rope_cos.shape[0], q_out.data_ptr(), *gp, float(threshold),
                                      cache.cache_seqlens.data_ptr(), stream_ptr(qkv.device))
        check(st, "wgkv_decode_prologue")

def load_gate_checkpoint(modules, state, prefix="model.layers.{i}.self_attn.g_predictors.", strict=True):
    """Load a WG-KV gate checkpoint into per-layer gates.

    ``state`` is the dict the reference's training script saves (``scripts/train.py:311-335``:
    ``{name: param}`` of the trainable parameters, loaded with ``load_state_dict(strict=False)`` at
    ``scripts/profiling.py:223-226``) or a path to it.  ``modules[i]`` is layer i's attention module
    (anything with ``.g_predictors``) or its :class:`GatingPredictor`.  Returns the keys used."""
    if isinstance(state, str):
        state = torch.load(state, map_location="cpu", weights_only=True)
    used = []
    for i, m in enumerate(modules):
        gp = m.g_predictors if hasattr(m, "g_predictors") else m
        pre = prefix.format(i=i)
        sub = {k[len(pre):]: torch.as_tensor(v) for k, v in state.items() if k.startswith(pre)}
        if not sub:
            if strict:
                raise KeyError(f"no gate parameters under {pre!r}")
            continue
        own = gp.state_dict()
        for k, v in sub.items():
            if k not in own:
                raise KeyError(f"unexpected gate parameter {pre + k}")
            if tuple(own[k].shape) != tuple(v.shape):
                raise ValueError(f"{pre + k}: shape {tuple(v.shape)} != {tuple(own[k].shape)}")
        gp.load_state_dict({k: v.to(own[k].dtype) for k, v in sub.items()}, strict=strict)
        used += [pre + k for k in sub]
    return used
