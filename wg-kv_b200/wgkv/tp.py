"""KV-head tensor parallelism around the admission path: one process per GPU.

The admission path never exchanges data: a KV head's gate, pages, ring, tables
and attention depend on that head alone.  A model split by KV head therefore
gives each rank whole GQA groups -- its KV heads and their query heads -- and
its own paged pool for them.  The one exchange sits after the path, in the
attention output projection (``o_proj``, src/modeling_llama.py:286): it becomes
row-parallel, each rank multiplying its heads' attention output by its column
slice of W_o, and the partial products are summed across ranks with one
all-reduce per layer (NCCL over NVLink).

The reference has no tensor parallelism (layers are placed whole on GPUs with
``device_map="auto"``, scripts/profiling.py:220); this module is the split that
BASELINE's 1/2/4/8-GPU decode configuration asks for.
"""
from __future__ import annotations

import torch

from .dist import kv_head_shard
from .gate import GatingPredictor


def shard_gate(gp: GatingPredictor, h0: int, h1: int) -> GatingPredictor:
    """A gate holding KV heads [h0, h1) of ``gp``.

    Both convolutions are grouped by KV head (src/modeling_layers.py:148-160), so a
    head's parameters are its own rows of conv1 / conv2 and the sliced gate scores
    those heads exactly as the full one does."""
    Hk = gp.num_kv_heads
    if not 0 <= h0 < h1 <= Hk:
        raise ValueError(f"head range [{h0}, {h1}) outside 0..{Hk}")
    g_act = "silu" if gp.act & 1 else "gelu"
    out = GatingPredictor(gp.head_dim, h1 - h0, gp.g_inputs, g_act, gp.inner_dim / gp.head_dim, gp.g_epsilon,
                          gp.g_rms, gp.g_fast_path)
    out = out.to(device=gp.conv1.weight.device, dtype=gp.conv1.weight.dtype)
    inner = gp.inner_dim
    with torch.no_grad():
        out.conv1.weight.copy_(gp.conv1.weight[h0 * inner:h1 * inner])
        out.conv1.bias.copy_(gp.conv1.bias[h0 * inner:h1 * inner])
        out.conv2.weight.copy_(gp.conv2.weight[h0:h1])
        out.conv2.bias.copy_(gp.conv2.bias[h0:h1])
        for name in ("pre_key_norm", "post_key_norm", "value_norm"):
            src = getattr(gp, name)
            if hasattr(src, "weight"):
                getattr(out, name).weight.copy_(src.weight)
    return out


def shard_o_proj(weight: torch.Tensor, q0: int, q1: int, head_dim: int) -> torch.Tensor:
    """Columns of W_o (hidden, Hq * D) that multiply query heads [q0, q1): the row-parallel slice."""
    return weight[:, q0 * head_dim:q1 * head_dim].contiguous()


class KVHeadParallelAttention:
    """One layer's attention for this rank's KV heads + the row-parallel ``o_proj`` + the sum over ranks.

    ``attn`` is an attention module prepared with :func:`wgkv.attach` whose ``g_predictors``
    holds this rank's heads (:func:`shard_gate`); its cache (``past_key_value``) is this rank's
    own pool.  ``o_proj_shard`` is (hidden, Hq_local * D) (:func:`shard_o_proj`).  ``group`` is
    the process group of the ranks sharing the layer; ``reduce=False`` returns this rank's
    partial product instead (the caller sums, e.g. a one-GPU emulation of several ranks).

    With ``timers`` set to a dict, per-call CUDA events are recorded for the phases
    ``attn``, ``o_proj`` and ``all_reduce`` (read them with :meth:`breakdown` after a sync).
    """

    def __init__(self, attn, o_proj_shard: torch.Tensor, group=None, reduce: bool = True):
        self.attn = attn
        self.w = o_proj_shard
        self.group = group
        self.reduce = reduce
        self.timers = None

    def _mark(self, key, start):
        if self.timers is None:
            return None
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        if start is not None:
            self.timers.setdefault(key, []).append((start, e))
        return e

    def __call__(self, past_key_value, input_shape, query_states, pre_key, key_states, value_states, out=None):
        """Inputs as ``self_attn_forward_patch`` takes them, for this rank's heads: query_states
        (B, Hq_local, T, D), pre_key / key_states / value_states (B, Hk_local, T, D).  Returns the
        o_proj output summed over the ranks, (B * T, hidden) (written into ``out`` when given)."""
        import torch.distributed as dist
        B, T = input_shape
        t0 = self._mark("attn", None)
        o, _, _ = self.attn.self_attn_forward_patch(self.attn, 3, None, past_key_value, input_shape, query_states,
                                                    pre_key, key_states, value_states)
        t1 = self._mark("attn", t0)
        a = o.reshape(B * T, -1)
        if a.shape[1] != self.w.shape[1]:
            raise ValueError(f"attention width {a.shape[1]} != o_proj shard width {self.w.shape[1]}")
        y = out if out is not None else torch.empty(B * T, self.w.shape[0], dtype=a.dtype, device=a.device)
        torch.matmul(a, self.w.t(), out=y)
        t2 = self._mark("o_proj", t1)
        if self.reduce and dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1:
            dist.all_reduce(y, group=self.group)
        self._mark("all_reduce", t2)
        return y

    def breakdown(self):
        """{phase: [ms per call]} of the recorded events (call after a synchronize)."""
        return {k: [a.elapsed_time(b) for a, b in v] for k, v in (self.timers or {}).items()}


def shard_layer(attn_full_gate: GatingPredictor, o_proj_weight: torch.Tensor, num_q_heads: int, rank: int,
                world: int, make_attn, group=None, reduce: bool = True) -> KVHeadParallelAttention:
    """Build this rank's :class:`KVHeadParallelAttention` from a layer's full gate and W_o.

    ``make_attn(gate)`` returns the attached attention module for the sharded gate (it sets the
    layer index, head_dim, scaling and config of the rank's pool)."""
    Hk = attn_full_gate.num_kv_heads
    (h0, h1), (q0, q1) = kv_head_shard(Hk, num_q_heads, rank, world)
    attn = make_attn(shard_gate(attn_full_gate, h0, h1))
    return KVHeadParallelAttention(attn, shard_o_proj(o_proj_weight, q0, q1, attn_full_gate.head_dim), group=group,
                                   reduce=reduce)
