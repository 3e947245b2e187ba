"""KV-head tensor parallelism around the admission path: one process per GPU.

The admission path never exchanges data: a KV head's gate, pages, ring, tables
and attention depend on that head alone.  A model split by KV head therefore
gives each rank whole GQA groups -- its KV heads and their query heads -- and
its own paged pool for them.  The one exchange sits after the path, in the
attention output projection (``o_proj``, src/modeling_llama.py:286): it becomes
row-parallel, each rank multiplying its heads' attention output by its column
slice of W_o, and the partial products are summed across ranks once per layer:
either a GEMM followed by an NCCL all-reduce, or one kernel that computes each
32-column tile of the product and sums the peers' copies of it over NVLink peer
memory as soon as they are published (``PeerGroup``, ``wgkv_oproj_allreduce``).

The reference has no tensor parallelism (layers are placed whole on GPUs with
``device_map="auto"``, scripts/profiling.py:220); this module is the split that
BASELINE's 1/2/4/8-GPU decode configuration asks for.
"""
from __future__ import annotations

import ctypes

import torch

from ._lib import check, lib
from .dist import kv_head_shard
from .gate import GatingPredictor
from .runtime import err_word, stream_ptr

MAX_WORLD = 8  # WGKV_TP_MAX_WORLD


class WgkvPeerGroup(ctypes.Structure):
    """Mirror of ``wgkv_peer_group`` in include/wgkv.h."""
    _fields_ = [("rank", ctypes.c_int32), ("world", ctypes.c_int32), ("max_rows", ctypes.c_int32),
                ("max_cols", ctypes.c_int32), ("partial", ctypes.c_void_p * MAX_WORLD),
                ("flags", ctypes.c_void_p * MAX_WORLD), ("ctr", ctypes.c_void_p)]


_opened: dict = {}  # IPC handle bytes -> [mapped base, users]; an allocation is opened once per process


def _ipc_open(handle: bytes) -> int:
    ent = _opened.get(handle)
    if ent is None:
        base = ctypes.c_void_p()
        check(lib.wgkv_ipc_open(handle, ctypes.byref(base)), "wgkv_ipc_open")
        ent = _opened[handle] = [base.value, 0]
    ent[1] += 1
    return ent[0]


def _ipc_release(handle: bytes):
    ent = _opened.get(handle)
    if ent is None:
        return
    ent[1] -= 1
    if ent[1] == 0:
        lib.wgkv_ipc_close(ent[0])
        del _opened[handle]


class PeerGroup:
    """The buffers of ``wgkv_oproj_allreduce`` for this process's GPU, mapped into every peer.

    One buffer per GPU holds the double-buffered partial products, the tile flags and the epoch
    counter; its CUDA IPC handle is exchanged once over ``group`` (a host-side all-gather) and the
    peers' buffers are mapped here.  Collective: every rank of ``group`` constructs it with the same
    ``max_rows`` / ``max_cols``.  Without an initialised process group it is a group of one (the
    fused call is then the plain GEMM)."""

    def __init__(self, max_rows: int, max_cols: int, group=None, device=None):
        import torch.distributed as dist
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        dist_on = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if dist_on else 0
        self.world = dist.get_world_size(group) if dist_on else 1
        if self.world > MAX_WORLD:
            raise ValueError(f"at most {MAX_WORLD} GPUs per group")
        align = lambda n: (n + 255) // 256 * 256  # noqa: E731
        pb = int(lib.wgkv_tp_partial_bytes(max_rows, max_cols))
        fb = int(lib.wgkv_tp_flag_bytes(max_cols))
        self.buf = torch.zeros(align(pb) + align(fb) + 256, dtype=torch.uint8, device=self.device)
        base = self.buf.data_ptr()
        own = (base, base + align(pb))
        self.struct = WgkvPeerGroup(rank=self.rank, world=self.world, max_rows=max_rows, max_cols=max_cols)
        self.struct.ctr = base + align(pb) + align(fb)
        self._handles = []
        if self.world == 1:
            self.struct.partial[0], self.struct.flags[0] = own
            return
        h = ctypes.create_string_buffer(64)
        off = ctypes.c_size_t()
        check(lib.wgkv_ipc_handle(base, h, ctypes.byref(off)), "wgkv_ipc_handle")
        torch.cuda.synchronize(self.device)  # the zeroed buffer must be visible before a peer maps it
        infos = [None] * self.world
        dist.all_gather_object(infos, (h.raw, off.value, align(pb)), group=group)
        error = None
        try:
            for r, (hr, offr, flag_off) in enumerate(infos):
                if r == self.rank:
                    self.struct.partial[r], self.struct.flags[r] = own
                    continue
                peer_base = _ipc_open(hr) + offr
                self._handles.append(hr)
                self.struct.partial[r] = peer_base
                self.struct.flags[r] = peer_base + flag_off
        except RuntimeError as e:  # every rank still takes part in the agreement below
            error = e
        # all ranks agree on the outcome, so a failure on one rank raises on every rank
        ok = torch.tensor([0 if error else 1], dtype=torch.int32, device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if int(ok.item()) == 0:
            self.close()
            raise RuntimeError(f"peer mapping failed on a rank of the group ({error or 'another rank'})")

    def close(self):
        """Unmap the peers' buffers (after the last call on every rank has completed)."""
        for hr in self._handles:
            _ipc_release(hr)
        self._handles = []

    def oproj_allreduce(self, a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, kernel: bool = False):
        """out (rows, n_out) = sum over the group of a (rows, k) @ w (n_out, k)^T (``wgkv_oproj_allreduce``).

        In a group of one there is nothing to sum and the product is cuBLAS's GEMM unless ``kernel``
        asks for the fused kernel (which then computes the same GEMM)."""
        assert a.dtype == w.dtype == out.dtype == torch.bfloat16 and a.stride(1) == 1 and out.stride(1) == 1
        if self.world == 1 and not kernel:
            return torch.matmul(a, w.t(), out=out)
        w = w if w.is_contiguous() else w.contiguous()
        check(lib.wgkv_oproj_allreduce(a.data_ptr(), a.stride(0), a.shape[0], a.shape[1], w.data_ptr(), w.shape[0],
                                       out.data_ptr(), out.stride(0), ctypes.byref(self.struct),
                                       err_word(a.device).data_ptr(), stream_ptr(a.device)), "wgkv_oproj_allreduce")
        return out


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

    With ``peers`` (a :class:`PeerGroup`) the projection and the sum run as one kernel over NVLink
    peer memory (``wgkv_oproj_allreduce``); otherwise the GEMM is followed by an NCCL all-reduce.

    With ``timers`` set to a dict, per-call CUDA events are recorded for the phases
    ``attn``, ``o_proj`` and ``all_reduce`` (``o_proj_allreduce`` for the fused kernel; read them
    with :meth:`breakdown` after a sync).
    """

    def __init__(self, attn, o_proj_shard: torch.Tensor, group=None, reduce: bool = True, peers=None):
        self.attn = attn
        self.w = o_proj_shard
        self.group = group
        self.reduce = reduce
        self.peers = peers
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
        if self.peers is not None and self.reduce:
            self.peers.oproj_allreduce(a, self.w, y)
            self._mark("o_proj_allreduce", t1)
            return y
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
