"""Per-device state shared by the ops: error word, scratch workspaces, streams.

Workspaces are cached per (device, stream, purpose) and only grow.  Their
leading counters must be zero when a kernel starts and the kernels leave them
zero; a cached buffer records how many leading bytes are known to be zero, and
a call that needs a longer counter prefix (more heads, more rows) zeroes the
extra bytes first, since they may hold an earlier call's partial results.
After a call only its own prefix is known to be zero.
"""
from __future__ import annotations

import torch

from ._lib import ERR_BITS, lib

_err_words: dict = {}
_workspaces: dict = {}


def require_cuda(t: torch.Tensor, name: str):
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (this library has no CPU path)")


def stream_ptr(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def err_word(device) -> torch.Tensor:
    d = torch.device(device)
    key = d.index if d.index is not None else torch.cuda.current_device()
    w = _err_words.get(key)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", key))
        _err_words[key] = w
    return w


def check_errors(device=None, reset: bool = True):
    """Synchronise and raise AssertionError if a kernel flagged an error.

    The device-side capacity checks mirror the reference's asserts
    (src/modeling_layers.py:1313-1321, :683-686, :702-704), so the raised type
    is the same."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    w = err_word(dev)
    v = int(w.item())
    if v:
        if reset:
            w.zero_()
        msgs = [m for bit, m in ERR_BITS.items() if v & bit]
        raise AssertionError("wgkv device error: " + "; ".join(msgs))


def workspace(device, purpose: str, nbytes: int, zero_prefix: int = 0) -> torch.Tensor:
    d = torch.device(device)
    key = (d.index, torch.cuda.current_stream(d).cuda_stream, purpose)
    ent = _workspaces.get(key)
    if ent is None or ent[0].numel() < nbytes:
        ws = torch.empty(max(nbytes, zero_prefix, 256), dtype=torch.uint8, device=d)
        zeroed = 0
    else:
        ws, zeroed = ent
    if zero_prefix > zeroed:
        # stream-ordered: runs after every earlier user of this buffer on this stream
        ws[zeroed:zero_prefix].zero_()
    # this call's kernels may write anything past its own prefix and leave the prefix zero
    _workspaces[key] = (ws, zero_prefix)
    return ws


def num_sms() -> int:
    return int(lib.wgkv_num_sms())
