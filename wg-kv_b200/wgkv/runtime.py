"""Per-device state shared by the ops: error word, scratch workspaces, streams.

Workspaces are cached per (device, stream, purpose) and only grow.  Their
leading counters are zeroed once at allocation; the kernels leave them zero.
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
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=d)
        if zero_prefix:
            ws[:zero_prefix].zero_()
        _workspaces[key] = ws
    return ws


def num_sms() -> int:
    return int(lib.wgkv_num_sms())
