"""Helpers for the GPU parity tests (numpy oracle arrays <-> torch bf16)."""
import numpy as np
import torch


def to_bf16(x, device="cuda"):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(device=device, dtype=torch.bfloat16)


def to_np(t):
    return t.detach().float().cpu().numpy()


def bits(t):
    """uint16 bf16 bit patterns of a bf16 tensor."""
    return t.detach().cpu().view(torch.int16).numpy().view(np.uint16)
