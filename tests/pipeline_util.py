"""Build reference-shaped attention "modules" around the golden pipeline cases."""
from types import SimpleNamespace

import numpy as np
import torch

from gpu_util import to_bf16


def make_config(case):
    return SimpleNamespace(num_hidden_layers=case.Ly, num_key_value_heads=case.Hk, num_attention_heads=case.Hq,
                           head_dim=case.D, block_size=case.T, max_total_tokens=case.max_total_tokens,
                           max_tokens_per_head=case.max_tokens_per_head, local_window_size=case.W,
                           g_defer=case.defer, g_threshold=case.threshold)


def make_gate(wgkv, case, l):
    p = case.params[l]
    gp = wgkv.GatingPredictor(case.D, case.Hk, list(case.inputs), case.act, case.inner / case.D, 1e-3, False, True)
    gp = gp.to(device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        gp.conv1.weight.copy_(to_bf16(p.w1.reshape(case.Hk * case.inner, -1, 1)))
        gp.conv1.bias.copy_(to_bf16(p.b1.reshape(-1)))
        gp.conv2.weight.copy_(to_bf16(p.w2.reshape(case.Hk, case.inner, 1)))
        gp.conv2.bias.copy_(to_bf16(p.b2))
    return gp


def make_layers(wgkv, case):
    cfg = make_config(case)
    out = []
    for l in range(case.Ly):
        a = SimpleNamespace(layer_idx=l, head_dim=case.D, scaling=case.D ** -0.5, g_predictors=make_gate(wgkv, case, l))
        wgkv.attach(a, cfg)
        out.append(a)
    return out


def bhld(x):
    """numpy (1, H, L, D) -> cuda bf16 (1, H, L, D) as a transposed view of (1, L, H, D), like HF's layout."""
    t = to_bf16(np.ascontiguousarray(np.transpose(x, (0, 2, 1, 3))))
    return t.transpose(1, 2)
