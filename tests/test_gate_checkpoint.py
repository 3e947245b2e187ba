"""Gate checkpoints in the reference's format load into wgkv.GatingPredictor; the oracle and the CUDA
gate reproduce the reference's scores for them (fixture from the reference's own GatingPredictor)."""
import numpy as np
import pytest
import torch

from golden_cases import O, load


def _state():
    z = load("gate_ckpt")
    return z, {k: torch.from_numpy(O.from_bf16_bits(v)).to(torch.bfloat16) for k, v in z.items()
               if k.startswith("model.")}


def _gates(wgkv):
    return [wgkv.GatingPredictor(64, 2, ["pre_k", "post_k"], "gelu", 1.5, 1e-3, True, True).to(torch.bfloat16)
            for _ in range(2)]


def test_checkpoint_keys_load_strict():
    import wgkv
    z, st = _state()
    gates = _gates(wgkv)
    used = wgkv.load_gate_checkpoint(gates, st)
    assert sorted(used) == sorted(st)
    for i, g in enumerate(gates):
        for k, v in g.state_dict().items():
            assert torch.equal(v, st[f"model.layers.{i}.self_attn.g_predictors.{k}"])
    with pytest.raises((KeyError, ValueError)):
        wgkv.load_gate_checkpoint([wgkv.GatingPredictor(64, 2, ["pre_k"], "gelu", 1.5, 1e-3, True, True)], st)


def test_oracle_rms_gate_matches_reference_scores():
    z, st = _state()
    for l in range(2):
        p = f"model.layers.{l}.self_attn.g_predictors."
        f = lambda k: st[p + k].float().numpy()
        params = O.GateParams(w1=f("conv1.weight").reshape(2, 96, 128), b1=f("conv1.bias").reshape(2, 96),
                              w2=f("conv2.weight").reshape(2, 96), b2=f("conv2.bias"), inputs=("pre_k", "post_k"),
                              rms=True, norms={"pre_k": f("pre_key_norm.weight"), "post_k": f("post_key_norm.weight")})
        s = O.gate_scores(params, pre_key=O.from_bf16_bits(z[f"pre_k_{l}"]), post_key=O.from_bf16_bits(z[f"post_k_{l}"]))
        ref = O.from_bf16_bits(z[f"scores_{l}"])
        assert (O.bf16_bits(s) != O.bf16_bits(ref)).sum() <= 1


@pytest.mark.gpu
def test_cuda_gate_from_checkpoint_matches_reference_scores():
    import wgkv
    z, st = _state()
    gates = [g.cuda() for g in _gates(wgkv)]
    wgkv.load_gate_checkpoint(gates, st)
    for l in range(2):
        pk = torch.from_numpy(O.from_bf16_bits(z[f"pre_k_{l}"])).cuda().bfloat16()
        kk = torch.from_numpy(O.from_bf16_bits(z[f"post_k_{l}"])).cuda().bfloat16()
        s = gates[l](pk, kk, None)
        torch.cuda.synchronize()
        got = s.cpu().view(torch.int16).numpy().view(np.uint16)
        assert (got != z[f"scores_{l}"]).sum() <= 1
