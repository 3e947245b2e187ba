"""Shared loader for the ``gate_conv`` fixture (the reference's ``g_fast_path=False`` gate)."""
from golden_cases import O, load

CASES = {"a": (["pre_k"], "gelu", False), "b": (["pre_k", "post_k", "v"], "silu", True)}


def conv_case(name):
    """Returns (params, inputs dict, reference scores, cfg, eps) for fixture case ``name``."""
    z = load("gate_conv")
    inputs, act, rms = CASES[name]
    D, Hk, L, inner = (int(v) for v in z[f"{name}_cfg"])
    f = lambda k: O.from_bf16_bits(z[f"{name}_{k}"])
    I = D * len(inputs)
    norms = {}
    if rms:
        norms = {"pre_k": f("pre_key_norm.weight"), "post_k": f("post_key_norm.weight"), "v": f("value_norm.weight")}
    p = O.GateParams(w1=f("conv1.weight").reshape(Hk, inner, I), b1=f("conv1.bias").reshape(Hk, inner),
                     w2=f("conv2.weight").reshape(Hk, inner), b2=f("conv2.bias"), inputs=tuple(inputs), act=act,
                     rms=rms, norms=norms, fast_path=False, epsilon=float(z[f"{name}_eps"]))
    xs = [O.from_bf16_bits(x) for x in z[f"{name}_x"]]
    ins = {"pre_key": xs[0], "post_key": xs[1], "value": xs[2]}
    return p, ins, O.from_bf16_bits(z[f"{name}_scores"]), (D, Hk, L, inner), float(z[f"{name}_eps"]), z, inputs, act, rms
