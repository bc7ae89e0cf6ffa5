"""The dense torch restatement that the GPU autograd tests compare against
(tests/test_gpu_fms_attention.py, tests/test_gpu_attn_dense.py), pinned on
CPU against the float64 oracle composition (projections, conv, merge
weights, tree, forward, sink, gate, output projection) for every position
mode: the restatement is test infrastructure, checked before it checks."""

import math

import numpy as np
import pytest
import torch

import test_gpu_fms_attention as TF
from oracle import numerics as O
from telescope_cache_b200.fms_attention import MultiHeadAttention


@pytest.mark.parametrize("ci", [0, 1, 2])
def test_dense_restatement_matches_oracle(ci):
    c = TF.CASES[ci]
    torch.manual_seed(ci)
    m = MultiHeadAttention(c["emb"], c["D"], c["D"], c["H"], c["Hkv"], fmap=c["fmap"], cache_size=c["cache"],
                           weight_mode=c["weight_mode"], use_kv_short_conv=c["conv"], use_sinks=c["sinks"],
                           use_gate=c["gate"], position_mode=c["pos"])
    P = {}
    for n, p in m.named_parameters():
        s = 0.3 if n.endswith("sconv.weight") or n == "sinks" else 1 / math.sqrt(p.shape[-1])
        P[n] = torch.randn(p.shape, dtype=torch.float64) * s
    B, N, H, Hkv, D = c["B"], c["N"], c["H"], c["Hkv"], c["D"]
    x = torch.randn(B, N, c["emb"], dtype=torch.float64)
    if c["pos"] == "rope":
        cs, sn = O.rope_tables(N, D)
        m._rope = (N, torch.from_numpy(cs).double(), torch.from_numpy(sn).double())
    got = TF._dense(P, x, m).numpy()
    xn = x.numpy()
    Pn = {k: v.numpy() for k, v in P.items()}
    q, k, v = np.split(xn @ Pn["in_proj.weight"].T, [H * D, H * D + Hkv * D], axis=-1)
    if c["conv"]:
        k, v = O.short_conv(k, Pn["k_sconv.weight"]), O.short_conv(v, Pn["v_sconv.weight"])
    q, k, v = q.reshape(B, N, H, D), k.reshape(B, N, Hkv, D), v.reshape(B, N, Hkv, D)
    w = O.linear_weights(xn, Pn["w.weight"]) if c["weight_mode"] == "linear" else O.qk_weights(q, k)
    kl, vl, _ = O.build_tree(k, v, w, len(c["fmap"]))
    if c["pos"] == "rope":
        pos = O.Positional("rope", cos=cs, sin=sn)
    elif c["pos"] == "relative":
        st = (xn @ Pn["relative_weight"].T).reshape(B, N, H, -1)
        pos = O.Positional("relative", states=st, proj=Pn["relative_proj"])
    else:
        pos = O.Positional()
    out, lse = O.forward(q, kl, vl, c["fmap"], c["cache"], m.softcap, pos)
    if c["sinks"]:
        out = O.sink_forward(out, lse, Pn["sinks"])
    if c["gate"]:
        out = O.output_gate(out, xn, Pn["gate_proj.weight"])
    want = out.reshape(B, N, H * D) @ Pn["dense.weight"].T
    assert np.linalg.norm(got - want) <= 1e-12 * np.linalg.norm(want)
