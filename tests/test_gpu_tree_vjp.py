"""Phase-1 VJP (build_dyadic_summaries through autograd) against the float64
oracle on shapes the golden cases do not reach: trees deeper than one
64-leaf tile (levels above it run on the fp32 scratch), ragged N with an
orphan node on several levels, GQA groups of 8 and 12, head dims that are
not whole 16-byte chunks (the scalar-chunk kernel), no tree at all (L = 0),
head dim 256, upstream gradients missing for some outputs, and the D = 128
16-bit kernel with one and with eight query heads per KV head."""

import zlib

import numpy as np
import pytest
import torch

import telescope_cache_b200 as T
from oracle import numerics as O

pytestmark = pytest.mark.gpu

CASES = {
    # name: B, N, Hq, Hkv, Dk, Dv, L, dtype, weights, conv, detach, grads
    "deep_gqa12": (1, 1000, 12, 1, 64, 64, 9, "bf16", "qk", 0, False, "kvw"),
    "f32_scalar_chunks": (2, 333, 4, 2, 10, 6, 5, "fp32", "qk", 3, False, "kvw"),
    "f32_deep_linear": (1, 777, 2, 2, 32, 32, 8, "fp32", "linear", 2, False, "kvw"),
    "no_tree": (2, 37, 4, 2, 16, 16, 0, "fp32", "qk", 3, False, "kvw"),
    "d256_linear": (1, 2061, 2, 1, 256, 256, 8, "bf16", "linear", 0, False, "kvw"),
    "k_only": (1, 515, 4, 2, 128, 128, 7, "bf16", "qk", 4, False, "k"),
    "w_only_detach": (2, 200, 2, 2, 32, 16, 4, "fp32", "qk", 0, True, "w"),
    # the D = 128 16-bit kernel: one query head per KV head, scratch levels above the tiles
    "d128_qk_deep": (2, 1500, 4, 4, 128, 128, 9, "bf16", "qk", 0, False, "kvw"),
    "d128_f16_gqa8": (1, 700, 8, 1, 128, 128, 5, "f16", "qk", 2, False, "kvw"),
}
DT = {"fp32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _inputs(name):
    B, N, Hq, Hkv, Dk, Dv, L, dt, weights, conv, detach, grads = CASES[name]
    r = np.random.default_rng(zlib.crc32(name.encode()))
    f = lambda *s: r.standard_normal(s).astype(np.float32)  # noqa: E731
    inp = dict(q=f(B, N, Hq, Dk), k=f(B, N, Hkv, Dk), v=f(B, N, Hkv, Dv))
    if weights == "linear":
        inp["x"] = f(B, N, 24)
        inp["w_proj"] = f(Hkv, 24) / np.float32(24 ** 0.5)
    if conv:
        inp["kcw"] = f(Hkv * Dk, conv) / np.float32(conv ** 0.5)
        inp["vcw"] = f(Hkv * Dv, conv) / np.float32(conv ** 0.5)
    total = sum(N >> l for l in range(L + 1))
    up = dict(dk=f(B, total, Hkv, Dk), dv=f(B, total, Hkv, Dv), dw=f(B, total, Hkv))
    tdt = DT[dt]
    # round to the device dtype so both sides start from the same values
    inp = {k: torch.from_numpy(v).to(tdt).float().numpy() for k, v in inp.items()}
    up = {k: torch.from_numpy(v).to(tdt).float().numpy() for k, v in up.items()}
    return inp, up, tdt


@pytest.mark.parametrize("name", sorted(CASES))
def test_tree_vjp_matches_oracle(name):
    B, N, Hq, Hkv, Dk, Dv, L, dt, weights, conv, detach, grads = CASES[name]
    inp, up, tdt = _inputs(name)
    dev = torch.device("cuda")
    leaves = {k: torch.from_numpy(v).to(dev, tdt).requires_grad_(True) for k, v in inp.items()}
    kw = {}
    if conv:
        kw.update(k_conv_weight=leaves["kcw"], v_conv_weight=leaves["vcw"])
    if weights == "linear":
        kw.update(x=leaves["x"], w_proj=leaves["w_proj"])
    kl, vl, wl = T.build_dyadic_summaries(leaves["q"], leaves["k"], leaves["v"], L, detach_weights=detach, **kw)
    kp, vp, wp = torch.cat(kl, 1), torch.cat(vl, 1), torch.cat(wl, 1)[..., 0]
    loss = 0.0
    use = {"k": (kp, "dk"), "v": (vp, "dv"), "w": (wp, "dw")}
    for g in grads:
        t, key = use[g]
        loss = loss + (t.float() * torch.from_numpy(up[key]).to(dev)).sum()
    loss.backward()
    zero = {key: np.zeros_like(up[key]) for key in ("dk", "dv", "dw")}
    ups = {key: (up[key] if key[1] in grads else zero[key]) for key in ("dk", "dv", "dw")}
    want = O.build_tree_vjp(inp["q"], inp["k"], inp["v"], L, ups["dk"], ups["dv"], ups["dw"],
                            x=inp.get("x"), w_proj=inp.get("w_proj"), k_conv_weight=inp.get("kcw"),
                            v_conv_weight=inp.get("vcw"), detach_weights=detach)
    names = {"q": "dq", "k": "dk", "v": "dv", "x": "dx", "w_proj": "dw_proj", "kcw": "dkcw", "vcw": "dvcw"}
    for leaf, key in names.items():
        if leaf not in leaves:
            continue
        g = leaves[leaf].grad
        got = np.zeros(leaves[leaf].shape) if g is None else g.double().cpu().numpy()
        ref = want.get(key, np.zeros_like(got))
        scale = float(np.abs(ref).max()) if ref.size else 0.0
        if dt == "fp32":
            err = np.abs(got - ref).max() if ref.size else 0.0
            assert err <= 1e-4 * max(scale, 1.0), (key, err, scale)
        else:
            # 16-bit inputs: |got - want| <= 2e-2 (|want| + max |want|)
            assert np.all(np.abs(got - ref) <= 2e-2 * (np.abs(ref) + scale) + 1e-6), (key, scale)
