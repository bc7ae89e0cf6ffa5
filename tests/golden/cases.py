"""Seeded case definitions shared by the golden-fixture generator and the
tests.

Inputs are regenerated from a numpy PCG64 seed on every machine, so a fixture
stores only the reference's OUTPUTS.  The geometries restate the reference
suite's (``test/test_reference.py:133-146``) plus two head-dim 64/128 shapes
for the tensor-core kernels.
"""

import json

import numpy as np

GEOS = {
    "tiny": dict(B=2, N=8, Hq=4, Hkv=2, Dk=8, Dv=16, fmap={1: 2, 2: 3}, cache=6),
    "evict": dict(B=1, N=64, Hq=4, Hkv=2, Dk=8, Dv=16, fmap={1: 2, 2: 3}, cache=6),
    "evict_gqa3": dict(B=1, N=64, Hq=6, Hkv=2, Dk=8, Dv=8, fmap={1: 2, 2: 3}, cache=6),
    "odd_n": dict(B=1, N=63, Hq=4, Hkv=2, Dk=8, Dv=16, fmap={1: 2, 2: 3}, cache=6),
    "four_levels": dict(B=1, N=96, Hq=8, Hkv=4, Dk=16, Dv=16,
                        fmap={1: 4, 2: 6, 3: 8}, cache=12),
    # config-1 windows (128 per level) at head dim 64
    "d64": dict(B=1, N=1024, Hq=2, Hkv=2, Dk=64, Dv=64,
                fmap={1: 128, 2: 256, 3: 384}, cache=512),
    # BASELINE config 1 exactly: B=1, H=4, T=1024, Dk=Dv=64, 4 levels x 128
    "config1": dict(B=1, N=1024, Hq=4, Hkv=4, Dk=64, Dv=64,
                    fmap={1: 128, 2: 256, 3: 384}, cache=512),
    # head dim 128, GQA 2:1, four levels all live inside N
    "d128": dict(B=1, N=512, Hq=2, Hkv=1, Dk=128, Dv=128,
                 fmap={1: 64, 2: 128, 3: 192}, cache=256),
    # head dim 128 with 1, 4 and 8 query heads per KV head (decode variants)
    "d128_mha": dict(B=2, N=512, Hq=2, Hkv=2, Dk=128, Dv=128,
                     fmap={1: 64, 2: 128, 3: 192}, cache=256),
    "d128_gqa4": dict(B=1, N=512, Hq=4, Hkv=1, Dk=128, Dv=128,
                      fmap={1: 64, 2: 128, 3: 192}, cache=256),
    "d128_gqa8": dict(B=1, N=512, Hq=8, Hkv=1, Dk=128, Dv=128,
                      fmap={1: 64, 2: 128, 3: 192}, cache=256),
    # head dim 128 with a ragged last 64-token chunk and odd level lengths
    "d128_odd": dict(B=2, N=301, Hq=2, Hkv=2, Dk=128, Dv=128,
                     fmap={1: 64, 2: 128, 3: 192}, cache=256),
    # cache 640 (the decode attention splits each head's entries over CTAs)
    "d128_dec": dict(B=2, N=900, Hq=2, Hkv=2, Dk=128, Dv=128,
                     fmap={1: 128, 2: 256, 3: 384, 4: 512}, cache=640),
    # eight levels: merges past one 64-token chunk
    "d128_deep": dict(B=1, N=700, Hq=2, Hkv=2, Dk=128, Dv=128,
                      fmap={l: 64 * l for l in range(1, 8)}, cache=512),
}

EMB, D_REL = 32, 6

# Schedules pinned by the golden range tables: the reference suite's
# SCHEDULE_CONFIGS (test_reference.py:818-826) plus the five BASELINE configs
# (fmap {l: l*W}, cache L*W).
SCHEDULES = [
    ("readme_tiny", 8, 6, {1: 2, 2: 3}),
    ("tiny_evict", 64, 12, {1: 2, 2: 3}),
    ("mid", 400, 40, {1: 8, 2: 12, 3: 16}),
    ("four_small", 300, 40, {1: 4, 2: 6, 3: 10, 4: 11}),
    ("baseline", 128, 512, {1: 64, 2: 72, 3: 80}),
    ("eviction", 1024, 160, {1: 64, 2: 72, 3: 80}),
    ("config1", 1024, 512, {1: 128, 2: 256, 3: 384}),
    ("config2", 8192, 1536, {l: 256 * l for l in range(1, 6)}),
    ("config3", 16384, 4096, {l: 512 * l for l in range(1, 8)}),
    ("config4", 32768 + 1024, 2048, {l: 256 * l for l in range(1, 8)}),
    ("config5", 131072, 10240, {l: 1024 * l for l in range(1, 10)}),
]


def case(name, kind, geo, *, dtype="fp32", weights="qk", conv=0, position="none",
         sink=False, gate=False, softcap=20.0, seed=0, tail=None):
    return dict(name=name, kind=kind, geo=geo, dtype=dtype, weights=weights, conv=conv,
                position=position, sink=sink, gate=gate, softcap=softcap, seed=seed,
                tail=tail)


CASES = [
    # Phase 1 tree
    case("tree_qk_tiny", "tree", "tiny", seed=10),
    case("tree_lin_odd", "tree", "odd_n", weights="linear", seed=11),
    case("tree_conv_four", "tree", "four_levels", conv=3, seed=12),
    case("tree_conv_lin_odd", "tree", "odd_n", conv=4, weights="linear", seed=13),
    case("tree_bf16_d128", "tree", "d128", dtype="bf16", conv=4, seed=14),
    case("tree_bf16_d128_odd", "tree", "d128_odd", dtype="bf16", conv=3, seed=15),
    case("tree_lin_d128_odd", "tree", "d128_odd", dtype="bf16", weights="linear", seed=16),
    case("tree_bf16_d128_deep", "tree", "d128_deep", dtype="bf16", conv=4, seed=17),
    # Phase 2 forward (boundary rows; sink applied post-attention)
    case("fwd_plain_tiny", "fwd", "tiny", seed=100),
    case("fwd_plain_evict", "fwd", "evict", seed=101),
    case("fwd_plain_gqa3", "fwd", "evict_gqa3", seed=102),
    case("fwd_plain_odd", "fwd", "odd_n", seed=103),
    case("fwd_plain_four", "fwd", "four_levels", seed=104),
    case("fwd_linear_odd", "fwd", "odd_n", weights="linear", seed=105),
    case("fwd_conv_four", "fwd", "four_levels", conv=4, seed=106),
    case("fwd_rope_tiny", "fwd", "tiny", position="rope", seed=107),
    case("fwd_rope_evict", "fwd", "evict", position="rope", seed=108),
    case("fwd_rel_tiny", "fwd", "tiny", position="relative", seed=109),
    case("fwd_rel_evict", "fwd", "evict", position="relative", seed=110),
    case("fwd_rel_four", "fwd", "four_levels", position="relative", seed=111),
    case("fwd_sink_evict", "fwd", "evict", sink=True, seed=112),
    case("fwd_gate_tiny", "fwd", "tiny", gate=True, sink=True, seed=113),
    case("fwd_nocap_tiny", "fwd", "tiny", softcap=None, seed=114),
    case("fwd_plain_d64", "fwd", "d64", softcap=None, seed=115),
    case("fwd_rope_d128_bf16", "fwd", "d128", dtype="bf16", position="rope", conv=4,
         weights="linear", sink=True, softcap=30.0, seed=116),
    case("fwd_rel_d128_bf16", "fwd", "d128", dtype="bf16", position="relative",
         sink=True, softcap=50.0, seed=117),
    # Phase 2 backward at the packed boundary
    case("bwd_none_tiny", "bwd", "tiny", seed=300),
    case("bwd_rope_tiny", "bwd", "tiny", position="rope", seed=304),
    case("bwd_rel_tiny", "bwd", "tiny", position="relative", seed=308),
    case("bwd_rel_evict", "bwd", "evict", position="relative", seed=312),
    case("bwd_nocap_tiny", "bwd", "tiny", softcap=None, seed=316),
    case("bwd_rope_sink_tiny", "bwd", "tiny", position="rope", sink=True, seed=324),
    case("bwd_rel_sink_tiny", "bwd", "tiny", position="relative", sink=True, seed=328),
    case("bwd_none_four", "bwd", "four_levels", seed=344),
    case("bwd_none_gqa3", "bwd", "evict_gqa3", seed=345),
    case("bwd_rel_sink_d128_bf16", "bwd", "d128", dtype="bf16", position="relative",
         sink=True, softcap=50.0, seed=346),
    case("bwd_rope_sink_d128_bf16", "bwd", "d128", dtype="bf16", position="rope",
         sink=True, softcap=30.0, seed=347),
    case("bwd_none_d128_bf16", "bwd", "d128", dtype="bf16", softcap=None, seed=348),
    # BASELINE config 1 at its own shape: fp32, qk weights, no position, no softcap
    case("bwd_config1", "bwd", "config1", softcap=None, seed=349),
    # incremental decode: prefill N - tail tokens, decode `tail`
    case("dec_plain_tiny", "decode", "tiny", tail=7, seed=500),
    case("dec_plain_evict", "decode", "evict", tail=40, seed=501),
    case("dec_plain_odd", "decode", "odd_n", tail=62, seed=502),
    case("dec_plain_four", "decode", "four_levels", tail=60, seed=503),
    case("dec_linear_odd", "decode", "odd_n", weights="linear", tail=7, seed=504),
    case("dec_conv_four", "decode", "four_levels", conv=4, tail=30, seed=505),
    case("dec_conv1_tiny", "decode", "tiny", conv=1, tail=3, seed=506),
    case("dec_rope_evict", "decode", "evict", position="rope", tail=20, seed=507),
    case("dec_rel_four", "decode", "four_levels", position="relative", tail=20, seed=508),
    case("dec_full_tiny", "decode", "tiny", weights="linear", conv=4, sink=True, gate=True,
         tail=7, seed=509),
    case("dec_nocap_tiny", "decode", "tiny", softcap=None, tail=3, seed=510),
    # head dim 128, 16-bit rings (the vectorised decode kernel), E = 1, 2, 4, 8
    case("dec_rope_d128_bf16", "decode", "d128_mha", dtype="bf16", weights="linear", conv=4,
         position="rope", sink=True, gate=True, tail=40, seed=511),
    case("dec_rel_d128_bf16", "decode", "d128", dtype="bf16", position="relative", sink=True,
         softcap=50.0, tail=24, seed=512),
    case("dec_plain_gqa4_bf16", "decode", "d128_gqa4", dtype="bf16", conv=4, tail=20, seed=513),
    case("dec_nocap_gqa8_bf16", "decode", "d128_gqa8", dtype="bf16", position="rope",
         softcap=None, tail=16, seed=514),
    # cache 640: the decode attention splits each head's entries over CTAs
    case("dec_rope_split_bf16", "decode", "d128_dec", dtype="bf16", conv=4, position="rope",
         sink=True, gate=True, tail=40, seed=515),
    case("dec_rel_split_bf16", "decode", "d128_dec", dtype="bf16", position="relative",
         tail=24, seed=516),
    # Phase-1 VJP (tree / merge weights / short conv backward): the gradients
    # of q, k, v (and x, w_proj, the conv weights) for seeded upstream
    # gradients of the packed k, v and w levels (make_tree_grads)
    case("vjp_qk_tiny", "treevjp", "tiny", seed=30),
    case("vjp_lin_odd", "treevjp", "odd_n", weights="linear", seed=31),
    case("vjp_conv_four", "treevjp", "four_levels", conv=3, seed=32),
    case("vjp_conv_lin_odd", "treevjp", "odd_n", conv=4, weights="linear", seed=33),
    dict(case("vjp_detach_four", "treevjp", "four_levels", conv=2, seed=34), detach=True),
    case("vjp_bf16_d128", "treevjp", "d128", dtype="bf16", conv=4, seed=35),
    case("vjp_bf16_d128_lin_odd", "treevjp", "d128_odd", dtype="bf16", weights="linear", seed=36),
    case("vjp_bf16_d128_deep", "treevjp", "d128_deep", dtype="bf16", conv=4, seed=37),
]

CASE_BY_NAME = {c["name"]: c for c in CASES}


def _rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def bf16_round(x):
    u = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32)
    u = (u + (((u >> 16) & 1) + 0x7FFF)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def make_inputs(c):
    """All float inputs of case `c` as float32 numpy arrays (bf16 cases are
    already rounded to bf16 values)."""
    g = GEOS[c["geo"]]
    B, N, Hq, Hkv, Dk, Dv = (g[k] for k in ("B", "N", "Hq", "Hkv", "Dk", "Dv"))
    r = _rng(c["seed"])
    f = lambda *s: r.standard_normal(s).astype(np.float32)  # noqa: E731
    inp = dict(q=f(B, N, Hq, Dk), k=f(B, N, Hkv, Dk), v=f(B, N, Hkv, Dv),
               x=f(B, N, EMB), dout=f(B, N, Hq, Dv))
    if c["weights"] == "linear":
        inp["w_proj"] = f(Hkv, EMB) / np.float32(EMB ** 0.5)
    if c["conv"]:
        kc = c["conv"]
        inp["kcw"] = f(Hkv * Dk, kc) / np.float32(kc ** 0.5)
        inp["vcw"] = f(Hkv * Dv, kc) / np.float32(kc ** 0.5)
    if c["position"] == "relative":
        bins = max(8, g["cache"])
        inp["rel_w"] = f(Hq * D_REL, EMB) / np.float32(EMB ** 0.5)
        inp["rel_proj"] = f(D_REL, bins) / np.float32(D_REL ** 0.5)
        inp["states"] = f(B, N, Hq, D_REL)
    if c["sink"]:
        inp["sinks"] = f(Hq)
    if c["gate"]:
        inp["gate_w"] = f(Hq * Dv, EMB) / np.float32(EMB ** 0.5)
    if c["dtype"] == "bf16":
        inp = {k: bf16_round(v) for k, v in inp.items()}
    return inp


def tree_total(c):
    """Packed length of case `c`'s tree (levels 0 .. len(fmap))."""
    g = GEOS[c["geo"]]
    return sum(g["N"] >> l for l in range(len(g["fmap"]) + 1))


def make_tree_grads(c):
    """Seeded upstream gradients of the packed k, v and w levels of a
    treevjp case: dk [B, total, Hkv, Dk], dv [B, total, Hkv, Dv],
    dw [B, total, Hkv] (bf16-rounded for bf16 cases)."""
    g = GEOS[c["geo"]]
    B, Hkv, Dk, Dv = (g[k] for k in ("B", "Hkv", "Dk", "Dv"))
    total = tree_total(c)
    r = _rng(c["seed"] + 1000)
    f = lambda *s: r.standard_normal(s).astype(np.float32)  # noqa: E731
    out = dict(dk=f(B, total, Hkv, Dk), dv=f(B, total, Hkv, Dv), dw=f(B, total, Hkv))
    if c["dtype"] == "bf16":
        out = {k: bf16_round(v) for k, v in out.items()}
    return out


def case_json(c):
    return json.dumps(c, sort_keys=True)
