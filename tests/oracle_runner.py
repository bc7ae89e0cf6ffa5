"""Run the CPU oracle on a golden case: the same keys the fixture stores.

Test infrastructure shared by the oracle-pinning tests (CPU) and the CUDA
parity tests (GPU).
"""

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")
if GOLDEN not in sys.path:
    sys.path.insert(0, GOLDEN)

import cases as C  # noqa: E402
from oracle import numerics as O  # noqa: E402
from oracle import schedule as S  # noqa: E402


def load_golden(name):
    z = np.load(os.path.join(GOLDEN, name + ".npz"))
    return {k: z[k] for k in z.files}


def oracle_tree(c, inp, g, store=O.identity):
    L = len(g["fmap"])
    k, v = inp["k"], inp["v"]
    B, N, Hkv, Dk = k.shape
    Dv = v.shape[-1]
    if c["conv"]:
        k = store(O.short_conv(k.reshape(B, N, Hkv * Dk), inp["kcw"])).reshape(B, N, Hkv, Dk)
        v = store(O.short_conv(v.reshape(B, N, Hkv * Dv), inp["vcw"])).reshape(B, N, Hkv, Dv)
    if c["weights"] == "linear":
        w = O.linear_weights(inp["x"], inp["w_proj"])
    else:
        w = O.qk_weights(inp["q"], k)
    return O.build_tree(k, v, w, L, store=store)


def positional(c, inp, g, n_pos):
    if c["position"] == "rope":
        cos, sin = O.rope_tables(n_pos, g["Dk"])
        return O.Positional("rope", cos=cos, sin=sin)
    if c["position"] == "relative":
        return O.Positional("relative", states=inp["states"], proj=inp["rel_proj"])
    return O.Positional()


def oracle_tree_vjp(c, inp=None):
    """The float64 Phase-1 VJP of a treevjp case (upstream gradients from
    make_tree_grads)."""
    g = C.GEOS[c["geo"]]
    inp = C.make_inputs(c) if inp is None else inp
    up = C.make_tree_grads(c)
    kw = {}
    if c["conv"]:
        kw.update(k_conv_weight=inp["kcw"], v_conv_weight=inp["vcw"])
    if c["weights"] == "linear":
        kw.update(x=inp["x"], w_proj=inp["w_proj"])
    return O.build_tree_vjp(inp["q"], inp["k"], inp["v"], len(g["fmap"]), up["dk"], up["dv"], up["dw"],
                            detach_weights=c.get("detach", False), **kw)


def oracle_case(c, inp=None, store=O.identity):
    if c["kind"] == "treevjp":
        return oracle_tree_vjp(c, inp)
    g = C.GEOS[c["geo"]]
    inp = C.make_inputs(c) if inp is None else inp
    res = {}
    kl, vl, wl = oracle_tree(c, inp, g, store)
    if c["kind"] == "tree":
        res["k_packed"] = O.pack(kl)
        res["v_packed"] = O.pack(vl)
        res["w_packed"] = O.pack(wl)
        res["offsets"] = np.asarray(S.level_offsets(g["N"], len(kl)))
        return res
    if c["kind"] in ("fwd", "bwd"):
        pos = positional(c, inp, g, g["N"])
        out, lse = O.forward(inp["q"], kl, vl, g["fmap"], g["cache"], c["softcap"], pos, store)
        res["out"], res["lse"] = out, lse
        if c["sink"]:
            res["out_sink"] = O.sink_forward(out, lse, inp["sinks"])
            if c["gate"]:
                res["out_gate"] = O.output_gate(res["out_sink"], inp["x"], inp["gate_w"])
        if c["kind"] == "fwd":
            return res
        dout, dlse = inp["dout"], None
        if c["sink"]:
            dout, dlse, dsinks = O.sink_backward(out, lse, inp["sinks"], dout)
            res["dout_pre"], res["dlse"], res["dsinks"] = dout, dlse, dsinks
        dq, dkl, dvl, drel = O.backward(inp["q"], kl, vl, out, lse, dout, g["fmap"], g["cache"],
                                        c["softcap"], pos, dlse=dlse, store=store)
        res["dq"], res["dk_packed"], res["dv_packed"] = dq, O.pack(dkl), O.pack(dvl)
        if drel is not None:
            res["dpos"] = drel
        return res
    # decode
    N, m = g["N"], c["tail"]
    n0 = N - m
    inp0 = {k: (v[:, :n0] if k in ("q", "k", "v", "x") else v) for k, v in inp.items()}
    g0 = dict(g, N=n0)
    kl0, vl0, wl0 = oracle_tree(c, inp0, g0, store)
    st = O.init_decode_state(kl0, vl0, wl0, g["fmap"], g["cache"],
                             k_pre=inp0["k"] if c["conv"] else None,
                             v_pre=inp0["v"] if c["conv"] else None,
                             kernel_size=c["conv"] or None, store=store)
    cos = sin = None
    if c["position"] == "rope":
        cos, sin = O.rope_tables(N, g["Dk"])
    outs, lses = [], []
    for i in range(m):
        ti = n0 + i
        sl = slice(ti, ti + 1)
        lin = c["weights"] == "linear"
        O.advance(st, inp["q"][:, sl], inp["k"][:, sl], inp["v"][:, sl],
                  x_t=inp["x"][:, sl] if lin else None, w_proj=inp.get("w_proj") if lin else None,
                  kcw=inp.get("kcw") if c["conv"] else None,
                  vcw=inp.get("vcw") if c["conv"] else None, store=store)
        if c["position"] == "rope":
            pos = O.Positional("rope", cos=cos, sin=sin)
        elif c["position"] == "relative":
            states = (inp["x"][:, sl] @ inp["rel_w"].astype(np.float64).T).reshape(
                inp["x"].shape[0], 1, g["Hq"], -1)
            pos = O.Positional("relative", states=states, proj=inp["rel_proj"])
        else:
            pos = O.Positional()
        out, lse = O.decode_attend(st, inp["q"][:, sl], c["softcap"], pos, store)
        if c["sink"]:
            out = O.sink_forward(out, lse, inp["sinks"])
        if c["gate"]:
            out = O.output_gate(out, inp["x"][:, sl], inp["gate_w"])
        outs.append(out)
        lses.append(lse)
    res["out"] = np.concatenate(outs, axis=1)
    res["lse"] = np.concatenate(lses, axis=1)
    res["ring_k"], res["ring_v"], res["ring_w"] = st.k, st.v, st.w
    res["caps"] = np.asarray(st.caps)
    if c["conv"]:
        res["conv_k"], res["conv_v"] = st.conv_k, st.conv_v
    return res
