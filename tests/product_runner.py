"""Run a golden case through the product API (telescope_cache_b200) on CUDA,
returning the same keys as the fixture / the oracle."""

import numpy as np
import torch

import cases as C
import telescope_cache_b200 as T

DT = {"fp32": torch.float32, "bf16": torch.bfloat16}


def to_dev(inp, dtype, device="cuda"):
    return {k: torch.from_numpy(np.ascontiguousarray(v)).to(device=device, dtype=dtype)
            for k, v in inp.items()}


def _tree(c, t, g, n=None):
    L = len(g["fmap"])
    sl = slice(None) if n is None else slice(0, n)
    kw = {}
    if c["conv"]:
        kw.update(k_conv_weight=t["kcw"], v_conv_weight=t["vcw"])
    if c["weights"] == "linear":
        kw.update(x=t["x"][:, sl], w_proj=t["w_proj"])
    return T.build_dyadic_summaries(t["q"][:, sl], t["k"][:, sl], t["v"][:, sl], L, **kw)


def _pos(c, t, g, n_pos):
    if c["position"] == "rope":
        cos, sin = T.rope_tables(n_pos, g["Dk"], device="cuda")
        return dict(position_mode="rope", rope_cos=cos, rope_sin=sin)
    if c["position"] == "relative":
        return dict(position_mode="relative", relative_states=t["states"],
                    relative_proj=t["rel_proj"])
    return {}


def f64(x):
    return x.detach().double().cpu().numpy()


def product_tree_vjp(c, inp=None):
    """Phase-1 VJP through the product's autograd path: the packed levels of
    build_dyadic_summaries reduced against the seeded upstream gradients."""
    g = C.GEOS[c["geo"]]
    inp = C.make_inputs(c) if inp is None else inp
    dt = DT[c["dtype"]]
    t = to_dev(inp, dt)
    up = to_dev(C.make_tree_grads(c), dt)
    names = ["q", "k", "v"] + (["kcw", "vcw"] if c["conv"] else []) + \
        (["x", "w_proj"] if c["weights"] == "linear" else [])
    leaves = {n_: t[n_].clone().requires_grad_(True) for n_ in names}
    kw = {}
    if c["conv"]:
        kw.update(k_conv_weight=leaves["kcw"], v_conv_weight=leaves["vcw"])
    if c["weights"] == "linear":
        kw.update(x=leaves["x"], w_proj=leaves["w_proj"])
    kl, vl, wl = T.build_dyadic_summaries(leaves["q"], leaves["k"], leaves["v"], len(g["fmap"]),
                                          detach_weights=c.get("detach", False), **kw)
    kp, vp, wp = torch.cat(kl, 1), torch.cat(vl, 1), torch.cat(wl, 1)[..., 0]
    loss = ((kp.float() * up["dk"].float()).sum() + (vp.float() * up["dv"].float()).sum()
            + (wp.float() * up["dw"].float()).sum())
    loss.backward()
    return {"d" + n_: (f64(x_.grad) if x_.grad is not None else np.zeros(tuple(x_.shape)))
            for n_, x_ in leaves.items()}


def product_case(c, inp=None, impl=None):
    if c["kind"] == "treevjp":
        return product_tree_vjp(c, inp)
    g = C.GEOS[c["geo"]]
    inp = C.make_inputs(c) if inp is None else inp
    t = to_dev(inp, DT[c["dtype"]])
    res = {}
    with torch.no_grad():
        kl, vl, wl = _tree(c, t, g)
        packed = T.pack_levels(kl, vl)
        if c["kind"] == "tree":
            res["k_packed"] = f64(packed.k)
            res["v_packed"] = f64(packed.v)
            res["w_packed"] = f64(torch.cat(wl, dim=1))[..., 0]
            res["offsets"] = np.asarray(packed.level_offsets)
            return res
        if c["kind"] in ("fwd", "bwd"):
            pos = _pos(c, t, g, g["N"])
            out, lse = T.multilevel_attention_forward(t["q"], packed, g["fmap"], g["cache"],
                                                      softcap=c["softcap"], impl=impl, **pos)
            res["out"], res["lse"] = f64(out), f64(lse)
            if c["sink"]:
                o_s = T.apply_attention_sink(out, lse, t["sinks"])
                res["out_sink"] = f64(o_s)
                if c["gate"]:
                    res["out_gate"] = f64(T.apply_output_gate(o_s, t["x"], t["gate_w"]))
            if c["kind"] == "fwd":
                return res
            dout, dlse = t["dout"], None
            if c["sink"]:
                dout, dlse, dsinks = T.attention_sink_backward(out, lse, t["sinks"], dout)
                res["dout_pre"], res["dlse"], res["dsinks"] = f64(dout), f64(dlse), f64(dsinks)
            dq, dk, dv, dpos, _ = T.multilevel_attention_backward(
                t["q"], packed, out, lse, dout, g["fmap"], g["cache"], softcap=c["softcap"],
                dlse=dlse, impl=impl, **pos)
            res["dq"], res["dk_packed"], res["dv_packed"] = f64(dq), f64(dk), f64(dv)
            if dpos is not None:
                res["dpos"] = f64(dpos)
            return res
        # decode
        N, m = g["N"], c["tail"]
        n0 = N - m
        kl0, vl0, wl0 = _tree(c, t, g, n0)
        ikw = {}
        if c["conv"]:
            ikw = dict(k_pre_conv=t["k"][:, :n0], v_pre_conv=t["v"][:, :n0],
                       conv_kernel_size=c["conv"])
        st = T.init_decode_state(kl0, vl0, wl0, g["fmap"], g["cache"], **ikw)
        cos = sin = None
        if c["position"] == "rope":
            cos, sin = T.rope_tables(N, g["Dk"], device="cuda")
        outs, lses = [], []
        for i in range(m):
            ti = n0 + i
            sl = slice(ti, ti + 1)
            o, lse = T.decode_step(
                t["x"][:, sl], t["q"][:, sl], t["k"][:, sl], t["v"][:, sl], st,
                weight_mode=c["weights"], w_proj=t.get("w_proj"),
                k_conv_weight=t.get("kcw"), v_conv_weight=t.get("vcw"), softcap=c["softcap"],
                position_mode=c["position"], rope_cos=cos, rope_sin=sin,
                relative_weight=t.get("rel_w"), relative_proj=t.get("rel_proj"),
                sinks=t.get("sinks"), gate_weight=t.get("gate_w"))
            outs.append(f64(o))
            lses.append(f64(lse))
        res["out"] = np.concatenate(outs, axis=1)
        res["lse"] = np.concatenate(lses, axis=1)
        res["ring_k"], res["ring_v"] = f64(st.k), f64(st.v)
        res["ring_w"] = f64(st.w)[..., 0]
        res["caps"] = np.asarray(st.caps)
        if c["conv"]:
            res["conv_k"], res["conv_v"] = f64(st.conv_k), f64(st.conv_v)
        return res
