"""Generate the golden fixtures in this directory by running the REFERENCE
implementation (Knarf04/telescope_cache ``reference.py`` and
``telescoping_attn/range_spec.py``) on the seeded cases of ``cases.py``.

Run from the repository root, in a container where the reference is mounted,
naming its checkout with --reference or the TC_REFERENCE_ROOT environment
variable:

    python tests/golden/make_golden.py --reference <reference checkout>

The reference expects to be importable as package ``telescope_cache`` with a
top-level ``range_spec`` module; this script builds that package as a
directory of symlinks under a temporary directory (nothing is copied) and
imports it from there.  Floating-point cases run the reference in float32 on
the (bf16-rounded, for bf16 cases) inputs: that is the parity target for both
precisions.  Only outputs are stored; inputs are re-created from the seed.
"""

import argparse
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import cases as C  # noqa: E402


def import_reference(root):
    tmp = tempfile.mkdtemp(prefix="tc_ref_shim_")
    pkg = os.path.join(tmp, "telescope_cache")
    os.makedirs(pkg)
    for name in ("reference.py", "minimal_reference.py", "telescoping_attn", "fms", "test"):
        os.symlink(os.path.join(root, name), os.path.join(pkg, name))
    os.symlink(os.path.join(root, "telescoping_attn", "range_spec.py"),
               os.path.join(pkg, "range_spec.py"))
    open(os.path.join(pkg, "__init__.py"), "w").close()
    sys.path.insert(0, tmp)
    import telescope_cache.range_spec as rs
    import telescope_cache.reference as ref
    return rs, ref


def t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))


def n(x):
    return x.detach().float().numpy()


def run_tree(ref, c, inp, g):
    L = len(g["fmap"])
    kw = {}
    if c["conv"]:
        kw.update(k_conv_weight=t(inp["kcw"]), v_conv_weight=t(inp["vcw"]))
    if c["weights"] == "linear":
        kw.update(x=t(inp["x"]), w_proj=t(inp["w_proj"]))
    return ref.build_dyadic_summaries(t(inp["q"]), t(inp["k"]), t(inp["v"]), L, **kw)


def positional(ref, c, inp, g, n_pos):
    if c["position"] == "rope":
        cos, sin = ref.rope_tables(n_pos, g["Dk"])
        return dict(position_mode="rope", rope_cos=cos, rope_sin=sin)
    if c["position"] == "relative":
        return dict(position_mode="relative", relative_states=t(inp["states"]),
                    relative_proj=t(inp["rel_proj"]))
    return {}


def gen_tree_vjp(ref, c):
    """Phase-1 VJP: the reference's forward tree under autograd (float32),
    reduced against the seeded upstream gradients of the packed k, v, w."""
    import torch
    g = C.GEOS[c["geo"]]
    inp = C.make_inputs(c)
    up = C.make_tree_grads(c)
    leaves = {k_: t(inp[k_]).requires_grad_(True) for k_ in ("q", "k", "v")}
    kw = {}
    if c["conv"]:
        leaves["kcw"] = t(inp["kcw"]).requires_grad_(True)
        leaves["vcw"] = t(inp["vcw"]).requires_grad_(True)
        kw.update(k_conv_weight=leaves["kcw"], v_conv_weight=leaves["vcw"])
    if c["weights"] == "linear":
        leaves["x"] = t(inp["x"]).requires_grad_(True)
        leaves["w_proj"] = t(inp["w_proj"]).requires_grad_(True)
        kw.update(x=leaves["x"], w_proj=leaves["w_proj"])
    kl, vl, wl = ref.build_dyadic_summaries(leaves["q"], leaves["k"], leaves["v"], len(g["fmap"]),
                                            detach_weights=c.get("detach", False), **kw)
    kp, vp, wp = torch.cat(kl, 1), torch.cat(vl, 1), torch.cat(wl, 1)[..., 0]
    loss = (kp * t(up["dk"])).sum() + (vp * t(up["dv"])).sum() + (wp * t(up["dw"])).sum()
    loss.backward()
    out = {}
    for k_, leaf in leaves.items():
        out["d" + k_] = n(leaf.grad) if leaf.grad is not None else np.zeros(leaf.shape, np.float32)
    return out


def gen_case(rs, ref, c):
    import torch
    if c["kind"] == "treevjp":
        return gen_tree_vjp(ref, c)
    g = C.GEOS[c["geo"]]
    inp = C.make_inputs(c)
    out = {}
    with torch.no_grad():
        kl, vl, wl = run_tree(ref, c, inp, g)
        packed = ref.pack_levels(kl, vl)
        if c["kind"] == "tree":
            out["k_packed"] = n(packed.k)
            out["v_packed"] = n(packed.v)
            out["w_packed"] = n(torch.cat(wl, dim=1))[..., 0]
            out["offsets"] = np.asarray(packed.level_offsets, dtype=np.int64)
            return out
        if c["kind"] in ("fwd", "bwd"):
            pos = positional(ref, c, inp, g, g["N"])
            o, lse = ref.multilevel_attention_forward(
                t(inp["q"]), packed, g["fmap"], g["cache"], softcap=c["softcap"], **pos)
            out["out"], out["lse"] = n(o), n(lse)
            if c["sink"]:
                o_s = ref.apply_attention_sink(o, lse, t(inp["sinks"]))
                out["out_sink"] = n(o_s)
                if c["gate"]:
                    out["out_gate"] = n(ref.apply_output_gate(o_s, t(inp["x"]), t(inp["gate_w"])))
            if c["kind"] == "fwd":
                return out
            dout = t(inp["dout"])
            dlse = None
            if c["sink"]:
                dout, dlse, dsinks = ref.attention_sink_backward(o, lse, t(inp["sinks"]), dout)
                out["dout_pre"], out["dlse"], out["dsinks"] = n(dout), n(dlse), n(dsinks)
            dq, dk, dv, dpos, _ = ref.multilevel_attention_backward(
                t(inp["q"]), packed, o, lse, dout, g["fmap"], g["cache"],
                softcap=c["softcap"], dlse=dlse, **pos)
            out["dq"], out["dk_packed"], out["dv_packed"] = n(dq), n(dk), n(dv)
            if dpos is not None:
                out["dpos"] = n(dpos)
            return out
        # decode
        N, m = g["N"], c["tail"]
        n0 = N - m
        c0 = dict(c)
        inp0 = {k: (v[:, :n0] if k in ("q", "k", "v", "x") else v) for k, v in inp.items()}
        g0 = dict(g, N=n0)
        kl0, vl0, wl0 = run_tree(ref, c0, inp0, g0)
        ikw = {}
        if c["conv"]:
            ikw = dict(k_pre_conv=t(inp0["k"]), v_pre_conv=t(inp0["v"]),
                       conv_kernel_size=c["conv"])
        st = ref.init_decode_state(kl0, vl0, wl0, g["fmap"], g["cache"], **ikw)
        outs, lses = [], []
        cos = sin = None
        if c["position"] == "rope":
            cos, sin = ref.rope_tables(N, g["Dk"])
        for i in range(m):
            ti = n0 + i
            sl = slice(ti, ti + 1)
            o, lse = ref.decode_step(
                t(inp["x"][:, sl]), t(inp["q"][:, sl]), t(inp["k"][:, sl]), t(inp["v"][:, sl]),
                st, weight_mode=c["weights"],
                w_proj=t(inp["w_proj"]) if c["weights"] == "linear" else None,
                k_conv_weight=t(inp["kcw"]) if c["conv"] else None,
                v_conv_weight=t(inp["vcw"]) if c["conv"] else None,
                softcap=c["softcap"], position_mode=c["position"], rope_cos=cos, rope_sin=sin,
                relative_weight=t(inp["rel_w"]) if c["position"] == "relative" else None,
                relative_proj=t(inp["rel_proj"]) if c["position"] == "relative" else None,
                sinks=t(inp["sinks"]) if c["sink"] else None,
                gate_weight=t(inp["gate_w"]) if c["gate"] else None)
            outs.append(n(o))
            lses.append(n(lse))
        out["out"] = np.concatenate(outs, axis=1)
        out["lse"] = np.concatenate(lses, axis=1)
        # live ring slots only (dead slots hold stale values by design)
        spec = st.spec(st.t)
        live = np.zeros(st.k.shape[1], dtype=bool)
        for lv in range(spec.num_levels):
            lo, hi = rs.range_bounds(spec, st.t - 1, lv)
            for j in range(lo, hi):
                live[ref.ring_slot(st, lv, j)] = True
        out["ring_live"] = live
        out["ring_k"] = n(st.k)
        out["ring_v"] = n(st.v)
        out["ring_w"] = n(st.w)[..., 0]
        out["caps"] = np.asarray(st.caps, dtype=np.int64)
        if c["conv"]:
            out["conv_k"], out["conv_v"] = n(st.conv_k), n(st.conv_v)
        return out


def gen_schedule(rs, ref, name, N, cache, fmap):
    spec = rs.RangeSpec.from_fmap(fmap, cache, N)
    a = spec.activation_times
    L = spec.num_levels
    if N <= 1024:
        qs = np.arange(N)
    else:
        r = np.random.Generator(np.random.PCG64(N))
        qs = np.unique(np.concatenate([
            np.arange(0, 64), np.asarray(a), np.asarray(a) - 1, np.asarray(a) + 1,
            r.integers(0, N, 3000), np.arange(N - 64, N)]))
        qs = qs[(qs >= 0) & (qs < N)]
    bounds = np.array([[rs.range_bounds(spec, int(q), lv) for lv in range(L)] for q in qs],
                      dtype=np.int64)
    out = dict(qs=qs.astype(np.int64), bounds=bounds, a=np.asarray(a, np.int64),
               offsets=np.asarray(spec.level_offsets(), np.int64),
               span=np.int64(rs.coarsest_lifetime_span(spec)),
               caps=np.asarray(ref.decode_capacities(a, cache), np.int64),
               fmap=np.asarray([fmap[k] for k in sorted(fmap)], np.int64),
               N=np.int64(N), cache=np.int64(cache))
    # hulls over aligned 128-query blocks / 128-node tiles and a few odd widths
    fw, bw = [], []
    for lv in range(L):
        for w in (1, 3, 128):
            for s in range(0, N, max(w, N // 200)):
                e = min(s + w, N)
                fw.append((lv, s, e) + rs.fwd_bounds(spec, s, e, lv))
            nl = spec.level_len(lv)
            for s in range(0, nl, max(w, nl // 200 if nl >= 200 else 1)):
                e = min(s + w, nl)
                bw.append((lv, s, e) + rs.bwd_bounds(spec, s, e, lv))
    out["fwd_hulls"] = np.asarray(fw, np.int64)
    out["bwd_hulls"] = np.asarray(bw, np.int64)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("TC_REFERENCE_ROOT"),
                    help="reference checkout (default: $TC_REFERENCE_ROOT)")
    ap.add_argument("--only", nargs="*")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or TC_REFERENCE_ROOT")
    rs, ref = import_reference(args.reference)
    for c in C.CASES:
        if args.only and c["name"] not in args.only:
            continue
        res = gen_case(rs, ref, c)
        np.savez_compressed(os.path.join(HERE, c["name"] + ".npz"), case=C.case_json(c), **res)
        print("case", c["name"], {k: v.shape for k, v in res.items()})
    for name, N, cache, fmap in C.SCHEDULES:
        if args.only and ("sched_" + name) not in args.only:
            continue
        res = gen_schedule(rs, ref, name, N, cache, fmap)
        np.savez_compressed(os.path.join(HERE, "sched_" + name + ".npz"),
                            case=json.dumps(dict(name=name)), **res)
        print("schedule", name, res["a"].tolist(), int(res["span"]), res["caps"].tolist())


if __name__ == "__main__":
    main()
