"""Benchmark of the telescoping-attention hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload c3|c5|c2]

A step is one training-layer pass of the hot path over one batch of seeded
synthetic inputs (the reference publishes no dataset): build the dyadic tree
(fused conv / merge weights / merges / packing), Phase-2 forward, attention
sink, sink backward and the Phase-2 backward with the dlse seam.  The default
workload is BASELINE config 3 (B=4, T=16384, H=16, D=128, bf16, qk weights,
relative bias, 8 levels x 512, softcap 50, sink).  Multi-GPU runs shard
(batch x head) units across ranks with no data-path collective: each rank
processes its own config-3 batch (weak scaling).

The metric is visible-entry TFLOP/s: per visible (query, entry) pair and query
head, 4 D FLOPs forward (QK^T and PV) + 10 D backward (five GEMMs); hull
padding, softcap, bias and RoPE are not counted.

``--impl reference`` times the reference's own ``reference.py`` (pure
Python over torch, installed under ``baseline/_ref``, which travels to the
GPU box) on the box's host cores, on a bounded sample of the same workload:
one (batch, head) slice of the workload's schedule and features at a shorter
sequence.  When that install is missing it falls back to the numpy oracle
port and says so.
"""

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    # name: (B, T, H, D, levels, window, weights, position, softcap, sink, conv, d_rel)
    "c3": dict(B=4, T=16384, H=16, D=128, levels=8, W=512, weights="qk", position="relative",
               softcap=50.0, sink=True, conv=0, d_rel=16,
               desc="BASELINE config 3: training-layer fwd+bwd, relative bias, sink"),
    "c5": dict(B=1, T=131072, H=32, D=128, levels=10, W=1024, weights="linear", position="rope",
               softcap=50.0, sink=True, conv=0, d_rel=0,
               desc="BASELINE config 5: long-context fwd+bwd, rope, linear weights, sink"),
    "c2": dict(B=2, T=8192, H=16, D=128, levels=6, W=256, weights="linear", position="rope",
               softcap=30.0, sink=True, conv=4, d_rel=0,
               desc="BASELINE config 2 shape (attention fwd+bwd)"),
    # reduced shapes of the same kernels for ncu captures (a few GB on the device)
    "c3_small": dict(B=1, T=16384, H=4, D=128, levels=8, W=512, weights="qk", position="relative",
                     softcap=50.0, sink=True, conv=0, d_rel=16,
                     desc="config 3 schedule and features at B=1, H=4 (profiling case)"),
    "c5_small": dict(B=1, T=32768, H=4, D=128, levels=10, W=1024, weights="linear", position="rope",
                     softcap=50.0, sink=True, conv=0, d_rel=0,
                     desc="config 5 schedule and features at T=32768, H=4 (profiling case)"),
}
EMB = 2048

# incremental decode after a 32768-token prefill.  The
# config names no softcap; decode_step's default (20.0) is used.
DECODE = dict(B=64, T=32768, H=16, D=128, levels=8, W=256, conv=4, softcap=20.0,
              desc="BASELINE config 4: decode_step after a 32768-token prefill, rope, conv 4, "
                   "sink, gate")
# the same decode schedule and features at B=8, for ncu captures (a few GB on the device)
DECODE_SMALL = dict(DECODE, B=8, desc="config 4 schedule and features at B=8 (profiling case)")


# DRAM bytes per launch of the dominant op (the backward: Pass A + Pass B), from
# the ncu capture of the c3_small case (profiles/attn_kernels_c3_small_full.txt)
# scaled by the 16x (batch, head) units of config 3; traffic is proportional to
# the units.  None where no capture covers the workload.
TRAFFIC = {"c3": 16 * (0.411784e9 + 1.043806e9 + 0.407769e9 + 0.063763e9)}


def schedule(wl):
    fmap = {l: l * wl["W"] for l in range(1, wl["levels"])}
    return fmap, wl["levels"] * wl["W"]


def flops_per_step(wl, total_visible):
    return (4 + 10) * wl["D"] * total_visible * wl["B"] * wl["H"]


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p.get("bf16_tflops", 1590.0), p.get("bf16_tflops_sustained", 1400.0), \
            p.get("hbm_gbs", 6650.0), "measured"
    except Exception:
        return 1590.0, 1400.0, 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clocks / throttle reasons during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        mhz.sort()
        med = mhz[len(mhz) // 2] if mhz else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(mhz)}


def make_inputs(wl, device, seed, rank):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed + 7919 * rank)
    B, T, H, D = wl["B"], wl["T"], wl["H"], wl["D"]
    bf = torch.bfloat16
    inp = dict(
        q=torch.randn(B, T, H, D, generator=g, device=device, dtype=bf),
        k=torch.randn(B, T, H, D, generator=g, device=device, dtype=bf),
        v=torch.randn(B, T, H, D, generator=g, device=device, dtype=bf),
        dout=torch.randn(B, T, H, D, generator=g, device=device, dtype=bf),
    )
    fmap, cache = schedule(wl)
    if wl["sink"]:
        inp["sinks"] = torch.randn(H, generator=g, device=device, dtype=torch.float32)
    if wl["position"] == "relative":
        inp["states"] = (0.02 * torch.randn(B, T, H, wl["d_rel"], generator=g, device=device)).to(bf)
        inp["proj"] = (0.02 * torch.randn(wl["d_rel"], cache, generator=g, device=device)).to(bf)
    if wl["weights"] == "linear":
        inp["x"] = torch.randn(B, T, EMB, generator=g, device=device, dtype=bf)
        inp["w_proj"] = (0.02 * torch.randn(H, EMB, generator=g, device=device)).to(bf)
    if wl["conv"]:
        inp["kcw"] = torch.randn(H * D, wl["conv"], generator=g, device=device) / math.sqrt(wl["conv"])
        inp["vcw"] = torch.randn(H * D, wl["conv"], generator=g, device=device) / math.sqrt(wl["conv"])
    return inp


def run_step(T, wl, inp, fmap, cache, tables, timers=None):
    """One pass of the hot path.  timers: dict of (start, end) CUDA events."""
    import torch
    kw = {}
    if wl["weights"] == "linear":
        kw.update(x=inp["x"], w_proj=inp["w_proj"])
    if wl["conv"]:
        kw.update(k_conv_weight=inp["kcw"], v_conv_weight=inp["vcw"])
    kl, vl, _ = T.build_dyadic_summaries(inp["q"], inp["k"], inp["v"], wl["levels"] - 1, **kw)
    packed = T.pack_levels(kl, vl)
    pos = {}
    if wl["position"] == "relative":
        pos = dict(position_mode="relative", relative_states=inp["states"], relative_proj=inp["proj"])
    elif wl["position"] == "rope":
        pos = dict(position_mode="rope", rope_cos=tables[0], rope_sin=tables[1])
    if timers:
        timers["fwd"][0].record()
    out, lse = T.multilevel_attention_forward(inp["q"], packed, fmap, cache, softcap=wl["softcap"],
                                              **pos)
    if timers:
        timers["fwd"][1].record()
    dout, dlse = inp["dout"], None
    if wl["sink"]:
        _ = T.apply_attention_sink(out, lse, inp["sinks"])
        dout, dlse, _ = T.attention_sink_backward(out, lse, inp["sinks"], inp["dout"])
    if timers:
        timers["bwd"][0].record()
    dq, dk, dv, dpos, _ = T.multilevel_attention_backward(
        inp["q"], packed, out, lse, dout, fmap, cache, softcap=wl["softcap"], dlse=dlse, **pos)
    if timers:
        timers["bwd"][1].record()
    return dq, dk, dv, dpos, out


def vjp_bench(T, wl, inp, grads, args, hbm, flush):
    """Phase-1 VJP (the backward of build_dyadic_summaries) at the workload's
    shapes: the explicit backward from the Phase-2 step's packed dK / dV
    (no weight-level upstream gradient), W warm-up and K timed calls with
    CUDA events, L2 flushed before each.  Algorithmic bytes: the upstream
    gradients and the forward rows every merge reads (children of levels
    0..L-1), q and dq in qk mode, x and dx in linear mode, the level-0
    gradients written once."""
    import torch

    from telescope_cache_b200 import _lib
    from telescope_cache_b200.telescoping_attn import summaries as S
    L = wl["levels"] - 1
    kw = {}
    if wl["weights"] == "linear":
        kw.update(x=inp["x"], w_proj=inp["w_proj"])
    if wl["conv"]:
        kw.update(k_conv_weight=inp["kcw"], v_conv_weight=inp["vcw"])
    kl, vl, wls = T.build_dyadic_summaries(inp["q"], inp["k"], inp["v"], L, **kw)
    packed = T.pack_levels(kl, vl)
    wp = torch.cat(wls, 1)[..., 0]
    dk, dv = grads

    def call():
        return S.build_dyadic_summaries_backward(inp["q"], inp["k"], inp["v"], L, packed.k, packed.v, wp,
                                                 dk, dv, None, **kw)

    for _ in range(max(args.warmup, 1)):
        call()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    n0 = _lib.launch_count()
    for a, b in ev:
        flush.zero_()
        a.record(st)
        call()
        b.record(st)
    torch.cuda.synchronize()
    launches = (_lib.launch_count() - n0) // args.steps
    ms = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
    B, N, H, D = wl["B"], wl["T"], wl["H"], wl["D"]
    total = sum(N >> lv for lv in range(L + 1))
    el = 2  # bf16
    rows = B * H
    nbytes = rows * total * 2 * D * el                   # upstream dK, dV (packed)
    nbytes += rows * (total - (N >> L)) * (2 * D * el + wp.element_size())  # children k, v, w
    nbytes += rows * N * 2 * D * el                      # dk, dv written
    if wl["weights"] == "qk":
        nbytes += 2 * rows * N * D * el                  # q read, dq written
    else:
        nbytes += 2 * B * N * inp["x"].shape[-1] * el    # x read (dw_proj), dx written
    if wl["conv"]:
        nbytes += rows * N * 2 * D * (4 + 4 + el)        # fp32 dk0 / dv0 written and read, pre-conv rows
    achieved = nbytes / (ms * 1e-3) / 1e9
    return {"what": "build_dyadic_summaries_backward (Phase-1 VJP: tree, merge weights"
                    + (", conv" if wl["conv"] else "") + ")",
            "ms": ms, "launches": launches, "bytes": nbytes, "achieved_gbs": achieved, "peak_gbs": hbm,
            "frac": achieved / hbm, "upstream": "the step's packed dK, dV (bf16); no dw upstream"}


def decode_visible(spec, t0, n):
    """Visible entries of the newest query at t0 .. t0 + n - 1."""
    from telescope_cache_b200 import range_spec as R
    return [sum(hi - lo for lo, hi in (R.range_bounds(spec, t, lv) for lv in range(spec.num_levels)))
            for t in range(t0, t0 + n)]


def handoff_bench(T, args, kl, vl, wl, fmap, cache, k_pre, v_pre, conv):
    """The prefill hand-off at config 4: init_decode_state (one tc_decode_init
    launch places every ring slot; the conv history is two small copies),
    W warm-up and K timed public calls with CUDA events.  Its inputs and the
    2 GB of rings it writes exceed L2, so no flush is needed.  Algorithmic
    bytes: every ring slot written once (k, v, w) and every live node read
    once."""
    import torch

    from telescope_cache_b200 import _lib
    from telescope_cache_b200 import range_spec as R

    def call():
        return T.init_decode_state(kl, vl, wl, fmap, cache, k_pre_conv=k_pre, v_pre_conv=v_pre,
                                   conv_kernel_size=conv)

    for _ in range(max(args.warmup, 1)):
        st = call()
    del st
    torch.cuda.synchronize()
    cur = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    n0 = _lib.launch_count()
    for a, b in ev:
        a.record(cur)
        st = call()
        b.record(cur)
        del st
    torch.cuda.synchronize()
    launches = (_lib.launch_count() - n0) // args.steps
    ms = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
    B, N, H, Dk = kl[0].shape
    Dv = vl[0].shape[-1]
    el, wel = kl[0].element_size(), wl[0].element_size()
    caps = T.decode_capacities(R.activation_times_from_fmap(fmap), cache)
    spec = R.RangeSpec.from_fmap(fmap, cache, N)
    live = sum(hi - lo for lo, hi in (R.range_bounds(spec, N - 1, lv) for lv in range(len(caps))))
    row = H * ((Dk + Dv) * el + wel)
    nbytes = B * (sum(caps) + live) * row
    _, _, hbm, src = peaks()
    achieved = nbytes / (ms * 1e-3) / 1e9
    return {"what": "init_decode_state (prefill hand-off: tc_decode_init ring placement + conv history)",
            "ms": ms, "launches_per_call": launches, "bytes": nbytes, "ring_slots": sum(caps),
            "live_nodes": live, "achieved_gbs": achieved, "peak_gbs": hbm,
            "peak_source": f"{src} hbm_gbs", "frac": achieved / hbm}


def decode_bench(args, dev, world, with_e2e=True):
    """Config 4: prefill (builder + init_decode_state) untimed, then W warm-up
    and K timed decode_step calls through the public API.  Returns a dict
    with tokens/s over all ranks (each rank its own batch of 64 rows) and the
    HBM roofline of the ring reads (K + V of every visible entry)."""
    import torch
    import torch.distributed as dist

    import telescope_cache_b200 as T
    from telescope_cache_b200 import range_spec as R

    c = DECODE_SMALL if args.workload == "c4_small" else DECODE
    B, N, H, D = c["B"], c["T"], c["H"], c["D"]
    fmap, cache = {l: l * c["W"] for l in range(1, c["levels"])}, c["levels"] * c["W"]
    bf = torch.bfloat16
    g = torch.Generator(device=dev)
    g.manual_seed(4321 + 7919 * int(os.environ.get("RANK", "0")))
    kcw = torch.randn(H * D, c["conv"], generator=g, device=dev) / math.sqrt(c["conv"])
    vcw = torch.randn(H * D, c["conv"], generator=g, device=dev) / math.sqrt(c["conv"])
    steps = args.warmup + args.steps
    cos, sin = T.rope_tables(N + 2 * steps + 1, D, device=dev)
    sinks = torch.randn(H, generator=g, device=dev)
    gate_w = (0.02 * torch.randn(H * D, EMB, generator=g, device=dev)).to(bf)
    q = torch.randn(B, N, H, D, generator=g, device=dev, dtype=bf)
    k = torch.randn(B, N, H, D, generator=g, device=dev, dtype=bf)
    v = torch.randn(B, N, H, D, generator=g, device=dev, dtype=bf)
    kl, vl, wl = T.build_dyadic_summaries(q, k, v, c["levels"] - 1, k_conv_weight=kcw, v_conv_weight=vcw)
    handoff = handoff_bench(T, args, kl, vl, wl, fmap, cache, k, v, c["conv"])
    state = T.init_decode_state(kl, vl, wl, fmap, cache, k_pre_conv=k, v_pre_conv=v,
                                conv_kernel_size=c["conv"])
    del q, k, v, kl, vl, wl
    tok = dict(x=torch.randn(steps, B, 1, EMB, generator=g, device=dev, dtype=bf),
               q=torch.randn(steps, B, 1, H, D, generator=g, device=dev, dtype=bf),
               k=torch.randn(steps, B, 1, H, D, generator=g, device=dev, dtype=bf),
               v=torch.randn(steps, B, 1, H, D, generator=g, device=dev, dtype=bf))
    kw = dict(k_conv_weight=kcw, v_conv_weight=vcw, softcap=c["softcap"], position_mode="rope",
              rope_cos=cos, rope_sin=sin, sinks=sinks, gate_weight=gate_w)

    def step(i, src):
        return T.decode_step(src["x"][i], src["q"][i], src["k"][i], src["v"][i], state, **kw)

    def sync():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    st = torch.cuda.current_stream()
    for i in range(args.warmup):
        step(i, tok)
    sync()
    t_first = state.t
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(st)
    for i in range(args.warmup, steps):
        step(i, tok)
    b.record(st)
    sync()
    ms = a.elapsed_time(b) / args.steps
    if world > 1:
        tm = torch.tensor([ms], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm.item())
    spec = R.RangeSpec.from_fmap(fmap, cache, t_first + args.steps)
    vis = decode_visible(spec, t_first, args.steps)
    ring_bytes = sum(vis) / len(vis) * B * H * 2 * D * 2
    _, _, hbm, src = peaks()
    gbs = ring_bytes / (ms * 1e-3) / 1e9
    res = {"metric": "decode tokens/s", "value": B * world / (ms * 1e-3), "unit": "tokens/s",
           "ms_per_step": ms, "steps": args.steps, "warmup": args.warmup,
           "config": {"workload": args.workload if args.workload.startswith("c4") else "c4", "desc": c["desc"], "B_per_rank": B, "prefill": N, "H": H,
                      "D": D, "fmap": fmap, "cache_size": cache, "caps": list(state.caps),
                      "softcap": c["softcap"], "visible_per_step": sum(vis) / len(vis)},
           "roofline": {"bound": "hbm", "kernel": "decode_step (whole public call)",
                        "achieved": gbs, "peak": hbm, "peak_source": f"{src} hbm_gbs", "unit": "GB/s",
                        "frac": gbs / hbm, "algorithmic_bytes_per_step": ring_bytes,
                        "traffic": None},
           "handoff": handoff}
    if with_e2e:
        # every step copies its token inputs from pinned host memory and reads
        # its output back; the next step's inputs are copied on a side stream
        # while this step runs (the tokens do not depend on the outputs), and
        # the read-back runs on a third stream
        host = {k_: t_.cpu().pin_memory() for k_, t_ in tok.items()}
        out_host = torch.empty(B, 1, H, D, dtype=bf, pin_memory=True)
        h2d = sum(t_[0].numel() * t_.element_size() for t_ in host.values())
        s_in = torch.cuda.Stream(device=dev)
        s_out = torch.cuda.Stream(device=dev)  # the read-back stays off the compute stream
        bufs = [{k_: torch.empty_like(t_[0]) for k_, t_ in tok.items()} for _ in range(2)]
        evs = [torch.cuda.Event() for _ in range(2)]
        used = [torch.cuda.Event() for _ in range(2)]

        def upload(i, slot):
            with torch.cuda.stream(s_in):
                s_in.wait_event(used[slot])
                for k_, t_ in host.items():
                    bufs[slot][k_].copy_(t_[i], non_blocking=True)
                evs[slot].record(s_in)

        def pipelined(idx):
            """decode_step over the tokens idx, inputs uploaded and outputs read
            back per step; returns ms per step (events on the compute stream)."""
            sync()
            a.record(st)
            upload(idx[0], 0)
            for n in range(len(idx)):
                slot = n & 1
                if n + 1 < len(idx):
                    upload(idx[n + 1], slot ^ 1)
                st.wait_event(evs[slot])
                d_ = bufs[slot]
                out, _ = T.decode_step(d_["x"], d_["q"], d_["k"], d_["v"], state, **kw)
                used[slot].record(st)
                s_out.wait_stream(st)
                with torch.cuda.stream(s_out):
                    out.record_stream(s_out)
                    out_host.copy_(out, non_blocking=True)
            st.wait_stream(s_out)  # the last read-back inside the timed region
            b.record(st)
            sync()
            return a.elapsed_time(b) / len(idx)

        # the state continues at t_first + K with the same token values
        if args.warmup:
            pipelined(list(range(args.warmup)))
        ems = pipelined(list(range(args.warmup, steps)))
        if world > 1:
            tm = torch.tensor([ems], device=dev)
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            ems = float(tm.item())
        res["e2e"] = {"value": B * world / (ems * 1e-3), "unit": "tokens/s", "ms_per_step": ems,
                      "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": out_host.numel() * 2}
    return res


def c5_sharded_bench(args, dev, world, rank):
    """Config 5 split by heads across the ranks (strong scaling): rank r owns
    query / KV heads [r H / N, (r + 1) H / N) (sharding.head_shard).  A step
    builds its heads' tree (linear merge weights from x and its rows of
    w_proj), runs the rope forward with softcap 50, the sink and its backward
    and the Phase-2 backward, and gathers the full out and dq onto every rank
    with one NCCL all_gather each (into one rank-major buffer, returned as a
    [B, T, ranks, H / ranks, D] view) -- all inside the timed region; out's
    gather is started before the backward and overlaps it.  value = the whole config-5
    step's visible-entry FLOPs / the max-over-ranks step time."""
    import torch
    import torch.distributed as dist

    import telescope_cache_b200 as T
    from telescope_cache_b200 import range_spec as R
    from telescope_cache_b200.sharding import head_shard

    wl = WORKLOADS["c5"]
    B, N, H, D = wl["B"], wl["T"], wl["H"], wl["D"]
    _, _, h0, h1 = head_shard(H, H, world, rank)
    hl = h1 - h0
    fmap, cache = schedule(wl)
    total_visible = R.visible_stats(R.RangeSpec.from_fmap(fmap, cache, N))[2]
    step_flops = flops_per_step(wl, total_visible)  # all H heads
    g = torch.Generator(device=dev)
    g.manual_seed(2025 + 7919 * rank)
    bf = torch.bfloat16
    q, k, v, dout = (torch.randn(B, N, hl, D, generator=g, device=dev, dtype=bf) for _ in range(4))
    gx = torch.Generator(device=dev)
    gx.manual_seed(77)  # x and the full w_proj are the same on every rank
    x = torch.randn(B, N, EMB, generator=gx, device=dev, dtype=bf)
    w_proj = (0.02 * torch.randn(H, EMB, generator=gx, device=dev)).to(bf)[h0:h1].contiguous()
    sinks = torch.randn(H, generator=gx, device=dev)[h0:h1].contiguous()
    cos, sin = T.rope_tables(N, D, device=dev)
    out_full = torch.empty(world, B, N, hl, D, device=dev, dtype=bf)
    dq_full = torch.empty_like(out_full)

    def gather_start(local, buf):
        """Start the all_gather of `local` into `buf` on NCCL's stream (it
        waits for the work already queued on this stream); returns the
        handle, or None with one rank."""
        if world == 1:
            return None
        return dist.all_gather_into_tensor(buf.view(world, -1), local.reshape(1, -1), async_op=True)

    def gather_finish(handle, local, buf):
        """The gathered tensor as a [B, N, world, hl, D] view of the rank-major
        buffer (head = rank * hl + local head): every head is present and
        addressable in place, with no reorder copy."""
        if handle is None:
            return local
        handle.wait()  # this stream waits for the collective
        return buf.permute(1, 2, 0, 3, 4)

    def step(timers=None):
        kl, vl, _ = T.build_dyadic_summaries(q, k, v, wl["levels"] - 1, x=x, w_proj=w_proj)
        packed = T.pack_levels(kl, vl)
        pos = dict(position_mode="rope", rope_cos=cos, rope_sin=sin)
        out, lse = T.multilevel_attention_forward(q, packed, fmap, cache, softcap=wl["softcap"], **pos)
        T.apply_attention_sink(out, lse, sinks)
        d_out, dlse, _ = T.attention_sink_backward(out, lse, sinks, dout)
        h_out = gather_start(out, out_full)  # overlaps the backward
        dq, _, _, _, _ = T.multilevel_attention_backward(q, packed, out, lse, d_out, fmap, cache,
                                                         softcap=wl["softcap"], dlse=dlse, **pos)
        if timers:
            timers[0].record()
        h_dq = gather_start(dq, dq_full)
        o_all = gather_finish(h_out, out, out_full)
        dq_all = gather_finish(h_dq, dq, dq_full)
        if timers:
            timers[1].record()
        return o_all, dq_all

    def sync():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        step()
    sync()
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    gev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sync()
    for i in range(args.steps):
        ev[i][0].record(st)
        step(gev[i])
        ev[i][1].record(st)
    sync()
    ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
    gms = sum(a.elapsed_time(b) for a, b in gev) / args.steps
    if world > 1:
        tm = torch.tensor([ms, gms], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms, gms = float(tm[0].item()), float(tm[1].item())
    burst, sustained, _, src = peaks()
    value = step_flops / (ms * 1e-3) / 1e12
    return {"metric": "multilevel attn fwd+bwd TFLOP/s (visible-entry FLOPs), config 5 split by heads",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "scaling": "strong",
            "ms_per_step": ms, "gather_exposed_ms": gms, "gather_exposed_share": gms / ms,
            "config": {"workload": "c5", "desc": wl["desc"], "B": B, "T": N, "H": H, "D": D,
                       "heads_per_rank": hl, "fmap": fmap, "cache_size": cache, "step_flops": step_flops,
                       "gathered": "out and dq, [B, T, H, D] bf16 each: NCCL all_gather_into_tensor into a "
                                   "rank-major buffer, presented as a [B, T, ranks, H / ranks, D] view (no "
                                   "reorder copy); out's gather runs during the backward, gather_exposed_ms is "
                                   "the time from the backward's end to the step's end"},
            "frac_of_peak": value / world / sustained, "peak_source": f"{src} bf16_tflops_sustained (per GPU)"}


def config2_bench(args, dev, flush):
    """BASELINE config 2, the full block forward: B=2, T=8192, H=16, D=128;
    x ~ N(0, 1) of width 2048 and q / k / v = x W^T with random-init weights
    (std 0.02; the projections are the caller's, made before the timed
    region).  A step is the reference API's block: short causal K/V conv of
    width 4, linear merge weights x w_proj^T, the dyadic tree, the rope forward
    with softcap 30, the sink and the SiLU output gate.  Value: the attention's
    visible-entry forward FLOPs (4 D per pair and head) over the block time;
    the parts are timed with CUDA events."""
    import torch

    import telescope_cache_b200 as T
    from telescope_cache_b200 import range_spec as R
    B, N, H, D, L, W, K = 2, 8192, 16, 128, 6, 256, 4
    fmap, cache = {l: l * W for l in range(1, L)}, L * W
    g = torch.Generator(device=dev)
    g.manual_seed(2002)
    bf = torch.bfloat16
    x = torch.randn(B, N, EMB, generator=g, device=dev, dtype=bf)
    proj = [(0.02 * torch.randn(H * D, EMB, generator=g, device=dev)).to(bf) for _ in range(4)]
    q, k, v = (x.matmul(w_.t()).reshape(B, N, H, D) for w_ in proj[:3])
    gate_w = proj[3]
    kcw = torch.randn(H * D, K, generator=g, device=dev) / math.sqrt(K)
    vcw = torch.randn(H * D, K, generator=g, device=dev) / math.sqrt(K)
    w_proj = (0.02 * torch.randn(H, EMB, generator=g, device=dev)).to(bf)
    sinks = torch.randn(H, generator=g, device=dev)
    cos, sin = T.rope_tables(N, D, device=dev)
    pairs = R.visible_stats(R.RangeSpec.from_fmap(fmap, cache, N))[2]
    fwd_flops = 4 * D * pairs * B * H
    ev_names = ("tree", "forward", "sink_gate")

    def step(evs=None):
        if evs:
            evs[0].record()
        kl, vl, _ = T.build_dyadic_summaries(q, k, v, L - 1, x=x, w_proj=w_proj, k_conv_weight=kcw,
                                             v_conv_weight=vcw)
        packed = T.pack_levels(kl, vl)
        if evs:
            evs[1].record()
        out, lse = T.multilevel_attention_forward(q, packed, fmap, cache, softcap=30.0, position_mode="rope",
                                                  rope_cos=cos, rope_sin=sin)
        if evs:
            evs[2].record()
        y = T.apply_output_gate(T.apply_attention_sink(out, lse, sinks), x, gate_w)
        if evs:
            evs[3].record()
        return y

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    for e in evs:
        flush.zero_()
        step(e)
    torch.cuda.synchronize()
    parts = {n: sum(e[i].elapsed_time(e[i + 1]) for e in evs) / len(evs) for i, n in enumerate(ev_names)}
    ms = sum(parts.values())
    _, sustained, _, src = peaks()
    return {"metric": "multilevel attn fwd TFLOP/s (visible-entry FLOPs) over the full block forward",
            "value": fwd_flops / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "ms_per_step": ms,
            "parts_ms": parts, "forward_tflops": fwd_flops / (parts["forward"] * 1e-3) / 1e12,
            "config": {"workload": "c2", "B": B, "T": N, "H": H, "D": D, "levels": L, "window": W, "conv": K,
                       "weights": "linear", "position": "rope", "softcap": 30.0, "sink": True,
                       "gate": "SiLU", "fwd_flops": fwd_flops,
                       "l2": "flushed between timed steps (256 MB write)"},
            "peak_source": f"{src} bf16_tflops_sustained"}


def builder_bench(args, wl, inp, flush):
    """The dyadic builder alone at the workload's shapes (build_dyadic_summaries
    + pack_levels: merge weights, merges, packing), W warm-up and K timed
    calls with CUDA events, L2 flushed before each.  Algorithmic bytes: read
    k, v (and q for qk weights, x for linear ones) once; write every packed
    level of k and v and the packed weights once."""
    import torch

    import telescope_cache_b200 as T
    L = wl["levels"] - 1
    kw = {}
    if wl["weights"] == "linear":
        kw.update(x=inp["x"], w_proj=inp["w_proj"])

    def call():
        kl, vl, wl_ = T.build_dyadic_summaries(inp["q"], inp["k"], inp["v"], L, **kw)
        return T.pack_levels(kl, vl)

    for _ in range(max(args.warmup, 1)):
        call()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for a, b in ev:
        flush.zero_()
        a.record()
        call()
        b.record()
    torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
    B, N, H, D = wl["B"], wl["T"], wl["H"], wl["D"]
    total = sum(N >> lv for lv in range(L + 1))
    nbytes = 2 * B * N * H * D * 2 + 2 * B * total * H * D * 2 + B * total * H * 2
    nbytes += B * N * H * D * 2 if wl["weights"] == "qk" else B * N * EMB * 2
    _, _, hbm, src = peaks()
    gbs = nbytes / (ms * 1e-3) / 1e9
    return {"what": "build_dyadic_summaries + pack_levels", "ms": ms, "bytes": nbytes, "achieved_gbs": gbs,
            "peak_gbs": hbm, "peak_source": f"{src} hbm_gbs", "frac": gbs / hbm}


def cpu_reference_sample(wl, seconds_budget=20.0):
    """Time the CPU oracle (fwd + bwd) on a bounded sample of the workload:
    consecutive query rows of one (batch, head) slice, in the steady state
    where every level is live, for about `seconds_budget` seconds.  Returns
    (TFLOP/s on visible-entry FLOPs, description)."""
    import numpy as np

    from oracle import numerics as O
    from oracle import schedule as S

    fmap, cache = schedule(wl)
    a = S.activation_times(fmap)
    D, T_ = wl["D"], wl["T"]
    r = np.random.Generator(np.random.PCG64(5))
    q = r.standard_normal((1, T_, 1, D)).astype(np.float32)
    k = r.standard_normal((1, T_, 1, D)).astype(np.float32)
    v = r.standard_normal((1, T_, 1, D)).astype(np.float32)
    kl, vl, _ = O.build_tree(k, v, O.qk_weights(q, k), wl["levels"] - 1)
    pos = O.Positional()
    if wl["position"] == "relative":
        st = (0.02 * r.standard_normal((1, T_, 1, wl["d_rel"]))).astype(np.float32)
        pj = (0.02 * r.standard_normal((wl["d_rel"], cache))).astype(np.float32)
        pos = O.Positional("relative", states=st, proj=pj)
    elif wl["position"] == "rope":
        cos, sin = O.rope_tables(T_, D)
        pos = O.Positional("rope", cos=cos, sin=sin)
    dout = r.standard_normal((1, T_, 1, D)).astype(np.float32)
    start = T_ - 1
    pairs = 0
    t0 = time.perf_counter()
    chunk = 16
    while time.perf_counter() - t0 < seconds_budget and start - chunk >= 0:
        rows = range(start - chunk, start)
        out, lse = O.forward(q, kl, vl, fmap, cache, wl["softcap"], pos, rows=rows)
        O.backward(q, kl, vl, out, lse, dout, fmap, cache, wl["softcap"], pos, rows=rows)
        pairs += sum(len(S.visible_entries(qi, a, cache)) for qi in rows)
        start -= chunk
    el = time.perf_counter() - t0
    n = T_ - 1 - start
    return (4 + 10) * D * pairs / el / 1e12, (
        f"{n} query rows (the last of T={T_}) of one (batch, head) slice, fwd+bwd in float64 "
        f"numpy, {el:.1f} s; throughput scales linearly with the slice count")


REF_SAMPLE_T = 2048  # tokens of the reference's (batch, head) sample slice


def reference_py_sample(wl, T_s=REF_SAMPLE_T, seed=5):
    """Time the reference's own public API (reference.py from baseline/_ref,
    fp32 on the host cores, all threads) on one (batch, head) slice of the
    workload's schedule and features at sequence length T_s: the tree build
    and packing, the forward, the sink and its backward, and the backward
    with the dlse seam -- the step this file times on the GPU.  Returns
    (TFLOP/s on visible-entry FLOPs, seconds, description), or None when the
    reference is not installed."""
    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "telescope_cache")):
        return None
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    import torch
    try:
        import telescope_cache.reference as ref
    except Exception:  # noqa: BLE001 - any import failure means: not installed here
        return None
    from telescope_cache_b200 import range_spec as R
    torch.set_num_threads(os.cpu_count() or 1)
    fmap, cache = schedule(wl)
    D, levels = wl["D"], wl["levels"]
    g = torch.Generator().manual_seed(seed)
    q, k, v, dout = (torch.randn(1, T_s, 1, D, generator=g) for _ in range(4))
    kw, pos = {}, {}
    if wl["weights"] == "linear":
        kw = dict(x=torch.randn(1, T_s, EMB, generator=g), w_proj=0.02 * torch.randn(1, EMB, generator=g))
    if wl["conv"]:
        kw.update(k_conv_weight=torch.randn(D, wl["conv"], generator=g) / math.sqrt(wl["conv"]),
                  v_conv_weight=torch.randn(D, wl["conv"], generator=g) / math.sqrt(wl["conv"]))
    if wl["position"] == "relative":
        pos = dict(position_mode="relative", relative_states=0.02 * torch.randn(1, T_s, 1, wl["d_rel"], generator=g),
                   relative_proj=0.02 * torch.randn(wl["d_rel"], cache, generator=g))
    elif wl["position"] == "rope":
        cos, sin = ref.rope_tables(T_s, D)
        pos = dict(position_mode="rope", rope_cos=cos, rope_sin=sin)
    sinks = torch.randn(1, generator=g)
    t0 = time.perf_counter()
    kl, vl, _ = ref.build_dyadic_summaries(q, k, v, levels - 1, **kw)
    packed = ref.pack_levels(kl, vl)
    out, lse = ref.multilevel_attention_forward(q, packed, fmap, cache, softcap=wl["softcap"], **pos)
    dlse = None
    if wl["sink"]:
        ref.apply_attention_sink(out, lse, sinks)
        dout, dlse, _ = ref.attention_sink_backward(out, lse, sinks, dout)
    ref.multilevel_attention_backward(q, packed, out, lse, dout, fmap, cache, softcap=wl["softcap"], dlse=dlse,
                                      **pos)
    el = time.perf_counter() - t0
    pairs = R.visible_stats(R.RangeSpec.from_fmap(fmap, cache, T_s))[2]
    desc = (f"reference.py (baseline/_ref) fp32 on {os.cpu_count()} host threads: one (batch, head) slice at "
            f"T={T_s} of the {args_workload_name(wl)} schedule and features (tree, forward, sink, sink "
            f"backward, backward), {el:.1f} s; visible-entry FLOPs of that slice / time")
    return (4 + 10) * D * pairs / el / 1e12, el, desc


def args_workload_name(wl):
    return next((n for n, w in WORKLOADS.items() if w is wl), "workload")


def reference_arm(args, wl):
    """--impl reference: the reference's own implementation timed on the host
    cores (rank 0 only; other ranks exit without work).  Each step is one
    bounded sample (reference_py_sample); the line reports the median of the
    timed steps.  Falls back to the numpy oracle port when the reference is
    not installed, and says so."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    times, secs = [], []
    sample, kind = "", "reference"
    for i in range(args.warmup + args.steps):
        got = reference_py_sample(wl)
        if got is None:
            tf, sample = cpu_reference_sample(wl, seconds_budget=max(5.0, 60.0 / (args.steps + args.warmup)))
            sample = "numpy oracle port (reference.py not installed under baseline/_ref): " + sample
            kind, el = "port", None
        else:
            tf, el, sample = got
        if i >= args.warmup:
            times.append(tf)
            secs.append(el)
    val = sorted(times)[len(times) // 2]
    fmap, cache = schedule(wl)
    sec = sorted(s_ for s_ in secs if s_ is not None)
    line = {
        "impl": "reference", "metric": "multilevel attn fwd+bwd TFLOP/s (visible-entry FLOPs)",
        "value": val, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": sec[len(sec) // 2] * 1e3 if sec else None,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "desc": wl["desc"], "B_per_rank": wl["B"], "T": wl["T"],
                   "H": wl["H"], "D": wl["D"], "fmap": fmap, "cache_size": cache,
                   "sample": f"one (batch, head) slice at T={REF_SAMPLE_T} per step"},
        "cpu_baseline": {"value": val, "unit": "TFLOP/s", "cores": threads, "kind": kind, "sample": sample},
        "e2e": {"value": val, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def decode_main(args):
    """--workload c4: the decode tokens/s line on its own."""
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable":
                              "the decode reference arm is not implemented; the default c3 line "
                              "carries the reference comparison"}))
        return 0
    import torch
    import torch.distributed as dist

    from telescope_cache_b200 import _lib
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    n0 = _lib.launch_count()
    with ClockSampler(local) as clocks:
        res = decode_bench(args, dev, world, with_e2e=not args.no_e2e)
    if rank == 0:
        res.update({"n_gpus": world, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                    "dtype": "bf16", "data": "synthetic", "cpu_baseline": None,
                    "clocks": clocks.summary(), "gpu_launches": _lib.launch_count() - n0})
        print(json.dumps(res))
    if world > 1:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="c3", choices=sorted(WORKLOADS) + ["c4", "c4_small"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-decode", action="store_true",
                    help="skip the config-4 decode measurement added to the c3 line")
    ap.add_argument("--no-c2", action="store_true",
                    help="skip the config-2 block-forward measurement added to the c3 line")
    ap.add_argument("--no-c5-sharded", action="store_true",
                    help="skip the config-5 head-sharded (strong scaling) measurement added to the c3 line")
    ap.add_argument("--no-vjp", action="store_true",
                    help="skip the Phase-1 VJP measurement added to the line")
    args = ap.parse_args()
    if args.workload in ("c4", "c4_small"):
        return decode_main(args)
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        return reference_arm(args, wl)

    import torch
    import torch.distributed as dist

    import telescope_cache_b200 as T
    from telescope_cache_b200 import _lib
    from telescope_cache_b200 import range_spec as R

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    fmap, cache = schedule(wl)
    spec = R.RangeSpec.from_fmap(fmap, cache, wl["T"])
    total_visible = R.visible_stats(spec)[2]
    step_flops = flops_per_step(wl, total_visible)
    inp = make_inputs(wl, dev, 1234, rank)
    tables = T.rope_tables(wl["T"], wl["D"], device=dev) if wl["position"] == "rope" else None
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)  # > L2 (126 MB)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        run_step(T, wl, inp, fmap, cache, tables)
    barrier()
    st = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    kt = [{"fwd": (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)),
           "bwd": (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))}
          for _ in range(args.steps)]
    launches_before = _lib.launch_count()
    with ClockSampler(local) as clocks:
        barrier()
        step_ms = []
        for i in range(args.steps):
            flush.zero_()  # L2 flush between timed iterations
            ev[i][0].record(st)
            run_step(T, wl, inp, fmap, cache, tables, timers=kt[i])
            ev[i][1].record(st)
        barrier()
    launches_timed = _lib.launch_count() - launches_before
    step_ms = [a.elapsed_time(b) for a, b in ev]
    fwd_ms = [t["fwd"][0].elapsed_time(t["fwd"][1]) for t in kt]
    bwd_ms = [t["bwd"][0].elapsed_time(t["bwd"][1]) for t in kt]
    ms = sum(step_ms) / len(step_ms)
    if world > 1:
        tm = torch.tensor([ms], device=dev)
        dist.all_reduce(tm, op=dist.ReduceOp.MAX)
        ms = float(tm.item())
    value = step_flops * world / (ms * 1e-3) / 1e12

    # end-to-end through the public API from pinned host buffers: every step
    # copies its inputs host->device and its dq device->host inside the timed
    # region; the copies run on their own streams, pipelined with the
    # neighbouring steps' compute (double-buffered device inputs)
    e2e = None
    if not args.no_e2e:
        host = {k: v.cpu().pin_memory() for k, v in inp.items()}
        h2d = sum(v.numel() * v.element_size() for v in host.values())
        dq_host = [torch.empty(inp["q"].shape, dtype=inp["q"].dtype, pin_memory=True) for _ in range(2)]
        d2h = dq_host[0].numel() * dq_host[0].element_size()
        bufs = [{k: torch.empty_like(v) for k, v in inp.items()} for _ in range(2)]
        s_in, s_out = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

        def pipelined(nsteps):
            copied = [torch.cuda.Event() for _ in range(nsteps)]
            done = [torch.cuda.Event() for _ in range(nsteps)]
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(s_in)
            with torch.cuda.stream(s_in):
                for k, v in host.items():
                    bufs[0][k].copy_(v, non_blocking=True)
                copied[0].record(s_in)
            for i in range(nsteps):
                st.wait_event(copied[i])
                dq, *_ = run_step(T, wl, bufs[i % 2], fmap, cache, tables)
                done[i].record(st)
                if i + 1 < nsteps:
                    with torch.cuda.stream(s_in):
                        if i >= 1:
                            s_in.wait_event(done[i - 1])  # step i-1 no longer reads this buffer
                        for k, v in host.items():
                            bufs[(i + 1) % 2][k].copy_(v, non_blocking=True)
                        copied[i + 1].record(s_in)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(done[i])
                    dq_host[i % 2].copy_(dq, non_blocking=True)
                    dq.record_stream(s_out)
            s_out.wait_stream(s_in)
            s_out.wait_stream(st)
            end.record(s_out)
            torch.cuda.synchronize()
            return start.elapsed_time(end) / nsteps

        barrier()
        if args.warmup:
            pipelined(args.warmup)
        barrier()
        em = pipelined(args.steps)
        if world > 1:
            tm = torch.tensor([em], device=dev)
            dist.all_reduce(tm, op=dist.ReduceOp.MAX)
            em = float(tm.item())
        e2e = {"value": step_flops * world / (em * 1e-3) / 1e12, "unit": "TFLOP/s",
               "ms_per_step": em, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "copies": "pinned host buffers, H2D and D2H on their own streams, pipelined "
                         "with the neighbouring steps"}

    burst, sustained, hbm, src = peaks()
    fwd_flops = 4 * wl["D"] * total_visible * wl["B"] * wl["H"]
    bwd_flops = 10 * wl["D"] * total_visible * wl["B"] * wl["H"]
    fms, bms = sum(fwd_ms) / len(fwd_ms), sum(bwd_ms) / len(bwd_ms)
    dom = ("backward", bwd_flops, bms) if bms >= fms else ("forward", fwd_flops, fms)
    achieved = dom[1] / (dom[2] * 1e-3) / 1e12
    roofline = {"bound": "tensor", "kernel": f"attention {dom[0]}", "achieved": achieved,
                "peak": sustained, "peak_source": f"{src} bf16_tflops_sustained", "unit": "TFLOP/s",
                "frac": achieved / sustained, "traffic": TRAFFIC.get(args.workload),
                "traffic_note": "DRAM bytes per backward (Pass A + Pass B), ncu c3_small x16"
                if args.workload in TRAFFIC else None,
                "forward_tflops": fwd_flops / (fms * 1e-3) / 1e12,
                "backward_tflops": bwd_flops / (bms * 1e-3) / 1e12,
                "forward_ms": fms, "backward_ms": bms}
    vjp = None
    if not args.no_vjp:
        _, dk_s, dv_s, _, _ = run_step(T, wl, inp, fmap, cache, tables)
        vjp = vjp_bench(T, wl, inp, (dk_s, dv_s), args, hbm, flush)
        del dk_s, dv_s
    bld = builder_bench(args, wl, inp, flush)
    c2 = None
    if args.workload == "c3" and world == 1 and not args.no_c2:
        c2 = config2_bench(args, dev, flush)
        torch.cuda.empty_cache()
    c5s = None
    if args.workload == "c3" and not args.no_c5_sharded:
        c5s = c5_sharded_bench(args, dev, world, rank)
        torch.cuda.empty_cache()
    dec = None
    if args.workload == "c3" and not args.no_decode:
        # before the CPU baseline, whose worker threads can linger on the host
        dec = decode_bench(args, dev, world, with_e2e=not args.no_e2e)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        got = reference_py_sample(wl)
        if got is not None:
            cpu = {"value": got[0], "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "reference",
                   "sample": got[2]}
        else:
            tf, sample = cpu_reference_sample(wl, seconds_budget=15.0)
            cpu = {"value": tf, "unit": "TFLOP/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": "numpy oracle port (reference.py not installed under baseline/_ref): " + sample}
    launches = launches_timed
    if rank == 0:
        line = {
            "metric": "multilevel attn fwd+bwd TFLOP/s (visible-entry FLOPs)",
            "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": args.workload, "desc": wl["desc"], "B_per_rank": wl["B"],
                       "T": wl["T"], "H": wl["H"], "D": wl["D"], "fmap": fmap, "cache_size": cache,
                       "global_batch": wl["B"] * world, "parallelism": f"dp{world} (batch x head shards)",
                       "l2": "flushed between timed steps (256 MB write)",
                       "step_flops": step_flops},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "clocks": clocks.summary(),
            "gpu_launches": launches,
        }
    if vjp is not None and rank == 0:
        line["phase1_vjp"] = vjp
    if dec is not None and rank == 0:
        line["decode"] = dec
    if c5s is not None and rank == 0:
        line["c5_sharded"] = c5s
    if rank == 0:
        line["builder"] = bld
    if c2 is not None and rank == 0:
        line["config2"] = c2
    if rank == 0:
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
