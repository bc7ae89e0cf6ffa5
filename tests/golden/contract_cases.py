"""The reference suite's API contracts, stated once against an API namespace so
that the same cases run against the reference (``make_contract_golden.py``
records each case's exception type and message) and against this build
(``tests/test_contracts.py`` asserts the same type and message).

Cases restate ``test/test_reference.py``:
- ``error_cases``: the ValueError matrix of ``test_error_paths``
  (test_reference.py:1888-2079) for the reference.py API: forward / backward
  positional-argument matrix, dlse seed, sink / gate / conv contracts, the
  summary-causality guard and the decode API.  The minimal_reference mirrors
  of that test are not part of the reference.py surface and are left out.
- ``NO_MUTATION_MODES``: no position mode may mutate the packed buffers
  (test_reference.py:1803-1816).
- ``NEVER_VISIBLE_GEOS``: never-visible packed nodes get exactly zero
  gradient (test_reference.py:1575-1596).

``api`` is any object with the reference.py names as attributes (the module
itself, or ``telescope_cache_b200.reference``) plus ``RangeSpec``.
"""

import torch

# test_reference.py:133-148 (GEOS["tiny"], _EMB, _DREL)
TINY = dict(B=2, N=8, Hq=4, Hkv=2, Dk=8, Dv=16, fmap={1: 2, 2: 3}, cache=6)
EMB, DREL = 32, 6

NO_MUTATION_MODES = ("none", "rope", "relative")
NEVER_VISIBLE_GEOS = (("evict", 340), ("four_levels", 344))


def error_cases(api, device):
    """[(label, thunk)]: each thunk must raise ValueError (the reference's
    test_error_paths); the inputs come from the reference test's seed 460."""
    g = TINY
    B, N, Hq, Hkv, Dk, Dv = (g[s] for s in ("B", "N", "Hq", "Hkv", "Dk", "Dv"))
    L = len(g["fmap"])
    torch.manual_seed(460)
    q = torch.randn(B, N, Hq, Dk).to(device)
    k = torch.randn(B, N, Hkv, Dk).to(device)
    v = torch.randn(B, N, Hkv, Dv).to(device)
    x = torch.randn(B, N, EMB).to(device)
    kl_r, vl_r, _ = api.build_dyadic_summaries(q, k, v, L)
    packed = api.pack_levels(kl_r, vl_r)
    spec = api.RangeSpec.from_fmap(g["fmap"], g["cache"], N)
    cos, sin = api.rope_tables(N, Dk, device=device)
    states = torch.randn(B, N, Hq, DREL).to(device)
    proj = torch.randn(DREL, 8).to(device)
    q_odd = torch.randn(B, N, Hq, 7).to(device)
    cases = []

    def ve(label, fn):
        cases.append((label, fn))

    def fwd(**kw):
        return api.multilevel_attention_forward(q, packed, g["fmap"], g["cache"], block_m=3, block_n=2, **kw)

    ve("unknown mode", lambda: fwd(position_mode="alibi"))
    ve("rope args with none", lambda: fwd(position_mode="none", rope_cos=cos, rope_sin=sin))
    ve("relative args with rope", lambda: fwd(position_mode="rope", rope_cos=cos, rope_sin=sin,
                                              relative_states=states, relative_proj=proj))
    ve("rope args with relative", lambda: fwd(position_mode="relative", relative_states=states,
                                              relative_proj=proj, rope_cos=cos, rope_sin=sin))
    ve("missing sin", lambda: fwd(position_mode="rope", rope_cos=cos))
    ve("short rope table", lambda: fwd(position_mode="rope", rope_cos=cos[:N - 1], rope_sin=sin[:N - 1]))
    ve("mismatched cos/sin", lambda: fwd(position_mode="rope", rope_cos=cos, rope_sin=sin[:N - 1]))
    ve("wrong proj shape", lambda: fwd(position_mode="relative", relative_states=states,
                                       relative_proj=torch.randn(5, 8).to(device)))
    ve("1-D proj", lambda: fwd(position_mode="relative", relative_states=states,
                               relative_proj=torch.randn(8).to(device)))
    ve("table too small", lambda: fwd(position_mode="relative", relative_states=states,
                                      relative_proj=torch.randn(DREL, 2).to(device)))
    ve("odd Dk", lambda: api.multilevel_attention_forward(q_odd, packed, g["fmap"], g["cache"], block_m=3,
                                                          block_n=2, position_mode="rope", rope_cos=cos,
                                                          rope_sin=sin))
    ve("invisible entry", lambda: api.relative_bin_distance(spec, 0, 0, 5))

    out_lse = {}

    def out_and_lse():
        if not out_lse:
            out_lse["v"] = fwd()
        return out_lse["v"]

    def bwd(**kw):
        out, lse = out_and_lse()
        dlse = kw.pop("dlse_of", None)
        if dlse is not None:
            kw["dlse"] = dlse(lse)
        return api.multilevel_attention_backward(q, packed, out, lse, torch.randn_like(out), g["fmap"],
                                                 g["cache"], block_m=3, block_n=2, **kw)

    ve("backward unknown mode", lambda: bwd(position_mode="alibi"))
    ve("backward rope args with none", lambda: bwd(position_mode="none", rope_cos=cos, rope_sin=sin))
    ve("backward missing sin", lambda: bwd(position_mode="rope", rope_cos=cos))
    ve("backward missing proj", lambda: bwd(position_mode="relative", relative_states=states))
    ve("backward table too small", lambda: bwd(position_mode="relative", relative_states=states,
                                               relative_proj=torch.randn(DREL, 2).to(device)))
    ve("dlse wrong shape", lambda: bwd(dlse_of=lambda lse: lse[:, :-1]))
    ve("dlse non-floating", lambda: bwd(dlse_of=lambda lse: torch.zeros_like(lse, dtype=torch.long)))

    sinks = torch.randn(Hq).to(device)
    ve("sinks wrong length", lambda: api.apply_attention_sink(*out_and_lse(), torch.randn(Hq + 1).to(device)))
    ve("sinks per KV head", lambda: api.apply_attention_sink(*out_and_lse(), torch.randn(Hkv).to(device)))
    ve("gate weight shape", lambda: api.apply_output_gate(out_and_lse()[0], x,
                                                          torch.randn(Hq * Dv + 1, EMB).to(device)))
    ve("sink-backward dout dtype", lambda: api.attention_sink_backward(
        *out_and_lse(), sinks, torch.randn_like(out_and_lse()[0]).to(torch.bfloat16)))

    kcw = torch.randn(Hkv * Dk, 3).to(device)
    ve("one-sided conv (ref)", lambda: api.build_dyadic_summaries(q, k, v, L, k_conv_weight=kcw))
    ve("conv wrong channels", lambda: api.short_conv(x, torch.randn(EMB + 1, 3).to(device)))
    ve("conv 1-D weight", lambda: api.short_conv(x, torch.randn(3).to(device)))
    ve("conv zero-width", lambda: api.short_conv(x, torch.randn(EMB, 0).to(device)))
    ve("summary causality", lambda: api.validate_summary_causality(
        api.RangeSpec(activation_times=(0, 0), cache_size=6, seq_len=8)))

    kl_w, vl_w, wl_w = api.build_dyadic_summaries(q, k, v, L)

    def fresh(**kw):
        return api.init_decode_state(kl_w, vl_w, wl_w, g["fmap"], g["cache"], **kw)

    q1, k1, v1, x1 = q[:, :1], k[:, :1], v[:, :1], x[:, :1]
    vcw = torch.randn(Hkv * Dv, 3).to(device)
    ve("decode q_t not one token", lambda: api.multilevel_attention_decode(q, fresh()))
    ve("decode Dk mismatch", lambda: api.multilevel_attention_decode(q_odd[:, :1], fresh()))
    ve("decode unknown mode", lambda: api.multilevel_attention_decode(q1, fresh(), position_mode="alibi"))
    ve("decode rope args with none", lambda: api.multilevel_attention_decode(q1, fresh(), rope_cos=cos,
                                                                             rope_sin=sin))
    ve("decode short rope table", lambda: api.multilevel_attention_decode(
        q1, fresh(), position_mode="rope", rope_cos=cos[:N - 1], rope_sin=sin[:N - 1]))
    ve("decode table too small", lambda: api.multilevel_attention_decode(
        q1, fresh(), position_mode="relative", relative_states=states[:, :1],
        relative_proj=torch.randn(DREL, 2).to(device)))
    ve("decode k_t shape", lambda: api.advance_decode_state(fresh(), q1, k1[:, :, :1], v1))
    ve("decode one-sided conv", lambda: api.advance_decode_state(fresh(), q1, k1, v1, k_conv_weight=kcw))
    ve("decode conv weights without conv state", lambda: api.advance_decode_state(
        fresh(), q1, k1, v1, k_conv_weight=kcw, v_conv_weight=vcw))
    ve("decode conv state without weights", lambda: api.advance_decode_state(
        fresh(k_pre_conv=k, v_pre_conv=v, conv_kernel_size=3), q1, k1, v1))
    ve("decode init pre-conv without kernel size", lambda: fresh(k_pre_conv=k, v_pre_conv=v))
    ve("decode init one-sided pre-conv", lambda: fresh(k_pre_conv=k, conv_kernel_size=3))
    ve("decode init zero kernel", lambda: fresh(k_pre_conv=k, v_pre_conv=v, conv_kernel_size=0))
    ve("decode linear without w_proj", lambda: api.decode_step(x1, q1, k1, v1, fresh(), weight_mode="linear"))
    ve("decode w_proj with qk", lambda: api.decode_step(x1, q1, k1, v1, fresh(),
                                                        w_proj=torch.randn(Hkv, EMB).to(device)))
    ve("decode relative without weight", lambda: api.decode_step(x1, q1, k1, v1, fresh(),
                                                                 position_mode="relative", relative_proj=proj))
    ve("decode relative weight with none", lambda: api.decode_step(
        x1, q1, k1, v1, fresh(), relative_weight=torch.randn(Hq * DREL, EMB).to(device)))
    ve("conv step state shape", lambda: api.short_conv_step(x1, torch.zeros(B, 5, EMB).to(device),
                                                            torch.randn(EMB, 3).to(device)))
    ve("conv step multi-token x", lambda: api.short_conv_step(x, torch.zeros(B, 2, EMB).to(device),
                                                              torch.randn(EMB, 3).to(device)))
    ve("caps bad a[0]", lambda: api.decode_capacities((1, 3), 6))
    ve("ring_slot negative", lambda: api.ring_slot(fresh(), 0, -1))
    ve("ring_slot level", lambda: api.ring_slot(fresh(), L + 1, 0))
    return cases


def run_case(fn):
    """(exception type name, message) that fn raises, or (None, None)."""
    try:
        fn()
    except Exception as e:  # noqa: BLE001 - the type is the recorded outcome
        return type(e).__name__, str(e)
    return None, None
