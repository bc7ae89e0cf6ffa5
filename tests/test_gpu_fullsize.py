"""Parity at the BASELINE configs' full sizes, through checks whose cost does
not grow with the problem:

* config 3 (B=4, T=16384, H=16, relative bias, softcap 50) and config 5
  (T=131072, H=32, rope, linear weights, softcap 50): the CUDA forward /
  backward over the whole problem, then sampled query rows of two (batch,
  head) slices against the float64 oracle (out, lse, dq, drel); sampled
  packed nodes of several levels (dK, dV), against the oracle backward over
  exactly the queries that see them; and the linear identity
  sum_nodes dV = sum_queries dO of every (batch, head) (each row of P sums
  to one);
* config 2 (the full block forward: B=2, T=8192, H=16, q/k/v projected from
  x, conv 4, linear merge weights, rope, sink, SiLU gate, softcap 30): the
  gated output and lse of sampled rows of two (batch, head) slices against
  the float64 oracle of the same block;
* config 4 (batch 64, 32768-token prefill, rope, conv 4, sink, gate): the
  fused decode steps against the float64 oracle's full-sequence rows (conv,
  tree, rope forward, sink, gate) of sampled (batch, head) slices, and
  against the CUDA forward's rows over every slice.

Tolerance: the bf16 rules of the golden tests, per checked tensor: normwise
relative error <= 2e-2, and |got - want| <= 2e-2 (|want| + max|want|)."""

import math

import numpy as np
import pytest
import torch

import telescope_cache_b200 as T
from oracle import numerics as O

pytestmark = pytest.mark.gpu
BF16_REL = 2e-2


def close(name, got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (name, got.shape, want.shape)
    scale = np.abs(want).max() if want.size else 0.0
    err = np.abs(got - want)
    wn = np.linalg.norm(want)
    if wn > 0:
        normrel = np.linalg.norm(got - want) / wn
        assert normrel <= BF16_REL, f"{name}: normwise relative error {normrel:.3e} > {BF16_REL}"
    bad = err > BF16_REL * (np.abs(want) + scale)
    assert not bad.any(), f"{name}: max err {err.max():.3e} vs scale {scale:.3e}, {int(bad.sum())} out of bound"


def f64(t):
    return t.detach().double().cpu().numpy()


class _RowBias:
    """Relative bias rows computed on demand (the oracle indexes
    rel[:, q]); shape as the full [B, N, H, R] tensor."""

    def __init__(self, states, proj):
        self.states, self.proj = states, proj
        self.shape = states.shape[:3] + (proj.shape[1],)

    def __getitem__(self, key):
        _, qi = key
        return np.einsum("bhd,dr->bhr", self.states[:, qi], self.proj)


def _slice_oracle(q, k, v, dout, w, fmap, cache, softcap, pos, rows, L):
    kl, vl, _ = O.build_tree(k, v, w, L)
    out, lse = O.forward(q, kl, vl, fmap, cache, softcap, pos, rows=rows)
    dq, _, _, drel = O.backward(q, kl, vl, out, lse, dout, fmap, cache, softcap, pos, rows=rows)
    return out, lse, dq, drel


def _node_rows(fmap, cache, N, nodes):
    """Every query that sees one of `nodes` ((level, j) pairs): the oracle
    backward over exactly these rows gives those nodes' complete dK / dV."""
    from telescope_cache_b200.range_spec import RangeSpec, node_query_bounds
    spec = RangeSpec.from_fmap(fmap, cache, N)
    rows = set()
    for lv, j in nodes:
        lo, hi = node_query_bounds(spec, j, lv)
        assert lo < hi, (lv, j)
        rows.update(range(lo, hi))
    return sorted(rows), spec.level_offsets()


def _check_nodes(name, dk_packed, dv_packed, b, h, q, k, v, dout, w, fmap, cache, softcap, pos, L, nodes):
    rows, off = _node_rows(fmap, cache, q.shape[1], nodes)
    kl, vl, _ = O.build_tree(k, v, w, L)
    out, lse = O.forward(q, kl, vl, fmap, cache, softcap, pos, rows=rows)
    _, dkl, dvl, _ = O.backward(q, kl, vl, out, lse, dout, fmap, cache, softcap, pos, rows=rows)
    idx = [off[lv] + j for lv, j in nodes]
    close(f"{name} dk_packed nodes", f64(dk_packed[b, idx, h]), np.stack([dkl[lv][0, j, 0] for lv, j in nodes]))
    close(f"{name} dv_packed nodes", f64(dv_packed[b, idx, h]), np.stack([dvl[lv][0, j, 0] for lv, j in nodes]))


@pytest.fixture(scope="module")
def dev():
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    return torch.device("cuda")


def _dv_sum_identity(dv_packed, dout, name):
    # per (batch, head, dim): sum over every node of dV == sum over queries of dO
    got = dv_packed.double().sum(dim=1)
    want = dout.double().sum(dim=1)
    close(name, got.cpu().numpy(), want.cpu().numpy())


def test_config3_full_size(dev):
    B, N, H, D, L, W = 4, 16384, 16, 128, 8, 512
    fmap, cache = {l: l * W for l in range(1, L)}, L * W
    g = torch.Generator(device=dev)
    g.manual_seed(303)
    bf = torch.bfloat16
    q, k, v, dout = (torch.randn(B, N, H, D, generator=g, device=dev, dtype=bf) for _ in range(4))
    states = (0.02 * torch.randn(B, N, H, 16, generator=g, device=dev)).to(bf)
    proj = (0.02 * torch.randn(16, cache, generator=g, device=dev)).to(bf)
    kl, vl, _ = T.build_dyadic_summaries(q, k, v, L - 1)
    packed = T.pack_levels(kl, vl)
    pos = dict(position_mode="relative", relative_states=states, relative_proj=proj)
    out, lse = T.multilevel_attention_forward(q, packed, fmap, cache, softcap=50.0, **pos)
    dq, dk, dv, drel, _ = T.multilevel_attention_backward(q, packed, out, lse, dout, fmap, cache,
                                                          softcap=50.0, **pos)
    _dv_sum_identity(dv, dout, "c3 sum dV")
    rows = [0, 1, 511, 4097, 9000, 16383]
    for b, h in ((1, 5), (3, 15)):
        sl = lambda t: f64(t[b:b + 1, :, h:h + 1])  # noqa: E731
        qs, ks, vs = sl(q), sl(k), sl(v)
        p = O.Positional()
        p.mode, p.rel = "relative", _RowBias(sl(states), f64(proj))
        o_out, o_lse, o_dq, o_drel = _slice_oracle(qs, ks, vs, sl(dout), O.qk_weights(qs, ks), fmap, cache,
                                                   50.0, p, rows, L - 1)
        close(f"c3 out {b},{h}", f64(out[b, rows, h]), o_out[0, rows, 0])
        close(f"c3 lse {b},{h}", f64(lse[b, rows, h]), o_lse[0, rows, 0])
        close(f"c3 dq {b},{h}", f64(dq[b, rows, h]), o_dq[0, rows, 0])
        close(f"c3 drel {b},{h}", f64(drel[b, rows, h]), o_drel[0, rows, 0])
        _check_nodes(f"c3 {b},{h}", dk, dv, b, h, qs, ks, vs, sl(dout), O.qk_weights(qs, ks), fmap, cache,
                     50.0, p, L - 1, [(0, 4000), (0, 16383), (1, 7935), (2, 3711), (3, 1599), (4, 543), (5, 15)])


def test_config5_full_size(dev):
    B, N, H, D, L, W, E = 1, 131072, 32, 128, 10, 1024, 2048
    fmap, cache = {l: l * W for l in range(1, L)}, L * W
    g = torch.Generator(device=dev)
    g.manual_seed(505)
    bf = torch.bfloat16
    q, k, v, dout = (torch.randn(B, N, H, D, generator=g, device=dev, dtype=bf) for _ in range(4))
    x = torch.randn(B, N, E, generator=g, device=dev, dtype=bf)
    w_proj = (0.02 * torch.randn(H, E, generator=g, device=dev)).to(bf)
    cos, sin = T.rope_tables(N, D, device=dev)
    kl, vl, _ = T.build_dyadic_summaries(q, k, v, L - 1, x=x, w_proj=w_proj)
    packed = T.pack_levels(kl, vl)
    pos = dict(position_mode="rope", rope_cos=cos, rope_sin=sin)
    out, lse = T.multilevel_attention_forward(q, packed, fmap, cache, softcap=50.0, **pos)
    dq, dk, dv, _, _ = T.multilevel_attention_backward(q, packed, out, lse, dout, fmap, cache, softcap=50.0,
                                                       **pos)
    _dv_sum_identity(dv, dout, "c5 sum dV")
    ocos, osin = O.rope_tables(N, D)
    rows = [0, 1023, 5000, 65536, 131071]
    for h in (0, 21):
        sl = lambda t: f64(t[:, :, h:h + 1])  # noqa: E731
        # merge weights x . w_proj[h] in float64 on the device
        w = (x.double() @ w_proj[h].double()).cpu().numpy()[:, :, None]
        p = O.Positional("rope", cos=ocos, sin=osin)
        o_out, o_lse, o_dq, _ = _slice_oracle(sl(q), sl(k), sl(v), sl(dout), w, fmap, cache, 50.0, p, rows,
                                              L - 1)
        close(f"c5 out {h}", f64(out[0, rows, h]), o_out[0, rows, 0])
        close(f"c5 lse {h}", f64(lse[0, rows, h]), o_lse[0, rows, 0])
        close(f"c5 dq {h}", f64(dq[0, rows, h]), o_dq[0, rows, 0])
        _check_nodes(f"c5 {h}", dk, dv, 0, h, sl(q), sl(k), sl(v), sl(dout), w, fmap, cache, 50.0, p, L - 1,
                     [(0, 131071), (1, 65023), (2, 31999), (3, 15487), (5, 3103), (7, 7)])


def test_config2_block_forward_full_size(dev):
    B, N, H, D, L, W, K, E = 2, 8192, 16, 128, 6, 256, 4, 2048
    fmap, cache = {l: l * W for l in range(1, L)}, L * W
    g = torch.Generator(device=dev)
    g.manual_seed(202)
    bf = torch.bfloat16
    x = torch.randn(B, N, E, generator=g, device=dev, dtype=bf)
    wq, wk, wv, wg = ((0.02 * torch.randn(H * D, E, generator=g, device=dev)).to(bf) for _ in range(4))
    q, k, v = (x.matmul(w_.t()).reshape(B, N, H, D) for w_ in (wq, wk, wv))
    kcw = torch.randn(H * D, K, generator=g, device=dev) / math.sqrt(K)
    vcw = torch.randn(H * D, K, generator=g, device=dev) / math.sqrt(K)
    w_proj = (0.02 * torch.randn(H, E, generator=g, device=dev)).to(bf)
    sinks = torch.randn(H, generator=g, device=dev)
    cos, sin = T.rope_tables(N, D, device=dev)
    kl, vl, _ = T.build_dyadic_summaries(q, k, v, L - 1, x=x, w_proj=w_proj, k_conv_weight=kcw,
                                         v_conv_weight=vcw)
    out, lse = T.multilevel_attention_forward(q, T.pack_levels(kl, vl), fmap, cache, softcap=30.0,
                                              position_mode="rope", rope_cos=cos, rope_sin=sin)
    y = T.apply_output_gate(T.apply_attention_sink(out, lse, sinks), x, wg)
    ocos, osin = O.rope_tables(N, D)
    opos = O.Positional("rope", cos=ocos, sin=osin)
    rows = [0, 255, 1000, 4097, 8191]
    for b, h in ((0, 3), (1, 14)):
        sl = lambda t: f64(t[b:b + 1, :, h:h + 1])  # noqa: E731
        kc = O.short_conv(sl(k).reshape(1, N, D), f64(kcw[h * D:(h + 1) * D])).reshape(1, N, 1, D)
        vc = O.short_conv(sl(v).reshape(1, N, D), f64(vcw[h * D:(h + 1) * D])).reshape(1, N, 1, D)
        w = O.linear_weights(f64(x[b:b + 1]), f64(w_proj[h:h + 1]))
        kl_o, vl_o, _ = O.build_tree(kc, vc, w, L - 1)
        o_out, o_lse = O.forward(sl(q), kl_o, vl_o, fmap, cache, 30.0, opos, rows=rows)
        sunk = O.sink_forward(o_out[:, rows], o_lse[:, rows], f64(sinks[h:h + 1]))
        gated = O.output_gate(sunk, f64(x[b:b + 1, rows]), f64(wg[h * D:(h + 1) * D]))
        close(f"c2 gated out {b},{h}", f64(y[b, rows, h]), gated[0, :, 0])
        close(f"c2 lse {b},{h}", f64(lse[b, rows, h]), o_lse[0, rows, 0])


def test_config4_decode_equals_forward(dev):
    B, H, D, L, W, K, E = 64, 16, 128, 8, 256, 4, 2048
    P, steps = 32768, 3
    N = P + steps
    fmap, cache = {l: l * W for l in range(1, L)}, L * W
    g = torch.Generator(device=dev)
    g.manual_seed(404)
    bf = torch.bfloat16
    q, k, v = (torch.randn(B, N, H, D, generator=g, device=dev, dtype=bf) for _ in range(3))
    x = torch.randn(B, N, E, generator=g, device=dev, dtype=bf)
    kcw = torch.randn(H * D, K, generator=g, device=dev) / math.sqrt(K)
    vcw = torch.randn(H * D, K, generator=g, device=dev) / math.sqrt(K)
    sinks = torch.randn(H, generator=g, device=dev)
    gate_w = (0.02 * torch.randn(H * D, E, generator=g, device=dev)).to(bf)
    cos, sin = T.rope_tables(N + 1, D, device=dev)
    rope = dict(position_mode="rope", rope_cos=cos, rope_sin=sin)
    # the whole sequence at once: builder, forward, sink, gate
    kl, vl, _ = T.build_dyadic_summaries(q, k, v, L - 1, k_conv_weight=kcw, v_conv_weight=vcw)
    out, lse = T.multilevel_attention_forward(q, T.pack_levels(kl, vl), fmap, cache, softcap=20.0, **rope)
    want = T.apply_output_gate(T.apply_attention_sink(out, lse, sinks), x, gate_w)[:, P:]
    want_lse = lse[:, P:]
    del kl, vl, out, lse
    # prefill the first P tokens, then decode the rest one token at a time
    kl, vl, wl = T.build_dyadic_summaries(q[:, :P], k[:, :P], v[:, :P], L - 1, k_conv_weight=kcw,
                                          v_conv_weight=vcw)
    st = T.init_decode_state(kl, vl, wl, fmap, cache, k_pre_conv=k[:, :P], v_pre_conv=v[:, :P],
                             conv_kernel_size=K)
    del kl, vl, wl
    dec_out, dec_lse = [], []
    for i in range(steps):
        t = P + i
        o, l = T.decode_step(x[:, t:t + 1], q[:, t:t + 1], k[:, t:t + 1], v[:, t:t + 1], st, k_conv_weight=kcw,
                             v_conv_weight=vcw, softcap=20.0, sinks=sinks, gate_weight=gate_w, **rope)
        close(f"c4 decode out t={t}", f64(o[:, 0]), f64(want[:, i]))
        close(f"c4 decode lse t={t}", f64(l[:, 0]), f64(want_lse[:, i]))
        dec_out.append(f64(o[:, 0]))
        dec_lse.append(f64(l[:, 0]))
    # the float64 oracle's full-sequence rows of two (batch, head) slices:
    # conv, qk merge weights, tree, rope forward, sink and SiLU gate
    ocos, osin = O.rope_tables(N + 1, D)
    opos = O.Positional("rope", cos=ocos, sin=osin)
    rows = list(range(P, N))
    for b, h in ((5, 3), (60, 12)):
        sl = lambda t: f64(t[b:b + 1, :, h:h + 1])  # noqa: E731
        qs = sl(q)
        kc = O.short_conv(sl(k).reshape(1, N, D), f64(kcw[h * D:(h + 1) * D])).reshape(1, N, 1, D)
        vc = O.short_conv(sl(v).reshape(1, N, D), f64(vcw[h * D:(h + 1) * D])).reshape(1, N, 1, D)
        kl_o, vl_o, _ = O.build_tree(kc, vc, O.qk_weights(qs, kc), L - 1)
        o_out, o_lse = O.forward(qs, kl_o, vl_o, fmap, cache, 20.0, opos, rows=rows)
        sunk = O.sink_forward(o_out[:, rows], o_lse[:, rows], f64(sinks[h:h + 1]))
        gated = O.output_gate(sunk, f64(x[b:b + 1, P:N]), f64(gate_w[h * D:(h + 1) * D]))
        for i in range(steps):
            close(f"c4 decode out vs oracle b={b} h={h} t={P + i}", dec_out[i][b, h], gated[0, i, 0])
            close(f"c4 decode lse vs oracle b={b} h={h} t={P + i}", dec_lse[i][b, h], o_lse[0, P + i, 0])
