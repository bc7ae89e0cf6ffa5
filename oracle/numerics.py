"""Float64 oracle for the numerics of the hot path (TEST INFRASTRUCTURE, see
``oracle/__init__.py``).

Per-query visible-entry enumeration with ordinary (non-online) softmax, in the
spirit of the reference's semantic oracle ``minimal_reference.py``, plus an
explicit float64 VJP.  Every function cites the reference lines it restates.

Mixed precision: the reference stores each intermediate that it returns (tree
levels, rotated Q/K, decode rings) in the input dtype.  The functions below
take a ``store`` rounding function (``identity``, ``to_fp32`` or ``to_bf16``)
that is applied exactly where the reference writes such a tensor, and compute
everything else in float64.
"""

import math
from typing import Dict, List, Optional, Sequence

import numpy as np

from . import schedule as S


# ----------------------------------------------------------------------------
# dtype emulation
# ----------------------------------------------------------------------------

def identity(x):
    return np.asarray(x, dtype=np.float64)


def to_fp32(x):
    return np.asarray(x, dtype=np.float32).astype(np.float64)


def to_bf16(x):
    """Round to bfloat16 (round-to-nearest-even on the float32 bit pattern)."""
    u = np.ascontiguousarray(np.asarray(x, dtype=np.float32)).view(np.uint32)
    u = (u + (((u >> 16) & 1) + 0x7FFF)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32).astype(np.float64)


STORE = {"fp64": identity, "fp32": to_fp32, "bf16": to_bf16}


# ----------------------------------------------------------------------------
# Phase 1: short conv, merge weights, dyadic tree
# ----------------------------------------------------------------------------

def _same_segment(seq_idx, n, back):
    """[B, n - back, 1] mask: rows t and t - back belong to one segment
    (all ones without segment ids)."""
    if seq_idx is None:
        return 1.0
    s = np.asarray(seq_idx)
    return (s[:, back:] == s[:, : n - back])[..., None].astype(np.float64)


def short_conv(x, weight, seq_idx=None):
    """y[b,t,c] = x[b,t,c] + sum_j weight[c,j] x[b,t-K+1+j,c], causal, zero
    left padding (reference.py:167-211).  Returns float64 (caller rounds).
    seq_idx [B, N] (the reset the reference leaves as a TODO at
    reference.py:186-189): a tap at row s reaches row t only when
    seq_idx[b, s] == seq_idx[b, t]."""
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(weight, dtype=np.float64)
    n = x.shape[1]
    kk = w.shape[1]
    y = np.zeros_like(x)
    for j in range(kk):
        back = kk - 1 - j
        if back < n:
            y[:, back:, :] += w[:, j] * x[:, : n - back, :] * _same_segment(seq_idx, n, back)
    return x + y


def qk_weights(q, k):
    """w[b,t,hkv] = logsumexp_e(q[b,t,hkv*E+e] . k[b,t,hkv] / sqrt(Dk))
    (reference.py:117-145).  -> [B, N, Hkv]."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    b, n, hq, dk = q.shape
    hkv = k.shape[2]
    s = np.einsum("bnhed,bnhd->bnhe", q.reshape(b, n, hkv, hq // hkv, dk), k) / math.sqrt(dk)
    m = s.max(axis=-1, keepdims=True)
    return (m + np.log(np.exp(s - m).sum(axis=-1, keepdims=True)))[..., 0]


def linear_weights(x, w_proj):
    """w = x @ w_proj^T (reference.py:148-164).  -> [B, N, Hkv]."""
    return np.asarray(x, np.float64) @ np.asarray(w_proj, np.float64).T


def build_tree(k, v, w, num_summary_levels, store=identity):
    """Dyadic K/V/w tree, level 0 = the inputs (reference.py:545-584).

    Each parent merges children (2j, 2j+1) with alpha = softmax(w0, w1) and
    takes w = logsumexp(w0, w1); odd trailing nodes are dropped.  Every level
    is rounded by `store` (the reference keeps levels in the input dtype).
    Returns lists (k_levels [B,n,Hkv,Dk], v_levels, w_levels [B,n,Hkv]).
    """
    kl = [store(k)]
    vl = [store(v)]
    wl = [store(w)]
    for _ in range(num_summary_levels):
        kp, vp, wp = kl[-1], vl[-1], wl[-1]
        half = kp.shape[1] // 2
        k0, k1 = kp[:, 0:2 * half:2], kp[:, 1:2 * half:2]
        v0, v1 = vp[:, 0:2 * half:2], vp[:, 1:2 * half:2]
        w0, w1 = wp[:, 0:2 * half:2], wp[:, 1:2 * half:2]
        m = np.maximum(w0, w1)
        e0, e1 = np.exp(w0 - m), np.exp(w1 - m)
        a0, a1 = e0 / (e0 + e1), e1 / (e0 + e1)
        kl.append(store(a0[..., None] * k0 + a1[..., None] * k1))
        vl.append(store(a0[..., None] * v0 + a1[..., None] * v1))
        wl.append(store(m + np.log(e0 + e1)))
    return kl, vl, wl


def short_conv_vjp(x, weight, dy, seq_idx=None):
    """VJP of short_conv: dx[s] = dy[s] + sum_j weight[c,j] dy[s+K-1-j] and
    dweight[c,j] = sum_{b,t} dy[t,c] x[t-K+1+j,c] (zero padding; with
    seq_idx only taps within one segment)."""
    x = np.asarray(x, np.float64)
    w = np.asarray(weight, np.float64)
    dy = np.asarray(dy, np.float64)
    n, kk = x.shape[1], w.shape[1]
    dx = dy.copy()
    dw = np.zeros_like(w)
    for j in range(kk):
        back = kk - 1 - j
        if back < n:
            g = dy[:, back:, :] * _same_segment(seq_idx, n, back)
            dx[:, : n - back, :] += w[:, j] * g
            dw[:, j] = np.einsum("btc,btc->c", g, x[:, : n - back, :])
    return dx, dw


def build_tree_vjp(q, k, v, num_summary_levels, dk_packed, dv_packed, dw_packed, x=None, w_proj=None,
                   k_conv_weight=None, v_conv_weight=None, detach_weights=False):
    """VJP of build_dyadic_summaries (reference.py:465-584) in float64 for
    upstream gradients of the packed levels dk_packed [B, total, Hkv, Dk],
    dv_packed [B, total, Hkv, Dv] and dw_packed [B, total, Hkv].

    Forward as the reference: optional short conv of k and v, merge weights
    (qk logsumexp over the GQA group, or x @ w_proj^T), then per level
    alpha = softmax(w0, w1), parent = alpha0 child0 + alpha1 child1,
    w_parent = logsumexp(w0, w1).  Backward from the coarsest level down:
      dchild_i += alpha_i dparent                       (k and v)
      dalpha_i  = dk_parent . k_child_i + dv_parent . v_child_i
      dw_i     += alpha_i (dalpha_i - sum_j alpha_j dalpha_j) + alpha_i dw_parent
    then level 0's dw through the weights (cut by detach_weights) and dk, dv
    through the conv.  Returns a dict of dq, dk, dv and, when present, dx,
    dw_proj, dkcw, dvcw (float64)."""
    q = np.asarray(q, np.float64)
    k_pre = np.asarray(k, np.float64)
    v_pre = np.asarray(v, np.float64)
    B, N, Hkv, Dk = k_pre.shape
    Dv = v_pre.shape[-1]
    k0, v0 = k_pre, v_pre
    if k_conv_weight is not None:
        k0 = short_conv(k_pre.reshape(B, N, Hkv * Dk), k_conv_weight).reshape(B, N, Hkv, Dk)
        v0 = short_conv(v_pre.reshape(B, N, Hkv * Dv), v_conv_weight).reshape(B, N, Hkv, Dv)
    w0 = linear_weights(x, w_proj) if x is not None else qk_weights(q, k0)
    kl, vl, wl = build_tree(k0, v0, w0, num_summary_levels)
    offs = np.cumsum([0] + [a.shape[1] for a in kl])
    gk = [np.array(dk_packed[:, offs[l]:offs[l + 1]], np.float64) for l in range(len(kl))]
    gv = [np.array(dv_packed[:, offs[l]:offs[l + 1]], np.float64) for l in range(len(kl))]
    gw = [np.array(dw_packed[:, offs[l]:offs[l + 1]], np.float64) for l in range(len(kl))]
    for l in range(len(kl) - 1, 0, -1):
        npar = kl[l].shape[1]
        if npar == 0:
            continue
        c0, c1 = slice(0, 2 * npar, 2), slice(1, 2 * npar, 2)
        wc0, wc1 = wl[l - 1][:, c0], wl[l - 1][:, c1]
        m = np.maximum(wc0, wc1)
        e0, e1 = np.exp(wc0 - m), np.exp(wc1 - m)
        a0, a1 = e0 / (e0 + e1), e1 / (e0 + e1)
        dkp, dvp, dwp = gk[l], gv[l], gw[l]
        gk[l - 1][:, c0] += a0[..., None] * dkp
        gk[l - 1][:, c1] += a1[..., None] * dkp
        gv[l - 1][:, c0] += a0[..., None] * dvp
        gv[l - 1][:, c1] += a1[..., None] * dvp
        da0 = (dkp * kl[l - 1][:, c0]).sum(-1) + (dvp * vl[l - 1][:, c0]).sum(-1)
        da1 = (dkp * kl[l - 1][:, c1]).sum(-1) + (dvp * vl[l - 1][:, c1]).sum(-1)
        sa = a0 * da0 + a1 * da1
        gw[l - 1][:, c0] += a0 * (da0 - sa) + a0 * dwp
        gw[l - 1][:, c1] += a1 * (da1 - sa) + a1 * dwp
    dk0, dv0, dw0 = gk[0], gv[0], gw[0]
    out = {"dq": np.zeros_like(q)}
    if not detach_weights:
        if x is not None:
            xx = np.asarray(x, np.float64)
            out["dx"] = dw0 @ np.asarray(w_proj, np.float64)
            out["dw_proj"] = np.einsum("bnh,bne->he", dw0, xx)
        else:
            Hq = q.shape[2]
            E = Hq // Hkv
            qg = q.reshape(B, N, Hkv, E, Dk)
            sc = 1.0 / math.sqrt(Dk)
            s_ = np.einsum("bnhed,bnhd->bnhe", qg, k0) * sc
            p = np.exp(s_ - s_.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            ds = dw0[..., None] * p
            out["dq"] = (ds[..., None] * k0[:, :, :, None, :] * sc).reshape(B, N, Hq, Dk)
            dk0 = dk0 + np.einsum("bnhe,bnhed->bnhd", ds, qg) * sc
    elif x is not None:
        out["dx"] = np.zeros(np.shape(x))
        out["dw_proj"] = np.zeros(np.shape(w_proj))
    if k_conv_weight is not None:
        dk, out["dkcw"] = short_conv_vjp(k_pre.reshape(B, N, Hkv * Dk), k_conv_weight,
                                         dk0.reshape(B, N, Hkv * Dk))
        dv, out["dvcw"] = short_conv_vjp(v_pre.reshape(B, N, Hkv * Dv), v_conv_weight,
                                         dv0.reshape(B, N, Hkv * Dv))
        out["dk"], out["dv"] = dk.reshape(B, N, Hkv, Dk), dv.reshape(B, N, Hkv, Dv)
    else:
        out["dk"], out["dv"] = dk0, dv0
    return out


def pack(levels):
    """Level-major concatenation [L0 | L1 | ...] along the sequence axis
    (reference.py:604-640)."""
    return np.concatenate(levels, axis=1)


# ----------------------------------------------------------------------------
# positional helpers
# ----------------------------------------------------------------------------

def rope_tables(n_pos, dim, base=10000.0):
    """cos/sin [n_pos, dim/2], theta_i = base^(-2i/dim), evaluated in float32
    exactly as the reference builds them (reference.py:240-264)."""
    inv = np.power(np.float32(base), -np.arange(0, dim, 2, dtype=np.float32) / np.float32(dim))
    inv = inv.astype(np.float32)
    ang = (np.arange(n_pos, dtype=np.float32)[:, None] * inv[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rotate(x, pos, cos, sin, inverse=False):
    """Rotate-half RoPE on the last axis at integer positions `pos`
    (broadcastable to x.shape[:-1]) (reference.py:267-302)."""
    x = np.asarray(x, np.float64)
    d = x.shape[-1]
    c = np.asarray(cos, np.float64)[pos]
    s = np.asarray(sin, np.float64)[pos]
    if inverse:
        s = -s
    x1, x2 = x[..., : d // 2], x[..., d // 2:]
    return np.concatenate([x1 * c - x2 * s, x2 * c + x1 * s], axis=-1)


# ----------------------------------------------------------------------------
# Phase 2 forward / backward by per-query enumeration
# ----------------------------------------------------------------------------

def _entries(q, a, cache):
    """Visible entries of q as arrays (levels, js, dists), oldest first."""
    rr = S.row_ranges(q, a, cache)
    lv, js = [], []
    for l, (lo, hi) in enumerate(rr):
        lv.extend([l] * (hi - lo))
        js.extend(range(lo, hi))
    lv = np.asarray(lv, dtype=np.int64)
    js = np.asarray(js, dtype=np.int64)
    order = np.argsort(js << lv, kind="stable")
    lv, js = lv[order], js[order]
    m = len(lv)
    return lv, js, (m - 1) - np.arange(m)


def _gather(levels, lv, js):
    """Stack the entries (lv[i], js[i]) of a list of [B, n, H, D] levels into
    [B, M, H, D]."""
    return np.stack([levels[l][:, j] for l, j in zip(lv, js)], axis=1)


class Positional:
    """Positional arguments of one call (reference.py:675-768 semantics)."""

    def __init__(self, mode="none", cos=None, sin=None, states=None, proj=None):
        self.mode = mode
        self.cos, self.sin = cos, sin
        self.rel = None
        if mode == "relative":
            self.rel = np.einsum("bnhd,dr->bnhr", np.asarray(states, np.float64),
                                 np.asarray(proj, np.float64))


def _row_scores(qrow, kent, lv, js, dists, qi, b_rel, pos: Positional, e, scale, store):
    """Raw pre-softcap logits X [B, Hq, M] of one query row and the rotated
    operands.  qrow [B, Hq, Dk]; kent [B, M, Hkv, Dk]."""
    if pos.mode == "rope":
        qrow = store(rotate(qrow, qi, pos.cos, pos.sin))
        kpos = (js + 1) * (np.left_shift(1, lv)) - 1
        kent = store(rotate(kent, kpos[None, :, None], pos.cos, pos.sin))
    kq = np.repeat(kent, e, axis=2)  # [B, M, Hq, Dk], hq = hkv*E + e
    x = np.einsum("bhd,bmhd->bhm", qrow, kq) * scale
    if pos.mode == "relative":
        rel = pos.rel[:, qi]  # [B, Hq, R]
        if dists.max() >= rel.shape[-1]:
            raise ValueError("relative bin distance exceeds max_relative_bins")
        x = x + rel[:, :, dists]
    return x, qrow, kq


def forward(q, k_levels, v_levels, fmap, cache, softcap, pos: Optional[Positional] = None,
            store=identity, rows=None):
    """(out [B,N,Hq,Dv], lse [B,N,Hq]) with S = c tanh(X/c) (or X), X = q.k/sqrt(Dk)
    [+ bias], softmax over exactly the visible set (reference.py:771-1071;
    minimal_reference.py semantics).  lse is the natural-log pre-sink LSE.
    `rows` restricts the computation to those query rows (others stay 0)."""
    pos = pos or Positional()
    a = S.activation_times(fmap)
    q = np.asarray(q, np.float64)
    b, n, hq, dk = q.shape
    hkv = k_levels[0].shape[2]
    e = hq // hkv
    dv = v_levels[0].shape[-1]
    scale = 1.0 / math.sqrt(dk)
    out = np.zeros((b, n, hq, dv))
    lse = np.zeros((b, n, hq))
    for qi in (range(n) if rows is None else rows):
        lv, js, dists = _entries(qi, a, cache)
        if len(lv) == 0:
            raise RuntimeError(f"query {qi} has no visible entries")
        kent = _gather(k_levels, lv, js)
        vent = np.repeat(_gather(v_levels, lv, js), e, axis=2)
        x, _, _ = _row_scores(q[:, qi], kent, lv, js, dists, qi, None, pos, e, scale, store)
        s = softcap * np.tanh(x / softcap) if softcap is not None else x
        m = s.max(axis=-1, keepdims=True)
        p = np.exp(s - m)
        ell = p.sum(axis=-1, keepdims=True)
        lse[:, qi] = (m + np.log(ell))[..., 0]
        out[:, qi] = np.einsum("bhm,bmhd->bhd", p / ell, vent)
    return out, lse


def backward(q, k_levels, v_levels, out, lse, dout, fmap, cache, softcap,
             pos: Optional[Positional] = None, dlse=None, store=identity, rows=None):
    """Explicit float64 VJP at the packed boundary (reference.py:1222-1672):
    P = exp(S - lse_saved), dP = dO.V, Delta = sum(dO*O) - dlse,
    dS = P (dP - Delta), dX = dS (1 - tanh^2), dQ = scale dX K, dK = scale dX^T Q,
    dV = P^T dO, dbias = dX; RoPE gradients are rotated back by R(-p).

    Returns (dq [B,N,Hq,Dk], dk_levels, dv_levels, drel [B,N,Hq,R] or None).
    """
    pos = pos or Positional()
    a = S.activation_times(fmap)
    q = np.asarray(q, np.float64)
    dout = np.asarray(dout, np.float64)
    b, n, hq, dk = q.shape
    hkv = k_levels[0].shape[2]
    e = hq // hkv
    scale = 1.0 / math.sqrt(dk)
    delta = (dout * np.asarray(out, np.float64)).sum(-1)
    if dlse is not None:
        delta = delta - np.asarray(dlse, np.float64)
    dq = np.zeros_like(q)
    dkl = [np.zeros(kl.shape) for kl in k_levels]
    dvl = [np.zeros(vl.shape) for vl in v_levels]
    drel = np.zeros(pos.rel.shape) if pos.mode == "relative" else None
    for qi in (range(n) if rows is None else rows):
        lv, js, dists = _entries(qi, a, cache)
        kent = _gather(k_levels, lv, js)
        vent = np.repeat(_gather(v_levels, lv, js), e, axis=2)
        x, qrow, kq = _row_scores(q[:, qi], kent, lv, js, dists, qi, None, pos, e, scale, store)
        if softcap is not None:
            t = np.tanh(x / softcap)
            s = softcap * t
            grad = 1.0 - t * t
        else:
            s, grad = x, 1.0
        p = np.exp(s - np.asarray(lse, np.float64)[:, qi, :, None])
        dp = np.einsum("bhd,bmhd->bhm", dout[:, qi], vent)
        ds = p * (dp - delta[:, qi, :, None])
        dx = ds * grad
        dq_rot = scale * np.einsum("bhm,bmhd->bhd", dx, kq)
        dk_c = scale * np.einsum("bhm,bhd->bmhd", dx, qrow)  # per query head
        dv_c = np.einsum("bhm,bhd->bmhd", p, dout[:, qi])
        dk_c = dk_c.reshape(b, len(lv), hkv, e, dk).sum(axis=3)
        dv_c = dv_c.reshape(b, len(lv), hkv, e, dv_c.shape[-1]).sum(axis=3)
        if pos.mode == "rope":
            dq[:, qi] = rotate(dq_rot, qi, pos.cos, pos.sin, inverse=True)
            kpos = (js + 1) * (np.left_shift(1, lv)) - 1
            dk_c = rotate(dk_c, kpos[None, :, None], pos.cos, pos.sin, inverse=True)
        else:
            dq[:, qi] = dq_rot
        for l in np.unique(lv):
            sel = lv == l
            dkl[l][:, js[sel]] += dk_c[:, sel]
            dvl[l][:, js[sel]] += dv_c[:, sel]
        if drel is not None:
            drel[:, qi][:, :, dists] = dx
    return dq, dkl, dvl, drel


# ----------------------------------------------------------------------------
# post-ops
# ----------------------------------------------------------------------------

def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def sink_forward(out, lse, sinks, store=identity):
    """out * sigmoid(lse - s_h), the scale rounded to out's dtype
    (reference.py:1082-1122)."""
    r = store(sigmoid(np.asarray(lse, np.float64) - np.asarray(sinks, np.float64)[None, None, :]))
    return np.asarray(out, np.float64) * r[..., None]


def sink_backward(out, lse, sinks, dout, store=identity):
    """(dout_pre, dlse, dsinks) (reference.py:1125-1184)."""
    r = sigmoid(np.asarray(lse, np.float64) - np.asarray(sinks, np.float64)[None, None, :])
    dout = np.asarray(dout, np.float64)
    dout_pre = dout * store(r)[..., None]
    g = (dout * np.asarray(out, np.float64)).sum(-1)
    dlse = g * r * (1.0 - r)
    return dout_pre, dlse, -dlse.sum(axis=(0, 1))


def silu(x):
    return x * sigmoid(x)


def output_gate(out, x, gate_weight):
    """SiLU(x @ W_g^T).reshape(B, N, Hq, Dv) * out (reference.py:1187-1219)."""
    out = np.asarray(out, np.float64)
    b, n, hq, dv = out.shape
    g = silu(np.asarray(x, np.float64) @ np.asarray(gate_weight, np.float64).T)
    return g.reshape(b, n, hq, dv) * out


# ----------------------------------------------------------------------------
# incremental decode
# ----------------------------------------------------------------------------

class DecodeState:
    """Ring cache (reference.py:1703-1736): k/v [B, sum(caps), Hkv, D],
    w [B, sum(caps), Hkv], conv rows [B, K-1, C] or None, t = next query."""

    def __init__(self, k, v, w, conv_k, conv_v, t, a, cache, caps):
        self.k, self.v, self.w = k, v, w
        self.conv_k, self.conv_v = conv_k, conv_v
        self.t = t
        self.a = tuple(a)
        self.cache = cache
        self.caps = tuple(caps)
        self.offsets = S.ring_offsets(caps)

    def slot(self, level, j):
        return S.ring_slot(self.offsets, self.caps, level, j)


def init_decode_state(k_levels, v_levels, w_levels, fmap, cache,
                      k_pre=None, v_pre=None, kernel_size=None, store=identity):
    """Prefill hand-off: the nodes live at query N-1 go to their ring slots;
    the last K-1 pre-conv rows seed the conv history (reference.py:1848-1945)."""
    a = S.activation_times(fmap)
    top = len(a) - 1
    b, n, hkv, dk = k_levels[0].shape
    dv = v_levels[0].shape[-1]
    caps = S.decode_caps(a, cache)
    total = sum(caps)
    st = DecodeState(np.zeros((b, total, hkv, dk)), np.zeros((b, total, hkv, dv)),
                     np.zeros((b, total, hkv)), None, None, n, a, cache, caps)
    rr = S.row_ranges(n - 1, a, cache)
    for lv in range(top + 1):
        lo, hi = rr[lv]
        for j in range(lo, hi):
            s = st.slot(lv, j)
            st.k[:, s] = k_levels[lv][:, j]
            st.v[:, s] = v_levels[lv][:, j]
            st.w[:, s] = w_levels[lv][:, j]
    if k_pre is not None:
        hist = kernel_size - 1

        def history(x):
            x = np.asarray(x, np.float64).reshape(b, n, -1)
            h = np.zeros((b, hist, x.shape[-1]))
            take = min(hist, n)
            if take:
                h[:, hist - take:] = x[:, n - take:]
            return h

        st.conv_k, st.conv_v = history(k_pre), history(v_pre)
    return st


def conv_step(x_row, hist, weight):
    """One-token short conv: y = x + sum_j w[:, j] full[j], full = hist ++ x
    (reference.py:1810-1845).  -> (y [B, C], new history)."""
    full = np.concatenate([hist, x_row[:, None, :]], axis=1)
    y = x_row + np.einsum("bkc,ck->bc", full, np.asarray(weight, np.float64))
    return y, full[:, 1:]


def advance(st: DecodeState, q_t, k_t, v_t, x_t=None, w_proj=None, kcw=None, vcw=None,
            store=identity):
    """Consume token t = st.t: conv step, merge weight, the single ruler-tick
    merge, then the level-0 write (reference.py:1948-2090)."""
    t = st.t
    b, _, hkv, dk = k_t.shape
    dv = v_t.shape[-1]
    k_t = np.asarray(k_t, np.float64)
    v_t = np.asarray(v_t, np.float64)
    if kcw is not None:
        kf, st.conv_k = conv_step(k_t.reshape(b, -1), st.conv_k, kcw)
        vf, st.conv_v = conv_step(v_t.reshape(b, -1), st.conv_v, vcw)
        st.conv_k, st.conv_v = store(st.conv_k), store(st.conv_v)
        k_t = store(kf).reshape(b, 1, hkv, dk)
        v_t = store(vf).reshape(b, 1, hkv, dv)
    if x_t is not None:
        w_t = store(linear_weights(x_t, w_proj))  # [B, 1, Hkv]
    else:
        w_t = store(qk_weights(q_t, k_t))
    a = st.a
    top = len(a) - 1
    for lv in range(1, top + 1):
        if t >= a[lv] and (t - a[lv]) % (1 << lv) == 0:
            j = (t - a[lv]) >> lv
            c0, c1, par = st.slot(lv - 1, 2 * j), st.slot(lv - 1, 2 * j + 1), st.slot(lv, j)
            w0, w1 = st.w[:, c0], st.w[:, c1]
            m = np.maximum(w0, w1)
            e0, e1 = np.exp(w0 - m), np.exp(w1 - m)
            a0, a1 = e0 / (e0 + e1), e1 / (e0 + e1)
            st.k[:, par] = store(a0[..., None] * st.k[:, c0] + a1[..., None] * st.k[:, c1])
            st.v[:, par] = store(a0[..., None] * st.v[:, c0] + a1[..., None] * st.v[:, c1])
            st.w[:, par] = store(m + np.log(e0 + e1))
    s0 = st.slot(0, t)
    st.k[:, s0] = k_t[:, 0]
    st.v[:, s0] = v_t[:, 0]
    st.w[:, s0] = w_t[:, 0]
    st.t = t + 1


def decode_attend(st: DecodeState, q_t, softcap, pos: Optional[Positional] = None,
                  store=identity):
    """Attention of query t = st.t - 1 over its ring entries
    (reference.py:2093-2239).  -> (out [B,1,Hq,Dv], lse [B,1,Hq])."""
    pos = pos or Positional()
    t = st.t - 1
    q_t = np.asarray(q_t, np.float64)
    b, _, hq, dk = q_t.shape
    hkv = st.k.shape[2]
    e = hq // hkv
    lv, js, dists = _entries(t, st.a, st.cache)
    slots = [st.slot(l, j) for l, j in zip(lv, js)]
    kent = st.k[:, slots]
    vent = np.repeat(st.v[:, slots], e, axis=2)
    scale = 1.0 / math.sqrt(dk)
    if pos.mode == "relative":
        # decode states are [B, 1, Hq, d_rel]: the row index is 0
        x, _, _ = _row_scores(q_t[:, 0], kent, lv, js, dists, 0, None, pos, e, scale, store)
    else:
        x, _, _ = _row_scores(q_t[:, 0], kent, lv, js, dists, t, None, pos, e, scale, store)
    s = softcap * np.tanh(x / softcap) if softcap is not None else x
    m = s.max(axis=-1, keepdims=True)
    p = np.exp(s - m)
    ell = p.sum(axis=-1, keepdims=True)
    out = np.einsum("bhm,bmhd->bhd", p / ell, vent)
    return out[:, None], (m + np.log(ell))[..., 0][:, None]
