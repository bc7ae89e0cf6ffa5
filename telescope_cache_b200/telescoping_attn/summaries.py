"""Phase 1: merge weights, the short causal conv and the dyadic tree builder
(reference ``telescoping_attn/summaries.py`` / ``reference.py:113-584``).

The builder is one fused CUDA launch (``tc_build_tree``) that writes every
level straight into a level-major packed buffer; the per-level tensors it
returns are views of that buffer, so ``pack_levels`` on them copies nothing.

When an input requires gradients the packed buffers come from a
``torch.autograd.Function`` whose backward is the Phase-1 VJP in CUDA
(``tc_build_tree_bwd``: the pair merges from the coarsest level down and the
qk merge weights; ``tc_short_conv_bwd``: the conv), with the linear merge
weights' two GEMMs through cuBLAS -- the gradients the reference obtains from
torch autograd on ``build_dyadic_summaries``.  The same VJP is the explicit
call ``build_dyadic_summaries_backward``.
"""

import ctypes
from typing import Optional

import torch

from .. import _lib
from . import linear as _proj


def _contig(t):
    return t if t.is_contiguous() else t.contiguous()


def _qk_weights(q, k):
    B, N, Hq, Dk = q.shape
    Hkv = k.shape[2]
    out = torch.empty(B, N, Hkv, 1, device=q.device, dtype=q.dtype)
    _lib.launch("tc_qk_weights", q.device, B, N, Hq, Hkv, Dk, _lib.dtype_code(q.dtype), _lib.ptr(q),
                                        _lib.ptr(k), _lib.dtype_code(out.dtype), _lib.ptr(out),
                                        _lib.stream_of(q))
    return out


class _QKWeights(torch.autograd.Function):
    """compute_summary_weights with its VJP (tc_qk_weights_bwd) as backward:
    the gradients torch autograd gives the reference's logsumexp."""

    @staticmethod
    def forward(ctx, q, k):
        ctx.save_for_backward(q, k)
        return _qk_weights(q, k)

    @staticmethod
    def backward(ctx, gw):
        q, k = ctx.saved_tensors
        B, N, Hq, Dk = q.shape
        Hkv = k.shape[2]
        g = _contig(gw)
        dq, dk = torch.empty_like(q), torch.empty_like(k)
        _lib.launch("tc_qk_weights_bwd", q.device, B, N, Hq, Hkv, Dk, _lib.dtype_code(q.dtype),
                    _lib.ptr(q), _lib.ptr(k), _lib.dtype_code(g.dtype), _lib.ptr(g), _lib.ptr(dq),
                    _lib.ptr(dk), _lib.stream_of(q))
        return dq, dk


def compute_summary_weights(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """w[b, t, hkv] = logsumexp over the KV head's query group of
    q_h . k / sqrt(Dk).  q [B, N, Hq, Dk], k [B, N, Hkv, Dk] -> [B, N, Hkv, 1]
    in q's dtype (reference.py:117-145); differentiable in q and k."""
    B, N, Hq, Dk = q.shape
    _, Nk, Hkv, Dkk = k.shape
    assert N == Nk
    assert Dk == Dkk
    assert Hq % Hkv == 0
    _lib.require_cuda(q, k)
    # k in q's type (the cast carries its own gradient back to k's type)
    q, k = _contig(q), _contig(k.to(q.dtype))
    if torch.is_grad_enabled() and (q.requires_grad or k.requires_grad):
        return _QKWeights.apply(q, k)
    return _qk_weights(q, k)


def compute_linear_weights(x: torch.Tensor, w_proj: torch.Tensor) -> torch.Tensor:
    """w = x @ w_proj^T, the trained-linear merge weight.  x [B, N, E],
    w_proj [Hkv, E] -> [B, N, Hkv, 1] (reference.py:148-164)."""
    B, N, E = x.shape
    Hkv, Ew = w_proj.shape
    assert E == Ew
    _lib.require_cuda(x, w_proj)
    if x.dtype == w_proj.dtype:
        # the reference's x @ w_proj^T (with its gradients) on tc_linear
        return _proj.project(x, w_proj).unsqueeze(-1)
    x, w_proj = _contig(x), _contig(w_proj)
    out = torch.empty(B, N, Hkv, 1, device=x.device, dtype=torch.result_type(x, w_proj))
    _lib.launch("tc_linear_weights", x.device,
        B * N, E, Hkv, _lib.dtype_code(x.dtype), _lib.ptr(x), _lib.dtype_code(w_proj.dtype),
        _lib.ptr(w_proj), _lib.dtype_code(out.dtype), _lib.ptr(out), _lib.stream_of(x))
    return out


def _check_conv_weight(weight, C):
    if weight.dim() != 2 or weight.shape[0] != C:
        raise ValueError(
            f"conv weight shape {tuple(weight.shape)} incompatible with C={C}; expected [C, K]")
    if weight.shape[1] <= 0:
        raise ValueError(f"conv kernel size must be positive, got {weight.shape[1]}")


def _check_seq_idx(seq_idx, B, N, device):
    """seq_idx [B, N] integer segment ids -> contiguous int32 on device."""
    if seq_idx is None:
        return None
    if not torch.is_tensor(seq_idx) or seq_idx.dtype.is_floating_point or seq_idx.dtype == torch.bool:
        raise ValueError("seq_idx must be an integer tensor [B, N]")
    if tuple(seq_idx.shape) != (B, N):
        raise ValueError(f"seq_idx shape {tuple(seq_idx.shape)} != {(B, N)}")
    _lib.require_cuda(seq_idx)
    if seq_idx.device != device:
        raise ValueError("seq_idx must be on the same device as x")
    return seq_idx.to(torch.int32).contiguous()


def _conv_forward(x, weight, seq):
    B, N, C = x.shape
    y = torch.empty_like(x)
    _lib.launch("tc_short_conv_seg", x.device, B, N, C, _lib.dtype_code(x.dtype), _lib.ptr(x),
                weight.shape[1], _lib.dtype_code(weight.dtype), _lib.ptr(weight), _lib.ptr(seq),
                _lib.ptr(y), _lib.stream_of(x))
    return y


class _ShortConv(torch.autograd.Function):
    """short_conv with its VJP (tc_short_conv_seg_bwd) as backward."""

    @staticmethod
    def forward(ctx, x, weight, seq):
        ctx.save_for_backward(x, weight, seq)
        return _conv_forward(x, weight, seq)

    @staticmethod
    def backward(ctx, gy):
        x, weight, seq = ctx.saved_tensors
        dx, dw = _short_conv_vjp(x, weight, _contig(gy.float()), seq)
        return dx, dw, None


def short_conv(x: torch.Tensor, weight: torch.Tensor, seq_idx: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal depthwise conv with an fp32 residual, cast once:
    y[b,t,c] = x[b,t,c] + sum_j weight[c,j] x[b,t-K+1+j,c]
    (reference.py:167-211).  x [B, N, C], weight [C, K]; differentiable in x
    and weight.

    seq_idx (an extension; the reference leaves it as a TODO at
    reference.py:186-189): optional integer segment ids [B, N] of packed
    examples; the tap at row s reaches row t only when seq_idx[b, s] ==
    seq_idx[b, t], so each example's conv starts from zero history."""
    B, N, C = x.shape
    _check_conv_weight(weight, C)
    _lib.require_cuda(x, weight)
    x, weight = _contig(x), _contig(weight)
    seq = _check_seq_idx(seq_idx, B, N, x.device)
    if torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad):
        return _ShortConv.apply(x, weight, seq)
    return _conv_forward(x, weight, seq)


def _build_packed(q, k, v, num_summary_levels, x, w_proj, k_conv_weight, v_conv_weight):
    """The forward builder: (k_packed, v_packed, w_packed, level offsets)."""
    if (k_conv_weight is None) != (v_conv_weight is None):
        raise ValueError(
            "k_conv_weight and v_conv_weight must both be provided or both be None")
    B, N, Hkv, Dk = k.shape
    Dv = v.shape[-1]
    Hq = q.shape[2]
    conv_k = 0
    if k_conv_weight is not None:
        _check_conv_weight(k_conv_weight, Hkv * Dk)
        _check_conv_weight(v_conv_weight, Hkv * Dv)
        if k_conv_weight.shape[1] != v_conv_weight.shape[1]:
            raise NotImplementedError("K and V conv widths must match")
        conv_k = k_conv_weight.shape[1]
    if (x is None) != (w_proj is None):
        raise ValueError(
            "x and w_proj must both be provided (linear weight mode) or both be None "
            "(QK weight mode)")
    _lib.require_cuda(q, k, v, x, w_proj, k_conv_weight, v_conv_weight)
    dtype = v.dtype
    q, k, v = _contig(q.to(dtype)), _contig(k.to(dtype)), _contig(v)
    w0 = None
    if x is not None:
        w0 = compute_linear_weights(x, w_proj)
        expected = (B, N, Hkv, 1)
        if tuple(w0.shape) != expected:
            raise ValueError(f"linear weights shape {tuple(w0.shape)} != {expected}")
        w_dtype = w0.dtype
    else:
        if q.shape[0] != B or q.shape[1] != N or Hq % Hkv or q.shape[3] != Dk:
            raise ValueError(f"q shape {tuple(q.shape)} incompatible with k {tuple(k.shape)}")
        w_dtype = dtype
    L = int(num_summary_levels)
    if L < 0:
        raise ValueError("num_summary_levels must be non-negative")
    if L + 1 > _lib.MAX_LEVELS:
        raise NotImplementedError(f"at most {_lib.MAX_LEVELS - 1} summary levels are supported")
    lens = [N >> lv for lv in range(L + 1)]
    offs = [0]
    for n in lens:
        offs.append(offs[-1] + n)
    total = offs[-1]
    kp = torch.empty(B, total, Hkv, Dk, device=k.device, dtype=dtype)
    vp = torch.empty(B, total, Hkv, Dv, device=k.device, dtype=dtype)
    wp = torch.empty(B, total, Hkv, device=k.device, dtype=w_dtype)
    if N > 0:
        kcw = _contig(k_conv_weight) if conv_k else None
        vcw = _contig(v_conv_weight.to(k_conv_weight.dtype)) if conv_k else None
        args = _lib.TreeArgs(
            B=B, N=N, Hq=Hq, Hkv=Hkv, Dk=Dk, Dv=Dv, num_summary_levels=L,
            dtype=_lib.dtype_code(dtype), w_dtype=_lib.dtype_code(w_dtype),
            q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(),
            w0=None if w0 is None else w0.data_ptr(),
            k_conv_w=None if kcw is None else kcw.data_ptr(),
            v_conv_w=None if vcw is None else vcw.data_ptr(),
            conv_dtype=_lib.dtype_code(kcw.dtype) if conv_k else 0, conv_k=conv_k,
            k_packed=kp.data_ptr(), v_packed=vp.data_ptr(), w_packed=wp.data_ptr(), total=total)
        _lib.launch("tc_build_tree", k.device, ctypes.byref(args), _lib.stream_of(k))
    return kp, vp, wp, offs


class _DyadicTree(torch.autograd.Function):
    """Packed tree with the Phase-1 VJP as its backward."""

    @staticmethod
    def forward(ctx, q, k, v, x, w_proj, k_conv_weight, v_conv_weight, num_summary_levels, detach):
        kp, vp, wp, offs = _build_packed(q, k, v, num_summary_levels, x, w_proj, k_conv_weight,
                                         v_conv_weight)
        ctx.save_for_backward(q, k, v, x, w_proj, k_conv_weight, v_conv_weight, kp, vp, wp)
        ctx.cfg = (int(num_summary_levels), bool(detach), tuple(offs))
        return kp, vp, wp

    @staticmethod
    def backward(ctx, gkp, gvp, gwp):
        q, k, v, x, w_proj, kcw, vcw, kp, vp, wp = ctx.saved_tensors
        L, detach, _ = ctx.cfg
        return (*build_dyadic_summaries_backward(
            q, k, v, L, kp, vp, wp, gkp, gvp, gwp, detach_weights=detach, x=x, w_proj=w_proj,
            k_conv_weight=kcw, v_conv_weight=vcw), None, None)


def build_dyadic_summaries_backward(q, k, v, num_summary_levels, k_packed, v_packed, w_packed,
                                    dk_packed, dv_packed, dw_packed, detach_weights=False, x=None,
                                    w_proj=None, k_conv_weight=None, v_conv_weight=None):
    """Explicit Phase-1 VJP: gradients of build_dyadic_summaries' inputs from
    the upstream gradients of its packed outputs (the backward the reference
    gets from torch autograd through reference.py:117-211, 465-584).

    k_packed / v_packed / w_packed are the forward's packed buffers
    ([B, total, Hkv, D] and [B, total, Hkv] or [..., 1]); dk_packed /
    dv_packed / dw_packed the upstream gradients in the same shapes and
    element types, any of them None for zero.  Returns (dq, dk, dv, dx,
    dw_proj, dk_conv_weight, dv_conv_weight), None where the input is absent
    (dq is zeros in linear mode or with detach_weights, dx / dw_proj None
    with detach_weights)."""
    L, detach = int(num_summary_levels), bool(detach_weights)
    kp, vp = k_packed, v_packed
    wp = w_packed[..., 0] if w_packed.dim() == 4 else w_packed
    kcw, vcw = k_conv_weight, v_conv_weight
    B, N, Hkv, Dk = k.shape
    Dv, Hq = v.shape[-1], q.shape[2]
    dtype = kp.dtype
    total = kp.shape[1]
    linear = x is not None
    conv = kcw is not None
    dev = k.device
    if dw_packed is not None and dw_packed.dim() == 4:
        dw_packed = dw_packed[..., 0]
    ups = [None if g is None else _contig(g) for g in (dk_packed, dv_packed, dw_packed)]
    for g, ref in zip(ups, (kp, vp, wp)):
        if g is not None and (g.shape != ref.shape or g.dtype != ref.dtype):
            raise ValueError(f"upstream gradient {tuple(g.shape)} {g.dtype} does not match the packed "
                             f"output {tuple(ref.shape)} {ref.dtype}")
    kp, vp, wp = _contig(kp), _contig(vp), _contig(wp)
    qc = dq = dw0 = None
    if not linear and not detach:
        qc = _contig(q.to(dtype))
        dq = torch.empty(qc.shape, device=dev, dtype=dtype)
    if linear and not detach:
        dw0 = torch.empty(B, N, Hkv, device=dev, dtype=torch.float32)
    d0 = torch.float32 if conv else dtype  # the conv VJP takes fp32 gradients
    dk0 = torch.empty(B, N, Hkv, Dk, device=dev, dtype=d0)
    dv0 = torch.empty(B, N, Hkv, Dv, device=dev, dtype=d0)

    def addr(t):
        return None if t is None else t.data_ptr()

    args = _lib.TreeBwdArgs(
        B=B, N=N, Hq=Hq, Hkv=Hkv, Dk=Dk, Dv=Dv, num_summary_levels=L, dtype=_lib.dtype_code(dtype),
        w_dtype=_lib.dtype_code(wp.dtype), detach=int(detach), q=addr(qc),
        k_packed=kp.data_ptr(), v_packed=vp.data_ptr(), w_packed=wp.data_ptr(),
        gk_packed=addr(ups[0]), gv_packed=addr(ups[1]), gw_packed=addr(ups[2]),
        dq=addr(dq), dq_dtype=_lib.dtype_code(dtype), d0_dtype=_lib.dtype_code(d0),
        dk0=dk0.data_ptr(), dv0=dv0.data_ptr(), dw0=addr(dw0), total=total)
    nbytes = _lib.lib().tc_tree_bwd_scratch_bytes(ctypes.byref(args))
    if nbytes < 0:
        raise ValueError("tc_tree_bwd_scratch_bytes: invalid arguments")
    scratch = torch.empty(max(int(nbytes), 1), device=dev, dtype=torch.uint8)
    args.scratch, args.scratch_bytes = scratch.data_ptr(), int(nbytes)
    _lib.launch("tc_build_tree_bwd", k.device, ctypes.byref(args), _lib.stream_of(k))
    dq_out = torch.zeros_like(q) if dq is None else dq.to(q.dtype)
    dx = dwp = None
    if dw0 is not None:
        # w0 = x @ w_proj^T: dx = g w_proj (tc_linear) and dw_proj = g^T x
        # (tc_linear_wgrad), fp32 accumulation, results rounded to the
        # inputs' precision as autograd's products on the reference's
        # x @ w_proj^T are; dw0 is rounded to that precision first
        ct = torch.promote_types(x.dtype, w_proj.dtype)
        g = dw0.to(ct).reshape(-1, Hkv)
        dx = _proj.linear(g, w_proj.to(ct).t().contiguous()).to(x.dtype).reshape(x.shape)
        dwp = _proj.linear_wgrad(g, x.reshape(-1, x.shape[-1]).to(ct), ct).to(w_proj.dtype)
    dkcw = dvcw = None
    if conv:
        dk, dkcw = _short_conv_vjp(k, kcw, dk0)
        dv, dvcw = _short_conv_vjp(v, vcw, dv0)
    else:
        dk, dv = dk0.to(k.dtype), dv0.to(v.dtype)
    return dq_out, dk, dv, dx, dwp, dkcw, dvcw


def _short_conv_vjp(x_pre, weight, dy, seq=None):
    """dx (x_pre's dtype) and dweight (weight's dtype) of short_conv for fp32
    dy [B, N, H, D] or [B, N, C] (tc_short_conv_seg_bwd; seq: int32 segment
    ids [B, N] or None)."""
    B, N = x_pre.shape[:2]
    C = x_pre[0, 0].numel()
    K = weight.shape[1]
    xc = _contig(x_pre)
    wc = _contig(weight)
    dx = torch.empty_like(xc)
    dw = torch.empty(C, K, device=x_pre.device, dtype=torch.float32)
    parts = torch.empty(max(1, B * ((N + 255) // 256) * C * K), device=x_pre.device, dtype=torch.float32)
    _lib.launch("tc_short_conv_seg_bwd", x_pre.device,
        B, N, C, _lib.dtype_code(xc.dtype), _lib.ptr(xc), K, _lib.dtype_code(wc.dtype), _lib.ptr(wc),
        _lib.ptr(seq), _lib.ptr(dy), _lib.ptr(dx), _lib.ptr(dw), _lib.ptr(parts), parts.numel(),
        _lib.stream_of(xc))
    return dx.reshape(x_pre.shape), dw.to(weight.dtype)


def build_dyadic_summaries(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    num_summary_levels: int,
    detach_weights: bool = False,
    x: Optional[torch.Tensor] = None,
    w_proj: Optional[torch.Tensor] = None,
    k_conv_weight: Optional[torch.Tensor] = None,
    v_conv_weight: Optional[torch.Tensor] = None,
    seq_idx: Optional[torch.Tensor] = None,
):
    """The canonical dyadic K/V tree, levels 0..L (reference.py:465-584).

    Level 0 is k/v after the optional short conv; parent j of level l merges
    children (2j, 2j+1) with alpha = softmax(w0, w1) and takes
    w = logsumexp(w0, w1); odd trailing nodes are dropped.  Merge weights are
    qk-logsumexp (x and w_proj None) or x @ w_proj^T (both given).

    Returns (k_levels, v_levels, w_levels): lists of L + 1 views
    [B, N >> l, Hkv, D] / [B, N >> l, Hkv, 1] of one level-major packed
    buffer per tensor.  With grad mode on and any input requiring gradients,
    the buffers carry the Phase-1 VJP; ``detach_weights`` then cuts the
    gradient through the merge weights (q / k in qk mode, x / w_proj in
    linear mode), as in the reference.

    seq_idx (an extension, see short_conv): segment ids [B, N] of packed
    examples; the short conv then restarts at each example (it has no
    effect without conv weights).  The conv runs as its own launch
    (short_conv) ahead of the builder, with its own VJP under autograd.
    """
    if seq_idx is not None and k_conv_weight is not None and v_conv_weight is not None:
        B, N, Hkv, Dk = k.shape
        Dv = v.shape[-1]
        k = short_conv(k.reshape(B, N, Hkv * Dk), k_conv_weight, seq_idx).reshape(B, N, Hkv, Dk)
        v = short_conv(v.reshape(B, N, Hkv * Dv), v_conv_weight, seq_idx).reshape(B, N, Hkv, Dv)
        k_conv_weight = v_conv_weight = None
    inputs = (q, k, v, x, w_proj, k_conv_weight, v_conv_weight)
    if torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in inputs):
        kp, vp, wp = _DyadicTree.apply(q, k, v, x, w_proj, k_conv_weight, v_conv_weight,
                                       int(num_summary_levels), bool(detach_weights))
        N = k.shape[1]
        offs = [0]
        for lv in range(int(num_summary_levels) + 1):
            offs.append(offs[-1] + (N >> lv))
    else:
        kp, vp, wp, offs = _build_packed(q, k, v, num_summary_levels, x, w_proj, k_conv_weight,
                                         v_conv_weight)
    L = int(num_summary_levels)
    k_levels, v_levels, w_levels = [], [], []
    for lv in range(L + 1):
        kl = kp[:, offs[lv]:offs[lv + 1]]
        vl = vp[:, offs[lv]:offs[lv + 1]]
        kl._tc_packed = (kp, lv, tuple(offs))
        vl._tc_packed = (vp, lv, tuple(offs))
        k_levels.append(kl)
        v_levels.append(vl)
        w_levels.append(wp[:, offs[lv]:offs[lv + 1]].unsqueeze(-1))
    return k_levels, v_levels, w_levels


__all__ = ["compute_summary_weights", "compute_linear_weights", "short_conv",
           "build_dyadic_summaries", "build_dyadic_summaries_backward"]
