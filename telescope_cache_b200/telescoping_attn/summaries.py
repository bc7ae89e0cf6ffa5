"""Phase 1: merge weights, the short causal conv and the dyadic tree builder
(reference ``telescoping_attn/summaries.py`` / ``reference.py:113-584``).

The builder is one fused CUDA launch (``tc_build_tree``) that writes every
level straight into a level-major packed buffer; the per-level tensors it
returns are views of that buffer, so ``pack_levels`` on them copies nothing.

The returned tensors are not attached to autograd (the Phase-1 VJP of the
reference is left to torch autograd; here it is not provided yet).
"""

import ctypes
from typing import Optional

import torch

from .. import _lib


def _contig(t):
    return t if t.is_contiguous() else t.contiguous()


def compute_summary_weights(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """w[b, t, hkv] = logsumexp over the KV head's query group of
    q_h . k / sqrt(Dk).  q [B, N, Hq, Dk], k [B, N, Hkv, Dk] -> [B, N, Hkv, 1]
    in q's dtype (reference.py:117-145)."""
    B, N, Hq, Dk = q.shape
    _, Nk, Hkv, Dkk = k.shape
    assert N == Nk
    assert Dk == Dkk
    assert Hq % Hkv == 0
    _lib.require_cuda(q, k)
    q, k = _contig(q), _contig(k.to(q.dtype))
    out = torch.empty(B, N, Hkv, 1, device=q.device, dtype=q.dtype)
    _lib.check(_lib.lib().tc_qk_weights(B, N, Hq, Hkv, Dk, _lib.dtype_code(q.dtype), _lib.ptr(q),
                                        _lib.ptr(k), _lib.dtype_code(out.dtype), _lib.ptr(out),
                                        _lib.stream_of(q)), "tc_qk_weights")
    return out


def compute_linear_weights(x: torch.Tensor, w_proj: torch.Tensor) -> torch.Tensor:
    """w = x @ w_proj^T, the trained-linear merge weight.  x [B, N, E],
    w_proj [Hkv, E] -> [B, N, Hkv, 1] (reference.py:148-164)."""
    B, N, E = x.shape
    Hkv, Ew = w_proj.shape
    assert E == Ew
    _lib.require_cuda(x, w_proj)
    if x.dtype == w_proj.dtype:
        # the reference's own op: one plain GEMM (cuBLAS through torch)
        return x.matmul(w_proj.t()).unsqueeze(-1)
    x, w_proj = _contig(x), _contig(w_proj)
    out = torch.empty(B, N, Hkv, 1, device=x.device, dtype=torch.result_type(x, w_proj))
    _lib.check(_lib.lib().tc_linear_weights(
        B * N, E, Hkv, _lib.dtype_code(x.dtype), _lib.ptr(x), _lib.dtype_code(w_proj.dtype),
        _lib.ptr(w_proj), _lib.dtype_code(out.dtype), _lib.ptr(out), _lib.stream_of(x)),
        "tc_linear_weights")
    return out


def _check_conv_weight(weight, C):
    if weight.dim() != 2 or weight.shape[0] != C:
        raise ValueError(
            f"conv weight shape {tuple(weight.shape)} incompatible with C={C}; expected [C, K]")
    if weight.shape[1] <= 0:
        raise ValueError(f"conv kernel size must be positive, got {weight.shape[1]}")


def short_conv(x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Causal depthwise conv with an fp32 residual, cast once:
    y[b,t,c] = x[b,t,c] + sum_j weight[c,j] x[b,t-K+1+j,c]
    (reference.py:167-211).  x [B, N, C], weight [C, K]."""
    B, N, C = x.shape
    _check_conv_weight(weight, C)
    _lib.require_cuda(x, weight)
    x, weight = _contig(x), _contig(weight)
    y = torch.empty_like(x)
    _lib.check(_lib.lib().tc_short_conv(B, N, C, _lib.dtype_code(x.dtype), _lib.ptr(x),
                                        weight.shape[1], _lib.dtype_code(weight.dtype),
                                        _lib.ptr(weight), _lib.ptr(y), _lib.stream_of(x)),
               "tc_short_conv")
    return y


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
):
    """The canonical dyadic K/V tree, levels 0..L (reference.py:465-584).

    Level 0 is k/v after the optional short conv; parent j of level l merges
    children (2j, 2j+1) with alpha = softmax(w0, w1) and takes
    w = logsumexp(w0, w1); odd trailing nodes are dropped.  Merge weights are
    qk-logsumexp (x and w_proj None) or x @ w_proj^T (both given).

    Returns (k_levels, v_levels, w_levels): lists of L + 1 views
    [B, N >> l, Hkv, D] / [B, N >> l, Hkv, 1] of one level-major packed
    buffer per tensor.  ``detach_weights`` only affects gradients in the
    reference; these outputs carry none, so it is accepted and ignored.
    """
    del detach_weights
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
        _lib.check(_lib.lib().tc_build_tree(ctypes.byref(args), _lib.stream_of(k)), "tc_build_tree")
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
           "build_dyadic_summaries"]
