"""Projections of hidden states, x @ W^T, and their gradients on this
library's kernels: ``tc_linear`` (tcgen05 tensor cores for bf16/f16
operands of one type, a SIMT kernel otherwise; optional fused SiLU(.) * out
epilogue) and ``tc_linear_wgrad`` (dW = dy^T x, deterministic).

The reference computes these with ``x.matmul(W.t())`` in
compute_linear_weights (reference.py:148-164), compute_relative_states
(reference.py:374-395) and apply_output_gate (reference.py:1187-1219); torch
autograd supplies their gradients.  ``Projection`` is the same function with
the same gradients (dx = dy W, dW = dy^T x), every product on this library.
"""

import ctypes
from typing import Optional

import torch

from .. import _lib


def _rows(t: torch.Tensor) -> torch.Tensor:
    """t as a 2-D row-major matrix (last dim contiguous)."""
    t2 = t.reshape(-1, t.shape[-1])
    if t2.stride(-1) != 1 or (t2.shape[0] > 1 and t2.stride(0) < t2.shape[1]):
        t2 = t2.contiguous()
    return t2


def _status(device):
    """The device status word (a bounded wait that gives up sets a bit)."""
    from .attention import device_status  # attention imports this module
    return ctypes.c_void_p(device_status(device).data_ptr())


def linear(x: torch.Tensor, w: torch.Tensor, *, out_dtype: Optional[torch.dtype] = None,
           gate_out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [..., K] @ w[N, K]^T -> [..., N] in out_dtype (default: the common
    type of x and w).  With gate_out ([..., N], out_dtype), returns
    SiLU(x @ w^T) * gate_out from one kernel (the product in the epilogue)."""
    if w.dim() != 2 or x.shape[-1] != w.shape[-1]:
        raise ValueError(f"linear: x {tuple(x.shape)} and w {tuple(w.shape)} do not share the last dim")
    _lib.require_cuda(x, w)
    K, N = x.shape[-1], w.shape[0]
    out_dtype = out_dtype or torch.result_type(x, w)
    a, b = _rows(x), _rows(w)
    M = a.shape[0]
    out = torch.empty(M, N, device=x.device, dtype=out_dtype)
    aux, ld_aux, epi = None, 0, _lib.TC_LIN_STORE
    if gate_out is not None:
        if gate_out.dtype != out_dtype or gate_out.numel() != M * N:
            raise ValueError("linear: gate_out must hold [..., N] elements of the output type")
        aux = _rows(gate_out.reshape(M, N))
        ld_aux, epi = aux.stride(0), _lib.TC_LIN_GATE
    if M and N:
        # split-K scratch (few rows, long K); torch's allocator, stream ordered
        nscratch = int(_lib.lib().tc_linear_scratch_floats(M, N, K, _lib.dtype_code(out_dtype)))
        scratch = torch.empty(nscratch, device=x.device, dtype=torch.float32) if nscratch > 0 else None
        _lib.launch("tc_linear", x.device, M, N, K, _lib.dtype_code(a.dtype), _lib.ptr(a), a.stride(0),
                    _lib.dtype_code(b.dtype), _lib.ptr(b), b.stride(0), _lib.dtype_code(out_dtype),
                    _lib.ptr(out), N, epi, _lib.ptr(aux), ld_aux, _lib.ptr(scratch), max(nscratch, 0),
                    _status(x.device), _lib.stream_of(x))
    return out.reshape(*x.shape[:-1], N)


def linear_wgrad(a: torch.Tensor, b: torch.Tensor, out_dtype: torch.dtype) -> torch.Tensor:
    """a [M, N1]^T @ b [M, N2] -> [N1, N2] (fp32 accumulation, chunked in a
    fixed order: deterministic)."""
    a2, b2 = _rows(a), _rows(b)
    if a2.shape[0] != b2.shape[0]:
        raise ValueError(f"linear_wgrad: row counts differ ({a2.shape[0]} vs {b2.shape[0]})")
    _lib.require_cuda(a2, b2)
    M, N1, N2 = a2.shape[0], a2.shape[1], b2.shape[1]
    out = torch.empty(N1, N2, device=a.device, dtype=out_dtype)
    nscratch = int(_lib.lib().tc_linear_wgrad_scratch_floats(M, N1, N2))
    if nscratch < 0:
        raise ValueError("linear_wgrad: invalid sizes")
    scratch = torch.empty(max(nscratch, 1), device=a.device, dtype=torch.float32)
    _lib.launch("tc_linear_wgrad", a.device, M, N1, N2, _lib.dtype_code(a2.dtype), _lib.ptr(a2), a2.stride(0),
                _lib.dtype_code(b2.dtype), _lib.ptr(b2), b2.stride(0), _lib.dtype_code(out_dtype), _lib.ptr(out),
                N2, _lib.ptr(scratch), nscratch, _status(a.device), _lib.stream_of(a))
    return out


class Projection(torch.autograd.Function):
    """y = x @ w^T with dx = dy w and dw = dy^T x, all on this library."""

    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        return linear(x, w)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dx = dw = None
        if ctx.needs_input_grad[0]:
            # dx [.., K] = dy [.., N] @ w [N, K]: the B operand is w^T as [K, N] rows
            dx = linear(dy.to(w.dtype), w.t().contiguous(), out_dtype=x.dtype)
        if ctx.needs_input_grad[1]:
            dw = linear_wgrad(dy, x.to(dy.dtype), w.dtype)
        return dx, dw


def project(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """x @ w^T through Projection when a gradient is wanted, else linear()."""
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad):
        return Projection.apply(x, w)
    return linear(x, w)


__all__ = ["linear", "linear_wgrad", "Projection", "project"]
