"""Post-attention ops over the frozen (out, lse) boundary: learned attention
sink and SiLU output gate (reference ``telescoping_attn/sink_gate.py`` /
``reference.py:1074-1219``).  Both run as CUDA kernels and are
differentiable through ``torch.autograd``."""

from typing import Tuple

import torch

from .. import _lib
from .linear import linear, project


def _sink_fwd(out, lse, sinks):
    B, N, Hq, Dv = out.shape
    out_c, lse_c = out.contiguous(), lse.contiguous().float()
    s = sinks.contiguous()
    y = torch.empty_like(out_c)
    _lib.launch("tc_sink_fwd", out.device, B * N, Hq, Dv, _lib.dtype_code(out.dtype), _lib.ptr(out_c),
                                      _lib.ptr(lse_c), _lib.dtype_code(s.dtype), _lib.ptr(s),
                                      _lib.ptr(y), _lib.stream_of(out))
    return y


def _sink_bwd(out, lse, sinks, dout):
    B, N, Hq, Dv = out.shape
    out_c, lse_c, g = out.contiguous(), lse.contiguous().float(), dout.contiguous()
    s = sinks.contiguous()
    dout_pre = torch.empty_like(g)
    dlse = torch.empty(B, N, Hq, device=out.device, dtype=torch.float32)
    dsinks = torch.empty(Hq, device=out.device, dtype=torch.float32)
    _lib.launch("tc_sink_bwd", out.device, B * N, Hq, Dv, _lib.dtype_code(out.dtype), _lib.ptr(out_c),
                                      _lib.ptr(lse_c), _lib.dtype_code(s.dtype), _lib.ptr(s),
                                      _lib.ptr(g), _lib.ptr(dout_pre), _lib.ptr(dlse),
                                      _lib.ptr(dsinks), _lib.stream_of(out))
    return dout_pre, dlse, dsinks.to(sinks.dtype)


class _Sink(torch.autograd.Function):
    @staticmethod
    def forward(ctx, out, lse, sinks):
        ctx.save_for_backward(out, lse, sinks)
        return _sink_fwd(out, lse, sinks)

    @staticmethod
    def backward(ctx, g):
        out, lse, sinks = ctx.saved_tensors
        dout_pre, dlse, dsinks = _sink_bwd(out, lse, sinks, g.to(out.dtype))
        return dout_pre, dlse.to(lse.dtype), dsinks


def apply_attention_sink(out: torch.Tensor, lse: torch.Tensor, sinks: torch.Tensor) -> torch.Tensor:
    """out * sigmoid(lse - sinks[h]), the scale computed in fp32 and cast to
    out's dtype: one extra softmax logit per query head with a zero value
    (reference.py:1082-1122)."""
    B, N, Hq, Dv = out.shape
    if tuple(lse.shape) != (B, N, Hq):
        raise ValueError(f"lse shape {tuple(lse.shape)} != {(B, N, Hq)}")
    if tuple(sinks.shape) != (Hq,):
        raise ValueError(f"sinks shape {tuple(sinks.shape)} != {(Hq,)} (one logit per query head)")
    _lib.require_cuda(out, lse, sinks)
    return _Sink.apply(out, lse, sinks)


def attention_sink_backward(out: torch.Tensor, lse: torch.Tensor, sinks: torch.Tensor,
                            dout: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """(dout_pre, dlse, dsinks) at the (out, lse) boundary, r = sigmoid(lse - s):
    dout_pre = r dout, dlse = <dout, out> r (1 - r), dsinks = -sum dlse
    (reference.py:1125-1184)."""
    B, N, Hq, Dv = out.shape
    if tuple(lse.shape) != (B, N, Hq):
        raise ValueError(f"lse shape {tuple(lse.shape)} != {(B, N, Hq)}")
    if tuple(sinks.shape) != (Hq,):
        raise ValueError(f"sinks shape {tuple(sinks.shape)} != {(Hq,)} (one logit per query head)")
    if tuple(dout.shape) != (B, N, Hq, Dv):
        raise ValueError(f"dout shape {tuple(dout.shape)} != {(B, N, Hq, Dv)}")
    if dout.dtype != out.dtype:
        raise ValueError(f"dout dtype {dout.dtype} must match out dtype {out.dtype}")
    _lib.require_cuda(out, lse, sinks, dout)
    with torch.no_grad():
        return _sink_bwd(out, lse, sinks, dout)


def _gate_fwd(out, g):
    y = torch.empty(out.shape, device=out.device, dtype=torch.result_type(out, g))
    oc, gc = out.contiguous(), g.contiguous()
    _lib.launch("tc_gate_apply", out.device, out.numel(), _lib.dtype_code(out.dtype), _lib.ptr(oc),
                                        _lib.dtype_code(g.dtype), _lib.ptr(gc),
                                        _lib.dtype_code(y.dtype), _lib.ptr(y), _lib.stream_of(out))
    return y


class _Gate(torch.autograd.Function):
    @staticmethod
    def forward(ctx, out, g):
        ctx.save_for_backward(out, g)
        return _gate_fwd(out, g)

    @staticmethod
    def backward(ctx, dy):
        out, g = ctx.saved_tensors
        gf = g.float()
        sig = torch.sigmoid(gf)
        silu = (gf * sig).to(g.dtype)
        d_out = (dy * silu).to(out.dtype)
        d_g = (dy.float() * out.float() * (sig * (1 + gf * (1 - sig)))).to(g.dtype)
        return d_out, d_g


def apply_output_gate(out: torch.Tensor, x: torch.Tensor, gate_weight: torch.Tensor) -> torch.Tensor:
    """SiLU(x @ gate_weight^T).reshape(B, N, Hq, Dv) * out
    (reference.py:1187-1219).  Without gradients: one tc_linear launch with
    SiLU and the product in its epilogue.  With gradients: the projection on
    tc_linear (Projection, whose backward is also this library's), then the
    SiLU-product kernel, which keeps the pre-activation for its backward."""
    B, N, Hq, Dv = out.shape
    if x.dim() != 3 or x.shape[0] != B or x.shape[1] != N:
        raise ValueError(
            f"x shape {tuple(x.shape)} incompatible with out {tuple(out.shape)}; expected "
            f"[B, N, emb_dim]")
    if tuple(gate_weight.shape) != (Hq * Dv, x.shape[-1]):
        raise ValueError(f"gate_weight shape {tuple(gate_weight.shape)} != {(Hq * Dv, x.shape[-1])}")
    _lib.require_cuda(out, x, gate_weight)
    grad = torch.is_grad_enabled() and (out.requires_grad or x.requires_grad or gate_weight.requires_grad)
    if not grad and out.dtype == torch.result_type(x, gate_weight):
        return linear(x, gate_weight, gate_out=out).reshape(B, N, Hq, Dv)
    g = project(x, gate_weight).reshape(B, N, Hq, Dv)
    return _Gate.apply(out, g)


__all__ = ["apply_attention_sink", "attention_sink_backward", "apply_output_gate"]
