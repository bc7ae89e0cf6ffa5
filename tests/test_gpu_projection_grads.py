"""Gradients through the public projection ops (apply_output_gate,
compute_linear_weights, compute_relative_states) against torch autograd of
the reference's formulas (reference.py:148-164, :374-395, :1187-1219) on the
same inputs in fp32.  Tolerance: fp32 normwise 1e-5; bf16 normwise 2e-2."""

import pytest
import torch

from telescope_cache_b200 import reference as R

pytestmark = pytest.mark.gpu


def _close(got, want, dtype):
    rel = ((got.double() - want.double()).norm() / max(want.double().norm(), 1e-30)).item()
    assert rel <= (1e-5 if dtype == torch.float32 else 2e-2), f"normwise {rel:.3e}"


def _leaf(t):
    return t.detach().clone().requires_grad_(True)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_output_gate_gradients(dtype):
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    B, N, Hq, Dv, E = 2, 96, 4, 32, 64
    out = torch.randn(B, N, Hq, Dv, generator=g, device="cuda").to(dtype)
    x = torch.randn(B, N, E, generator=g, device="cuda").to(dtype)
    w = (torch.randn(Hq * Dv, E, generator=g, device="cuda") / 8).to(dtype)
    dy = torch.randn(B, N, Hq, Dv, generator=g, device="cuda").to(dtype)
    o1, x1, w1 = _leaf(out), _leaf(x), _leaf(w)
    y = R.apply_output_gate(o1, x1, w1)
    grads = torch.autograd.grad(y, (o1, x1, w1), dy)
    o2, x2, w2 = _leaf(out.float()), _leaf(x.float()), _leaf(w.float())
    y2 = torch.nn.functional.silu(x2.matmul(w2.t())).reshape(B, N, Hq, Dv) * o2
    want = torch.autograd.grad(y2, (o2, x2, w2), dy.float())
    _close(y.detach(), y2.detach(), dtype)
    for a, b_ in zip(grads, want):
        _close(a, b_, dtype)
    # without gradients the fused epilogue gives the same values
    with torch.no_grad():
        _close(R.apply_output_gate(out, x, w), y2.detach(), dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_linear_weights_and_relative_states_gradients(dtype):
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(12)
    B, N, E, Hkv, Hq, drel = 2, 80, 64, 4, 8, 16
    x = torch.randn(B, N, E, generator=g, device="cuda").to(dtype)
    wp = (torch.randn(Hkv, E, generator=g, device="cuda") / 8).to(dtype)
    wr = (torch.randn(Hq * drel, E, generator=g, device="cuda") / 8).to(dtype)
    x1, wp1, wr1 = _leaf(x), _leaf(wp), _leaf(wr)
    lw = R.compute_linear_weights(x1, wp1)
    rs = R.compute_relative_states(x1, wr1, Hq)
    d_lw = torch.randn(lw.shape, generator=g, device="cuda").to(dtype)
    d_rs = torch.randn(rs.shape, generator=g, device="cuda").to(dtype)
    grads = torch.autograd.grad((lw, rs), (x1, wp1, wr1), (d_lw, d_rs))
    x2, wp2, wr2 = _leaf(x.float()), _leaf(wp.float()), _leaf(wr.float())
    lw2 = x2.matmul(wp2.t()).unsqueeze(-1)
    rs2 = x2.matmul(wr2.t()).reshape(B, N, Hq, drel)
    want = torch.autograd.grad((lw2, rs2), (x2, wp2, wr2), (d_lw.float(), d_rs.float()))
    _close(lw.detach(), lw2.detach(), dtype)
    _close(rs.detach(), rs2.detach(), dtype)
    for a, b_ in zip(grads, want):
        _close(a, b_, dtype)
