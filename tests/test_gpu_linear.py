"""tc_linear / tc_linear_wgrad (the projections x @ W^T of
compute_linear_weights, compute_relative_states, apply_output_gate and the
relative-bias band, and their gradients) against plain PyTorch fp32 products
of the same (rounded) inputs.

Tolerances: fp32 results (fp32 accumulation, another summation order)
normwise relative 1e-5; 16-bit results additionally carry one rounding of the
output, so normwise 1e-2 and elementwise |got - want| <= 1e-2 (|want| +
1e-2 max|want|).
"""

import pytest
import torch

from telescope_cache_b200 import _lib
from telescope_cache_b200.telescoping_attn.linear import Projection, linear, linear_wgrad

pytestmark = pytest.mark.gpu


def _close(got, want, out_dtype):
    got, want = got.double(), want.double()
    rel = (got - want).norm() / max(want.norm(), 1e-30)
    if out_dtype == torch.float32:
        assert rel <= 1e-5, f"normwise {rel:.3e}"
    else:
        assert rel <= 1e-2, f"normwise {rel:.3e}"
        bound = 1e-2 * (want.abs() + 1e-2 * want.abs().max())
        assert bool(((got - want).abs() <= bound + 1e-6).all()), f"max err {(got - want).abs().max():.3e}"


# (M, N, K): tiny, ragged, the band (K = 16), the decode gate (M = 64), the
# linear merge weights (N = 32), wide and square-ish
SHAPES = [(1, 16, 16), (77, 40, 96), (300, 130, 200), (1024, 2048, 2048), (513, 4368, 16),
          (64, 2048, 2048), (1000, 32, 2048), (129, 17, 64), (256, 256, 24)]


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("dtype,out_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float16, torch.float16),
                                             (torch.bfloat16, torch.float32), (torch.float32, torch.float32)])
def test_linear_matches_fp32_product(M, N, K, dtype, out_dtype):
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(M * 7 + N * 13 + K)
    x = torch.randn(M, K, generator=g, device="cuda").to(dtype)
    w = (torch.randn(N, K, generator=g, device="cuda") / K ** 0.5).to(dtype)
    before = _lib.launch_count()
    y = linear(x, w, out_dtype=out_dtype)
    torch.cuda.synchronize()
    # one launch, or two when few row blocks and a long K split K (partial sums, then their reduction)
    split = _lib.lib().tc_linear_scratch_floats(M, N, K, _lib.dtype_code(out_dtype)) > 0 and dtype != torch.float32
    assert _lib.launch_count() == before + (2 if split else 1)
    assert y.dtype == out_dtype and y.shape == (M, N)
    _close(y, x.float() @ w.float().t(), out_dtype)


@pytest.mark.parametrize("M,N,K", [(300, 130, 200), (1024, 2048, 2048), (33, 16, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_gate_epilogue(M, N, K, dtype):
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(91 + M)
    x = torch.randn(M, K, generator=g, device="cuda").to(dtype)
    w = (torch.randn(N, K, generator=g, device="cuda") / K ** 0.5).to(dtype)
    aux = torch.randn(M, N, generator=g, device="cuda").to(dtype)
    y = linear(x, w, gate_out=aux)
    want = torch.nn.functional.silu(x.float() @ w.float().t()) * aux.float()
    _close(y, want, dtype)


def test_strided_operands():
    """A row stride that is a multiple of 8 with an aligned start (tensor-core
    path) and the same rows from a misaligned start (SIMT path) give the
    products."""
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    big = torch.randn(200, 136, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(48, 100, generator=g, device="cuda") / 10).to(torch.bfloat16)
    for x in (big[:, :100], big[:, 3:103]):
        y = linear(x, w)
        _close(y, x.float() @ w.float().t(), torch.bfloat16)


@pytest.mark.parametrize("M,N1,N2", [(1, 16, 16), (5000, 32, 2048), (4097, 17, 300), (300, 130, 64),
                                     (9001, 32, 200)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_wgrad(M, N1, N2, dtype):
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(M + N1 + N2)
    a = torch.randn(M, N1, generator=g, device="cuda").to(dtype)
    b = torch.randn(M, N2, generator=g, device="cuda").to(dtype)
    out = linear_wgrad(a, b, torch.float32)
    _close(out, a.float().t() @ b.float(), torch.float32)
    again = linear_wgrad(a, b, torch.float32)
    assert torch.equal(out, again), "wgrad must be deterministic"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_projection_gradients(dtype):
    torch.cuda.set_device(0)
    g = torch.Generator(device="cuda")
    g.manual_seed(77)
    x = torch.randn(3, 170, 256, generator=g, device="cuda").to(dtype).requires_grad_(True)
    w = (torch.randn(96, 256, generator=g, device="cuda") / 16).to(dtype).requires_grad_(True)
    dy = torch.randn(3, 170, 96, generator=g, device="cuda").to(dtype)
    y = Projection.apply(x, w)
    dx, dw = torch.autograd.grad(y, (x, w), dy)
    xf, wf = x.detach().float().requires_grad_(True), w.detach().float().requires_grad_(True)
    yf = xf @ wf.t()
    dxf, dwf = torch.autograd.grad(yf, (xf, wf), dy.float())
    _close(y.detach(), yf.detach(), dtype)
    _close(dx, dxf, dtype)
    _close(dw, dwf, dtype)
