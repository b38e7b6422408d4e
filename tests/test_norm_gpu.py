"""The fused RMS norm (m3_rms_norm) against the reference's formula (layer.py:190-198) in
torch: fp32 / bf16 rows, strided 2-D views (the B / C slices of the in_proj output) and
contiguous 3-D inputs, rows that do and do not allow 16-byte vectors."""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(x, w, eps):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


@pytest.mark.parametrize("dtype,wdtype", [(torch.float32, torch.float32), (torch.bfloat16, torch.bfloat16),
                                          (torch.bfloat16, torch.float32)])
@pytest.mark.parametrize("shape", [(256, 128), (3, 7, 2048), (5, 100), (64, 8192)])
def test_fused_matches_formula(dtype, wdtype, shape):
    from mamba3_b200 import layer as LY

    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(*shape, device="cuda", generator=g).to(dtype) * 3
    w = (1 + 0.1 * torch.randn(shape[-1], device="cuda", generator=g)).to(wdtype)
    with torch.no_grad():
        y = LY.rms_norm(x, w, 1e-5)
    assert LY._fused_norm_ok(x, w)
    ref = _ref(x, w, 1e-5)
    tol = 1e-6 if dtype == torch.float32 else 1e-2
    assert torch.allclose(y.float(), ref.float(), rtol=tol, atol=tol)


def test_strided_rows_and_autograd_path():
    from mamba3_b200 import layer as LY

    proj = torch.randn(256, 8672, device="cuda", dtype=torch.bfloat16)
    b = proj[:, 8192:8320]  # a (256, 128) view with row stride 8672
    w = torch.ones(128, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        y = LY.rms_norm(b, w, 1e-5)
    assert torch.allclose(y.float(), _ref(b, w, 1e-5).float(), rtol=1e-2, atol=1e-2)
    xg = torch.randn(4, 64, device="cuda", requires_grad=True)
    assert not LY._fused_norm_ok(xg, torch.ones(64, device="cuda"))
    LY.rms_norm(xg, torch.ones(64, device="cuda"), 1e-5).sum().backward()
    assert xg.grad is not None


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("dim", [128, 512, 2048])
def test_fused_backward_matches_autograd(dtype, dim):
    """The fused autograd path (m3_rms_norm + m3_rms_norm_bwd) against torch autograd of the
    formula, on a strided 3-D view of a wider row (the B / C slices of the in_proj output)."""
    from mamba3_b200 import layer as LY

    g = torch.Generator(device="cuda").manual_seed(9)
    base = torch.randn(3, 50, dim + 64, device="cuda", generator=g).to(dtype)
    w0 = (1 + 0.1 * torch.randn(dim, device="cuda", generator=g))
    dy = torch.randn(3, 50, dim, device="cuda", generator=g).to(dtype)

    xa = base.clone().requires_grad_(True)
    wa = w0.clone().requires_grad_(True)
    ya = LY.rms_norm(xa[..., 32:32 + dim], wa, 1e-5)
    ya.backward(dy)
    xb = base.clone().requires_grad_(True)
    wb = w0.clone().requires_grad_(True)
    yb = _ref(xb[..., 32:32 + dim], wb, 1e-5)
    yb.backward(dy)
    tol = 1e-5 if dtype == torch.float32 else 2e-2
    rel = lambda a, b: float((a.detach().float() - b.detach().float()).norm() / b.detach().float().norm())
    assert rel(ya, yb) < tol
    assert rel(xa.grad, xb.grad) < tol
    assert rel(wa.grad, wb.grad) < (1e-4 if dtype == torch.float32 else 2e-2)
