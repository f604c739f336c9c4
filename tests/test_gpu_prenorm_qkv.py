"""Fused RMSNorm -> QKV projection (one tcgen05 GEMM, csrc/prenorm_qkv.cu)
against the unfused fp32 formulation of scree/examples/03_train_step.py:36-41:
h = x / sqrt(mean(x^2) + eps) * gamma, qkv = h @ Wqkv.

Tolerance: 1e-2 absolute plus 2^-7 relative.  The kernel's result is rounded
once to the 16-bit output type (2^-9 relative) and uses gamma * Wqkv rounded to
16 bits; the unfused 16-bit path of the reference rounds h instead, which is an
error of the same order."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu

ATOL, RTOL = 1e-2, 2.0**-7


def _ref(x, gamma, w, eps):
    xf = x.float()
    h = xf / torch.sqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    if gamma is not None:
        h = h * gamma.float()
    return h @ w.float(), 1.0 / torch.sqrt(xf.pow(2).mean(-1) + eps)


def _check(got, want):
    err = (got.float() - want).abs() - (ATOL + RTOL * want.abs())
    assert float(err.max()) <= 0, f"max excess {float(err.max()):.3e}, max abs {float((got.float() - want).abs().max()):.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("T,C,N", [(300, 256, 768), (128, 64, 384), (1, 512, 256), (1000, 1024, 3072), (4100, 512, 3072)])
@pytest.mark.parametrize("with_gamma", [True, False])
def test_rmsnorm_qkv_forward(cuda, dtype, T, C, N, with_gamma):
    from scree_b200.kernels.native import rmsnorm_qkv

    g = torch.Generator().manual_seed(T + C + N)
    x = torch.randn((T, C), generator=g).to(dtype).to(cuda)
    gamma = (1 + 0.02 * torch.randn(C, generator=g)).to(cuda) if with_gamma else None
    w = (torch.randn((C, N), generator=g) / math.sqrt(C)).to(dtype).to(cuda)
    y, rstd = rmsnorm_qkv(x, gamma, w, 1e-6, want_rstd=True)
    torch.cuda.synchronize()
    ref, rref = _ref(x, gamma, w, 1e-6)
    _check(y, ref)
    torch.testing.assert_close(rstd, rref, atol=1e-5, rtol=1e-4)
    from scree_b200 import _lib

    assert _lib.device_status() == 0


def test_rmsnorm_qkv_strided_rows_and_shapes(cuda):
    from scree_b200.kernels.native import rmsnorm_qkv

    g = torch.Generator().manual_seed(1)
    big = torch.randn((200, 384), generator=g).to(torch.bfloat16).to(cuda)
    x = big[:, :256]  # row stride 384
    w = (torch.randn((256, 512), generator=g) / 16).to(torch.bfloat16).to(cuda)
    _check(rmsnorm_qkv(x, None, w, 1e-5), _ref(x, None, w, 1e-5)[0])
    with pytest.raises(NotImplementedError):
        rmsnorm_qkv(x, None, torch.zeros((256, 200), dtype=torch.bfloat16, device=cuda))


def test_rmsnorm_qkv_autograd_matches_fp32(cuda):
    """Gradients of sum(qkv * dY) for x, gamma and Wqkv against fp32 autograd."""
    from scree_b200.kernels.native import rmsnorm_qkv_autograd

    g = torch.Generator().manual_seed(2)
    T, C, N = 333, 256, 768
    x0 = torch.randn((T, C), generator=g)
    gam0 = 1 + 0.02 * torch.randn(C, generator=g)
    w0 = torch.randn((C, N), generator=g) / 16
    dy = torch.randn((T, N), generator=g).to(cuda)
    x = x0.to(torch.bfloat16).to(cuda).requires_grad_(True)
    gam = gam0.to(cuda).requires_grad_(True)
    w = w0.to(torch.bfloat16).to(cuda).requires_grad_(True)
    y = rmsnorm_qkv_autograd(x, gam, w, 1e-6)
    (y.float() * dy).sum().backward()
    xr = x.detach().float().requires_grad_(True)
    gr = gam.detach().clone().requires_grad_(True)
    wr = w.detach().float().requires_grad_(True)
    yr = (xr / torch.sqrt(xr.pow(2).mean(-1, keepdim=True) + 1e-6) * gr) @ wr
    (yr * dy).sum().backward()
    for got, want, name in ((x.grad, xr.grad, "dx"), (gam.grad, gr.grad, "dgamma"), (w.grad, wr.grad, "dW")):
        scale = float(want.abs().max())
        err = float((got.float() - want).abs().max())
        assert err <= 2e-2 * scale, f"{name}: max err {err:.3e} vs max |ref| {scale:.3e}"
