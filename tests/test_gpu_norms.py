"""Parity of the varlen RMSNorm / LayerNorm kernels with the oracle (GPU only).

Bar: forward and dx within 1e-3 absolute of the fp64 oracle plus the rounding
of the output dtype (half an ulp: 2^-9 relative for bf16, 2^-12 for fp16, 0 for
fp32); dweight / dbias (fp32 sums over all rows) within 1e-3 relative.
"""

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden
from gpu_helpers import to64

pytestmark = pytest.mark.gpu

REL = {torch.float32: 0.0, torch.float16: 2.0**-11, torch.bfloat16: 2.0**-8}


def _assert_close(got, want, dtype, atol=1e-3):
    g = to64(got)
    w = np.asarray(want, dtype=np.float64)
    lim = atol + REL[dtype] * np.abs(w)
    bad = np.abs(g - w) > lim
    assert not bad.any(), f"max err {np.abs(g - w).max():.3e}, {bad.sum()} elements over the bound"


def _inputs(T, C, dtype, device, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn((T, C), generator=g).to(dtype).to(device)
    dy = torch.randn((T, C), generator=g).to(dtype).to(device)
    w = (1 + 0.02 * torch.randn(C, generator=g)).to(device)
    b = (0.02 * torch.randn(C, generator=g)).to(device)
    return x, dy, w, b


CASES = [
    (1710, 128, torch.float32),   # cfg1 rmsnorm shape
    (19794, 4096, torch.bfloat16),  # cfg3
    (3000, 4096, torch.float16),
    (257, 100, torch.float32),    # vectorised, odd row count
    (129, 33, torch.float16),     # scalar path (C*2 bytes not a multiple of 16)
    (64, 8192, torch.bfloat16),
    (333, 2048, torch.bfloat16),    # streamed kernels, last row block ragged
    (500, 2048, torch.float32),     # streamed kernels, 32-bit rows
    (5, 4096, torch.float16),       # fewer rows than SMs
    (1, 8, torch.float32),
]


@pytest.mark.parametrize("T,C,dtype", CASES, ids=lambda c: str(c))
@pytest.mark.parametrize("wdtype", ["f32", "same", "none"])
def test_rmsnorm(cuda, T, C, dtype, wdtype):
    from scree_b200.kernels.native import varlen_rmsnorm_autograd, varlen_rmsnorm_triton

    x, dy, w, _ = _inputs(T, C, dtype, cuda)
    w = None if wdtype == "none" else (w if wdtype == "f32" else w.to(dtype))
    eps = 1e-6
    y = varlen_rmsnorm_triton(x, w, eps)
    wn = None if w is None else to64(w)
    _assert_close(y, oracle.rmsnorm_fwd(to64(x), wn, eps), dtype)
    xr = x.clone().requires_grad_(True)
    wr = None if w is None else w.clone().requires_grad_(True)
    y2 = varlen_rmsnorm_autograd(xr, wr, eps)
    y2.backward(dy)
    dx, dw = oracle.rmsnorm_bwd(to64(dy), to64(x), wn, eps)
    _assert_close(xr.grad, dx, dtype)
    if w is not None:
        np.testing.assert_allclose(to64(wr.grad), dw, rtol=1e-3 + REL[w.dtype], atol=1e-3)


@pytest.mark.parametrize("T,C,dtype", CASES, ids=lambda c: str(c))
@pytest.mark.parametrize("affine", [True, False])
def test_layernorm(cuda, T, C, dtype, affine):
    from scree_b200.kernels.native import varlen_layernorm_autograd, varlen_layernorm_triton

    x, dy, w, b = _inputs(T, C, dtype, cuda, seed=1)
    if not affine:
        w = b = None
    eps = 1e-5
    y = varlen_layernorm_triton(x, w, b, eps)
    wn = None if w is None else to64(w)
    bn = None if b is None else to64(b)
    _assert_close(y, oracle.layernorm_fwd(to64(x), wn, bn, eps), dtype)
    xr = x.clone().requires_grad_(True)
    wr = None if w is None else w.clone().requires_grad_(True)
    br = None if b is None else b.clone().requires_grad_(True)
    varlen_layernorm_autograd(xr, wr, br, eps).backward(dy)
    dx, dw, db = oracle.layernorm_bwd(to64(dy), to64(x), wn, bn, eps)
    _assert_close(xr.grad, dx, dtype)
    if affine:
        np.testing.assert_allclose(to64(wr.grad), dw, rtol=1e-3, atol=1e-3)
        np.testing.assert_allclose(to64(br.grad), db, rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("name", ["norm_ref_small", "norm_ref_small_w", "norm_c128"])
def test_norms_golden(cuda, name):
    """Against the reference's own outputs and autograd gradients (fp32 inputs)."""
    from scree_b200.kernels.native import varlen_layernorm_autograd, varlen_rmsnorm_autograd

    g = load_golden(name)
    x = torch.tensor(g["x"], device=cuda)
    dy = torch.tensor(g["dy"], device=cuda)
    w = torch.tensor(g["w"], device=cuda) if "w" in g else None
    b = torch.tensor(g["b"], device=cuda) if "b" in g else None
    for kind in ("rms", "ln"):
        xr = x.clone().requires_grad_(True)
        wr = None if w is None else w.clone().requires_grad_(True)
        br = None if b is None else b.clone().requires_grad_(True)
        if kind == "rms":
            y = varlen_rmsnorm_autograd(xr, wr, float(g["eps_rms"]))
        else:
            y = varlen_layernorm_autograd(xr, wr, br, float(g["eps_ln"]))
        y.backward(dy)
        np.testing.assert_allclose(to64(y), g[f"y_{kind}"], atol=1e-5)
        np.testing.assert_allclose(to64(xr.grad), g[f"dx_{kind}"], atol=1e-5)
        if w is not None:
            np.testing.assert_allclose(to64(wr.grad), g[f"dw_{kind}"], atol=1e-4)
        if b is not None and kind == "ln":
            np.testing.assert_allclose(to64(br.grad), g["db_ln"], atol=1e-4)


def test_norm_multidim_and_strided(cuda):
    """(T, heads, C) input and a row-strided view keep shape and values."""
    from scree_b200.kernels.native import varlen_rmsnorm_triton

    base = torch.randn((50, 3, 256), device=cuda, dtype=torch.bfloat16)
    y = varlen_rmsnorm_triton(base, None, 1e-6)
    assert y.shape == base.shape
    _assert_close(y, oracle.rmsnorm_fwd(to64(base), None, 1e-6), torch.bfloat16)
    wide = torch.randn((40, 512), device=cuda, dtype=torch.float16)
    view = wide[:, :256]
    y = varlen_rmsnorm_triton(view, None, 1e-6)
    _assert_close(y, oracle.rmsnorm_fwd(to64(view), None, 1e-6), torch.float16)
    wide = torch.randn((40, 2048), device=cuda, dtype=torch.bfloat16)
    view = wide[:, :1024]  # 2 KB rows 4 KB apart: streamed forward with a row stride
    w = torch.rand(1024, device=cuda) + 0.5
    b = torch.randn(1024, device=cuda) * 0.1
    from scree_b200.kernels.native import varlen_layernorm_triton
    y = varlen_layernorm_triton(view, w, b, 1e-5)
    _assert_close(y, oracle.layernorm_fwd(to64(view), to64(w), to64(b), 1e-5), torch.bfloat16)


def test_array_level_norms(cuda):
    import scree_b200 as scree
    from scree_b200.kernels import varlen_layernorm, varlen_rmsnorm

    seqs = [torch.randn(n, 8, device=cuda) for n in [3, 5, 2]]
    arr = scree.pack(seqs)
    w = torch.ones(8, device=cuda, requires_grad=True)
    b = torch.zeros(8, device=cuda, requires_grad=True)
    out = varlen_layernorm(arr, w, b, eps=1e-5)
    assert out.offsets is arr.offsets
    out.values.sum().backward()
    assert torch.isfinite(w.grad).all() and torch.isfinite(b.grad).all()
    r = varlen_rmsnorm(arr, eps=1e-6)
    rows = scree.unpack(r)
    for i, s in enumerate(seqs):
        ref = oracle.rmsnorm_fwd(to64(s), None, 1e-6)
        np.testing.assert_allclose(to64(rows[i]), ref, atol=1e-5)
