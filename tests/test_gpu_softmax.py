"""varlen_softmax on the GPU against the oracle and the reference's own outputs.

Bar: within 1e-3 absolute of the fp64 oracle plus the output dtype's rounding
(2^-9 relative for bf16, 2^-12 for fp16, none for fp32 beyond 1e-5 absolute)."""

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden
from gpu_helpers import to64

pytestmark = pytest.mark.gpu

REL = {torch.float32: 0.0, torch.float16: 2.0**-11, torch.bfloat16: 2.0**-8}
ABS = {torch.float32: 1e-5, torch.float16: 1e-3, torch.bfloat16: 1e-3}


def _close(got, want, dtype, atol=None):
    g, w = to64(got), np.asarray(want, dtype=np.float64)
    lim = (ABS[dtype] if atol is None else atol) + REL[dtype] * np.abs(w)
    assert np.all(np.abs(g - w) <= lim), f"max err {np.abs(g - w).max():.3e}"


@pytest.mark.parametrize("name", ["softmax_ref_small", "softmax_2d"])
def test_softmax_golden(cuda, name):
    from scree_b200.kernels.native import varlen_softmax_packed

    g = load_golden(name)
    offs = np.concatenate([[0], np.cumsum(g["lengths"])])
    x = torch.tensor(g["x"], device=cuda, requires_grad=True)
    cu = torch.tensor(offs, dtype=torch.int32, device=cuda)
    y = varlen_softmax_packed(x, cu)
    y.backward(torch.tensor(g["dy"], device=cuda))
    _close(y, g["y"], torch.float32)
    _close(x.grad, g["dx"], torch.float32, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16], ids=str)
@pytest.mark.parametrize("feat", [(4096,), (7,), (3, 40)], ids=str)
def test_softmax_against_oracle(cuda, dtype, feat):
    from scree_b200.kernels.native import varlen_softmax_packed

    lengths = [1, 0, 300, 17, 1000, 2]
    offs = np.concatenate([[0], np.cumsum(lengths)])
    g = torch.Generator().manual_seed(3)
    x = (2.0 * torch.randn((offs[-1], *feat), generator=g)).to(dtype).to(cuda).requires_grad_(True)
    dy = torch.randn((offs[-1], *feat), generator=g).to(dtype).to(cuda)
    cu = torch.tensor(offs, dtype=torch.int64, device=cuda)
    y = varlen_softmax_packed(x, cu)
    y.backward(dy)
    ry = oracle.softmax_fwd(to64(x), offs)
    _close(y, ry, dtype)
    rdx = oracle.softmax_bwd(to64(dy), to64(y), offs)  # gradient at the kernel's y
    _close(x.grad, rdx, dtype)


def test_softmax_array_level_cfg3(cuda):
    import scree_b200 as scree
    from scree_b200 import workloads
    from scree_b200.kernels import varlen_softmax

    lengths = workloads.cfg3_lengths()
    offs = np.concatenate([[0], np.cumsum(lengths)])
    x = torch.randn((offs[-1], 4096), device=cuda).to(torch.bfloat16)
    arr = scree.from_cu_seqlens(x, torch.tensor(offs, dtype=torch.int32, device=cuda))
    out = varlen_softmax(arr)
    assert out.offsets is arr.offsets
    sums = torch.stack([r.float().sum(0) for r in scree.unpack(out)])
    torch.testing.assert_close(sums, torch.ones_like(sums), atol=2e-2, rtol=0)
    for b in (0, int(np.argmax(lengths))):
        s, e = int(offs[b]), int(offs[b + 1])
        _close(out.values[s:e], oracle.softmax_fwd(to64(x[s:e]), [0, e - s]), torch.bfloat16)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=str)
def test_softmax_chunk_boundaries(cuda, dtype):
    """Sequences at the 128-row chunk and 512-row residency limits of the staged
    16-bit forward (resident below 513 rows, streamed above), a ragged last
    column block (F = 200) and a column whose inputs include -inf."""
    from scree_b200.kernels.native import varlen_softmax_packed

    lengths = [128, 129, 0, 511, 512, 513, 640, 1, 1537]
    offs = np.concatenate([[0], np.cumsum(lengths)])
    g = torch.Generator().manual_seed(11)
    x = (3.0 * torch.randn((offs[-1], 200), generator=g)).to(dtype)
    x[offs[4] : offs[4] + 7, 5] = float("-inf")
    x = x.to(cuda)
    cu = torch.tensor(offs, dtype=torch.int32, device=cuda)
    y = varlen_softmax_packed(x, cu)
    _close(y, oracle.softmax_fwd(to64(x), offs), dtype)
