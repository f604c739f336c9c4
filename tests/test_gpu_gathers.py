"""pack / unpack / to_padded / from_padded on the GPU: bit-exact against the oracle
and against the reference's own outputs (golden fixtures)."""

import numpy as np
import pytest
import torch

import oracle
from conftest import load_golden

pytestmark = pytest.mark.gpu


def _np(t):
    """Host numpy copy; bf16 (no numpy dtype) as its int16 bit pattern."""
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return t.numpy()


@pytest.mark.parametrize("name", ["gather_2d", "gather_3d"])
def test_gathers_golden(cuda, name):
    import scree_b200 as scree

    g = load_golden(name)
    offs = g["offsets"]
    seqs = [torch.tensor(s, device=cuda) for s in oracle.unpack(g["values"], offs)]
    arr = scree.pack(seqs)
    assert arr.offsets.dtype == torch.int32
    assert np.array_equal(_np(arr.values), g["values"]) and np.array_equal(_np(arr.offsets), offs)
    for side in ("right", "left"):
        p, m = scree.to_padded(arr, side=side, fill_value=int(g["fill"]))
        assert np.array_equal(_np(p), g[f"padded_{side}"])
        assert np.array_equal(_np(m), g[f"mask_{side}"])
    back = scree.from_padded(torch.tensor(g["padded_right"], device=cuda), torch.tensor(g["mask_right"], device=cuda))
    assert np.array_equal(_np(back.values), g["from_padded_values"])
    assert np.array_equal(_np(back.offsets), g["from_padded_offsets"])


DTYPES = [torch.uint8, torch.int16, torch.bfloat16, torch.float32, torch.float64, torch.bool]


@pytest.mark.parametrize("dtype", DTYPES, ids=str)
@pytest.mark.parametrize("feat", [(), (3,), (4, 8), (4096,)], ids=str)
def test_roundtrips(cuda, dtype, feat):
    import scree_b200 as scree

    rng = np.random.default_rng(7)
    lengths = [5, 0, 1, 37, 2, 16]
    seqs = []
    for n in lengths:
        a = rng.integers(0, 200, size=(n, *feat))
        seqs.append(torch.tensor(a).to(dtype).to(cuda))
    arr = scree.pack(seqs)
    ref_vals, ref_offs = oracle.pack([_np(s) for s in seqs])
    assert np.array_equal(_np(arr.values), ref_vals)
    assert np.array_equal(_np(arr.offsets), ref_offs)
    rows = scree.unpack(arr)
    for r, s in zip(rows, seqs):
        assert torch.equal(r, s)
    for side in ("right", "left"):
        fill = 1 if dtype == torch.bool else 3
        p, m = scree.to_padded(arr, side=side, fill_value=fill)
        fill_ref = fill
        if dtype == torch.bfloat16:  # oracle works on the int16 bit patterns
            fill_ref = int(torch.tensor([fill], dtype=torch.bfloat16).view(torch.int16)[0])
        rp, rm = oracle.to_padded(ref_vals, ref_offs, side=side, fill_value=fill_ref)
        assert np.array_equal(_np(p), rp) and np.array_equal(_np(m), rm)
        if side == "right":
            back = scree.from_padded(p, m)
            assert np.array_equal(_np(back.values), ref_vals)
            assert np.array_equal(_np(back.offsets), ref_offs)


def test_pack_unaligned_sources(cuda):
    """Sources at odd byte offsets (views) fall back to narrower accesses."""
    import scree_b200 as scree

    base = torch.arange(1000, dtype=torch.int16, device=cuda)
    seqs = [base[1:8].reshape(7, 1), base[3:13].reshape(5, 2)[:, :1].contiguous(), base[101:140].reshape(39, 1)]
    arr = scree.pack(seqs)
    assert torch.equal(arr.values, torch.cat(seqs))


def test_to_padded_cfg3_size(cuda):
    """cfg3: 64 sequences, hidden 4096 bf16, pack(unpack(x)) round trip and padding."""
    import scree_b200 as scree
    from scree_b200 import workloads

    lengths = workloads.cfg3_lengths()
    T = sum(lengths)
    x = torch.randn((T, 4096), device=cuda).to(torch.bfloat16)
    offs = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=cuda)
    arr = scree.from_cu_seqlens(x, offs)
    again = scree.pack(scree.unpack(arr))
    assert torch.equal(again.values, x) and torch.equal(again.offsets, offs)
    p, m = scree.to_padded(arr)
    assert p.shape == (64, max(lengths), 4096)
    assert int(m.sum()) == T
    back = scree.from_padded(p, m)
    assert torch.equal(back.values, x)


def test_pack_autograd(cuda):
    """reference tests/test_autograd.py:15-25: gradients flow through pack/unpack."""
    import scree_b200 as scree

    seqs = [torch.randn(n, 4, device=cuda, requires_grad=True) for n in [3, 5, 2]]
    arr = scree.pack(seqs)
    loss = sum(t.sum() for t in scree.unpack(arr))
    loss.backward()
    for s in seqs:
        assert s.grad is not None and torch.equal(s.grad, torch.ones_like(s))


def test_array_invariants_and_errors(cuda):
    import scree_b200 as scree

    with pytest.raises(ValueError, match="empty list"):
        scree.pack([])
    v = torch.zeros(5, 2, device=cuda)
    with pytest.raises(ValueError, match=r"offsets\[-1\]"):
        scree.Array(values=v, offsets=torch.tensor([0, 3], device=cuda))
    with pytest.raises(ValueError, match=r"offsets\[0\]"):
        scree.Array(values=v, offsets=torch.tensor([1, 5], device=cuda))
    arr = scree.Array(values=v, offsets=torch.tensor([0, 2, 5], device=cuda))
    with pytest.raises(ValueError, match="side"):
        scree.to_padded(arr, side="middle")
    with pytest.raises(NotImplementedError):
        scree.to_padded(scree.Array(values=torch.zeros(2, 5, device=cuda), offsets=torch.tensor([0, 5]), ragged_dim=1))
