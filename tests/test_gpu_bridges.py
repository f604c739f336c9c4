"""Bridges (scree/bridges) on the GPU: HF padded <-> packed with the int64
attention_mask read / written by the gather kernels, jagged NestedTensor
wrapping without a copy, and the host-side to_torch / to_numpy.  Mirrors the
reference's tests/test_bridges.py cases on CUDA tensors, checked bit-exactly
against the oracle's to_padded / from_padded."""

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _seqs(lens, feat, dtype, cuda, seed=0):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn((n, *feat), generator=g).to(dtype).to(cuda) for n in lens]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("lens", [[3, 5, 2], [1], [0, 4, 7], [300, 1, 129]])
def test_hf_padded_roundtrip(cuda, dtype, lens):
    import scree_b200 as scree
    from scree_b200.bridges import from_hf_padded, to_hf_padded

    arr = scree.pack(_seqs(lens, (4, 3), dtype, cuda))
    hidden, mask = to_hf_padded(arr)
    assert mask.dtype == torch.int64 and hidden.dtype == dtype
    vals = arr.values.float().cpu().numpy()
    ref_p, ref_m = oracle.to_padded(vals, np.concatenate([[0], np.cumsum(lens)]), side="right")
    assert np.array_equal(mask.cpu().numpy(), ref_m.astype(np.int64))
    assert np.array_equal(hidden.float().cpu().numpy(), ref_p)
    arr2 = from_hf_padded(hidden, mask)
    assert torch.equal(arr2.values, arr.values)
    assert arr2.offsets.tolist() == arr.offsets.tolist()


@pytest.mark.parametrize("mask_dtype", [torch.int64, torch.int32, torch.int16, torch.uint8, torch.bool])
def test_from_hf_padded_mask_widths(cuda, mask_dtype):
    """The lengths kernel reads each mask width as is (nonzero = token)."""
    from scree_b200.bridges import from_hf_padded

    B, S = 3, 6
    hidden = torch.arange(B * S * 2, dtype=torch.float32, device=cuda).reshape(B, S, 2)
    lens = [2, 6, 0]
    mask = torch.zeros((B, S), dtype=mask_dtype, device=cuda)
    for b, n in enumerate(lens):
        mask[b, :n] = 1
    arr = from_hf_padded(hidden, mask)
    assert arr.offsets.tolist() == [0, 2, 8, 8]
    want = torch.cat([hidden[b, :n] for b, n in enumerate(lens)])
    assert torch.equal(arr.values, want)


def test_hf_mask_convention(cuda):
    import scree_b200 as scree
    from scree_b200.bridges import to_hf_padded

    arr = scree.pack(_seqs([2, 5], (4,), torch.float32, cuda))
    _, mask = to_hf_padded(arr)
    assert mask[0].tolist() == [1, 1, 0, 0, 0]
    assert mask[1].tolist() == [1, 1, 1, 1, 1]


def test_torch_nested_roundtrip_no_copy(cuda):
    import scree_b200 as scree
    from scree_b200.bridges import from_torch_nested, to_torch_nested

    arr = scree.pack(_seqs([3, 5, 2], (4,), torch.float32, cuda))
    nt = to_torch_nested(arr)
    assert nt.is_nested
    assert nt.values().data_ptr() == arr.values.data_ptr()  # wraps, does not copy
    rows = list(nt.unbind())
    for r, want in zip(rows, scree.unpack(arr)):
        assert torch.equal(r, want)
    arr2 = from_torch_nested(nt)
    assert torch.equal(arr2.values, arr.values)
    assert arr2.offsets.tolist() == arr.offsets.tolist()


def test_to_numpy_and_back(cuda):
    import scree_b200 as scree
    from scree_b200.bridges import to_numpy, to_torch

    arr = scree.pack(_seqs([3, 1], (2,), torch.float32, cuda))
    a_np = to_numpy(arr)
    assert isinstance(a_np.values, np.ndarray) and a_np.offsets.dtype == np.int32
    a_t = to_torch(a_np)
    assert torch.equal(a_t.values, arr.values.cpu())
    assert to_torch(arr) is arr and to_numpy(a_np) is a_np
