"""Seeded random batches on the GPU (the reference's property-test style,
tests/test_properties.py): attention forward + backward on random lengths
(empty and length-1 sequences included), head counts, head dims, dtypes and
masks, against the fp64 oracle with the bar of tests/attn_cases.py; and the
gathers on random shapes and dtypes, bit-exact against the oracle."""

import numpy as np
import pytest
import torch

import oracle
from attn_cases import measure

pytestmark = pytest.mark.gpu


def _lengths(rng):
    B = int(rng.integers(1, 9))
    kinds = rng.integers(0, 4, size=B)
    out = []
    for k in kinds:
        if k == 0:
            out.append(int(rng.integers(0, 3)))          # empty / tiny
        elif k == 1:
            out.append(int(rng.integers(120, 140)))      # around a tile boundary
        else:
            out.append(int(rng.integers(1, 600)))
    if sum(out) == 0:
        out[0] = 1
    return out


@pytest.mark.parametrize("seed", range(12))
def test_random_attention_batches(cuda, seed):
    from scree_b200 import _lib

    rng = np.random.default_rng(1000 + seed)
    lengths = _lengths(rng)
    H = int(rng.integers(1, 4))
    D = int(rng.choice([32, 64, 128]))
    dtype = torch.bfloat16 if rng.integers(0, 2) else torch.float16
    causal = bool(rng.integers(0, 2))
    offs = torch.int64 if rng.integers(0, 2) else torch.int32
    stats = measure(lengths, H, D, dtype, causal, cuda, seed=seed, offs_dtype=offs)
    bad = [s for s in stats if s.verdict == "FAIL"]
    assert not bad, (lengths, H, D, dtype, causal, bad)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("seed", range(8))
def test_random_gathers_bit_exact(cuda, seed):
    import scree_b200 as scree

    rng = np.random.default_rng(2000 + seed)
    lengths = _lengths(rng)
    feat = tuple(int(f) for f in rng.integers(1, 6, size=int(rng.integers(0, 3))))
    dtype = [torch.float32, torch.bfloat16, torch.float16, torch.int8, torch.int64, torch.uint8][seed % 6]
    rows = []
    for n in lengths:
        t = torch.from_numpy(rng.integers(-100, 100, size=(n, *feat)).astype(np.int64)).to(dtype)
        rows.append(t.to(cuda))
    arr = scree.pack(rows)

    def host(t):  # numpy has no bfloat16; the values are small integers, exact in fp32
        return (t.float() if t.dtype == torch.bfloat16 else t).cpu().numpy()

    flat = [host(r) for r in rows]
    ref_vals, ref_offs = oracle.pack(flat)
    assert np.array_equal(host(arr.values), ref_vals)
    assert arr.offsets.cpu().tolist() == ref_offs.tolist()
    for side in ("right", "left"):
        padded, mask = scree.to_padded(arr, side=side, fill_value=7)
        rp, rm = oracle.to_padded(ref_vals, ref_offs, side=side, fill_value=7)
        assert np.array_equal(host(padded), rp) and np.array_equal(mask.cpu().numpy(), rm)
    padded, mask = scree.to_padded(arr)
    back = scree.from_padded(padded, mask)
    assert torch.equal(back.values, arr.values)
    assert back.offsets.tolist() == arr.offsets.tolist()
    for got, want in zip(scree.unpack(arr), rows):
        assert torch.equal(got, want)
