"""Host-side checks that need no GPU: the C ABI library loads and exports every
symbol include/scree_b200.h declares, argument validation maps to the
reference's exception types, workloads match their documented sizes, and the
Array container keeps the reference's invariants."""

import re
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent


def _header_symbols():
    text = (ROOT / "include" / "scree_b200.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:int|size_t|long long)\s+(scree_\w+)\s*\(", text, re.M)))


def test_library_exports_every_header_symbol():
    from scree_b200 import _lib

    lib = _lib.load()
    syms = _header_symbols()
    assert len(syms) >= 18
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(_lib.EXPORTED)
    assert lib.scree_version() == 1


def test_argument_validation_without_gpu():
    """Invalid sizes are rejected before any CUDA call."""
    from scree_b200 import _lib

    lib = _lib.load()
    rc = lib.scree_attn_fwd(None, None, None, 0, 0, 0, 0, 0, 0, None, 0, 1, 10, 1, 96, 1, 0, 1.0, 0, None, 0, 0, None, None, 0, None)
    assert rc == _lib.SCREE_ERR_UNSUPPORTED
    with pytest.raises(NotImplementedError, match="head_dim 96"):
        _lib.check(rc, "attn")
    rc = lib.scree_attn_fwd(None, None, None, 0, 0, 0, 0, 0, 0, None, 0, 0, 10, 1, 64, 1, 0, 1.0, 0, None, 0, 0, None, None, 0, None)
    assert rc == _lib.SCREE_ERR_INVALID
    with pytest.raises(ValueError):
        _lib.check(rc, "attn")
    rc = lib.scree_attn_bwd(None, None, None, None, None, None, None, 0, 1, 10, 1, 64, 2, 0, 1.0, 0, None, None, None, None, 0, None)
    assert rc == _lib.SCREE_ERR_INVALID  # null pointers are rejected before any CUDA call
    assert lib.scree_pack(None, None, 0, 0, 0, 0, 0, 16, None, None) == _lib.SCREE_ERR_INVALID
    assert lib.scree_to_padded(None, None, 0, 1, 1, 4, 3, None, 0, None, None, None) == _lib.SCREE_ERR_INVALID


def test_workspace_sizes():
    from scree_b200 import _lib

    lib = _lib.load()
    T, H, D, B = 158330, 32, 128, 64
    ws = lib.scree_attn_bwd_workspace_size(B, T, H, D)
    assert ws >= T * H * D * 4 + 2 * T * H * 4
    assert lib.scree_attn_fwd_workspace_size(B, T, H, D) == 16 + 16 * B  # one schedule entry per sequence


def test_workloads_match_documented_sizes():
    from scree_b200 import workloads as w

    assert sum(w.cfg1_lengths()) == 1710
    assert sum(w.cfg2_lengths()) == 12160 and max(w.cfg2_lengths()) == 1712
    assert sum(w.cfg3_lengths()) == 19794 and max(w.cfg3_lengths()) == 830
    l4 = w.cfg4_lengths()
    assert sum(l4) == 158330 and max(l4) == 6639 and min(l4) >= 16
    l5 = w.cfg5_lengths()
    assert sum(l5) == 36568 and max(l5) == 5278 and l5[:4] == [1, 1, 1, 1]
    assert abs(w.attn_flops(l4, 32, 128) / 1e9 - 14816.9) < 1
    assert abs(w.attn_flops(w.cfg2_lengths(), 16, 64) / 1e9 - 83.18) < 0.01


def test_lpt_partition_balance():
    from scree_b200 import workloads as w

    l4 = w.cfg4_lengths()
    costs = [L * L for L in l4]
    for n in (1, 2, 4, 8):
        parts = w.lpt_partition(costs, n)
        assert sorted(i for p in parts for i in p) == list(range(len(l4)))
        loads = [sum(costs[i] for i in p) for p in parts]
        assert max(loads) / (sum(loads) / n) < 1.02


def test_array_invariants_cpu():
    import scree_b200 as scree

    v = torch.zeros(5, 2)
    a = scree.Array(values=v, offsets=torch.tensor([0, 2, 5]))
    assert a.batch_size == 2 and a.total_length == 5 and a.feature_shape == (2,)
    assert a.lengths.tolist() == [2, 3]
    with pytest.raises(ValueError, match=r"offsets\[0\] must be 0"):
        scree.Array(values=v, offsets=torch.tensor([1, 5]))
    with pytest.raises(ValueError, match=r"must equal"):
        scree.Array(values=v, offsets=torch.tensor([0, 4]))
    with pytest.raises(ValueError, match="length >= 2"):
        scree.Array(values=v, offsets=torch.tensor([0]))
    with pytest.raises(ValueError, match="1-D"):
        scree.Array(values=v, offsets=torch.zeros(2, 2, dtype=torch.int64))
    with pytest.raises(ValueError, match="out of range"):
        scree.Array(values=v, offsets=torch.tensor([0, 5]), ragged_dim=2)
    # numpy container works too (validation only)
    b = scree.from_cu_seqlens(np.zeros((3, 1)), np.array([0, 1, 3]))
    assert len(b) == 2 and "batch_size=2" in repr(b)
    # unpack of a CPU array is view slicing only
    rows = scree.unpack(a)
    assert [r.shape[0] for r in rows] == [2, 3]


def test_data_ops_refuse_cpu_tensors():
    """No CPU fallback: the data-moving ops and kernels demand CUDA tensors."""
    import scree_b200 as scree
    from scree_b200.kernels import native

    with pytest.raises(TypeError, match="CUDA"):
        scree.pack([torch.zeros(2, 3)])
    with pytest.raises(TypeError, match="CUDA"):
        scree.to_padded(scree.Array(values=torch.zeros(3, 1), offsets=torch.tensor([0, 3])))
    with pytest.raises(AssertionError, match="CUDA"):
        native.varlen_rmsnorm_triton(torch.zeros(3, 8))
    q = torch.zeros(3, 1, 64, dtype=torch.float16)
    with pytest.raises(AssertionError, match="CUDA"):
        native.varlen_attention_triton(q, q, q, torch.tensor([0, 3], dtype=torch.int32))


def test_triton_module_path_is_drop_in():
    from scree_b200.kernels import triton as t

    for name in ("varlen_attention_triton", "varlen_attention_triton_autograd", "varlen_layernorm_triton", "varlen_rmsnorm_triton", "TRITON_AVAILABLE"):
        assert hasattr(t, name)
    assert t.TRITON_AVAILABLE is True


def test_norm_workspace_size_on_odd_and_wide_rows():
    """The backward workspace query plans every layout, including rows too wide
    for one CTA (rejected later by the kernel), without faulting."""
    from scree_b200 import _lib

    lib = _lib.load()
    for rows, C in [(100, 33), (19794, 4096), (1, 8), (64, 8192), (10, 100000), (0, 7)]:
        assert lib.scree_norm_bwd_workspace_size(rows, C) >= 8 * C
