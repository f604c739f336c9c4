"""The allocation-free attention forward, scree_attn_fwd_noalloc (GPU only).

It exists for callers that cannot allocate device memory when they run
attention (an engine working from a fixed memory arena, or a binding that only
holds raw pointers).  Called through the C ABI, twice in a row, it must match
scree_attn_fwd with a caller workspace, within the attention tolerance the
other tests use (it runs the same kernels, so the results are in fact equal).
This file is collected last so a failure here comes after every other test.
"""

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(lib, fn, q, k, v, cu, o, lse, ws=None):
    from scree_b200 import _lib

    T, H, D = q.shape
    B = cu.numel() - 1
    args = [
        q.data_ptr(), k.data_ptr(), v.data_ptr(), q.stride(0), q.stride(1), k.stride(0), k.stride(1),
        v.stride(0), v.stride(1), cu.data_ptr(), 0, B, T, H, D, _lib.dtype_code(q.dtype), 1,
        1.0 / math.sqrt(D), 0, o.data_ptr(), o.stride(0), o.stride(1), lse.data_ptr(),
    ]
    if ws is not None:
        args += [ws.data_ptr(), ws.numel()]
    args.append(torch.cuda.current_stream().cuda_stream)
    return getattr(lib, fn)(*args)


def test_noalloc_forward_matches_workspace_forward(cuda):
    from scree_b200 import _lib, workloads

    lib = _lib.load()
    for seed, lengths in ((0, [1, 300, 77, 128, 5]), (1, [513, 2, 64])):
        q, k, v = workloads.make_qkv(lengths, 4, 128, "bfloat16", cuda, seed=seed, with_do=False)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=cuda)
        T, H, _ = q.shape
        o_ref = torch.empty_like(q)
        l_ref = torch.empty((T, H), dtype=torch.float32, device=cuda)
        ws = torch.empty(lib.scree_attn_fwd_workspace_size(len(lengths), T, H, 128), dtype=torch.uint8, device=cuda)
        _lib.check(_call(lib, "scree_attn_fwd", q, k, v, cu, o_ref, l_ref, ws), "scree_attn_fwd")
        for _ in range(2):  # two calls in a row share the built-in scratch
            o = torch.full_like(q, float("nan"))
            lse = torch.full((T, H), float("nan"), dtype=torch.float32, device=cuda)
            _lib.check(_call(lib, "scree_attn_fwd_noalloc", q, k, v, cu, o, lse), "scree_attn_fwd_noalloc")
            torch.cuda.synchronize()
            torch.testing.assert_close(o.float(), o_ref.float(), atol=1e-2, rtol=2.0**-8)
            torch.testing.assert_close(lse, l_ref, atol=1e-3, rtol=0)
    assert _lib.device_status() == 0


def test_noalloc_rejects_batches_over_the_limit(cuda):
    from scree_b200 import _lib

    lib = _lib.load()
    B = 4096  # one more than the 64 KiB scratch holds
    q = torch.zeros((B, 1, 64), dtype=torch.float16, device=cuda)
    cu = torch.arange(B + 1, dtype=torch.int32, device=cuda)
    o = torch.empty_like(q)
    lse = torch.empty((B, 1), dtype=torch.float32, device=cuda)
    rc = _call(lib, "scree_attn_fwd_noalloc", q, q, q, cu, o, lse)
    assert rc == _lib.SCREE_ERR_INVALID
    assert "4095" in _lib.last_error()
