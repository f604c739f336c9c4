"""Grouped-query attention (fewer K/V heads than query heads) on the GPU
kernels, forward and backward, against the fp64 oracle run on K/V expanded to
every query head (query head h reads K/V head h // G; dk / dv are the sums over
the G query heads of a group).  Same bar as the plain attention tests
(tests/attn_cases.py) for the output and dq; for the group-summed dk / dv see
the comment in the test.  The reference lists GQA as not yet supported
(docs/kernels.md:177), so the expansion is the definition checked here."""

import numpy as np
import pytest
import torch

from gpu_helpers import ATTN_REL, ATTN_TOL, attn_bwd_emulated, attn_reference, excess, max_err, round_to, to64

pytestmark = pytest.mark.gpu


def _inputs(lengths, H, Hkv, D, dtype, cuda, seed):
    g = torch.Generator().manual_seed(seed)
    T = sum(lengths)
    q, do = (torch.randn((T, H, D), generator=g).to(dtype).to(cuda) for _ in range(2))
    k, v = (torch.randn((T, Hkv, D), generator=g).to(dtype).to(cuda) for _ in range(2))
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lengths)]), dtype=torch.int32, device=cuda)
    return q, k, v, do, cu


def _group_sum(x, G):
    T, H, D = x.shape
    return x.reshape(T, H // G, G, D).sum(axis=2)


@pytest.mark.parametrize("H,Hkv", [(8, 2), (4, 1), (6, 3)])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gqa_fwd_bwd_16bit(cuda, H, Hkv, D, causal, dtype):
    from scree_b200 import _lib
    from scree_b200.kernels.native import varlen_attention_triton, varlen_attention_triton_backward

    lengths = [1, 130, 257, 5]
    G = H // Hkv
    q, k, v, do, cu = _inputs(lengths, H, Hkv, D, dtype, cuda, seed=H + D)
    out, lse = varlen_attention_triton(q, k, v, cu, causal=causal, return_lse=True)
    dq, dk, dv = varlen_attention_triton_backward(do, q, k, v, out, lse, cu, causal=causal)
    torch.cuda.synchronize()
    assert dk.shape == k.shape and dv.shape == v.shape and dq.shape == q.shape
    ke, ve = (t.repeat_interleave(G, dim=1) for t in (k, v))
    ref = list(attn_reference(q, ke, ve, do, lengths, causal))
    ref[3], ref[4] = _group_sum(ref[3], G), _group_sum(ref[4], G)
    tol, rel = ATTN_TOL[dtype], ATTN_REL[dtype]
    emul = None
    for name, got, want in zip(("out", "lse", "dq", "dk", "dv"), (out, lse, dq, dk, dv), ref):
        g = to64(got)
        if name == "lse":
            assert max_err(g, want) <= 1e-3
            continue
        err = max_err(g, want)
        if excess(g, want, tol, rel) <= 0:
            continue
        # dk / dv here sum G query heads' contributions, so they are larger than
        # any single-head gradient and their 16-bit storage rounding grows with
        # them.  Past the bound, the kernel must stay within twice the error of
        # the fp64 oracle evaluated with a tensor-core backward's 16-bit P / dS
        # / O and with its result stored in the output dtype.
        assert name != "out", (name, err)
        if emul is None:
            e = attn_bwd_emulated(do, q, ke, ve, lengths, causal, dtype)
            emul = {"dq": round_to(e[0], dtype), "dk": round_to(_group_sum(e[1], G), dtype),
                    "dv": round_to(_group_sum(e[2], G), dtype)}
        e_emul = max_err(emul[name], want)
        assert err <= 2 * e_emul, (name, err, e_emul)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("causal", [False, True])
def test_gqa_fp32(cuda, causal):
    from scree_b200.kernels.native import varlen_attention_fp32, varlen_attention_fp32_backward

    lengths = [3, 64, 1, 77]
    H, Hkv, D, G = 8, 2, 32, 4
    q, k, v, do, cu = _inputs(lengths, H, Hkv, D, torch.float32, cuda, seed=7)
    out, lse = varlen_attention_fp32(q, k, v, cu, causal)
    dq, dk, dv = varlen_attention_fp32_backward(do, q, k, v, out, lse, cu, causal)
    torch.cuda.synchronize()
    ke, ve = (t.repeat_interleave(G, dim=1) for t in (k, v))
    ref = list(attn_reference(q, ke, ve, do, lengths, causal))
    ref[3], ref[4] = _group_sum(ref[3], G), _group_sum(ref[4], G)
    for name, got, want in zip(("out", "lse", "dq", "dk", "dv"), (out, lse, dq, dk, dv), ref):
        assert max_err(to64(got), want) <= 1e-4, name


def test_gqa_autograd_and_shape_errors(cuda):
    from scree_b200.kernels.native import varlen_attention_triton, varlen_attention_triton_autograd

    lengths = [40, 9]
    q, k, v, do, cu = _inputs(lengths, 4, 2, 64, torch.bfloat16, cuda, seed=3)
    for t in (q, k, v):
        t.requires_grad_(True)
    out = varlen_attention_triton_autograd(q, k, v, cu, causal=True)
    out.backward(do)
    assert k.grad.shape == k.shape and q.grad.shape == q.shape
    bad = torch.zeros((49, 3, 64), dtype=torch.bfloat16, device=cuda)
    with pytest.raises(AssertionError, match="multiple"):
        varlen_attention_triton(q.detach(), bad, bad, cu)
