"""KV-cache support on the GPU: the append gather (bit-exact against a
per-sequence concatenation) and attention of new queries against cached + new
keys with end-aligned causal masking (query i of Lq sees keys j <= i + Lk - Lq),
checked against a float64 numpy evaluation of that definition with the
attention bar of tests/attn_cases.py (out: 1e-2 + 2^-8 |ref| bf16, 2e-3 +
2^-11 |ref| fp16; LSE 1e-3).  The reference plans this feature
(docs/kernels.md:178) without an implementation, so the definition is the
plain softmax attention restricted by that mask."""

import math

import numpy as np
import pytest
import torch

from gpu_helpers import ATTN_REL, ATTN_TOL, excess, max_err, to64

pytestmark = pytest.mark.gpu


def _arr(lens, feat, dtype, cuda, g):
    import scree_b200 as scree

    vals = torch.randn((sum(lens), *feat), generator=g).to(dtype).to(cuda)
    offs = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int64, device=cuda)
    return scree.from_cu_seqlens(vals, offs)


@pytest.mark.parametrize("feat", [(2, 64), (3,), (8, 128)])
def test_kv_append_bit_exact(cuda, feat):
    from scree_b200.kvcache import kv_append

    g = torch.Generator().manual_seed(0)
    cl, nl = [5, 0, 300, 17, 0], [1, 4, 0, 33, 0]
    cache, new = _arr(cl, feat, torch.bfloat16, cuda, g), _arr(nl, feat, torch.bfloat16, cuda, g)
    out = kv_append(cache, new)
    co, no = np.concatenate([[0], np.cumsum(cl)]), np.concatenate([[0], np.cumsum(nl)])
    want = torch.cat([torch.cat([cache.values[co[b]:co[b + 1]], new.values[no[b]:no[b + 1]]]) for b in range(len(cl))])
    assert torch.equal(out.values, want)
    assert out.offsets.tolist() == list(np.concatenate([[0], np.cumsum(np.add(cl, nl))]))
    from scree_b200 import _lib

    assert _lib.device_status() == 0


def _ref_kv(q, k, v, lq, lk, causal):
    qn, kn, vn = (to64(t) for t in (q, k, v))
    H, Hkv, D = qn.shape[1], kn.shape[1], qn.shape[2]
    G = H // Hkv
    kn, vn = np.repeat(kn, G, axis=1), np.repeat(vn, G, axis=1)
    out = np.zeros_like(qn)
    lse = np.full(qn.shape[:2], -np.inf)
    qo, ko = np.concatenate([[0], np.cumsum(lq)]), np.concatenate([[0], np.cumsum(lk)])
    for b in range(len(lq)):
        Lq, Lk = lq[b], lk[b]
        if Lq == 0:
            continue
        qs, ks, vs = qn[qo[b]:qo[b + 1]], kn[ko[b]:ko[b + 1]], vn[ko[b]:ko[b + 1]]
        s = np.einsum("ihd,jhd->hij", qs, ks) / math.sqrt(D)
        if causal:
            i = np.arange(Lq)[:, None]
            j = np.arange(Lk)[None, :]
            s = np.where(j > i + (Lk - Lq), -np.inf, s)
        for h in range(H):
            for r in range(Lq):
                row = s[h, r]
                if not np.isfinite(row).any():
                    continue
                m = row.max()
                e = np.exp(row - m)
                out[qo[b] + r, h] = (e / e.sum()) @ vs[:, h]
                lse[qo[b] + r, h] = m + np.log(e.sum())
    return out, lse


CASES = {
    "decode": ([1, 1, 1, 1], [1, 300, 129, 2048]),
    "chunked_prefill": ([37, 128, 5], [37 + 100, 128 + 256, 5 + 1]),
    "fewer_keys": ([40, 3], [10, 3]),
    "empty_queries": ([0, 65, 1], [17, 65, 0]),
}


@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("D,H,Hkv", [(128, 4, 2), (64, 2, 2)])
def test_attention_with_cache(cuda, case, causal, D, H, Hkv):
    from scree_b200.kvcache import varlen_attention_kv

    lq, lk = CASES[case]
    g = torch.Generator().manual_seed(len(case) + D)
    dt = torch.bfloat16
    q = _arr(lq, (H, D), dt, cuda, g)
    k = _arr(lk, (Hkv, D), dt, cuda, g)
    v = _arr(lk, (Hkv, D), dt, cuda, g)
    out, lse = varlen_attention_kv(q, k, v, causal=causal, return_lse=True)
    torch.cuda.synchronize()
    ro, rl = _ref_kv(q.values, k.values, v.values, lq, lk, causal)
    assert excess(to64(out.values), ro, ATTN_TOL[dt], ATTN_REL[dt]) <= 0
    got_l = to64(lse)
    fin = np.isfinite(rl)
    assert np.array_equal(np.isfinite(got_l), fin)
    if fin.any():
        assert max_err(got_l[fin], rl[fin]) <= 1e-3
    from scree_b200 import _lib

    assert _lib.device_status() == 0


def test_cache_attention_equals_self_attention_without_cache(cuda):
    """With keys = queries (empty cache) it is the ordinary causal attention."""
    import scree_b200 as scree
    from scree_b200.kernels.native import varlen_attention_triton
    from scree_b200.kvcache import kv_append, varlen_attention_kv

    g = torch.Generator().manual_seed(9)
    lens = [70, 1, 300]
    q, k, v = (_arr(lens, (2, 64), torch.float16, cuda, g) for _ in range(3))
    empty = scree.from_cu_seqlens(torch.zeros((0, 2, 64), dtype=torch.float16, device=cuda),
                                  torch.zeros(4, dtype=torch.int64, device=cuda))
    kk = kv_append(empty, k)
    out = varlen_attention_kv(q, kk, kv_append(empty, v), causal=True)
    ref = varlen_attention_triton(q.values, k.values, v.values, q.offsets, causal=True)
    torch.testing.assert_close(out.values, ref, atol=0, rtol=0)
