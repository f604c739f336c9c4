"""Pin the oracle against golden vectors produced by the real reference
(tests/golden/make_golden.py) and against the reference's own known-answer
tests (tests/test_varlen_kernels.py, tests/test_core.py of jvoltci/scree)."""

import numpy as np
import pytest

from conftest import decode16, load_golden
import oracle

ATTN_CASES = ["attn_ref_small_c0", "attn_ref_small_c1", "attn_d32_f16_c0", "attn_d32_f16_c1", "attn_d128_bf16_c1"]


@pytest.mark.parametrize("name", ATTN_CASES)
def test_oracle_attention_matches_reference(name):
    g = load_golden(name)
    dt = str(g["dtype"])
    q, k, v, do = (decode16(g[n], dt) for n in ("q", "k", "v", "do"))
    offs = oracle.pack([np.zeros((int(n), 1)) for n in g["lengths"]])[1]
    out, lse = oracle.attention_fwd(q, k, v, offs, causal=bool(g["causal"]))
    np.testing.assert_allclose(out, g["out"], atol=2e-6, rtol=1e-5)
    np.testing.assert_allclose(out, g["out_torch"], atol=2e-6, rtol=1e-5)
    dq, dk, dv = oracle.attention_bwd(do, q, k, v, offs, causal=bool(g["causal"]))
    for mine, ref in ((dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"])):
        np.testing.assert_allclose(mine, ref, atol=1e-5, rtol=1e-4)
    assert np.isfinite(lse).all()


def test_oracle_attention_per_sequence_baseline():
    """reference tests/test_varlen_kernels.py:19-43: each row equals isolated attention."""
    rng = np.random.default_rng(0)
    lengths = [3, 5, 2]
    seqs = [[rng.standard_normal((n, 2, 4)).astype(np.float32) for n in lengths] for _ in range(3)]
    (q, offs), (k, _), (v, _) = (oracle.pack(s) for s in seqs)
    out, _ = oracle.attention_fwd(q, k, v, offs)
    for i, rows in enumerate(oracle.unpack(out, offs)):
        qi, ki, vi = seqs[0][i], seqs[1][i], seqs[2][i]
        sc = np.einsum("ihd,jhd->hij", qi, ki) / 2.0
        a = np.exp(sc - sc.max(-1, keepdims=True))
        a /= a.sum(-1, keepdims=True)
        np.testing.assert_allclose(rows, np.einsum("hij,jhd->ihd", a, vi), atol=1e-5)


def test_oracle_causal_first_token_is_v0():
    """reference tests/test_varlen_kernels.py:46-63."""
    rng = np.random.default_rng(0)
    seqs = [[rng.standard_normal((n, 1, 4)) for n in [4, 6]] for _ in range(3)]
    (q, offs), (k, _), (v, _) = (oracle.pack(s) for s in seqs)
    out, _ = oracle.attention_fwd(q, k, v, offs, causal=True)
    for i, rows in enumerate(oracle.unpack(out, offs)):
        np.testing.assert_allclose(rows[0], seqs[2][i][0], atol=1e-12)


@pytest.mark.parametrize("name", ["norm_ref_small", "norm_ref_small_w", "norm_c128"])
def test_oracle_norms_match_reference(name):
    g = load_golden(name)
    w = g.get("w")
    b = g.get("b")
    y = oracle.rmsnorm_fwd(g["x"], w, float(g["eps_rms"]))
    np.testing.assert_allclose(y, g["y_rms"], atol=1e-5)
    y = oracle.layernorm_fwd(g["x"], w, b, float(g["eps_ln"]))
    np.testing.assert_allclose(y, g["y_ln"], atol=1e-5)
    dx, dw = oracle.rmsnorm_bwd(g["dy"], g["x"], w, float(g["eps_rms"]))
    np.testing.assert_allclose(dx, g["dx_rms"], atol=1e-5)
    if w is not None:
        np.testing.assert_allclose(dw, g["dw_rms"], atol=1e-4)
    dx, dw, db = oracle.layernorm_bwd(g["dy"], g["x"], w, b, float(g["eps_ln"]))
    np.testing.assert_allclose(dx, g["dx_ln"], atol=1e-5)
    if w is not None:
        np.testing.assert_allclose(dw, g["dw_ln"], atol=1e-4)
    if b is not None:
        np.testing.assert_allclose(db, g["db_ln"], atol=1e-4)


def test_oracle_norm_closed_forms():
    """reference tests/test_varlen_kernels.py:78-116."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((10, 8)).astype(np.float32)
    m = x.mean(-1, keepdims=True)
    np.testing.assert_allclose(oracle.layernorm_fwd(x, eps=1e-5), (x - m) / np.sqrt(x.var(-1, keepdims=True) + 1e-5), atol=1e-6)
    np.testing.assert_allclose(oracle.rmsnorm_fwd(x, eps=1e-6), x / np.sqrt((x * x).mean(-1, keepdims=True) + 1e-6), atol=1e-6)


@pytest.mark.parametrize("name", ["gather_2d", "gather_3d"])
def test_oracle_gathers_match_reference(name):
    g = load_golden(name)
    offs = g["offsets"]
    seqs = oracle.unpack(g["values"], offs)
    vals, o2 = oracle.pack(seqs)
    assert np.array_equal(vals, g["values"]) and np.array_equal(o2, offs) and o2.dtype == np.int32
    for side in ("right", "left"):
        p, m = oracle.to_padded(g["values"], offs, side=side, fill_value=int(g["fill"]))
        assert np.array_equal(p, g[f"padded_{side}"]) and np.array_equal(m, g[f"mask_{side}"])
    v3, o3 = oracle.from_padded(g["padded_right"], g["mask_right"])
    assert np.array_equal(v3, g["from_padded_values"]) and np.array_equal(o3, g["from_padded_offsets"])


def test_oracle_roundtrip_left_padding_mask():
    """reference tests/test_core.py:71-78: left padding puts the mask on the right."""
    vals, offs = oracle.pack([np.ones((2, 3)), np.ones((4, 3))])
    p, m = oracle.to_padded(vals, offs, side="left")
    assert m.tolist() == [[False, False, True, True], [True, True, True, True]]


@pytest.mark.parametrize("name", ["softmax_ref_small", "softmax_2d"])
def test_oracle_softmax_matches_reference(name):
    """varlen_softmax (reference/varlen_softmax.py): values and torch-autograd gradient."""
    g = load_golden(name)
    offs = np.concatenate([[0], np.cumsum(g["lengths"])])
    y = oracle.softmax_fwd(g["x"], offs)
    np.testing.assert_allclose(y, g["y"], atol=1e-6)
    np.testing.assert_allclose(y, g["y_torch"], atol=1e-6)
    np.testing.assert_allclose(oracle.softmax_bwd(g["dy"], y, offs), g["dx"], atol=1e-5)


def test_oracle_softmax_columns_sum_to_one():
    """reference tests/test_varlen_kernels.py:119-140: per-sequence sums are 1."""
    rng = np.random.default_rng(0)
    vals, offs = oracle.pack([rng.standard_normal((n, 3)) for n in [3, 5, 2]])
    y = oracle.softmax_fwd(vals, offs)
    for rows in oracle.unpack(y, offs):
        np.testing.assert_allclose(rows.sum(axis=0), np.ones(3), atol=1e-12)
