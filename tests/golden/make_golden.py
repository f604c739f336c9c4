"""Generate golden vectors for the oracle by running the real scree reference.

Usage:  python tests/golden/make_golden.py --ref <scree checkout>/src

Imports ``scree`` (jvoltci/scree) from the given source directory and stores,
for small seeded inputs, the reference's own outputs:
  * forward values from the reference's numpy branch
    (src/scree/kernels/reference/varlen_attention.py:115-138,
     varlen_rmsnorm.py:58-65, varlen_layernorm.py:64-74, _core.py pack /
     to_padded / from_padded numpy branches);
  * gradients from torch autograd (float64) through the reference's torch
    branch (the path tests/test_autograd.py:28-64 exercises), since the
    reference has no explicit backward.
The fixtures (golden_*.npz next to this script) are committed; the GPU box never
needs the reference.  16-bit inputs are stored as their bit patterns (uint16)
so every value is exact.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def bf16_bits(x32: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = x32.astype(np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def bf16_value(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def attn_case(scree, ref, torch, lengths, H, D, dtype, causal, seed):
    rng = np.random.default_rng(seed)
    T = sum(lengths)
    raw = [rng.standard_normal((T, H, D)).astype(np.float32) for _ in range(4)]
    if dtype == "float16":
        bits = [r.astype(np.float16).view(np.uint16) for r in raw]
        vals = [b.view(np.float16).astype(np.float64) for b in bits]
    elif dtype == "bfloat16":
        bits = [bf16_bits(r) for r in raw]
        vals = [bf16_value(b).astype(np.float64) for b in bits]
    else:
        bits = raw
        vals = [r.astype(np.float64) for r in raw]
    q, k, v, do = vals
    offs = np.zeros(len(lengths) + 1, dtype=np.int32)
    offs[1:] = np.cumsum(lengths)
    A = lambda x: scree.Array(values=x, offsets=offs)  # noqa: E731
    out = ref.varlen_attention(A(q), A(k), A(v), causal=causal).values
    tq, tk, tv = (torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (q, k, v))
    toffs = torch.tensor(offs)
    TA = lambda x: scree.Array(values=x, offsets=toffs)  # noqa: E731
    tout = ref.varlen_attention(TA(tq), TA(tk), TA(tv), causal=causal).values
    tout.backward(torch.tensor(do))
    return {
        "lengths": np.array(lengths, dtype=np.int64),
        "H": H,
        "D": D,
        "causal": int(causal),
        "dtype": dtype,
        "q": bits[0], "k": bits[1], "v": bits[2], "do": bits[3],
        "out": out.astype(np.float32),
        "out_torch": tout.detach().numpy().astype(np.float32),
        "dq": tq.grad.numpy().astype(np.float32),
        "dk": tk.grad.numpy().astype(np.float32),
        "dv": tv.grad.numpy().astype(np.float32),
    }


def norm_case(scree, ref, torch, lengths, C, with_weight, with_bias, seed, eps_rms, eps_ln):
    rng = np.random.default_rng(seed)
    T = sum(lengths)
    x = rng.standard_normal((T, C)).astype(np.float32)
    dy = rng.standard_normal((T, C)).astype(np.float32)
    w = (1.0 + 0.02 * rng.standard_normal(C)).astype(np.float32) if with_weight else None
    b = (0.02 * rng.standard_normal(C)).astype(np.float32) if with_bias else None
    offs = np.zeros(len(lengths) + 1, dtype=np.int32)
    offs[1:] = np.cumsum(lengths)
    arr = scree.Array(values=x.astype(np.float64), offsets=offs)
    w64 = None if w is None else w.astype(np.float64)
    b64 = None if b is None else b.astype(np.float64)
    y_rms = ref.varlen_rmsnorm(arr, weight=w64, eps=eps_rms).values
    y_ln = ref.varlen_layernorm(arr, weight=w64, bias=b64, eps=eps_ln).values
    res = {"lengths": np.array(lengths), "x": x, "dy": dy, "eps_rms": eps_rms, "eps_ln": eps_ln,
           "y_rms": y_rms.astype(np.float32), "y_ln": y_ln.astype(np.float32)}
    if w is not None:
        res["w"] = w
    if b is not None:
        res["b"] = b
    toffs = torch.tensor(offs)
    for name, fn in (("rms", "varlen_rmsnorm"), ("ln", "varlen_layernorm")):
        tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
        tw = torch.tensor(w, dtype=torch.float64, requires_grad=True) if w is not None else None
        tb = torch.tensor(b, dtype=torch.float64, requires_grad=True) if b is not None else None
        tarr = scree.Array(values=tx, offsets=toffs)
        if name == "rms":
            ty = ref.varlen_rmsnorm(tarr, weight=tw, eps=eps_rms).values
        else:
            ty = ref.varlen_layernorm(tarr, weight=tw, bias=tb, eps=eps_ln).values
        ty.backward(torch.tensor(dy, dtype=torch.float64))
        res[f"dx_{name}"] = tx.grad.numpy().astype(np.float32)
        if tw is not None:
            res[f"dw_{name}"] = tw.grad.numpy().astype(np.float32)
        if tb is not None and name == "ln":
            res["db_ln"] = tb.grad.numpy().astype(np.float32)
    return res


def softmax_case(scree, ref, torch, lengths, feat, seed):
    rng = np.random.default_rng(seed)
    T = sum(lengths)
    x = (3.0 * rng.standard_normal((T, *feat))).astype(np.float32)
    dy = rng.standard_normal((T, *feat)).astype(np.float32)
    offs = np.zeros(len(lengths) + 1, dtype=np.int32)
    offs[1:] = np.cumsum(lengths)
    y = ref.varlen_softmax(scree.Array(values=x.astype(np.float64), offsets=offs)).values
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    ty = ref.varlen_softmax(scree.Array(values=tx, offsets=torch.tensor(offs))).values
    ty.backward(torch.tensor(dy, dtype=torch.float64))
    return {"lengths": np.array(lengths), "x": x, "dy": dy, "y": y.astype(np.float32),
            "y_torch": ty.detach().numpy().astype(np.float32), "dx": tx.grad.numpy().astype(np.float32)}


def gather_case(scree, lengths, feat, seed, fill):
    rng = np.random.default_rng(seed)
    seqs = [rng.integers(-1000, 1000, size=(n, *feat)).astype(np.int32) for n in lengths]
    arr = scree.pack(seqs)
    right, mright = scree.to_padded(arr, side="right", fill_value=fill)
    left, mleft = scree.to_padded(arr, side="left", fill_value=fill)
    back = scree.from_padded(right, mright)
    return {
        "lengths": np.array(lengths), "values": arr.values, "offsets": arr.offsets,
        "padded_right": right, "mask_right": mright, "padded_left": left, "mask_left": mleft,
        "fill": fill, "from_padded_values": back.values, "from_padded_offsets": back.offsets,
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path to the scree source dir (contains scree/)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    import torch
    import scree
    import scree.kernels.reference as ref

    # Attention: the reference test's shape, then GPU-sized head dims.
    cases = {
        "attn_ref_small_c0": attn_case(scree, ref, torch, [3, 5, 2], 2, 4, "float32", False, 0),
        "attn_ref_small_c1": attn_case(scree, ref, torch, [3, 5, 2], 2, 4, "float32", True, 0),
        "attn_d32_f16_c0": attn_case(scree, ref, torch, [1, 17, 128, 129, 64], 2, 32, "float16", False, 1),
        "attn_d32_f16_c1": attn_case(scree, ref, torch, [1, 17, 128, 129, 64], 2, 32, "float16", True, 1),
        "attn_d128_bf16_c1": attn_case(scree, ref, torch, [1, 130, 70], 1, 128, "bfloat16", True, 2),
    }
    for name, c in cases.items():
        np.savez_compressed(OUT / f"golden_{name}.npz", **c)
    norms = {
        "norm_ref_small": norm_case(scree, ref, torch, [3, 5, 2], 8, False, False, 0, 1e-6, 1e-5),
        "norm_ref_small_w": norm_case(scree, ref, torch, [3, 5, 2], 8, True, True, 0, 1e-6, 1e-5),
        "norm_c128": norm_case(scree, ref, torch, [3, 5, 2, 60], 128, True, True, 3, 1e-6, 1e-5),
    }
    for name, c in norms.items():
        np.savez_compressed(OUT / f"golden_{name}.npz", **c)
    for name, c in {
        "softmax_ref_small": softmax_case(scree, ref, torch, [3, 5, 2], (4,), 6),
        "softmax_2d": softmax_case(scree, ref, torch, [1, 7, 40, 13], (3, 24), 7),
    }.items():
        np.savez_compressed(OUT / f"golden_{name}.npz", **c)
    gathers = {
        "gather_2d": gather_case(scree, [3, 1, 5, 2], (3,), 4, -7),
        "gather_3d": gather_case(scree, [4, 7, 1, 6, 2], (2, 4), 5, 9),
    }
    for name, c in gathers.items():
        np.savez_compressed(OUT / f"golden_{name}.npz", **c)
    print("wrote", sorted(p.name for p in OUT.glob("golden_*.npz")))


if __name__ == "__main__":
    main()
