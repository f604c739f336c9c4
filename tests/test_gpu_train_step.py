"""End-to-end training step through the drop-in API (the caller side of the
hot path): the pre-norm transformer block of the reference's
examples/03_train_step.py:26-48, with scree_b200's varlen_rmsnorm and
varlen_attention (bf16 q/k/v, causal) in place of scree.kernels.reference,
plain torch matmuls around them.  Checked against the same block written
with per-sequence torch fp32 ops, and for a decreasing loss under Adam."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _block(x_vals, offsets, host, W, n_heads, native):
    import scree_b200 as scree
    from scree_b200.kernels import varlen_attention, varlen_rmsnorm

    Wqkv, Wo, W1, W2 = W
    T, C = x_vals.shape
    D = C // n_heads

    def rms(v):
        if native:
            return varlen_rmsnorm(scree.Array(values=v, offsets=offsets, _host=host), eps=1e-6).values
        return v / torch.sqrt(v.pow(2).mean(-1, keepdim=True) + 1e-6)

    h = rms(x_vals)
    qkv = (h @ Wqkv).reshape(T, 3, n_heads, D)
    if native:
        q, k, v = (scree.Array(values=qkv[:, i].to(torch.bfloat16), offsets=offsets, _host=host) for i in range(3))
        attn = varlen_attention(q, k, v, causal=True).values.float()
    else:
        outs = []
        for b in range(len(host) - 1):
            s, e = host[b], host[b + 1]
            qi, ki, vi = (qkv[s:e, i].to(torch.bfloat16).float() for i in range(3))
            sc = torch.einsum("ihd,jhd->hij", qi, ki) / math.sqrt(D)
            mask = torch.triu(torch.ones(e - s, e - s, dtype=torch.bool, device=sc.device), diagonal=1)
            p = torch.softmax(sc.masked_fill(mask, float("-inf")), dim=-1)
            outs.append(torch.einsum("hij,jhd->ihd", p, vi))
        attn = torch.cat(outs)
    h1 = x_vals + attn.reshape(T, C) @ Wo
    ff = torch.nn.functional.gelu(rms(h1) @ W1) @ W2
    return h1 + ff


def _params(C, F, device, seed=0):
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / math.sqrt(C)
    shapes = [(C, 3 * C, s), (C, C, s), (C, F, s), (F, C, 1.0 / math.sqrt(F))]
    return [torch.nn.Parameter((torch.randn(a, b, generator=g) * sc).to(device)) for a, b, sc in shapes]


def test_train_step_matches_torch_and_learns(cuda):
    import scree_b200 as scree

    torch.manual_seed(0)
    lengths, C, H, F = [6, 40, 130, 1], 128, 4, 256
    seqs = [torch.randn(n, C, device=cuda) for n in lengths]
    x = scree.pack(seqs)
    host = list(x._host)
    target = x.values.detach().clone()

    # Step-0 agreement with the torch fp32 formulation (same bf16 q/k/v rounding).
    W_n = _params(C, F, cuda)
    W_t = [torch.nn.Parameter(w.detach().clone()) for w in W_n]
    loss_n = ((_block(x.values, x.offsets, host, W_n, H, True) - target) ** 2).mean()
    loss_t = ((_block(x.values, x.offsets, host, W_t, H, False) - target) ** 2).mean()
    loss_n.backward()
    loss_t.backward()
    assert abs(loss_n.item() - loss_t.item()) <= 2e-2 * abs(loss_t.item())
    for wn, wt in zip(W_n, W_t):
        rel = (wn.grad - wt.grad).norm() / wt.grad.norm()
        assert rel < 5e-2, float(rel)

    # A few Adam steps on the copy task decrease the loss (reference example).
    W = _params(C, F, cuda, seed=1)
    opt = torch.optim.Adam(W, lr=3e-3)
    losses = []
    for _ in range(20):
        opt.zero_grad()
        loss = ((_block(x.values, x.offsets, host, W, H, True) - target) ** 2).mean()
        loss.backward()
        opt.step()
        losses.append(loss.item())
    assert losses[-1] < 0.7 * losses[0], losses
    from scree_b200 import _lib

    assert _lib.device_status() == 0
