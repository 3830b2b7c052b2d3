"""The oracle's analytic gradients against torch autograd (float64, CPU)
through the reference's eager formulas (src/agents/mappo.py:192-231
topk_gather, 361-373 dense). Pins the gradient oracle the GPU backward tests
use."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle


def _eager_gather(q, k, v, idx):
    # topk_gather / zorder_k contraction with a fixed index set
    B, N, d = q.shape
    kk = idx.shape[-1]
    flat = idx.reshape(B, N * kk, 1).expand(B, N * kk, d)
    kg = k.gather(1, flat).view(B, N, kk, d)
    vg = v.gather(1, flat).view(B, N, kk, d)
    s = torch.matmul(q.unsqueeze(-2), kg.transpose(-1, -2)) / (d ** 0.5)
    w = torch.softmax(s, dim=-1)
    return torch.matmul(w, vg).squeeze(-2)


def _eager_dense(q, k, v):
    N = q.shape[1]
    s = torch.matmul(q, k.transpose(-1, -2)) / (k.shape[-1] ** 0.5)
    s = s.masked_fill(torch.eye(N, dtype=torch.bool), float("-inf"))
    return torch.matmul(torch.softmax(s, -1), v)


def _leaf(x):
    return torch.from_numpy(x.astype(np.float64)).requires_grad_(True)


@pytest.mark.parametrize("B,N,d,kk,dup", [(3, 7, 5, 2, False), (2, 20, 16, 4, False),
                                          (2, 9, 8, 5, True)])
def test_gather_grad_matches_autograd(B, N, d, kk, dup):
    rng = np.random.default_rng(B * 100 + N)
    q, k, v, g = (rng.standard_normal((B, N, d)) for _ in range(4))
    if dup:   # repeated peers in a row are summed by autograd as well
        idx = rng.integers(0, N, size=(B, N, kk))
    else:
        idx = np.stack([np.stack([rng.choice(N, kk, replace=False)
                                  for _ in range(N)]) for _ in range(B)])
    tq, tk, tv = _leaf(q), _leaf(k), _leaf(v)
    out = _eager_gather(tq, tk, tv, torch.from_numpy(idx))
    out.backward(torch.from_numpy(g))
    dq, dk, dv = oracle.gather_attention_grad(q, k, v, idx, g)
    np.testing.assert_allclose(dq, tq.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dk, tk.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dv, tv.grad.numpy(), rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("B,N,d", [(2, 2, 3), (3, 6, 16), (2, 33, 8)])
def test_dense_grad_matches_autograd(B, N, d):
    rng = np.random.default_rng(N * 7 + d)
    q, k, v, g = (rng.standard_normal((B, N, d)) for _ in range(4))
    tq, tk, tv = _leaf(q), _leaf(k), _leaf(v)
    _eager_dense(tq, tk, tv).backward(torch.from_numpy(g))
    dq, dk, dv = oracle.dense_attention_grad(q, k, v, g)
    np.testing.assert_allclose(dq, tq.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dk, tk.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dv, tv.grad.numpy(), rtol=1e-10, atol=1e-12)


def test_topk_grad_is_gather_grad_of_the_selection():
    """Gradients of the eager top-k path (torch.topk then gather) equal the
    fixed-set gradient at the selected indices: the selection carries none."""
    rng = np.random.default_rng(5)
    B, N, d, kk = 2, 12, 8, 3
    q, k, v, g = (rng.standard_normal((B, N, d)) for _ in range(4))
    tq, tk, tv = _leaf(q), _leaf(k), _leaf(v)
    s = torch.matmul(tq, tk.transpose(-1, -2)) / (d ** 0.5)
    s = s.masked_fill(torch.eye(N, dtype=torch.bool), float("-inf"))
    ts, ti = s.topk(kk, dim=-1)
    w = torch.softmax(ts, -1)
    vg = tv.gather(1, ti.reshape(B, N * kk, 1).expand(B, N * kk, d)).view(B, N, kk, d)
    torch.matmul(w.unsqueeze(-2), vg).squeeze(-2).backward(torch.from_numpy(g))
    dq, dk, dv = oracle.gather_attention_grad(q, k, v, ti.numpy(), g)
    np.testing.assert_allclose(dq, tq.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dk, tk.grad.numpy(), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(dv, tv.grad.numpy(), rtol=1e-10, atol=1e-12)
