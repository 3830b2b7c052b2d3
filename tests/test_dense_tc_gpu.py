"""GPU parity: the tensor-core (tcgen05) bf16 dense attention kernel vs the
CPU oracle.

bf16 episodes of 128 or more agents run Q K^T and P V on the tensor cores
(bf16 operands, fp32 accumulation in tensor memory, bf16 softmax weights as
in the reference's `tl.dot(p.to(v.dtype), v)`). Bar: outputs within 2e-2
(bf16) of the oracle's float64 softmax over the same bf16 inputs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _parity import BF16_TOL, host, qkv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from tarmac_b200 import ops as _ops
    return _ops


def bf16(B, N, d, seed):
    return qkv(B, N, d, seed, dtype=torch.bfloat16)


def check(ops, q, k, v, **tol):
    out = ops.dense_attention(q, k, v)
    assert out.dtype == torch.bfloat16
    ref = oracle.dense_attention(host(q), host(k), host(v))
    np.testing.assert_allclose(host(out), ref, **(tol or BF16_TOL))
    return out


@pytest.mark.parametrize("N", [128, 129, 200, 256, 300, 512, 1000, 2048])
def test_dense_tc_episode_sizes(ops, N):
    q, k, v = bf16(6 if N < 1000 else 2, N, 16, seed=1234 + 7 * N + 16)
    check(ops, q, k, v)


@pytest.mark.parametrize("d", [1, 8, 12, 16, 24, 32, 48, 64, 100, 128])
def test_dense_tc_head_dims(ops, d):
    for N in (256, 512):
        q, k, v = bf16(4, N, d, seed=d * 31 + N)
        check(ops, q, k, v)


def test_dense_tc_large_scores_move_the_reference(ops):
    """Scores of magnitude ~100 in random key order: the reference maximum
    moves across tiles and the accumulator in tensor memory is rescaled."""
    q, k, v = bf16(4, 512, 16, seed=3)
    q = (q.float() * 40.0).to(torch.bfloat16)
    out = check(ops, q, k, v)
    assert torch.isfinite(out.float()).all()
    # keys sorted so each tile's best score beats the previous tiles'
    g = torch.Generator().manual_seed(4)
    base = torch.randn(2, 1, 16, generator=g)
    ramp = torch.linspace(0.1, 6.0, 384).view(1, 384, 1)
    kt = (base * ramp).to(torch.bfloat16).cuda()
    qt = (base.expand(2, 384, 16) * 3.0).to(torch.bfloat16).cuda()
    vt = torch.randn(2, 384, 16, generator=g).to(torch.bfloat16).cuda()
    check(ops, qt, kt, vt)


def test_dense_tc_strided_and_misaligned_views(ops):
    g = torch.Generator().manual_seed(9)
    qkv3 = torch.randn(4, 256, 192, generator=g).to(torch.bfloat16).cuda()
    q, k, v = qkv3.chunk(3, dim=-1)
    out = ops.dense_attention(q, k, v)
    ref = oracle.dense_attention(host(q), host(k), host(v))
    np.testing.assert_allclose(host(out), ref, **BF16_TOL)
    odd = torch.randn(4, 200, 53, generator=g).to(torch.bfloat16).cuda()
    q2, k2, v2 = odd[..., 1:17], odd[..., 18:34], odd[..., 35:51]
    out2 = ops.dense_attention(q2, k2, v2)
    ref2 = oracle.dense_attention(host(q2), host(k2), host(v2))
    np.testing.assert_allclose(host(out2), ref2, **BF16_TOL)


def test_dense_tc_large_batch(ops):
    q, k, v = bf16(600, 128, 16, seed=17)
    check(ops, q, k, v)


def test_dense_tc_matches_topk_with_all_peers(ops):
    """k = N - 1 keeps every peer: the top-k kernel's softmax over all
    retained scores equals dense attention (test_comm_module.py:33-67)."""
    q, k, v = bf16(4, 200, 16, seed=21)
    a = ops.dense_attention(q, k, v)
    b = ops.topk_attention(q.float(), k.float(), v.float(), 199)
    np.testing.assert_allclose(host(a), host(b), **BF16_TOL)
