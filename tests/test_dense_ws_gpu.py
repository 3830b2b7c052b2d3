"""GPU parity: the persistent warp-specialized dense kernel (csrc/dense_ws.cu).

It serves bf16 batches of at least 592 episodes (four per SM) of 320 to 512
agents with d a multiple of 8 up to 64. Two checks per case, through the
C ABI:

* a seeded sample of episodes against the CPU oracle's float64 softmax over
  the same bf16 inputs (bf16 tolerance, 2e-2);
* bit equality with the per-block tensor-core dense kernel (csrc/dense_tc.cu):
  the same episodes called in a batch below the persistent kernel's
  threshold take that kernel, and both run the same tiles, products and
  online-softmax steps in the same order.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _parity import BF16_TOL, host, qkv

pytestmark = pytest.mark.gpu

B_WS = 600


@pytest.fixture(scope="module")
def ops():
    from tarmac_b200 import ops as _ops
    return _ops


def _check(ops, q, k, v):
    out = ops.dense_attention(q, k, v)
    assert out.dtype == torch.bfloat16
    rng = np.random.default_rng(q.shape[1] + q.shape[2])
    sel = torch.from_numpy(np.sort(rng.choice(q.shape[0], size=10, replace=False))).cuda()
    qs, ks, vs, os_ = (t.index_select(0, sel) for t in (q, k, v, out))
    ref = oracle.dense_attention(host(qs), host(ks), host(vs))
    np.testing.assert_allclose(host(os_), ref, **BF16_TOL)
    head = ops.dense_attention(q[:8], k[:8], v[:8])
    assert torch.equal(head, out[:8])


@pytest.mark.parametrize("N", [320, 384, 385, 448, 512])
@pytest.mark.parametrize("d", [16, 32, 64])
def test_episode_sizes_and_widths(ops, N, d):
    q, kt, v = qkv(B_WS, N, d, seed=N * 3 + d, dtype=torch.bfloat16)
    _check(ops, q, kt, v)


@pytest.mark.parametrize("d", [8, 24, 32, 40])
def test_other_widths(ops, d):
    q, kt, v = qkv(B_WS, 500, d, seed=d, dtype=torch.bfloat16)
    _check(ops, q, kt, v)


def test_large_scores_rescale_the_accumulator(ops):
    """Scores of magnitude ~100: the reference maximum moves across tiles and
    the output accumulator in tensor memory is rescaled."""
    q, kt, v = qkv(B_WS, 512, 32, seed=11, dtype=torch.bfloat16)
    q = (q.float() * 30.0).to(torch.bfloat16)
    out = ops.dense_attention(q, kt, v)
    assert torch.isfinite(out.float()).all()
    _check(ops, q, kt, v)


def test_strided_views(ops):
    base = qkv(B_WS, 512, 96, seed=4, dtype=torch.bfloat16)[0]
    q, kt, v = base[..., :32], base[..., 32:64], base[..., 64:]
    _check(ops, q, kt, v)
