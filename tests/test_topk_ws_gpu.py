"""GPU parity: the persistent warp-specialized top-k kernel (csrc/topk_ws.cu).

It serves fp32 batches of at least 296 episodes (two per SM) of 352 to 512
agents with d in {8, 16} and k <= 2, and bf16 batches of at least 148 (one
per SM) of 320 to 512 agents with d a multiple of 8 from 24 to 64 and
k <= 4. Two checks per case, through the C ABI:

* a seeded sample of episodes against the CPU oracle (the bar of every
  top-k test: indices equal on unambiguous rows, outputs within rtol = atol
  = 1e-5 fp32 / 2e-2 bf16);
* bit equality with the per-block tensor-core kernel (csrc/topk_tc.cu): the
  same episodes called in a batch below the persistent kernel's threshold
  take that kernel, and both form every score with the same products.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _parity import check_topk, qkv

pytestmark = pytest.mark.gpu

B_WS = 600          # >= 4 episodes per SM on a 148-SM B200


@pytest.fixture(scope="module")
def ops():
    from tarmac_b200 import ops as _ops
    return _ops


def _sample(B, seed, n=12):
    rng = np.random.default_rng(seed)
    return torch.from_numpy(np.sort(rng.choice(B, size=n, replace=False))).cuda()


def _check(ops, q, k, v, kk, mode="argmax", tie="low"):
    out, idx = ops.topk_attention(q, k, v, kk, mode=mode, return_indices=True)
    sel = _sample(q.shape[0], q.shape[1] * 7 + kk)
    qs, ks, vs, os_, is_ = (t.index_select(0, sel) for t in (q, k, v, out, idx))
    check_topk(qs, ks, vs, kk, os_, tie=tie, idx=is_)
    # the first 8 episodes alone run the per-block kernel: same bits
    o8, i8 = ops.topk_attention(q[:8], k[:8], v[:8], kk, mode=mode,
                                return_indices=True)
    assert torch.equal(o8, out[:8])
    assert torch.equal(i8, idx[:8])


@pytest.mark.parametrize("N", [352, 384, 385, 448, 500, 512])
@pytest.mark.parametrize("k", [1, 2])
def test_fp32_episode_sizes(ops, N, k):
    q, kt, v = qkv(B_WS, N, 16, seed=N + k)
    _check(ops, q, kt, v, k)


@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high")])
def test_fp32_d8_and_tie_rules(ops, mode, tie):
    q, kt, v = qkv(B_WS, 470, 8, seed=8)
    _check(ops, q, kt, v, 2, mode=mode, tie=tie)


@pytest.mark.parametrize("d", [24, 32, 40, 64])
@pytest.mark.parametrize("k", [1, 2])
def test_bf16_widths(ops, d, k):
    q, kt, v = qkv(B_WS, 512, d, seed=d + k, dtype=torch.bfloat16)
    _check(ops, q, kt, v, k)


@pytest.mark.parametrize("N,d,k", [(401, 32, 3), (512, 24, 4), (450, 48, 2)])
def test_bf16_ragged_and_k4(ops, N, d, k):
    q, kt, v = qkv(B_WS, N, d, seed=N + d, dtype=torch.bfloat16)
    _check(ops, q, kt, v, k, mode="sort", tie="high")


def test_strided_views_and_streaming_entry(ops):
    """q, k, v as column slices of one packed [B, N, 3d] tensor (row stride
    3d), and the streaming entry point, which dispatches the same way."""
    base = qkv(B_WS, 512, 48, seed=5)[0]
    q, kt, v = base[..., :16], base[..., 16:32], base[..., 32:]
    _check(ops, q, kt, v, 2)
    a = ops.streaming_topk_attention(q, kt, v, 2)
    b = ops.topk_attention(q, kt, v, 2)
    assert torch.equal(a, b)


@pytest.mark.parametrize("B,N,d,k", [(148, 320, 32, 2), (150, 333, 64, 1),
                                     (300, 384, 24, 4), (296, 512, 64, 2)])
def test_bf16_small_batches_and_three_query_tiles(ops, B, N, d, k):
    """Batches from one episode per SM and episodes of three query tiles
    (320-384 agents) take the persistent kernel as well."""
    q, kt, v = qkv(B, N, d, seed=B + N + d, dtype=torch.bfloat16)
    _check(ops, q, kt, v, k)


def test_fp32_two_episodes_per_sm(ops):
    q, kt, v = qkv(296, 360, 16, seed=296)
    _check(ops, q, kt, v, 2)
