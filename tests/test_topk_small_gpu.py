"""GPU parity: the short-episode top-k kernel (csrc/topk_small.cu: d <= 16,
k <= 8, episodes the tensor-core kernel does not take — up to 64 agents, up
to 95 for k > 4, and up to 128 when d is not a multiple of 8 or rows are off
the 16-byte grid; two lanes per query row up to 64 agents, else one) vs the
CPU oracle, through the C ABI. Episodes of 65-127 agents in these tests that
the tensor-core kernel takes check its part-filled tile as well.

Bar as for every top-k kernel: retained indices equal to the oracle's on
every row whose k-th and (k+1)-th scores are not within fp32 rounding of
each other; outputs within rtol = atol = 1e-5 (fp32) or 2e-2 (bf16) there.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _parity import check_topk, host, qkv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from tarmac_b200 import ops as _ops
    return _ops


# episode sizes at the warps-per-episode edges (1 warp to 32 agents, 2 to
# 64, 4 to 127) and batch sizes that leave the last block part empty
@pytest.mark.parametrize("B", [1, 3, 5, 7])
@pytest.mark.parametrize("N", [2, 17, 32, 33, 64, 65, 127])
def test_episode_edges_and_partial_blocks(ops, B, N):
    k = min(2, N - 1)
    q, kt, v = qkv(B, N, 16, seed=100 * B + N)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    check_topk(q, kt, v, k, out, idx=idx)


@pytest.mark.parametrize("k", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high")])
def test_every_k_and_tie_rule(ops, k, mode, tie):
    q, kt, v = qkv(40, 50, 16, seed=7 * k + len(mode))
    out, idx = ops.topk_attention(q, kt, v, k, mode=mode, return_indices=True)
    check_topk(q, kt, v, k, out, tie=tie, idx=idx)


@pytest.mark.parametrize("N,d,k", [(20, 7, 3), (60, 12, 2), (45, 1, 1),
                                   (100, 8, 4), (9, 16, 8), (127, 5, 6),
                                   (80, 16, 6), (127, 12, 2), (90, 16, 8)])
def test_widths_below_16(ops, N, d, k):
    """d < 16: columns past d are zero in shared memory; d not a multiple
    of 4 takes the 4-byte path. (80, 16, 6), (90, 16, 8) and (127, 12, 2)
    reach the one-lane-per-row form above 64 agents."""
    q, kt, v = qkv(12, N, d, seed=N * 3 + d)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    check_topk(q, kt, v, k, out, idx=idx)


@pytest.mark.parametrize("N,d,k", [(128, 12, 3), (128, 5, 8), (128, 1, 1),
                                   (128, 16, 2)])
@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high")])
def test_full_128_agent_episode(ops, N, d, k, mode, tie):
    """N = 128, the kernel's largest episode (four warps, one lane per row,
    every lane of the block busy): widths the tensor-core kernel declines
    (d not a multiple of 8), and d = 16 reached through a row stride off the
    16-byte grid, under both tie rules."""
    if d == 16:
        base = qkv(10, N, d + 1, seed=N + d + k)
        q, kt, v = (x[..., :d] for x in base)        # row stride 17 floats
    else:
        q, kt, v = qkv(10, N, d, seed=N + d + k)
    out, idx = ops.topk_attention(q, kt, v, k, mode=mode, return_indices=True)
    check_topk(q, kt, v, k, out, tie=tie, idx=idx)


@pytest.mark.parametrize("N,k", [(32, 1), (64, 2), (100, 4), (48, 8)])
def test_bf16(ops, N, k):
    q, kt, v = qkv(24, N, 16, seed=N + k, dtype=torch.bfloat16)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    assert out.dtype == torch.bfloat16
    check_topk(q, kt, v, k, out, idx=idx)


def test_unaligned_rows_and_strided_views(ops):
    """q, k, v as chunk views of one [B, N, 48] tensor (row stride 48) and
    as views one element off the 16-byte grid: same results."""
    g = torch.Generator().manual_seed(5)
    base = torch.randn(9, 70, 48, generator=g).cuda()
    q, kt, v = base.chunk(3, dim=-1)
    out = ops.topk_attention(q, kt, v, 3)
    check_topk(q.contiguous(), kt.contiguous(), v.contiguous(), 3, out)
    flat = [torch.empty(x.numel() + 1, device="cuda") for x in (q, kt, v)]
    qo, ko, vo = (f[1:].view(x.shape) for f, x in zip(flat, (q, kt, v)))
    for dst, src in zip((qo, ko, vo), (q, kt, v)):
        dst.copy_(src)
    out2 = ops.topk_attention(qo, ko, vo, 3)
    np.testing.assert_allclose(host(out2), host(out), rtol=1e-6, atol=1e-6)


def test_tie_rules_on_duplicated_keys(ops, golden):
    """The reference's tie fixture (episodes of 16 agents with duplicated
    keys) through the short-episode kernel, both tie rules; with the lowest
    index rule and k a power of two the indices equal the reference
    streaming kernel's own."""
    g = golden("topk_ties")
    q, kt, v = (torch.from_numpy(g[x]).cuda() for x in ("q", "k", "v"))
    assert q.shape[1] < 128
    s = oracle.scores_f32(g["q"], g["k"])
    for kk in (1, 2, 3, 5):
        for mode, tie, key in (("argmax", "low", "tiled"), ("sort", "high", "sort")):
            out, idx = ops.topk_attention(q, kt, v, kk, mode=mode,
                                          return_indices=True)
            np.testing.assert_array_equal(idx.long().cpu().numpy(),
                                          oracle.topk_indices(s, kk, tie))
            np.testing.assert_allclose(host(out), g[f"{key}_k{kk}"],
                                       rtol=1e-5, atol=1e-5)
            # the reference streaming kernel is defined for k a power of
            # two only (other k carry a padding word in its buffer)
            if mode == "argmax" and kk & (kk - 1) == 0:
                np.testing.assert_array_equal(idx.long().cpu().numpy(),
                                              g[f"stream_idx_k{kk}"])


def test_streaming_entry_point_same_result(ops):
    q, kt, v = qkv(16, 90, 16, seed=11)
    a = ops.topk_attention(q, kt, v, 4)
    b = ops.streaming_topk_attention(q, kt, v, 4)
    assert torch.equal(a, b)
