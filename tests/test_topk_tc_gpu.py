"""GPU parity: the tensor-core (tcgen05) bf16 top-k kernel vs the CPU oracle.

bf16 episodes of 128 or more agents with k <= 8 (argmax or sort mode, fused
or streaming entry point) form their scores on the tensor cores, 128 keys per
round: bf16 x bf16 products accumulated in fp32 in tensor memory. Same bar as every top-k kernel: retained indices equal
to the oracle's on every unambiguous row, outputs within 2e-2 (bf16).
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


def bf16(B, N, d, seed):
    return qkv(B, N, d, seed, dtype=torch.bfloat16)


@pytest.mark.parametrize("N", [128, 130, 200, 256, 300, 384, 500, 512])
@pytest.mark.parametrize("k", [1, 2, 4, 8])
def test_tc_episode_sizes(ops, N, k):
    q, kt, v = bf16(12, N, 16, seed=7 * N + k)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    assert out.dtype == torch.bfloat16
    check_topk(q, kt, v, k, out, idx=idx)


@pytest.mark.parametrize("d", [1, 8, 12, 16, 24, 32, 48, 64, 100, 128])
def test_tc_head_dims(ops, d):
    for N, k in ((256, 3), (512, 2)):
        q, kt, v = bf16(6, N, d, seed=d * 13 + N)
        out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
        check_topk(q, kt, v, k, out, idx=idx)


@pytest.mark.parametrize("k", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high")])
def test_tc_every_small_k_and_tie_rule(ops, k, mode, tie):
    q, kt, v = bf16(8, 300, 32, seed=97 * k)
    out, idx = ops.topk_attention(q, kt, v, k, mode=mode, return_indices=True)
    check_topk(q, kt, v, k, out, tie=tie, idx=idx)


@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high")])
def test_tc_duplicated_keys_follow_the_tie_rule(ops, mode, tie):
    """Every key appears several times, so each score row is made of exact
    ties; the retained indices must follow the mode's tie rule exactly."""
    g = torch.Generator().manual_seed(11)
    B, N, d = 4, 320, 16
    base = torch.randn(B, 40, d, generator=g).to(torch.bfloat16)
    perm = torch.randint(0, 40, (N,), generator=g)
    kt = base[:, perm].contiguous()
    q = torch.randn(B, N, d, generator=g).to(torch.bfloat16)
    v = torch.randn(B, N, d, generator=g).to(torch.bfloat16)
    qn, kn = host(q), host(kt)
    s = oracle.scores_f64(qn, kn).astype(np.float32)
    for kk in (1, 2, 3, 5, 8):
        out, idx = ops.topk_attention(q.cuda(), kt.cuda(), v.cuda(), kk,
                                      mode=mode, return_indices=True)
        want = oracle.topk_indices(s, kk, tie)
        np.testing.assert_array_equal(np.sort(idx.long().cpu().numpy(), -1),
                                      np.sort(want, -1))
        ref, _ = oracle.topk_attention(qn, kn, host(v), kk, tie=tie)
        np.testing.assert_allclose(host(out), ref, rtol=2e-2, atol=2e-2)


def test_tc_strided_and_misaligned_views(ops):
    """Views of one [B, N, 3d] tensor (16-byte staging copies), an odd row
    stride and a base address off the 16-byte grid (element staging)."""
    g = torch.Generator().manual_seed(3)
    qkv3 = torch.randn(8, 256, 96, generator=g).to(torch.bfloat16).cuda()
    q, kt, v = qkv3.chunk(3, dim=-1)
    out, idx = ops.topk_attention(q, kt, v, 4, return_indices=True)
    check_topk(q.contiguous(), kt.contiguous(), v.contiguous(), 4, out, idx=idx)
    odd = torch.randn(8, 200, 53, generator=g).to(torch.bfloat16).cuda()
    q2, k2, v2 = odd[..., 1:17], odd[..., 18:34], odd[..., 35:51]
    out2, idx2 = ops.topk_attention(q2, k2, v2, 2, return_indices=True)
    check_topk(q2.contiguous(), k2.contiguous(), v2.contiguous(), 2, out2,
               idx=idx2)


def test_tc_matches_ffma_kernel_on_clean_rows(ops):
    """The tensor-core path and the fp32 FFMA path agree on the inputs the
    two share (bf16 values widened to fp32) wherever no near tie exists."""
    q, kt, v = bf16(16, 512, 16, seed=5)
    a, ia = ops.topk_attention(q, kt, v, 2, return_indices=True)
    b, ib = ops.topk_attention(q.float(), kt.float(), v.float(), 2,
                               return_indices=True)
    amb = oracle.ambiguous_rows(host(q), host(kt), 2)
    ok = ~amb
    np.testing.assert_array_equal(ia.cpu().numpy()[ok], ib.cpu().numpy()[ok])
    np.testing.assert_allclose(host(a)[ok], host(b)[ok], rtol=2e-2, atol=2e-2)


def test_tc_large_batch(ops):
    """Many episodes per launch (grid well beyond one wave of 148 SMs)."""
    q, kt, v = bf16(600, 256, 16, seed=77)
    out, idx = ops.topk_attention(q, kt, v, 2, return_indices=True)
    check_topk(q, kt, v, 2, out, idx=idx)


@pytest.mark.parametrize("N,k", [(640, 2), (1024, 1), (1024, 4), (2000, 8),
                                 (4096, 2)])
def test_tc_large_n_both_entry_points(ops, N, k):
    """Episodes beyond one 128-key round stream K through the ring; the
    fused and the streaming entry points share the kernel."""
    q, kt, v = bf16(3, N, 16, seed=N + 3 * k)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    check_topk(q, kt, v, k, out, idx=idx)
    out2, idx2 = ops.streaming_topk_attention(q, kt, v, k, return_indices=True)
    np.testing.assert_array_equal(idx2.cpu().numpy(), idx.cpu().numpy())
    np.testing.assert_array_equal(host(out2), host(out))
