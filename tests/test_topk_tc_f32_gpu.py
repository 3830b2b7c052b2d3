"""GPU parity: fp32 top-k on the tensor cores (three exact bf16 planes per
operand, six plane products per score) vs the CPU oracle.

fp32 episodes of 128 or more agents (from 65 for k <= 4, from 96 for k <= 8)
with d a multiple of 8 up to 16, k <= 8 and 16-byte aligned rows form their
scores this way; other fp32 problems run the FFMA kernels. Same bar as every fp32 top-k kernel: retained indices
equal to the oracle's on every row whose k-th and (k+1)-th exact scores are
not within fp32 rounding of each other (oracle.ambiguous_rows), outputs
within rtol = atol = 1e-5.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _parity import FP32_TOL, check_topk, host, qkv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from tarmac_b200 import ops as _ops
    return _ops


def _offset_copy(x: torch.Tensor) -> torch.Tensor:
    """The same values in a buffer whose base is 4 bytes off the 16-byte grid
    (the fp32 FFMA kernels take such rows; the split path needs 16-byte
    rows)."""
    flat = torch.empty(x.numel() + 1, dtype=x.dtype, device=x.device)
    y = flat[1:].view(x.shape)
    y.copy_(x)
    return y


@pytest.mark.parametrize("N", [128, 129, 192, 200, 256, 333, 384, 512, 640,
                               1000, 1024])
@pytest.mark.parametrize("k", [1, 2, 4, 8])
def test_f32_tc_episode_sizes(ops, N, k):
    q, kt, v = qkv(8, N, 16, seed=11 * N + k)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    assert out.dtype == torch.float32
    check_topk(q, kt, v, k, out, idx=idx)


@pytest.mark.parametrize("d", [8, 16])
@pytest.mark.parametrize("N,k", [(256, 3), (512, 2), (300, 5)])
def test_f32_tc_head_dims(ops, d, N, k):
    q, kt, v = qkv(6, N, d, seed=d * 31 + N + k)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    check_topk(q, kt, v, k, out, idx=idx)


@pytest.mark.parametrize("k", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high")])
def test_f32_tc_every_small_k_and_tie_rule(ops, k, mode, tie):
    q, kt, v = qkv(8, 300, 16, seed=193 * k)
    out, idx = ops.topk_attention(q, kt, v, k, mode=mode, return_indices=True)
    check_topk(q, kt, v, k, out, tie=tie, idx=idx)


@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high")])
def test_f32_tc_duplicated_keys_follow_the_tie_rule(ops, mode, tie):
    """Every key appears several times, so each score row is made of exact
    ties (equal keys give bit-equal tensor-core scores); the retained indices
    must follow the mode's tie rule exactly."""
    g = torch.Generator().manual_seed(12)
    B, N, d = 4, 320, 16
    base = torch.randn(B, 40, d, generator=g)
    perm = torch.randint(0, 40, (N,), generator=g)
    kt = base[:, perm].contiguous()
    q = torch.randn(B, N, d, generator=g)
    v = torch.randn(B, N, d, generator=g)
    qn, kn = host(q), host(kt)
    s = oracle.scores_f32(qn, kn)
    for kk in (1, 2, 3, 5, 8):
        out, idx = ops.topk_attention(q.cuda(), kt.cuda(), v.cuda(), kk,
                                      mode=mode, return_indices=True)
        want = oracle.topk_indices(s, kk, tie)
        np.testing.assert_array_equal(np.sort(idx.long().cpu().numpy(), -1),
                                      np.sort(want, -1))
        ref, _ = oracle.topk_attention(qn, kn, host(v), kk, tie=tie)
        np.testing.assert_allclose(host(out), ref, **FP32_TOL)


@pytest.mark.parametrize("kk", [1, 2, 4])
def test_f32_tc_near_ties_resolved_within_the_fp32_bound(ops, kk):
    """Keys come in groups of kk + 1 near-equal rows (base + 2e-5 z), so the
    k-th and (k+1)-th best scores of a row usually sit a few fp32 ulps
    apart. Wherever their exact gap exceeds the fp32 dot-product rounding
    bound the kernel must still order them as exact arithmetic does: the
    split-plane scores carry an error of the size of an fp32 FFMA dot
    product's."""
    g = torch.Generator().manual_seed(2024 + kk)
    G = kk + 1
    B, N, d = 16, 510, 16
    q = torch.randn(B, N, d, generator=g)
    base = torch.randn(B, N // G, 1, d, generator=g)
    near = base + 2e-5 * torch.randn(B, N // G, G, d, generator=g)
    kt = near.reshape(B, N, d).contiguous()
    v = torch.randn(B, N, d, generator=g)
    out, idx = ops.topk_attention(q.cuda(), kt.cuda(), v.cuda(), kk,
                                  return_indices=True)
    amb = oracle.ambiguous_rows(host(q), host(kt), kk)
    # a real stress: many rows near the bound, most of them decided
    assert 0.05 < amb.mean() < 0.8, amb.mean()
    check_topk(q, kt, v, kk, out, idx=idx, max_amb_frac=1.0)


def test_f32_tc_matches_ffma_kernel_on_clean_rows(ops):
    """The split tensor-core path and the fp32 FFMA kernel (taken for rows
    off the 16-byte grid) agree wherever no near tie exists."""
    q, kt, v = qkv(16, 512, 16, seed=6)
    a, ia = ops.topk_attention(q, kt, v, 2, return_indices=True)
    qo, ko, vo = (_offset_copy(x) for x in (q, kt, v))
    b, ib = ops.topk_attention(qo, ko, vo, 2, return_indices=True)
    ok = ~oracle.ambiguous_rows(host(q), host(kt), 2)
    np.testing.assert_array_equal(ia.cpu().numpy()[ok], ib.cpu().numpy()[ok])
    np.testing.assert_allclose(host(a)[ok], host(b)[ok], **FP32_TOL)


def test_f32_tc_strided_views(ops):
    """q, k, v as views of one [B, N, 3d] tensor (the comm module's
    qkv.chunk(3, -1): row stride 48 floats, 16-byte aligned pieces) run the
    split path without a copy; a 4-byte offset view runs the FFMA kernel."""
    g = torch.Generator().manual_seed(4)
    qkv3 = torch.randn(8, 256, 48, generator=g).cuda()
    q, kt, v = qkv3.chunk(3, dim=-1)
    out, idx = ops.topk_attention(q, kt, v, 4, return_indices=True)
    check_topk(q.contiguous(), kt.contiguous(), v.contiguous(), 4, out,
               idx=idx)
    odd = torch.randn(8, 200, 53, generator=g).cuda()
    q2, k2, v2 = odd[..., 1:17], odd[..., 18:34], odd[..., 35:51]
    out2, idx2 = ops.topk_attention(q2, k2, v2, 2, return_indices=True)
    check_topk(q2.contiguous(), k2.contiguous(), v2.contiguous(), 2, out2,
               idx=idx2)


def test_f32_tc_large_batch(ops):
    """Many episodes per launch (grid well beyond one wave of 148 SMs)."""
    q, kt, v = qkv(600, 256, 16, seed=78)
    out, idx = ops.topk_attention(q, kt, v, 2, return_indices=True)
    check_topk(q, kt, v, 2, out, idx=idx)


@pytest.mark.parametrize("N,k", [(2000, 8), (4096, 2)])
def test_f32_tc_large_n_both_entry_points(ops, N, k):
    """Episodes far beyond one round stream K through the ring; the fused and
    the streaming entry points share the kernel."""
    q, kt, v = qkv(2, N, 16, seed=N + 5 * k)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    check_topk(q, kt, v, k, out, idx=idx)
    out2, idx2 = ops.streaming_topk_attention(q, kt, v, k, return_indices=True)
    np.testing.assert_array_equal(idx2.cpu().numpy(), idx.cpu().numpy())
    np.testing.assert_array_equal(host(out2), host(out))


def test_f32_tc_special_rows(ops):
    """A zero query row scores every key 0 (all ties: the lowest indices
    win); large-magnitude rows (|x| ~ 1e30) keep their order."""
    q, kt, v = qkv(4, 256, 16, seed=99)
    q[:, 5] = 0.0
    q[:, 7] *= 1e30
    kt[:, 9] *= 1e-30
    out, idx = ops.topk_attention(q, kt, v, 3, return_indices=True)
    got = idx.long().cpu().numpy()
    np.testing.assert_array_equal(got[:, 5], np.tile([0, 1, 2], (4, 1)))
    check_topk(q, kt, v, 3, out, idx=idx)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("N,k", [(65, 1), (65, 4), (72, 2), (95, 3), (96, 5),
                                 (100, 8), (112, 2), (127, 4), (127, 7)])
@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high")])
def test_part_filled_tile_below_128(ops, dtype, N, k, mode, tie):
    """Episodes of 65-127 agents run one part-filled 128-row tile (k <= 4
    from 65 agents, k <= 8 from 96): query rows and keys past N are masked."""
    q, kt, v = qkv(20, N, 16, seed=3 * N + k, dtype=dtype)
    out, idx = ops.topk_attention(q, kt, v, k, mode=mode, return_indices=True)
    check_topk(q, kt, v, k, out, tie=tie, idx=idx)
