"""GPU parity: fp32 dense attention on the tensor cores vs the CPU oracle.

fp32 episodes of 96 or more agents with d in {8, 16} and 16-byte aligned
rows run Q K^T and P V on the tensor cores with every operand (Q, K, V and
the softmax weights P) split exactly into three bf16 planes and six plane
products per product, an fp32-accurate result; other fp32 shapes run the
FFMA kernel. Bar: rtol = atol = 1e-5 against the oracle's float64 softmax
over the fp32 inputs (the fp32 parity tolerance).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _parity import FP32_TOL, host, qkv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from tarmac_b200 import ops as _ops
    return _ops


def check(ops, q, k, v, **tol):
    out = ops.dense_attention(q, k, v)
    assert out.dtype == torch.float32
    ref = oracle.dense_attention(host(q), host(k), host(v))
    np.testing.assert_allclose(host(out), ref, **(tol or FP32_TOL))
    return out


@pytest.mark.parametrize("N", [128, 129, 192, 200, 256, 333, 512, 640, 1000,
                               1024])
@pytest.mark.parametrize("d", [8, 16])
def test_f32_dense_tc_episode_sizes(ops, N, d):
    q, k, v = qkv(6, N, d, seed=1234 + 7 * N + d)
    check(ops, q, k, v)


def test_f32_dense_tc_large_batch(ops):
    """Many episodes per launch (grid well beyond one wave)."""
    q, k, v = qkv(400, 256, 16, seed=5)
    check(ops, q, k, v)


def test_f32_dense_tc_strided_views(ops):
    """q, k, v as views of one [B, N, 3d] tensor (row stride 48 floats): the
    split path reads them in place."""
    g = torch.Generator().manual_seed(8)
    qkv3 = torch.randn(6, 300, 48, generator=g).cuda()
    q, k, v = qkv3.chunk(3, dim=-1)
    out = ops.dense_attention(q, k, v)
    ref = oracle.dense_attention(host(q.contiguous()), host(k.contiguous()),
                                 host(v.contiguous()))
    np.testing.assert_allclose(host(out), ref, **FP32_TOL)


def test_f32_dense_tc_large_scores(ops):
    """Scores of magnitude ~100: the base-2 online softmax moves its
    reference maximum many times (each move rescales the accumulator in
    tensor memory); any fp32 evaluation of a score carries an error up to
    about (d+2) u sum|q_c k_c| scale, so the tolerance adds that bound times
    max|v| to the usual 1e-5."""
    q, k, v = qkv(2, 300, 16, seed=3)
    q = q * 40.0
    out = ops.dense_attention(q, k, v)
    qn, kn, vn = host(q), host(k), host(v)
    ref = oracle.dense_attention(qn, kn, vn)
    assert torch.isfinite(out).all()
    mag = np.einsum("bid,bjd->bij", np.abs(qn), np.abs(kn)).max() / 4.0
    ds = 2 * 18 * 2.0 ** -24 * mag
    atol = 1e-5 + 2 * ds * np.abs(vn).max()
    np.testing.assert_allclose(host(out), ref, rtol=1e-5, atol=atol)


def test_f32_dense_tc_matches_ffma_kernel(ops):
    """The split tensor-core kernel and the FFMA kernel (taken for rows off
    the 16-byte grid) agree to fp32 accuracy."""
    q, k, v = qkv(8, 512, 16, seed=9)
    a = ops.dense_attention(q, k, v)
    flat = [torch.empty(x.numel() + 1, device=x.device) for x in (q, k, v)]
    qo, ko, vo = (f[1:].view(x.shape) for f, x in zip(flat, (q, k, v)))
    for dst, src in zip((qo, ko, vo), (q, k, v)):
        dst.copy_(src)
    b = ops.dense_attention(qo, ko, vo)
    np.testing.assert_allclose(host(a), host(b), rtol=1e-5, atol=1e-5)


def test_f32_dense_tc_zero_and_tiny_rows(ops):
    """A zero query row gives the plain mean of the other V rows; a tiny K
    row (|k| ~ 1e-30) scores ~0 without breaking the split."""
    q, k, v = qkv(2, 256, 16, seed=21)
    q[:, 3] = 0.0
    k[:, 7] *= 1e-30
    out = check(ops, q, k, v)
    vm = (v[:, :, :].sum(1) - v[:, 3]) / 255.0
    np.testing.assert_allclose(host(out[:, 3]), host(vm), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("N,d,dtype", [(96, 16, torch.float32),
                                       (100, 8, torch.float32),
                                       (127, 16, torch.float32),
                                       (65, 16, torch.bfloat16),
                                       (100, 64, torch.bfloat16),
                                       (127, 32, torch.bfloat16)])
def test_dense_tc_part_filled_tile_below_128(ops, N, d, dtype):
    """Dense episodes below 128 agents on one part-filled 128-row tile (bf16
    from 65 agents, fp32 from 96): query rows and keys past N are masked."""
    from _parity import tol_for
    q, k, v = qkv(12, N, d, seed=5 * N + d, dtype=dtype)
    out = ops.dense_attention(q, k, v)
    assert out.dtype == dtype
    ref = oracle.dense_attention(host(q), host(k), host(v))
    np.testing.assert_allclose(host(out), ref, **tol_for(dtype))
