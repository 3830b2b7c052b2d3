"""GPU parity: fused score-then-select top-k kernels vs the CPU oracle.

All calls go through the C ABI (tarmac_b200.ops -> libtarmac_b200.so).
Bar: retained indices equal to the oracle's (lowest-index tie rule unless
stated) on every row whose k-th and (k+1)-th scores are not within fp32
rounding of each other; outputs within rtol = atol = 1e-5 (fp32) or 2e-2
(bf16) on those rows.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _parity import check_topk, host, qkv, tol_for

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from tarmac_b200 import ops as _ops
    return _ops


# C2 shapes (B reduced from 1024 for the oracle's sake), k in {1, 2, 4}
@pytest.mark.parametrize("N", [32, 64, 128, 256, 384, 512])
@pytest.mark.parametrize("k", [1, 2, 4])
def test_c2_shapes_fp32(ops, N, k):
    q, kt, v = qkv(48, N, 16, seed=1234 + 7 * N + 16)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    check_topk(q, kt, v, k, out, idx=idx)


def test_c1_config(ops):
    q, kt, v = qkv(256, 6, 16, seed=1234 + 7 * 6 + 16)
    out, idx = ops.topk_attention(q, kt, v, 2, return_indices=True)
    check_topk(q, kt, v, 2, out, idx=idx)


@pytest.mark.parametrize("N,d,k", [
    (2, 16, 1), (3, 16, 2), (5, 7, 3), (31, 16, 8), (33, 8, 5), (100, 12, 4),
    (257, 16, 2), (63, 1, 1), (70, 24, 3), (129, 32, 6), (96, 48, 2),
    (200, 64, 4), (50, 100, 3), (40, 128, 8), (1000, 16, 1)])
def test_ragged_shapes(ops, N, d, k):
    q, kt, v = qkv(6, N, d, seed=N * 131 + d * 17 + k)
    out, idx = ops.topk_attention(q, kt, v, k, return_indices=True)
    check_topk(q, kt, v, k, out, idx=idx)


@pytest.mark.parametrize("N,k", [(16, 15), (40, 9), (64, 32), (130, 100),
                                 (512, 64), (1024, 17), (300, 299)])
def test_large_k_resident_rows(ops, N, k):
    q, kt, v = qkv(4, N, 16, seed=N + k)
    out = ops.topk_attention(q, kt, v, k)
    check_topk(q, kt, v, k, out)


def test_k_equals_n_minus_1_is_dense(ops):
    """Keeping every peer reproduces dense attention (test_comm_module.py:33-67)."""
    for N in (3, 6, 12, 24, 200):
        q, kt, v = qkv(8, N, 16, seed=N)
        a = ops.topk_attention(q, kt, v, N - 1)
        b = ops.dense_attention(q, kt, v)
        np.testing.assert_allclose(host(a), host(b), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high"),
                                      ("threshold", "all")])
def test_tie_rules_on_duplicated_keys(ops, golden, mode, tie):
    g = golden("topk_ties")
    q, kt, v = (torch.from_numpy(g[x]).cuda() for x in ("q", "k", "v"))
    for kk in g["ks"]:
        kk = int(kk)
        out = ops.topk_attention(q, kt, v, kk, mode=mode)
        ref, _ = oracle.topk_attention(g["q"], g["k"], g["v"], kk, tie=tie)
        np.testing.assert_allclose(host(out), ref, rtol=1e-5, atol=1e-5)
        # and the reference kernel with that tie rule, directly
        key = {"argmax": "tiled", "sort": "sort", "threshold": "masked"}[mode]
        np.testing.assert_allclose(host(out), g[f"{key}_k{kk}"], rtol=1e-5,
                                   atol=1e-5)


@pytest.mark.parametrize("mode,tie", [("sort", "high"), ("threshold", "all")])
@pytest.mark.parametrize("k", [1, 3, 12])
def test_modes_on_random_rows(ops, mode, tie, k):
    q, kt, v = qkv(8, 96, 16, seed=4321 + k)
    out = ops.topk_attention(q, kt, v, k, mode=mode)
    check_topk(q, kt, v, k, out, tie=tie)


def test_sort_mode_indices_highest_on_ties(ops, golden):
    g = golden("topk_ties")
    q, kt, v = (torch.from_numpy(g[x]).cuda() for x in ("q", "k", "v"))
    s = oracle.scores_f32(g["q"], g["k"])
    for kk in (1, 2, 3, 5):
        _, idx = ops.topk_attention(q, kt, v, kk, mode="sort", return_indices=True)
        np.testing.assert_array_equal(idx.long().cpu().numpy(),
                                      oracle.topk_indices(s, kk, "high"))
        _, idx = ops.topk_attention(q, kt, v, kk, mode="argmax", return_indices=True)
        np.testing.assert_array_equal(idx.long().cpu().numpy(),
                                      oracle.topk_indices(s, kk, "low"))


@pytest.mark.parametrize("N,k", [(512, 1), (512, 2), (768, 4), (1024, 8),
                                 (1500, 2), (2048, 4)])
def test_streaming_large_n(ops, N, k):
    q, kt, v = qkv(4, N, 16, seed=1234 + 7 * N + 16)
    out, idx = ops.streaming_topk_attention(q, kt, v, k, return_indices=True)
    check_topk(q, kt, v, k, out, idx=idx)


@pytest.mark.parametrize("N,d,k,mode,tie", [
    (4096, 16, 2, "argmax", "low"), (3000, 16, 5, "argmax", "low"),
    (512, 128, 2, "argmax", "low"), (700, 100, 3, "sort", "high"),
    (4096, 16, 1, "sort", "high")])
def test_keys_beyond_shared_memory_use_streaming_tiles(ops, N, d, k, mode, tie):
    """Episodes whose keys do not fit the chunked kernel's shared memory run
    on the tiled streaming kernel; same function."""
    q, kt, v = qkv(2, N, d, seed=N + d + k)
    out, idx = ops.topk_attention(q, kt, v, k, mode=mode, return_indices=True)
    check_topk(q, kt, v, k, out, tie=tie, idx=idx)


@pytest.mark.parametrize("k", [1, 2, 3, 4, 5, 6, 7, 8])
@pytest.mark.parametrize("mode,tie", [("argmax", "low"), ("sort", "high")])
def test_every_small_k_and_tie_rule(ops, k, mode, tie):
    q, kt, v = qkv(8, 200, 16, seed=31 * k)
    out, idx = ops.topk_attention(q, kt, v, k, mode=mode, return_indices=True)
    check_topk(q, kt, v, k, out, tie=tie, idx=idx)


@pytest.mark.parametrize("N,d,k", [(512, 16, 1), (512, 16, 2), (1024, 16, 4),
                                   (128, 32, 2), (512, 64, 1)])
def test_bf16_inputs(ops, N, d, k):
    q, kt, v = qkv(8, N, d, seed=99 + N, dtype=torch.bfloat16)
    out, idx = ops.streaming_topk_attention(q, kt, v, k, return_indices=True)
    assert out.dtype == torch.bfloat16
    check_topk(q, kt, v, k, out, idx=idx)


def test_strided_views_no_copy(ops):
    """q, k, v as chunks of one [B, N, 3d] tensor (the comm module's qkv
    output) and a non-multiple-of-4 row stride (scalar load path)."""
    g = torch.Generator().manual_seed(5)
    qkv3 = torch.randn(16, 100, 48, generator=g).cuda()
    q, kt, v = qkv3.chunk(3, dim=-1)
    out, idx = ops.topk_attention(q, kt, v, 3, return_indices=True)
    check_topk(q.contiguous(), kt.contiguous(), v.contiguous(), 3, out, idx=idx)
    odd = torch.randn(8, 64, 51, generator=g).cuda()
    q2, k2, v2 = odd[..., :16], odd[..., 17:33], odd[..., 34:50]
    out2 = ops.topk_attention(q2, k2, v2, 2)
    check_topk(q2.contiguous(), k2.contiguous(), v2.contiguous(), 2, out2)


def test_golden_replay(ops, golden):
    """The kernels on the reference's own fixture inputs vs the reference's
    own outputs (eager path and Triton kernels)."""
    for case in ("topk_c1", "topk_n40", "topk_n64_d32", "topk_n33_d8"):
        g = golden(case)
        q, kt, v = (torch.from_numpy(g[x]).cuda() for x in ("q", "k", "v"))
        for kk in g["ks"]:
            kk = int(kk)
            out = host(ops.topk_attention(q, kt, v, kk))
            np.testing.assert_allclose(out, g[f"eager_k{kk}"], rtol=1e-5, atol=1e-5)
            np.testing.assert_allclose(out, g[f"tiled_k{kk}"], rtol=1e-5, atol=1e-5)
    g = golden("topk_modes")
    q, kt, v = (torch.from_numpy(g[x]).cuda() for x in ("q", "k", "v"))
    for kk in g["ks"]:
        kk = int(kk)
        np.testing.assert_allclose(host(ops.topk_attention(q, kt, v, kk, "threshold")),
                                   g[f"masked_k{kk}"], rtol=1e-5, atol=1e-5)
        np.testing.assert_allclose(host(ops.topk_attention(q, kt, v, kk, "sort")),
                                   g[f"sort_k{kk}"], rtol=1e-5, atol=1e-5)


def test_errors_raise(ops):
    from tarmac_b200 import TarmacError
    q, kt, v = qkv(2, 2000, 16, seed=1)
    with pytest.raises(TarmacError):
        ops.topk_attention(q, kt, v, 20)            # k > 8 needs N <= 1024
    with pytest.raises(TarmacError):
        ops.streaming_topk_attention(q, kt, v, 9)   # streaming k <= 8
    with pytest.raises(TarmacError):
        ops.topk_attention(q, kt, v, 2000)          # k > N - 1
    q, kt, v = qkv(2, 50, 16, seed=1)
    with pytest.raises(TarmacError):
        ops.topk_attention(q, kt, v, 3, "threshold", return_indices=True)
