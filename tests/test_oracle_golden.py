"""Pin the CPU oracle to the reference's own outputs (golden vectors).

The fixtures in tests/golden were produced by running the unmodified
reference (eager PyTorch functions and its Triton kernels under Triton's CPU
interpreter) — see tests/golden/make_golden.py. Tolerances: outputs within
rtol = atol = 1e-5 (fp32), retained indices and Morton codes bit-exact.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle

RTOL = ATOL = 1e-5

TOPK_CASES = ["topk_c1", "topk_n40", "topk_n64_d32", "topk_n33_d8"]


def _stream_ok(kk: int) -> bool:
    """The reference's streaming kernel (bitonic merge, its default) is only
    defined for k a power of two: for other k its candidate buffer keeps one
    INT64_MAX padding word, which sorts first and is decoded as a NaN score
    (streaming_topk_attention.py:103, 118-123, 152-158). Those outputs are
    pinned as NaN and not compared."""
    return kk & (kk - 1) == 0


def _close(a, b, rows=None):
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    if rows is not None:
        a, b = a[rows], b[rows]
    np.testing.assert_allclose(a, b, rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("case", TOPK_CASES)
def test_topk_matches_reference_eager_and_kernels(golden, case):
    g = golden(case)
    q, k, v = g["q"], g["k"], g["v"]
    for kk in g["ks"]:
        kk = int(kk)
        amb = oracle.ambiguous_rows(q, k, kk)
        assert not amb.any(), "fixture rows should be unambiguous"
        out, _ = oracle.topk_attention(q, k, v, kk, tie="low")
        _close(out, g[f"eager_k{kk}"])
        _close(out, g[f"tiled_k{kk}"])
        if f"stream_k{kk}" in g:
            if _stream_ok(kk):
                _close(out, g[f"stream_k{kk}"])
            else:
                assert np.isnan(g[f"stream_k{kk}"]).any()


@pytest.mark.parametrize("case", TOPK_CASES)
def test_topk_indices_match_reference_streaming_kernel(golden, case):
    g = golden(case)
    q, k = g["q"], g["k"]
    s = oracle.scores_f32(q, k)
    for kk in g["ks"]:
        kk = int(kk)
        if f"stream_idx_k{kk}" not in g or not _stream_ok(kk):
            continue
        ref = g[f"stream_idx_k{kk}"].astype(np.int64)
        got = oracle.topk_indices(s, kk, tie="low")
        np.testing.assert_array_equal(np.sort(got, -1), np.sort(ref, -1))
        # the reference's buffer comes out score-descending, as ours does
        np.testing.assert_array_equal(got, ref)


def test_tie_rules_match_reference_kernels(golden):
    g = golden("topk_ties")
    q, k, v = g["q"], g["k"], g["v"]
    s = oracle.scores_f32(q, k)
    for kk in g["ks"]:
        kk = int(kk)
        low, _ = oracle.topk_attention(q, k, v, kk, tie="low")
        high, _ = oracle.topk_attention(q, k, v, kk, tie="high")
        every, m_all = oracle.topk_attention(q, k, v, kk, tie="all")
        _close(low, g[f"tiled_k{kk}"])
        _close(high, g[f"sort_k{kk}"])
        _close(every, g[f"masked_k{kk}"])
        if _stream_ok(kk):
            _close(low, g[f"stream_k{kk}"])
            ref_idx = g[f"stream_idx_k{kk}"].astype(np.int64)
            np.testing.assert_array_equal(oracle.topk_indices(s, kk, "low"),
                                          ref_idx)
        # the all-equal episode really exercises the rules
        assert (m_all[0].sum(-1) == q.shape[1] - 1).all()
        if kk < q.shape[1] - 1:
            assert not np.allclose(low[0], high[0])


def test_threshold_and_sort_kernels_on_random_rows(golden):
    g = golden("topk_modes")
    q, k, v = g["q"], g["k"], g["v"]
    for kk in g["ks"]:
        kk = int(kk)
        low, _ = oracle.topk_attention(q, k, v, kk, tie="low")
        high, _ = oracle.topk_attention(q, k, v, kk, tie="high")
        every, _ = oracle.topk_attention(q, k, v, kk, tie="all")
        _close(low, g[f"eager_k{kk}"])
        _close(low, g[f"rowwise_k{kk}"])
        _close(high, g[f"sort_k{kk}"])
        _close(every, g[f"masked_k{kk}"])


@pytest.mark.parametrize("case", ["dense_n40", "dense_c1", "dense_n70_d32"])
def test_dense_matches_reference(golden, case):
    g = golden(case)
    out = oracle.dense_attention(g["q"], g["k"], g["v"])
    _close(out, g["eager"])
    _close(out, g["flash"])


def test_morton_codes_bit_exact(golden):
    g = golden("morton_n50")
    np.testing.assert_array_equal(oracle.morton_code(g["pos"], 10), g["code10"])
    np.testing.assert_array_equal(oracle.morton_code(g["pos"], 16), g["code16"])
    e = golden("morton_edge")
    for bits, key in ((10, "code10"), (16, "code16"), (4, "code4")):
        np.testing.assert_array_equal(oracle.morton_code(e["pos"], bits), e[key])


def test_morton_window_matches_reference(golden):
    g = golden("morton_n50")
    clean = ~g["dup10"].astype(bool)  # the reference's argsort is unstable
    assert clean.any()
    for kk in g["ks"]:
        kk = int(kk)
        got = oracle.morton_window(g["pos"], kk, 10)
        np.testing.assert_array_equal(got[clean], g[f"win_k{kk}"][clean])
        # with duplicate codes the peer sets are still k distinct non-self
        self_idx = np.arange(got.shape[1])[None, :, None]
        assert not (got == self_idx).any()


def test_prescore_matches_reference(golden):
    g = golden("morton_n50")
    for kk in g["ks"]:
        kk = int(kk)
        idx = g[f"win_k{kk}"]
        out = oracle.prescore_attention(g["q"], g["k"], g["v"], idx)
        _close(out, g[f"prescore_k{kk}"])
        _close(out, g[f"fused_prescore_k{kk}"])


def test_prescore_bad_index_rows_are_nan():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((2, 8, 16)).astype(np.float32) for _ in range(3))
    idx = np.tile(np.array([1, 2]), (2, 8, 1))
    idx[1, 3, 1] = 8
    out = oracle.prescore_attention(q, k, v, idx)
    assert np.isnan(out[1, 3]).all()
    assert np.isfinite(np.delete(out.reshape(16, 16), 11, axis=0)).all()


def test_ambiguity_classifier_flags_near_ties_only():
    rng = np.random.default_rng(1)
    q = rng.standard_normal((1, 4, 16)).astype(np.float32)
    k = rng.standard_normal((1, 4, 16)).astype(np.float32)
    k[0, 3] = k[0, 2]
    k[0, 3, 0] = np.nextafter(k[0, 2, 0], np.float32(np.inf))
    amb = oracle.ambiguous_rows(q, k, 1)
    s = oracle.scores_f64(q, k)
    top = np.argsort(-s[0], axis=-1)[:, :2]
    for i in range(4):
        near = set(top[i]) == {2, 3}
        if near:
            assert amb[0, i]


@pytest.mark.parametrize("name", ["knn_n50", "knn_n600", "knn_n3000"])
def test_knn_selectors_match_reference(golden, name):
    """select_radius_knn and select_grid_knn (exact fallback at N=50, grid
    path at N=600 and 3000) against the reference's own outputs: the same
    peer set on every row whose k-th and (k+1)-th distances are not within
    rounding of each other."""
    g = golden(name)
    pos = g["pos"]
    for kk in g["ks"]:
        kk = int(kk)
        amb = oracle.knn_ambiguous(pos, kk)
        ok = ~amb
        assert tuple(g[f"shape_k{kk}"]) == oracle.grid_knn_shape(pos.shape[1], kk)
        np.testing.assert_array_equal(
            np.sort(oracle.knn_exact(pos, kk), -1)[ok],
            np.sort(g[f"radius_k{kk}"], -1)[ok])
        np.testing.assert_array_equal(
            np.sort(oracle.grid_knn(pos, kk), -1)[ok],
            np.sort(g[f"grid_k{kk}"], -1)[ok])
