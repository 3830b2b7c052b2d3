"""Helpers for the GPU parity tests: seeded inputs and comparisons against the
CPU oracle (tests only)."""

from __future__ import annotations

import numpy as np
import torch

import oracle

# Tolerances stated by the parity target: fp32 outputs within 1e-5 relative
# (with a 1e-5 absolute floor for values near zero), bf16 within 2e-2.
FP32_TOL = dict(rtol=1e-5, atol=1e-5)
BF16_TOL = dict(rtol=2e-2, atol=2e-2)


def qkv(B: int, N: int, d: int, seed: int, dtype=torch.float32,
        device="cuda"):
    """Q, K, V drawn i.i.d. N(0, 1) on the CPU from one seeded generator, in
    that order (scripts/bench_attention_core.py:341-344), then moved."""
    g = torch.Generator().manual_seed(seed)
    t = [torch.randn(B, N, d, generator=g) for _ in range(3)]
    t = [x.to(dtype) for x in t]
    return [x.to(device) for x in t]


def host(x: torch.Tensor) -> np.ndarray:
    """float32 numpy copy (bf16 values are exact in fp32)."""
    return x.detach().float().cpu().numpy()


def tol_for(dtype) -> dict:
    return BF16_TOL if dtype == torch.bfloat16 else FP32_TOL


def check_topk(q, k, v, topk, out, tie="low", idx=None, max_amb_frac=1e-2):
    """Compare a top-k attention output (and optional rank-ordered indices)
    with the oracle on every unambiguous row; returns the ambiguous-row count.

    Ambiguous rows (k-th and (k+1)-th exact scores closer than fp32 rounding
    of a length-d dot product) are expected at about 0.1 % of rows when k
    sits in the dense middle of a score row; more than 1 % fails the test.
    """
    qn, kn, vn = host(q), host(k), host(v)
    ref, mask = oracle.topk_attention(qn, kn, vn, topk, tie=tie)
    amb = oracle.ambiguous_rows(qn, kn, topk)
    ok = ~amb
    assert amb.mean() <= max_amb_frac, f"{amb.sum()} ambiguous rows"
    got = host(out)
    np.testing.assert_allclose(got[ok], ref[ok], **tol_for(out.dtype))
    if idx is not None:
        s = oracle.scores_f32(qn, kn)
        want = oracle.topk_indices(s, topk, tie)
        gi = idx.long().cpu().numpy()
        np.testing.assert_array_equal(np.sort(gi[ok], -1), np.sort(want[ok], -1))
        # rank order holds wherever no near tie sits inside the retained set
        s64 = oracle.scores_f64(qn, kn)
        vals = np.take_along_axis(s64, want, -1)
        gaps = -np.diff(vals, axis=-1) if topk > 1 else np.ones(vals.shape[:-1] + (1,))
        clean = ok & (np.abs(gaps).min(-1) > 1e-4)
        np.testing.assert_array_equal(gi[clean], want[clean])
    return int(amb.sum())
