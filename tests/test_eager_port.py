"""The eager-PyTorch restatement that bench.py times as the CPU baseline
(oracle/eager_torch.py) against the reference's own outputs: the committed
golden vectors were made by running the reference's eager functions on the
same inputs, and the restatement issues the same ATen calls, so on the same
host it reproduces them bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import eager_torch as et


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a))


@pytest.mark.parametrize("name", ["topk_n40", "topk_c1", "topk_n33_d8",
                                  "topk_n64_d32"])
def test_topk_gather_reproduces_reference_eager(golden, name):
    g = golden(name)
    q, k, v = (_t(g[x]) for x in ("q", "k", "v"))
    for kk in g["ks"]:
        got = et.topk_gather(q, k, v, int(kk)).numpy()
        np.testing.assert_allclose(got, g[f"eager_k{int(kk)}"], rtol=1e-6,
                                   atol=1e-6)


@pytest.mark.parametrize("name", ["dense_n40", "dense_c1", "dense_n70_d32"])
def test_dense_reproduces_reference_eager(golden, name):
    g = golden(name)
    q, k, v = (_t(g[x]) for x in ("q", "k", "v"))
    np.testing.assert_allclose(et.dense(q, k, v).numpy(), g["eager"],
                               rtol=1e-6, atol=1e-6)


def test_morton_window_and_prescore_reproduce_reference(golden):
    g = golden("morton_n50")
    pos = _t(g["pos"])
    q, k, v = (_t(g[x]) for x in ("q", "k", "v"))
    clean = ~g["dup10"]          # episodes where the unstable argsort is determined
    for kk in g["ks"]:
        kk = int(kk)
        idx = et.morton_window(pos, kk, 10)
        np.testing.assert_array_equal(idx.numpy()[clean], g[f"win_k{kk}"][clean])
        want = _t(g[f"win_k{kk}"])
        np.testing.assert_allclose(et.prescore(q, k, v, want).numpy(),
                                   g[f"prescore_k{kk}"], rtol=1e-6, atol=1e-6)
