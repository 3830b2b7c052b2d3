"""GPU parity of the positional and random selectors (csrc/selectors.cu).

The kNN selectors use the oracle's arithmetic (fp32 squared distances, each
step rounded) and its order (increasing distance, then index), so their
index lists are compared bit for bit; the oracle is pinned against the
reference's own select_radius_knn / select_grid_knn outputs
(test_oracle_golden.py). The random selector is checked for its contract
(k distinct peers, self excluded) and its distribution.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from tarmac_b200 import ops as _ops
    return _ops


def _pos(B, N, seed):
    return torch.rand(B, N, 2, generator=torch.Generator().manual_seed(seed))


@pytest.mark.parametrize("N,k", [(2, 1), (3, 2), (50, 5), (600, 2), (1000, 8),
                                 (3000, 16), (300, 32), (8192, 2)])
def test_knn_exact_bit_exact(ops, N, k):
    pos = _pos(2 if N < 4096 else 1, N, N + k)
    got = ops.knn_select(pos.cuda(), k).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.knn_exact(pos.numpy(), k))


@pytest.mark.parametrize("N,k", [(600, 1), (600, 2), (1000, 4), (3000, 2),
                                 (3000, 8), (8192, 2), (50, 3)])
def test_grid_knn_bit_exact(ops, N, k):
    pos = _pos(1 if N >= 3000 else 3, N, 7 * N + k)
    got = ops.grid_knn_select(pos.cuda(), k).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.grid_knn(pos.numpy(), k))


def test_selectors_on_degenerate_positions(ops):
    """Duplicated positions (exact distance ties: lowest index first), a zero
    span on one axis, clustered agents that overflow grid cells."""
    pos = _pos(4, 700, 3)
    pos[0, 100:120] = pos[0, 5]                 # 21 agents on one point
    pos[1, :, 1] = 0.25                         # zero span in y
    pos[2, :400] = pos[2, :400] * 0.02          # a dense cluster
    pos[3] = (pos[3] * 8).floor() / 8           # lattice: many equal distances
    for k in (1, 2, 5):
        np.testing.assert_array_equal(ops.knn_select(pos.cuda(), k).cpu().numpy(),
                                      oracle.knn_exact(pos.numpy(), k))
        np.testing.assert_array_equal(
            ops.grid_knn_select(pos.cuda(), k).cpu().numpy(),
            oracle.grid_knn(pos.numpy(), k))


def test_reference_fixtures_and_recall(golden):
    """The drop-in functions on the reference's fixture positions: the
    reference's own peer sets on unambiguous rows, and its recall figure."""
    from src.kernels import prescore_selection as ps
    for name in ("knn_n50", "knn_n600", "knn_n3000"):
        g = golden(name)
        pos = torch.from_numpy(g["pos"]).cuda()
        for kk in g["ks"]:
            kk = int(kk)
            ok = ~oracle.knn_ambiguous(g["pos"], kk)
            for fn, key in ((ps.select_radius_knn, "radius"),
                            (ps.select_grid_knn, "grid")):
                got = np.sort(fn(pos, kk).cpu().numpy(), -1)
                np.testing.assert_array_equal(got[ok],
                                              np.sort(g[f"{key}_k{kk}"], -1)[ok])
            assert abs(ps.grid_knn_recall(pos, kk) - float(g[f"recall_k{kk}"])) < 1e-3


def test_random_select_contract_and_distribution(ops):
    B, N, k = 4000, 6, 2
    torch.manual_seed(11)
    idx = ops.random_select(B, N, k, "cuda").cpu().numpy()
    assert idx.shape == (B, N, k)
    rows = np.arange(N)[None, :, None]
    assert ((idx >= 0) & (idx < N)).all()
    assert (idx != rows).all()                             # self excluded
    assert (idx[..., 0] != idx[..., 1]).all()              # distinct
    # every one of the C(5, 2) = 10 pairs of other agents equally likely
    for i in range(N):
        pairs = np.sort(idx[:, i, :], -1)
        keys, counts = np.unique(pairs[:, 0] * N + pairs[:, 1], return_counts=True)
        assert len(keys) == 10
        chi2 = ((counts - B / 10) ** 2 / (B / 10)).sum()
        assert chi2 < 40.0, chi2                           # 9 dof; p ~ 1e-5
    torch.manual_seed(11)
    again = ops.random_select(B, N, k, "cuda").cpu().numpy()
    np.testing.assert_array_equal(idx, again)              # seeded by torch
    big = ops.random_select(2, 1000, 32, "cuda").cpu().numpy()
    assert all(len(set(r)) == 32 for r in big.reshape(-1, 32))


def test_prescore_full_every_selector():
    from src.kernels import prescore_selection as ps
    from _parity import host, qkv
    q, k, v = qkv(3, 700, 16, seed=9)
    pos = _pos(3, 700, 10).cuda()
    for sel in ("radius_knn", "grid_knn", "morton_window"):
        out = ps.prescore_full(q, k, v, pos, 2, sel)
        idx = ps.SELECTORS[sel](pos, 2).cpu().numpy()
        ref = oracle.prescore_attention(host(q), host(k), host(v), idx)
        np.testing.assert_allclose(host(out), ref, rtol=1e-5, atol=1e-5)


def test_random_k_comm_mode_trains():
    from src.agents.mappo import AttentionComm, MAPPOConfig
    cfg = MAPPOConfig(obs_dim=18, n_actions=5, n_agents=12, hidden=32,
                      use_comm=True, msg_dim=8, attn_mode="random_k", topk=3)
    comm = AttentionComm(cfg, in_dim=32).cuda()
    out, info = comm(torch.randn(4, 12, 32, device="cuda"))
    assert info["effective_k"] == 3.0 and torch.isfinite(out).all()
    out.sum().backward()
    assert torch.isfinite(comm.qkv.weight.grad).all()
    assert comm.qkv.weight.grad.abs().sum() > 0
