"""GPU parity of the fused communication-module kernel (csrc/comm.cu):
qkv projection -> attention core -> GELU -> output projection in one launch,
against the oracle's float64 restatement of AttentionComm.forward
(src/agents/mappo.py:332-353, 361-373, 419-420).

Bar: outputs within rtol = atol = 1e-5 on every row whose k-th and (k+1)-th
scores are not within fp32 rounding of the projections (a relative gap of
1e-5 of the row's largest score); for dense attention, every row.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


def _weights(D, m, seed):
    g = torch.Generator().manual_seed(seed)
    w_qkv = torch.randn(3 * m, D, generator=g) / D ** 0.5
    b_qkv = torch.randn(3 * m, generator=g) * 0.1
    w_proj = torch.randn(m, m, generator=g) / m ** 0.5
    b_proj = torch.randn(m, generator=g) * 0.1
    return w_qkv, b_qkv, w_proj, b_proj


def _near_tie_rows(q, k, topk):
    if topk == 0:
        return np.zeros(q.shape[:2], dtype=bool)
    B, N, m = q.shape
    s = np.einsum("bid,bjd->bij", q, k) / np.sqrt(m)
    s[:, np.arange(N), np.arange(N)] = -np.inf
    srt = -np.sort(-s, axis=-1)
    if topk >= N - 1:
        return np.zeros((B, N), dtype=bool)
    gap = srt[..., topk - 1] - srt[..., topk]
    return gap <= 1e-5 * np.abs(srt[..., 0])


@pytest.mark.parametrize("B,N,D,m,topk", [
    (256, 6, 64, 16, 2), (64, 6, 36, 16, 0), (32, 40, 64, 16, 4),
    (8, 512, 64, 16, 2), (4, 1024, 32, 16, 1), (16, 100, 256, 64, 8),
    (8, 200, 48, 8, 0), (16, 3, 5, 3, 2), (4, 2, 16, 16, 1)])
def test_comm_forward_matches_module_oracle(B, N, D, m, topk):
    from tarmac_b200 import ops
    x = torch.randn(B, N, D, generator=torch.Generator().manual_seed(N + D))
    w = _weights(D, m, seed=m + topk)
    out = ops.comm_forward(x.cuda(), *(t.cuda() for t in w), topk)
    ref, q, k = oracle.comm_forward(x.numpy(), *(t.numpy() for t in w), topk)
    ok = ~_near_tie_rows(q, k, topk)
    assert ok.mean() > 0.99
    np.testing.assert_allclose(out.cpu().numpy()[ok], ref[ok], rtol=1e-5,
                               atol=1e-5)


@pytest.mark.parametrize("B,N,D,m,topk", [
    (4096, 6, 64, 16, 2), (4096, 6, 64, 16, 0), (1000, 32, 36, 8, 3),
    (3001, 17, 64, 32, 1), (700, 6, 33, 16, 0), (1500, 5, 20, 3, 2),
    (600, 8, 64, 64, 4), (149, 9, 64, 16, 8)])
def test_comm_forward_large_batches(B, N, D, m, topk):
    """Batches of at least one episode per SM take the multi-episode tile
    form (weights staged once per block, tiles of several episodes, a ragged
    last tile): every sampled episode matches the oracle, and a slice of the
    batch run on its own (one block per episode) gives the same bits. Covers
    4-byte staging (odd input width), padded message columns (m=3) and
    m=64."""
    from tarmac_b200 import ops
    x = torch.randn(B, N, D, generator=torch.Generator().manual_seed(B + N))
    w = [t.cuda() for t in _weights(D, m, seed=m + topk + 1)]
    xc = x.cuda()
    out = ops.comm_forward(xc, *w, topk)
    sel = np.sort(np.random.default_rng(B).choice(B, size=64, replace=False))
    sel[-1] = B - 1                                   # the ragged last tile
    ref, q, k = oracle.comm_forward(x.numpy()[sel], *(t.cpu().numpy() for t in w),
                                    topk)
    ok = ~_near_tie_rows(q, k, topk)
    assert ok.mean() > 0.99
    np.testing.assert_allclose(out.cpu().numpy()[sel][ok], ref[ok], rtol=1e-5,
                               atol=1e-5)
    head = ops.comm_forward(xc[:16].contiguous(), *w, topk)
    assert torch.equal(head, out[:16])


@pytest.mark.parametrize("mode,k", [("topk", 2), ("topk_gather", 3),
                                    ("dense", 0), ("dense_sdpa", 0)])
def test_module_inference_uses_one_kernel_with_same_result(mode, k):
    """Under no_grad the comm module runs the fused kernel; its output equals
    the layer-by-layer path (qkv Linear, attention kernel, GELU, proj)."""
    from src.agents.mappo import AttentionComm, MAPPOConfig
    cfg = MAPPOConfig(obs_dim=18, n_actions=5, n_agents=6, hidden=64,
                      use_comm=True, msg_dim=16, attn_mode=mode, topk=k)
    torch.manual_seed(3)
    comm = AttentionComm(cfg, in_dim=64).cuda()
    x = torch.randn(256, 6, 64, device="cuda")
    assert comm._fused_ok(x.detach(), mode, 6) is False   # params need grad
    with torch.no_grad():
        assert comm._fused_ok(x, mode, 6)
        fused, info = comm(x)
    layered, info2 = comm(x)                                # autograd path
    assert info == info2
    assert (fused - layered.detach()).abs().max().item() < 1e-5


def test_limits_raise_and_module_falls_back():
    from tarmac_b200 import TarmacError, ops
    from src.agents.mappo import AttentionComm, MAPPOConfig
    x = torch.randn(2, 2048, 16, device="cuda")
    w = [t.cuda() for t in _weights(16, 16, 1)]
    with pytest.raises(TarmacError):
        ops.comm_forward(x, *w, 2)              # K, V exceed shared memory
    cfg = MAPPOConfig(obs_dim=18, n_actions=5, n_agents=2048, hidden=16,
                      use_comm=True, msg_dim=16, attn_mode="topk", topk=2)
    comm = AttentionComm(cfg, in_dim=16).cuda()
    with torch.no_grad():
        out, _ = comm(x)                        # layer-by-layer path
    assert out.shape == (2, 2048, 16) and torch.isfinite(out).all()


def test_weights_on_another_device_raise():
    from tarmac_b200 import ops
    x = torch.randn(4, 6, 16, device="cuda")
    w = list(_weights(16, 16, 1))                 # left on the CPU
    with pytest.raises(ValueError):
        ops.comm_forward(x, *w, 2)


@pytest.mark.parametrize("B,N,D,m,topk,offset", [
    (64, 8, 64, 16, 2, 0),     # N * 16 = 128: the last (agent, column) size
    (64, 9, 64, 16, 2, 0),     # one agent past it: a thread per agent
    (64, 16, 20, 8, 3, 0),     # N * 8 = 128 with 16-byte rows of 20 words
    (64, 6, 64, 16, 2, 1),     # x one word off the 16-byte grid: 4-byte copies
    (64, 6, 33, 16, 0, 0),     # odd input width: 4-byte copies, dense
    (32, 4, 64, 32, 2, 0),     # N * 32 = 128
    (32, 2, 64, 64, 1, 0),     # N * 64 = 128
    (8, 150, 256, 64, 4, 0)])  # W_qkv left in global memory
def test_comm_forward_copy_forms_and_phase2_forms(B, N, D, m, topk, offset):
    """The 16-byte and 4-byte staging forms and both phase-2 forms (one
    thread per (agent, message column) up to N * padded m = 128, one thread
    per agent above) against the float64 module oracle."""
    from tarmac_b200 import ops
    g = torch.Generator().manual_seed(B + N + D + m)
    x = torch.randn(B, N, D, generator=g)
    w = _weights(D, m, seed=N * m + topk)
    xd = torch.empty(B * N * D + offset, device="cuda")[offset:].view(B, N, D)
    xd.copy_(x)
    out = ops.comm_forward(xd, *(t.cuda() for t in w), topk)
    ref, q, k = oracle.comm_forward(x.numpy(), *(t.numpy() for t in w), topk)
    ok = ~_near_tie_rows(q, k, topk)
    assert ok.mean() > 0.99
    np.testing.assert_allclose(out.cpu().numpy()[ok], ref[ok], rtol=1e-5,
                               atol=1e-5)
