"""GPU tests of the drop-in modules (reference names and signatures) against
the contracts the reference's own tests pin:

* tests/test_comm_module.py:33-67 — top-k with k = N-1 equals dense (1e-6);
  322-344 — `topk` and `topk_gather` compute the same function; 457-475 —
  `dense_sdpa` equals `dense`;
* tests/test_zorder_comm.py:46-105 — Z-order peers are k distinct non-self
  agents, the curve-order neighbours; the message equals dense attention
  restricted to them and ignores the other peers.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _parity import check_topk, host, qkv

pytestmark = pytest.mark.gpu


def _cfg(**kw):
    from src.agents.mappo import MAPPOConfig
    base = dict(obs_dim=18, n_actions=5, n_agents=6, hidden=32, use_comm=True,
                msg_dim=8, attn_mode="dense")
    base.update(kw)
    return MAPPOConfig(**base)


def test_topk_at_n_minus_1_equals_dense_across_n():
    from src.agents.mappo import AttentionComm
    for N in (3, 6, 12, 24):
        torch.manual_seed(N)
        dense = AttentionComm(_cfg(n_agents=N), in_dim=32).cuda()
        topk = AttentionComm(_cfg(n_agents=N, attn_mode="topk", topk=N - 1),
                             in_dim=32).cuda()
        topk.load_state_dict(dense.state_dict())
        x = torch.randn(3, N, 32, device="cuda")
        with torch.no_grad():
            a, _ = dense(x)
            b, info = topk(x)
        assert info["effective_k"] == float(N - 1)
        # two different kernels (resident-row top-k, dense online softmax)
        # sum in different orders: the identity holds to fp32 rounding (the
        # reference's 1e-6 compares two paths sharing one softmax)
        assert (a - b).abs().max().item() < 1e-5, f"failed at N={N}"


def test_topk_and_topk_gather_and_sdpa_modes():
    from src.agents.mappo import AttentionComm
    torch.manual_seed(0)
    for N, k in ((6, 1), (12, 3), (24, 2)):
        mods = {m: AttentionComm(_cfg(n_agents=N, attn_mode=m, topk=k),
                                 in_dim=32).cuda()
                for m in ("topk", "topk_gather", "dense", "dense_sdpa")}
        sd = mods["dense"].state_dict()
        for m in mods.values():
            m.load_state_dict(sd)
        x = torch.randn(4, N, 32, device="cuda")
        with torch.no_grad():
            out = {m: mod(x)[0] for m, mod in mods.items()}
        assert torch.equal(out["topk"], out["topk_gather"])
        assert torch.equal(out["dense"], out["dense_sdpa"])


def test_comm_module_matches_oracle_core():
    """qkv Linear -> oracle top-k core -> gelu -> proj equals the module."""
    from src.agents.mappo import AttentionComm
    torch.manual_seed(1)
    N, k = 12, 2
    comm = AttentionComm(_cfg(n_agents=N, attn_mode="topk_gather", topk=k),
                         in_dim=32).cuda()
    x = torch.randn(8, N, 32, device="cuda")
    with torch.no_grad():
        got, _ = comm(x)
        q, kk, v = comm.qkv(x).chunk(3, -1)
        core, _ = oracle.topk_attention(host(q), host(kk), host(v), k)
        ref = comm.proj(torch.nn.functional.gelu(torch.from_numpy(core).cuda()))
    assert (got - ref).abs().max().item() < 1e-5


def test_zorder_selector_contract():
    from src.kernels.prescore_selection import select_morton_window
    for N, k in ((6, 1), (6, 2), (6, 4), (12, 3)):
        torch.manual_seed(N * 10 + k)
        pos = (torch.rand(16, N, 2) * 2 - 1).cuda()
        idx = select_morton_window(pos, k)
        assert idx.shape == (16, N, k) and idx.dtype == torch.int64
        assert not (idx == torch.arange(N, device="cuda").view(1, N, 1)).any()
        srt = idx.sort(-1).values
        assert (srt[..., 1:] != srt[..., :-1]).all()
        np.testing.assert_array_equal(idx.cpu().numpy(),
                                      oracle.morton_window(pos.cpu().numpy(), k, 10))


def test_zorder_message_equals_restricted_dense_and_ignores_others():
    from src.agents.mappo import AttentionComm
    from src.kernels.prescore_selection import select_morton_window
    torch.manual_seed(0)
    N, B = 6, 5
    comm = AttentionComm(_cfg(obs_dim=36, attn_mode="zorder_k", topk=2),
                         in_dim=32).cuda().eval()
    x = torch.randn(B, N, 32, device="cuda")
    pos = (torch.rand(B, N, 2) * 2 - 1).cuda()
    with torch.no_grad():
        got, info = comm(x, pos)
        q, kk, v = comm.qkv(x).chunk(3, dim=-1)
        scores = q @ kk.transpose(-1, -2) / kk.shape[-1] ** 0.5
        keep = torch.zeros(B, N, N, dtype=torch.bool, device="cuda")
        keep.scatter_(-1, select_morton_window(pos, 2), True)
        w = torch.softmax(scores.masked_fill(~keep, float("-inf")), -1)
        ref = comm.proj(torch.nn.functional.gelu(w @ v))
    assert info["effective_k"] == 2.0
    assert (got - ref).abs().max().item() < 1e-6
    sel = select_morton_window(pos[:1], 2)[0, 0].tolist()
    other = next(j for j in range(1, N) if j not in sel)
    x2 = x[:1].clone()
    x2[0, other] += 10.0
    with torch.no_grad():
        m1, _ = comm(x[:1], pos[:1])
        m2, _ = comm(x2, pos[:1])
    assert torch.allclose(m1[0, 0], m2[0, 0], atol=1e-6)


def _eager_comm(x, pos, sd, mode, k):
    """float64 CPU restatement of the reference module's forward
    (src/agents/mappo.py:332-420) for one attention mode."""
    import torch.nn.functional as F
    qkv = x @ sd["qkv.weight"].T + sd["qkv.bias"]
    q, kt, v = qkv.chunk(3, dim=-1)
    B, N, d = q.shape
    if mode == "zorder_k":
        idx = torch.from_numpy(oracle.morton_window(pos.float().numpy(), k, 10))
    else:
        s = torch.matmul(q, kt.transpose(-1, -2)) / d ** 0.5
        s = s.masked_fill(torch.eye(N, dtype=torch.bool), float("-inf"))
        if mode == "dense":
            msg = torch.matmul(torch.softmax(s, -1), v)
        else:
            idx = s.topk(k, dim=-1).indices
    if mode != "dense":
        flat = idx.reshape(B, N * k, 1).expand(B, N * k, d)
        kg = kt.gather(1, flat).view(B, N, k, d)
        vg = v.gather(1, flat).view(B, N, k, d)
        w = torch.softmax(torch.matmul(q.unsqueeze(-2), kg.transpose(-1, -2))
                          / d ** 0.5, -1)
        msg = torch.matmul(w, vg).squeeze(-2)
    return F.gelu(msg) @ sd["proj.weight"].T + sd["proj.bias"]


@pytest.mark.parametrize("mode,k", [("dense", 0), ("topk", 2),
                                    ("topk_gather", 3), ("zorder_k", 2)])
def test_training_gradients_match_the_eager_module(mode, k):
    """loss.backward() through the comm module: every parameter's gradient
    equals the one autograd forms through the reference's eager path."""
    from src.agents.mappo import AttentionComm
    N = 12
    torch.manual_seed(7)
    comm = AttentionComm(_cfg(n_agents=N, attn_mode=mode, topk=k),
                         in_dim=32).cuda()
    x = torch.randn(3, N, 32)
    pos = torch.rand(3, N, 2)
    out, _ = comm(x.cuda(), pos.cuda())
    (out ** 2).sum().backward()
    sd = {n: p.detach().double().cpu().requires_grad_(True)
          for n, p in comm.named_parameters() if not n.startswith("k_gate")}
    ref = _eager_comm(x.double(), pos, sd, mode, k)
    (ref ** 2).sum().backward()
    assert (out.detach().cpu().double() - ref.detach()).abs().max() < 1e-5
    for n, p in sd.items():
        got = dict(comm.named_parameters())[n].grad.double().cpu()
        want = p.grad
        tol = 1e-4 * max(1.0, want.abs().max().item())
        assert (got - want).abs().max().item() < tol, n


def test_kernel_modules_reference_signatures():
    from src.kernels import fused_dense_attention as fda
    from src.kernels import fused_prescore_attention as fpa
    from src.kernels import fused_topk_attention as fta
    from src.kernels import streaming_topk_attention as sta
    q, k, v = qkv(8, 100, 16, seed=3)
    for fn in (fta.fused_topk_attention, fta.fused_topk_attention_tiled):
        check_topk(q, k, v, 2, fn(q, k, v, 2))
    check_topk(q, k, v, 3, fta.fused_topk_attention_sort(q, k, v, 3), tie="high")
    check_topk(q, k, v, 3, fta.fused_topk_attention_masked(q, k, v, 3), tie="all")
    out, idx = sta.streaming_topk_attention(q, k, v, 4, return_indices=True)
    assert idx.dtype == torch.int32 and idx.shape == (8, 100, 4)
    check_topk(q, k, v, 4, out, idx=idx)
    # k clamps to N - 1 exactly as the reference launchers do
    q6, k6, v6 = qkv(4, 6, 16, seed=4)
    np.testing.assert_allclose(host(fta.fused_topk_attention_tiled(q6, k6, v6, 50)),
                               host(fda.fused_dense_attention(q6, k6, v6)),
                               rtol=1e-5, atol=1e-6)
    idx64 = torch.randint(0, 100, (8, 100, 3), device="cuda")
    a = fpa.fused_prescore_attention(q, k, v, idx64)
    b = fpa.fused_prescore_attention(q, k, v, idx64.int())
    assert torch.equal(a, b)
    ref = fta.reference_topk_attention(q, k, v, 2)   # the eager baseline, on GPU
    np.testing.assert_allclose(host(fta.fused_topk_attention_tiled(q, k, v, 2)),
                               host(ref), rtol=1e-5, atol=1e-5)


def test_launch_form_kernel_calls():
    from src.kernels import fused_dense_attention as fda
    from src.kernels import fused_topk_attention as fta
    q, k, v = qkv(4, 64, 16, seed=9)
    o = torch.empty_like(q)
    st = [*q.stride(), *k.stride(), *v.stride(), *o.stride()]
    fta._fused_topk_tiled_kernel[(2, 4)](q, k, v, o, *st, 64, 0.25, TOPK=2,
                                         BLOCK_M=32, BLOCK_N=64, BLOCK_D=16,
                                         BLOCK_DC=16, HEAD_D=16, num_warps=4)
    check_topk(q, k, v, 2, o)
    o2 = torch.empty_like(q)
    fda._flash_dense_kernel[(1, 4)](q, k, v, o2, *st, 64, 0.25, BLOCK_M=64,
                                    BLOCK_KN=64, BLOCK_D=16, HEAD_D=16,
                                    PRECISION="ieee", num_warps=4, num_stages=2)
    np.testing.assert_allclose(host(o2), oracle.dense_attention(host(q), host(k), host(v)),
                               rtol=1e-5, atol=1e-5)
