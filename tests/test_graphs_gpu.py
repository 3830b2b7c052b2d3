"""GPU: GraphedCall (tarmac_b200/graphs.py) replays a captured call of the
library's operations; on new inputs its output equals a direct call's, bit
for bit (the same kernel on the same values)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _inputs(B, N, d, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(B, N, d, generator=g).to(dtype).cuda() for _ in range(3)]


def test_topk_replay_matches_direct_calls():
    from tarmac_b200 import ops
    from tarmac_b200.graphs import GraphedCall
    q, k, v = _inputs(64, 128, 16, 1)
    step = GraphedCall(ops.topk_attention, q, k, v, 2)
    for seed in (2, 3):
        q2, k2, v2 = _inputs(64, 128, 16, seed)
        got = step(q2, k2, v2, 2).clone()
        assert torch.equal(got, ops.topk_attention(q2, k2, v2, 2))
    # the example tensors are the graph's buffers: updated in place, seen
    q.copy_(_inputs(64, 128, 16, 4)[0])
    assert torch.equal(step(q, k, v, 2), ops.topk_attention(q, k, v, 2))


def test_comm_module_replay_matches_direct_calls():
    from tarmac_b200 import ops
    from tarmac_b200.graphs import GraphedCall
    g = torch.Generator().manual_seed(5)
    B, N, D, m = 256, 6, 64, 16
    w = [(torch.randn(3 * m, D, generator=g) / D ** 0.5).cuda(),
         (0.1 * torch.randn(3 * m, generator=g)).cuda(),
         (torch.randn(m, m, generator=g) / m ** 0.5).cuda(),
         (0.1 * torch.randn(m, generator=g)).cuda()]
    x = torch.randn(B, N, D, generator=g).cuda()
    step = GraphedCall(ops.comm_forward, x, *w, 2)
    for _ in range(2):
        x2 = torch.randn(B, N, D, generator=g).cuda()
        got = step(x2, *w, 2).clone()
        assert torch.equal(got, ops.comm_forward(x2, *w, 2))


def test_mismatched_arguments_raise():
    from tarmac_b200 import ops
    from tarmac_b200.graphs import GraphedCall
    q, k, v = _inputs(8, 64, 16, 7)
    step = GraphedCall(ops.dense_attention, q, k, v)
    with pytest.raises(ValueError):
        step(*_inputs(8, 32, 16, 8))          # other shape
    step2 = GraphedCall(ops.topk_attention, q, k, v, 2)
    with pytest.raises(ValueError):
        step2(q, k, v, 3)                     # other k


@pytest.mark.parametrize("op", ["topk", "dense"])
def test_training_step_graphed_with_torch(op):
    """The autograd functions are capturable: torch.cuda.make_graphed_callables
    records forward and backward (kernels, workspace and gradient buffers
    allocated through torch on the capturing stream) and the replays give the
    gradients of eager calls. The dense gradients are deterministic (equal
    bits); the fixed-peer kernel adds into dk and dv atomically (order not
    fixed), so those are compared to within fp32 rounding."""
    from tarmac_b200 import autograd as ag

    def fn(q, k, v):
        return ag.topk_attention(q, k, v, 2) if op == "topk" else ag.dense_attention(q, k, v)

    B, N, d = 256, 6, 16
    sample = [t.requires_grad_(True) for t in _inputs(B, N, d, 11)]
    graphed = torch.cuda.make_graphed_callables(fn, tuple(sample))
    for seed in (12, 13):
        x = [t.requires_grad_(True) for t in _inputs(B, N, d, seed)]
        go = _inputs(B, N, d, seed + 100)[0]
        out = graphed(*x)
        got = torch.autograd.grad(out, x, go)
        y = [t.detach().clone().requires_grad_(True) for t in x]
        ref_out = fn(*y)
        want = torch.autograd.grad(ref_out, y, go)
        assert torch.equal(out, ref_out)
        for a, b in zip(got, want):
            if op == "dense":
                assert torch.equal(a, b)
            else:
                torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)
