"""GPU parity of the gradient kernels (csrc/backward.cu) against the oracle's
gradients (float64, pinned against torch autograd in test_oracle_grad.py).

Bar: fp32 gradients within rtol = 1e-4 plus an absolute floor of 1e-5 times
the largest gradient magnitude (sums over up to N terms in fp32); gradients
returned in bf16 within 2e-2.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _parity import host, qkv

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tb():
    from tarmac_b200 import autograd, ops
    return ops, autograd


def close(got, want, rtol=1e-4, floor=1e-5):
    got = got.detach().float().cpu().numpy() if torch.is_tensor(got) else got
    atol = floor * max(1.0, float(np.abs(want).max()))
    np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)


@pytest.mark.parametrize("N,d", [(2, 16), (6, 16), (64, 16), (300, 16),
                                 (512, 16), (100, 8), (128, 64), (70, 100),
                                 (40, 128), (33, 3)])
def test_dense_backward(tb, N, d):
    ops, _ = tb
    q, k, v = qkv(4, N, d, seed=N + d)
    g = torch.randn(4, N, d, generator=torch.Generator().manual_seed(N)).cuda()
    out = ops.dense_attention(q, k, v)
    dq, dk, dv = ops.dense_attention_backward(q, k, v, out, g)
    want = oracle.dense_attention_grad(host(q), host(k), host(v), host(g))
    for a, b in zip((dq, dk, dv), want):
        close(a, b)


@pytest.mark.parametrize("N,d,scale_in,strided", [
    (128, 16, 1.0, False), (129, 16, 1.0, False), (1000, 16, 1.0, False),
    (256, 16, 6.0, False), (300, 16, 1.0, True)])
def test_dense_backward_tensor_cores(tb, N, d, scale_in, strided):
    """fp32 with d = 16 and at least 128 agents: the tensor-core kernels
    (backward_tc.cu), partial tiles, large scores (the log-sum-exp's
    reference point moves) and strided views included."""
    ops, _ = tb
    if strided:
        base = qkv(3, N, 3 * d, seed=N + 7)[0]
        q, k, v = base[..., :d], base[..., d:2 * d], base[..., 2 * d:]
    else:
        q, k, v = qkv(3, N, d, seed=N * 11 + d)
        q = q * scale_in
    g = torch.randn(3, N, d, generator=torch.Generator().manual_seed(N + 1)).cuda()
    out = ops.dense_attention(q, k, v)
    dq, dk, dv = ops.dense_attention_backward(q, k, v, out, g)
    want = oracle.dense_attention_grad(host(q), host(k), host(v), host(g))
    for a, b in zip((dq, dk, dv), want):
        close(a, b)


@pytest.mark.parametrize("N,d", [(6, 16), (128, 16), (300, 32), (512, 64)])
def test_dense_backward_bf16(tb, N, d):
    """bf16 inputs (fp32 arithmetic on the widened values); D from the
    bf16 forward output the kernel is given."""
    ops, _ = tb
    q, k, v = qkv(3, N, d, seed=N * 5 + d, dtype=torch.bfloat16)
    g = torch.randn(3, N, d, generator=torch.Generator().manual_seed(N))
    g = g.to(torch.bfloat16).cuda()
    out = ops.dense_attention(q, k, v)
    dq, dk, dv = ops.dense_attention_backward(q, k, v, out, g)
    want = oracle.dense_attention_grad(host(q), host(k), host(v), host(g),
                                       out=host(out))
    for a, b in zip((dq, dk, dv), want):
        close(a, b)


@pytest.mark.parametrize("N,d,kk,itype,dup", [
    (8, 16, 2, torch.int64, False), (64, 16, 4, torch.int32, False),
    (300, 32, 3, torch.int64, True), (512, 16, 8, torch.int32, False),
    (50, 100, 12, torch.int64, True), (20, 5, 2, torch.int32, False),
    (128, 128, 2, torch.int64, False)])
def test_gather_backward(tb, N, d, kk, itype, dup):
    ops, _ = tb
    q, k, v = qkv(3, N, d, seed=N * 3 + kk)
    gen = torch.Generator().manual_seed(N + kk)
    g = torch.randn(3, N, d, generator=gen).cuda()
    if dup:
        idx = torch.randint(0, N, (3, N, kk), generator=gen)
    else:
        idx = torch.stack([torch.stack([torch.randperm(N, generator=gen)[:kk]
                                        for _ in range(N)]) for _ in range(3)])
    idx = idx.to(itype)
    dq, dk, dv = ops.gather_attention_backward(q, k, v, g, idx.cuda())
    want = oracle.gather_attention_grad(host(q), host(k), host(v), idx.numpy(),
                                        host(g))
    for a, b in zip((dq, dk, dv), want):
        close(a, b)


def test_gather_backward_bad_index_rows(tb):
    """A row naming a peer outside [0, N) gets a NaN dq row and adds nothing
    to dk / dv."""
    ops, _ = tb
    q, k, v = qkv(2, 16, 16, seed=4)
    idx = torch.randint(0, 16, (2, 16, 3),
                        generator=torch.Generator().manual_seed(1)).cuda()
    idx[1, 5, 2] = 16
    g = torch.ones(2, 16, 16).cuda()
    dq, dk, dv = ops.gather_attention_backward(q, k, v, g, idx)
    assert torch.isnan(dq[1, 5]).all()
    assert torch.isfinite(dq[0]).all()
    good = idx.clone()
    good[1, 5] = 0
    g_masked = host(g).copy()
    g_masked[1, 5] = 0
    want = oracle.gather_attention_grad(host(q), host(k), host(v),
                                        good.cpu().numpy(), g_masked)
    close(dk, want[1])
    close(dv, want[2])


@pytest.mark.parametrize("N,d,k,dtype", [(6, 16, 2, torch.float32),
                                         (64, 16, 1, torch.float32),
                                         (300, 16, 4, torch.float32),
                                         (512, 16, 2, torch.float32),
                                         (200, 32, 8, torch.float32),
                                         (256, 16, 2, torch.bfloat16),
                                         (512, 64, 3, torch.bfloat16)])
def test_topk_autograd(tb, N, d, k, dtype):
    ops, ag = tb
    q, kt, v = (t.requires_grad_(True) for t in qkv(3, N, d, seed=N + k, dtype=dtype))
    out, idx = ag.TopkAttention.apply(q, kt, v, k)
    g = torch.randn(3, N, d, generator=torch.Generator().manual_seed(k)).cuda()
    out.backward(g.to(dtype))
    want = oracle.gather_attention_grad(host(q), host(kt), host(v),
                                        idx.long().cpu().numpy(),
                                        host(g.to(dtype)))
    for t, b in zip((q, kt, v), want):
        assert t.grad.dtype == dtype
        if dtype == torch.bfloat16:
            close(t.grad, b, rtol=2e-2, floor=2e-2)
        else:
            close(t.grad, b)


def test_dense_and_morton_autograd(tb):
    _, ag = tb
    B, N, d = 4, 200, 16
    q, k, v = (t.requires_grad_(True) for t in qkv(B, N, d, seed=21))
    g = torch.randn(B, N, d, generator=torch.Generator().manual_seed(2)).cuda()
    ag.dense_attention(q, k, v).backward(g)
    want = oracle.dense_attention_grad(host(q), host(k), host(v), host(g))
    for t, b in zip((q, k, v), want):
        close(t.grad, b)
    pos = torch.rand(B, N, 2, generator=torch.Generator().manual_seed(3)).cuda()
    q2, k2, v2 = (t.detach().clone().requires_grad_(True) for t in (q, k, v))
    out, idx = ag.MortonPrescoreAttention.apply(q2, k2, v2, pos, 2, 16)
    out.backward(g)
    np.testing.assert_array_equal(idx.cpu().numpy(),
                                  oracle.morton_window(host(pos), 2, bits=16))
    want = oracle.gather_attention_grad(host(q), host(k), host(v),
                                        idx.cpu().numpy(), host(g))
    for t, b in zip((q2, k2, v2), want):
        close(t.grad, b)


def test_strided_views_receive_gradients(tb):
    """q, k, v as chunks of one [B, N, 3d] tensor (the comm module's qkv
    output): the gradient lands in the parent tensor's three column blocks."""
    _, ag = tb
    g0 = torch.Generator().manual_seed(8)
    x = torch.randn(4, 96, 48, generator=g0).cuda().requires_grad_(True)
    q, k, v = x.chunk(3, dim=-1)
    g = torch.randn(4, 96, 16, generator=g0).cuda()
    ag.topk_attention(q, k, v, 2).backward(g)
    _, idx = ag.TopkAttention.apply(q.detach(), k.detach(), v.detach(), 2)
    want = oracle.gather_attention_grad(host(q), host(k), host(v),
                                        idx.long().cpu().numpy(), host(g))
    close(x.grad, np.concatenate(want, axis=-1))


def test_gather_backward_gradients_off_the_16_byte_grid(tb):
    """Through the C ABI with dk and dv starting 4 bytes past a 16-byte
    boundary: the kernel falls back from four-column vector reductions to
    scalar ones and returns the same gradients."""
    ops, _ = tb
    from tarmac_b200 import _lib
    B, N, d, kk = 3, 64, 16, 4
    q, k, v = qkv(B, N, d, seed=77)
    gen = torch.Generator().manual_seed(78)
    g = torch.randn(B, N, d, generator=gen).cuda()
    idx = torch.randint(0, N, (B, N, kk), generator=gen).cuda()
    want = ops.gather_attention_backward(q, k, v, g, idx)
    dq = torch.empty(B, N, d, device="cuda")
    dk_buf = torch.full((B * N * d + 4,), float("nan"), device="cuda")
    dv_buf = torch.full((B * N * d + 4,), float("nan"), device="cuda")
    dk, dv = dk_buf[1:1 + B * N * d], dv_buf[1:1 + B * N * d]
    assert dk.data_ptr() % 16 == 4
    strides = ops._strides_n(q, k, v, g)
    with ops._on(q.device):
        _lib.call("tarmac_gather_attention_backward", q.data_ptr(), k.data_ptr(),
                  v.data_ptr(), g.data_ptr(), strides, idx.data_ptr(), 1, kk, B, N,
                  d, _lib.F32, 1.0 / d ** 0.5, dq.data_ptr(), dk.data_ptr(),
                  dv.data_ptr(), ops._stream(q.device))
    torch.cuda.synchronize()
    close(dq, host(want[0]))
    close(dk.view(B, N, d), host(want[1]))
    close(dv.view(B, N, d), host(want[2]))
    assert torch.isnan(dk_buf[0]) and torch.isnan(dk_buf[-3:]).all()
