"""The no-allocation entry point tarmac_dense_attention_backward_noalloc.

It serves callers that cannot allocate device memory (a host memory manager
owns every device allocation, or a running loop must not allocate because an
allocation can synchronise the device): it returns the same dense-attention
gradients as tarmac_dense_attention_backward while keeping the row
statistics in the library's fixed device array instead of a caller
workspace. Called here through the C ABI (ctypes), against the regular entry
point, on two calls in a row (the second reuses the array the first left
behind). This file is collected last.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from _parity import qkv

pytestmark = pytest.mark.gpu


def _strides(*ts):
    vals = []
    for t in ts:
        vals += [t.stride(0), t.stride(1)]
    return (ctypes.c_int64 * len(vals))(*vals)


def _grads(so, fn, q, k, v, out, g, with_work):
    B, N, d = q.shape
    assert q.dtype == k.dtype == v.dtype == out.dtype == g.dtype
    dq, dk, dv = (torch.empty(B, N, d, device="cuda") for _ in range(3))
    st = _strides(q, k, v, out, g)
    args = [q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
            g.data_ptr(), ctypes.addressof(st), B, N, d,
            1 if q.dtype == torch.bfloat16 else 0, 1.0 / d ** 0.5,
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr()]
    work = None
    if with_work:
        work = torch.empty(2, B, N, device="cuda")
        args.append(work.data_ptr())
    args.append(torch.cuda.current_stream().cuda_stream)
    status = getattr(so, fn)(*args)
    assert status == 0, so.tarmac_strerror(status)
    torch.cuda.synchronize()
    return dq, dk, dv


def test_noalloc_matches_regular_entry_point_twice():
    from tarmac_b200 import _lib, ops
    so = _lib.lib()
    for B, N, d, dtype in ((8, 300, 16, torch.float32),
                           (64, 128, 32, torch.bfloat16)):
        q, k, v = qkv(B, N, d, seed=B + N, dtype=dtype)
        g = torch.randn(B, N, d, generator=torch.Generator().manual_seed(N))
        g = g.to(dtype).cuda()      # every operand in the one declared dtype
        out = ops.dense_attention(q, k, v)
        want = _grads(so, "tarmac_dense_attention_backward", q, k, v, out, g,
                      True)
        got = _grads(so, "tarmac_dense_attention_backward_noalloc", q, k, v,
                     out, g, False)
        for a, b in zip(got, want):
            a, b = a.cpu().numpy(), b.cpu().numpy()
            np.testing.assert_allclose(a, b, rtol=1e-4,
                                       atol=1e-5 * max(1.0, np.abs(b).max()))


def test_noalloc_rejects_problems_beyond_its_scratch():
    from tarmac_b200 import _lib
    so = _lib.lib()
    t = torch.zeros(1, 2, 16, device="cuda")
    st = _strides(t, t, t, t, t)
    # 2 * B * N floats exceed the 4 MiB array: rejected before any launch
    status = so.tarmac_dense_attention_backward_noalloc(
        t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(),
        ctypes.addressof(st), 1024, 1024, 16, 0, 0.25, t.data_ptr(),
        t.data_ptr(), t.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert status == _lib.ERR_SCRATCH
    assert b"scratch" in so.tarmac_strerror(status)
