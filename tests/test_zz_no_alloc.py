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


def _reject_status(so, B, N):
    t = torch.zeros(1, 2, 16, device="cuda")
    st = _strides(t, t, t, t, t)
    return so.tarmac_dense_attention_backward_noalloc(
        t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(),
        ctypes.addressof(st), B, N, 16, 0, 0.25, t.data_ptr(),
        t.data_ptr(), t.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_noalloc_rejects_problems_beyond_its_scratch():
    from tarmac_b200 import _lib
    so = _lib.lib()
    # 2 * B * N floats exceed the 4 MiB array: rejected before any launch
    # (the pointers are never dereferenced)
    for B, N in ((1024, 1024), (3, 174763)):       # 2^20 and 2^19 + 1 rows
        status = _reject_status(so, B, N)
        assert status == _lib.ERR_SCRATCH
        assert b"scratch" in so.tarmac_strerror(status)


def test_noalloc_at_its_limit_allocates_nothing():
    """B * N = 2^19 query rows, which fills the whole array, matches the
    regular entry point; a warmed call changes neither torch's allocated
    bytes nor the device's free memory."""
    from tarmac_b200 import _lib, ops
    so = _lib.lib()
    B, N, d = 4096, 128, 8
    q, k, v = qkv(B, N, d, seed=19)
    g = torch.randn(B, N, d, generator=torch.Generator().manual_seed(3)).cuda()
    out = ops.dense_attention(q, k, v)
    want = _grads(so, "tarmac_dense_attention_backward", q, k, v, out, g, True)
    got = _grads(so, "tarmac_dense_attention_backward_noalloc", q, k, v, out,
                 g, False)
    for a, b in zip(got, want):
        a, b = a.cpu().numpy(), b.cpu().numpy()
        np.testing.assert_allclose(a, b, rtol=1e-4,
                                   atol=1e-5 * max(1.0, np.abs(b).max()))
    dq, dk, dv = got
    st = _strides(q, k, v, out, g)
    torch.cuda.synchronize()
    alloc0 = torch.cuda.memory_allocated()
    free0, _ = torch.cuda.mem_get_info()
    status = so.tarmac_dense_attention_backward_noalloc(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(),
        g.data_ptr(), ctypes.addressof(st), B, N, d, 0, 1.0 / d ** 0.5,
        dq.data_ptr(), dk.data_ptr(), dv.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert status == 0, so.tarmac_strerror(status)
    assert torch.cuda.memory_allocated() == alloc0
    assert torch.cuda.mem_get_info()[0] == free0


# Runs in a fresh process with no torch: the driver API makes a second
# context current on the same device, in which the library's module (and so
# its scratch array) lives at another address than in the primary context.
_CONTEXT_SCRIPT = r"""
import ctypes, importlib.util, sys
from ctypes import byref, c_int, c_size_t, c_uint64, c_void_p
import numpy as np

spec = importlib.util.spec_from_file_location("tarmac_lib", sys.argv[1])
tl = importlib.util.module_from_spec(spec)
spec.loader.exec_module(tl)
so = tl.lib()
cu = ctypes.CDLL("libcuda.so.1")

def ck(r, what):
    if r != 0:
        raise SystemExit(f"{what} returned {r}")

# device pointers are kept as Python ints and passed to the driver as
# 64-bit values (the library's own argtypes take them as c_void_p)
def dev_buf(a):
    p = c_uint64()
    ck(cu.cuMemAlloc_v2(byref(p), c_size_t(max(a.nbytes, 4))), "cuMemAlloc")
    ck(cu.cuMemcpyHtoD_v2(p, a.ctypes.data_as(c_void_p), c_size_t(a.nbytes)),
       "cuMemcpyHtoD")
    return p.value

def host(p, shape):
    a = np.empty(shape, np.float32)
    ck(cu.cuMemcpyDtoH_v2(a.ctypes.data_as(c_void_p), c_uint64(p),
                          c_size_t(a.nbytes)), "cuMemcpyDtoH")
    return a

def run(seed):
    B, N, d = 6, 200, 16
    rng = np.random.default_rng(seed)
    q, k, v, g = (rng.standard_normal((B, N, d)).astype(np.float32)
                  for _ in range(4))
    zeros = np.zeros((B, N, d), np.float32)
    bq, bk, bv, bg = (dev_buf(x) for x in (q, k, v, g))
    bo, dq0, dk0, dv0, dq1, dk1, dv1 = (dev_buf(zeros) for _ in range(7))
    work = dev_buf(np.zeros((2, B, N), np.float32))
    sc = 1.0 / d ** 0.5
    ck(so.tarmac_dense_attention(bq, bk, bv, bo, None, B, N, d, 0, sc, None),
       "dense forward")
    ck(so.tarmac_dense_attention_backward(bq, bk, bv, bo, bg, None, B, N, d,
                                          0, sc, dq0, dk0, dv0, work, None),
       "backward")
    free = []
    for _ in range(2):                      # two calls in a row
        f, t = c_size_t(), c_size_t()
        ck(cu.cuMemGetInfo_v2(byref(f), byref(t)), "cuMemGetInfo")
        free.append(f.value)
        ck(so.tarmac_dense_attention_backward_noalloc(
            bq, bk, bv, bo, bg, None, B, N, d, 0, sc, dq1, dk1, dv1, None),
           "backward_noalloc")
        ck(cu.cuCtxSynchronize(), "cuCtxSynchronize")
        for p0, p1 in ((dq0, dq1), (dk0, dk1), (dv0, dv1)):
            a, b = host(p1, (B, N, d)), host(p0, (B, N, d))
            np.testing.assert_allclose(a, b, rtol=1e-4,
                                       atol=1e-5 * max(1.0, np.abs(b).max()))
    f, t = c_size_t(), c_size_t()
    ck(cu.cuMemGetInfo_v2(byref(f), byref(t)), "cuMemGetInfo")
    assert free[1] == f.value, (free, f.value)  # the warmed call allocated nothing
    for p in (bq, bk, bv, bg, bo, dq0, dk0, dv0, dq1, dk1, dv1, work):
        ck(cu.cuMemFree_v2(c_uint64(p)), "cuMemFree")

ck(cu.cuInit(0), "cuInit")
dev = c_int()
ck(cu.cuDeviceGet(byref(dev), 0), "cuDeviceGet")
primary = c_void_p()
ck(cu.cuDevicePrimaryCtxRetain(byref(primary), dev), "cuDevicePrimaryCtxRetain")
ck(cu.cuCtxSetCurrent(primary), "cuCtxSetCurrent")
run(1)                                      # primary context
other = c_void_p()
ck(cu.cuCtxCreate_v2(byref(other), 0, dev), "cuCtxCreate")   # now current
run(2)                                      # a second context on the device
ck(cu.cuCtxDestroy_v2(other), "cuCtxDestroy")
ck(cu.cuCtxSetCurrent(primary), "cuCtxSetCurrent")
run(3)                                      # back in the primary context
ck(cu.cuDevicePrimaryCtxRelease_v2(dev), "cuDevicePrimaryCtxRelease")
print("contexts ok")
"""


def test_noalloc_follows_the_current_context():
    """The scratch array's device address belongs to a CUDA context. A caller
    that makes its own context current through the driver API gets the
    array's address in that context, not the one cached in the first:
    results match the regular entry point in the primary context, in a
    second context on the same device, and back in the primary one."""
    import subprocess
    import sys
    from pathlib import Path

    from tarmac_b200 import _lib
    lib_py = Path(_lib.__file__).resolve()
    r = subprocess.run([sys.executable, "-c", _CONTEXT_SCRIPT, str(lib_py)],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "contexts ok" in r.stdout
