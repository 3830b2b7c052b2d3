"""GPU parity: dense attention, attention over a given peer set, Morton codes,
Z-order window selection and the fused select-before-scoring kernel, all
through the C ABI, against the CPU oracle (tolerance rtol = atol = 1e-5 fp32,
2e-2 bf16; Morton codes and selected indices bit-exact)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from _parity import host, qkv, tol_for

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    from tarmac_b200 import ops as _ops
    return _ops


@pytest.mark.parametrize("N,d", [(2, 16), (6, 16), (32, 16), (64, 16),
                                 (128, 16), (512, 16), (1000, 16), (77, 8),
                                 (128, 32), (512, 64), (100, 3), (60, 100),
                                 (33, 128)])
def test_dense_fp32(ops, N, d):
    q, k, v = qkv(8, N, d, seed=1234 + 7 * N + d)
    out = ops.dense_attention(q, k, v)
    ref = oracle.dense_attention(host(q), host(k), host(v))
    np.testing.assert_allclose(host(out), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("N,d", [(128, 16), (512, 16), (128, 64), (512, 32)])
def test_dense_bf16(ops, N, d):
    q, k, v = qkv(4, N, d, seed=7 + N, dtype=torch.bfloat16)
    out = ops.dense_attention(q, k, v)
    assert out.dtype == torch.bfloat16
    ref = oracle.dense_attention(host(q), host(k), host(v))
    np.testing.assert_allclose(host(out), ref, **tol_for(torch.bfloat16))


def test_dense_large_scores_stay_finite(ops):
    """Scores of magnitude ~100: the online softmax must stay finite and
    accurate. Any fp32 evaluation of a score carries an error up to about
    (d+2) u sum|q_c k_c| scale, which moves a weight by that much relative;
    the tolerance adds that bound times max|v| to the usual 1e-5."""
    q, k, v = qkv(2, 300, 16, seed=3)
    q = q * 40.0
    out = ops.dense_attention(q, k, v)
    qn, kn, vn = host(q), host(k), host(v)
    ref = oracle.dense_attention(qn, kn, vn)
    assert torch.isfinite(out).all()
    mag = np.einsum("bid,bjd->bij", np.abs(qn), np.abs(kn)).max() / 4.0
    ds = 2 * 18 * 2.0 ** -24 * mag
    atol = 1e-5 + 2 * ds * np.abs(vn).max()
    np.testing.assert_allclose(host(out), ref, rtol=1e-5, atol=atol)


def test_dense_golden_replay(ops, golden):
    for case in ("dense_n40", "dense_c1", "dense_n70_d32"):
        g = golden(case)
        q, k, v = (torch.from_numpy(g[x]).cuda() for x in ("q", "k", "v"))
        out = host(ops.dense_attention(q, k, v))
        np.testing.assert_allclose(out, g["eager"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("bits", [1, 4, 10, 16])
def test_morton_code_bit_exact(ops, bits):
    g = torch.Generator().manual_seed(bits)
    pos = torch.rand(64, 300, 2, generator=g)
    got = ops.morton_code(pos.cuda(), bits).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.morton_code(pos.numpy(), bits))


def test_morton_golden(ops, golden):
    g = golden("morton_n50")
    pos = torch.from_numpy(g["pos"]).cuda()
    np.testing.assert_array_equal(ops.morton_code(pos, 10).cpu().numpy(), g["code10"])
    np.testing.assert_array_equal(ops.morton_code(pos, 16).cpu().numpy(), g["code16"])
    e = golden("morton_edge")
    pe = torch.from_numpy(e["pos"]).cuda()
    for bits, key in ((10, "code10"), (16, "code16"), (4, "code4")):
        np.testing.assert_array_equal(ops.morton_code(pe, bits).cpu().numpy(), e[key])
    clean = ~g["dup10"].astype(bool)
    for kk in g["ks"]:
        kk = int(kk)
        got = ops.morton_select(pos, kk, 10).cpu().numpy()
        np.testing.assert_array_equal(got[clean], g[f"win_k{kk}"][clean])
        np.testing.assert_array_equal(got, oracle.morton_window(g["pos"], kk, 10))


@pytest.mark.parametrize("N,k,bits", [(2, 1, 16), (6, 2, 10), (64, 2, 16),
                                      (256, 2, 16), (512, 2, 16), (512, 3, 10),
                                      (1000, 4, 16), (4096, 2, 16), (37, 36, 16)])
def test_morton_window_bit_exact(ops, N, k, bits):
    g = torch.Generator().manual_seed(4242 + N)
    pos = torch.rand(16, N, 2, generator=g)
    got = ops.morton_select(pos.cuda(), k, bits).cpu().numpy()
    np.testing.assert_array_equal(got, oracle.morton_window(pos.numpy(), k, bits))


@pytest.mark.parametrize("N", [31, 32, 33, 65, 127, 129, 255, 257, 511, 512,
                               513, 1023, 1024, 1025])
def test_morton_window_sort_tiers_and_equal_codes(ops, N):
    """Episode sizes at the edges of the register-sort tiers (32 to 1024
    keys over up to 4 warps, up to 8 per lane; the shared-memory sort above
    1024), with duplicated
    positions (equal codes keep index order), a collapsed episode (every
    code 0) and a collapsed axis; selector and fused kernel both follow the
    stable order."""
    g = torch.Generator().manual_seed(N)
    pos = torch.rand(8, N, 2, generator=g)
    pos[0, N // 2:] = pos[0, : N - N // 2].clone()
    pos[1] = 0.5
    pos[2, :, 0] = 0.25
    q, kt, v = qkv(8, N, 16, seed=N + 1)
    for k, bits in ((1, 16), (2, 16), (3, 10)):
        if k >= N:
            continue
        want = oracle.morton_window(pos.numpy(), k, bits)
        got = ops.morton_select(pos.cuda(), k, bits).cpu().numpy()
        np.testing.assert_array_equal(got, want)
        out, idx = ops.morton_prescore_attention(q, kt, v, pos.cuda(), k, bits,
                                                 return_indices=True)
        np.testing.assert_array_equal(idx.cpu().numpy(), want)
        ref = oracle.prescore_attention(host(q), host(kt), host(v), want)
        np.testing.assert_allclose(host(out), ref, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("N,d,kk,itype", [(64, 16, 2, torch.int64),
                                          (512, 16, 2, torch.int32),
                                          (100, 8, 5, torch.int64),
                                          (50, 32, 3, torch.int32),
                                          (40, 64, 7, torch.int64),
                                          (33, 100, 4, torch.int64)])
def test_prescore(ops, N, d, kk, itype):
    q, k, v = qkv(16, N, d, seed=N * 977 + kk)
    g = torch.Generator().manual_seed(N)
    idx = torch.randint(0, N, (16, N, kk), generator=g)
    out = ops.prescore_attention(q, k, v, idx.to(itype).cuda())
    ref = oracle.prescore_attention(host(q), host(k), host(v), idx.numpy())
    np.testing.assert_allclose(host(out), ref, rtol=1e-5, atol=1e-5)


def test_prescore_bad_indices_give_nan_rows(ops):
    q, k, v = qkv(2, 20, 16, seed=1)
    idx = torch.tensor([[1, 2]]).repeat(2, 20, 1)
    idx[0, 4, 1] = 20
    idx[1, 7, 0] = -1
    out = ops.prescore_attention(q, k, v, idx.cuda())
    assert torch.isnan(out[0, 4]).all() and torch.isnan(out[1, 7]).all()
    mask = torch.ones(2, 20, dtype=torch.bool)
    mask[0, 4] = False
    mask[1, 7] = False
    assert torch.isfinite(out[mask.cuda()]).all()


def test_prescore_golden(ops, golden):
    g = golden("morton_n50")
    q, k, v = (torch.from_numpy(g[x]).cuda() for x in ("q", "k", "v"))
    for kk in g["ks"]:
        kk = int(kk)
        idx = torch.from_numpy(g[f"win_k{kk}"]).cuda()
        out = host(ops.prescore_attention(q, k, v, idx))
        np.testing.assert_allclose(out, g[f"prescore_k{kk}"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("N,d,k,bits,dtype", [
    (64, 16, 2, 16, torch.float32), (256, 16, 2, 16, torch.float32),
    (512, 16, 2, 16, torch.float32), (6, 16, 2, 10, torch.float32),
    (300, 32, 3, 10, torch.float32), (128, 16, 4, 16, torch.bfloat16),
    (2048, 16, 2, 16, torch.float32)])
def test_fused_morton_prescore(ops, N, d, k, bits, dtype):
    q, kt, v = qkv(16, N, d, seed=4242 + N, dtype=dtype)
    g = torch.Generator().manual_seed(N)
    pos = torch.rand(16, N, 2, generator=g)
    out, idx = ops.morton_prescore_attention(q, kt, v, pos.cuda(), k, bits,
                                             return_indices=True)
    want_idx = oracle.morton_window(pos.numpy(), k, bits)
    np.testing.assert_array_equal(idx.cpu().numpy(), want_idx)
    ref = oracle.prescore_attention(host(q), host(kt), host(v), want_idx)
    np.testing.assert_allclose(host(out), ref, **tol_for(dtype))
    # without the index output, same result
    out2 = ops.morton_prescore_attention(q, kt, v, pos.cuda(), k, bits)
    assert torch.equal(out, out2)
