"""Host-side logic of the drop-in modules, without a GPU: reference
signatures, clamping and assertions, error behaviour (no CPU fallback), the
launch-form shims and the tuned-table reader."""

from __future__ import annotations

import inspect

import pytest
import torch

import oracle

from src.agents import mappo
from src.kernels import fused_dense_attention as fda
from src.kernels import fused_prescore_attention as fpa
from src.kernels import fused_topk_attention as fta
from src.kernels import prescore_selection as ps
from src.kernels import streaming_topk_attention as sta


def test_signatures_match_reference_parameters():
    want = {
        fta.fused_topk_attention_tiled: ["q", "k", "v", "topk", "block_m",
                                         "block_dc", "num_warps", "num_stages",
                                         "precision"],
        fta.fused_topk_attention: ["q", "k", "v", "topk"],
        fta.fused_topk_attention_masked: ["q", "k", "v", "topk", "bisect"],
        fta.fused_topk_attention_sort: ["q", "k", "v", "topk", "block_m"],
        fda.fused_dense_attention: ["q", "k", "v", "block_m", "block_kn",
                                    "num_warps", "num_stages", "precision"],
        sta.streaming_topk_attention: ["q", "k", "v", "topk", "block_m",
                                       "block_n", "num_warps", "num_stages",
                                       "tuned", "bitonic", "early_exit",
                                       "precision", "return_indices"],
        fpa.fused_prescore_attention: ["q", "k", "v", "idx", "block_m"],
        ps.select_morton_window: ["pos", "k", "bits"],
        ps.prescore_attention: ["q", "k", "v", "idx"],
        ps.prescore_full: ["q", "k", "v", "pos", "kk", "selector"],
    }
    for fn, params in want.items():
        assert list(inspect.signature(fn).parameters) == params, fn.__name__


def test_next_pow2():
    for mod in (fta, fda, sta, fpa):
        assert [mod._next_pow2(x) for x in (1, 2, 3, 5, 16, 17, 1000)] == \
            [1, 2, 4, 8, 16, 32, 1024]


def test_resident_cap_and_streaming_k_assertions():
    big = torch.zeros(1, 1025, 16)
    for fn in (fta.fused_topk_attention, fta.fused_topk_attention_tiled,
               fta.fused_topk_attention_masked, fta.fused_topk_attention_sort):
        with pytest.raises(AssertionError):
            fn(big, big, big, 2)
    x = torch.zeros(1, 40, 16)
    with pytest.raises(AssertionError):
        sta.streaming_topk_attention(x, x, x, 9)


def test_cpu_tensors_fail_loudly():
    x = torch.zeros(2, 8, 16)
    with pytest.raises(RuntimeError, match="CUDA"):
        fta.fused_topk_attention_tiled(x, x, x, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        fda.fused_dense_attention(x, x, x)
    with pytest.raises(RuntimeError, match="CUDA"):
        ps.select_morton_window(torch.zeros(2, 8, 2), 2)


def test_selectors_need_cuda_and_ledger_needs_reference_tree():
    pos = torch.zeros(1, 8, 2)
    for fn in (ps.select_radius_knn, ps.select_grid_knn, ps.grid_knn_recall):
        with pytest.raises(RuntimeError, match="CUDA"):
            fn(pos, 2)
    # outside the reference tree there is no src.analysis package
    with pytest.raises(NotImplementedError):
        ps.analytic_flops("morton_window", 1, 8, 16, 2)
    assert ps.grid_knn_shape(512, 2) == (16, 8)
    assert ps.grid_knn_shape(600, 2) == oracle.grid_knn_shape(600, 2)


def test_analytic_flops_delegates_to_the_reference_ledger(monkeypatch):
    """Inside the reference tree, analytic_flops returns partial_counts'
    result unchanged (prescore_selection.py:203-212)."""
    import sys
    import types
    seen = {}

    def partial_counts(selector, B, N, d, kk):
        seen["args"] = (selector, B, N, d, kk)
        return {"selector": 1, "count_model": "stub"}

    pkg = types.ModuleType("src.analysis")
    mod = types.ModuleType("src.analysis.selector_costs")
    mod.partial_counts = partial_counts
    pkg.selector_costs = mod
    monkeypatch.setitem(sys.modules, "src.analysis", pkg)
    monkeypatch.setitem(sys.modules, "src.analysis.selector_costs", mod)
    got = ps.analytic_flops("grid_knn", 4, 64, 16, 2)
    assert got == {"selector": 1, "count_model": "stub"}
    assert seen["args"] == ("grid_knn", 4, 64, 16, 2)


def test_tuned_cfg_absent_table_is_none():
    assert sta._tuned_cfg(16, 512, 2, 256) is None


def test_attention_comm_contract_without_gpu():
    cfg = mappo.MAPPOConfig(obs_dim=36, n_actions=5, n_agents=6, hidden=32,
                            use_comm=True, msg_dim=8, attn_mode="zorder_k",
                            topk=2)
    comm = mappo.AttentionComm(cfg, in_dim=32)
    assert set(comm.state_dict()) == {"qkv.weight", "qkv.bias", "proj.weight",
                                      "proj.bias", "k_gate.weight",
                                      "k_gate.bias"}
    with pytest.raises(ValueError):
        comm(torch.randn(1, 6, 32))              # zorder_k needs positions
    comm.cfg.attn_mode = "entmax"
    with pytest.raises(NotImplementedError):
        comm(torch.randn(1, 6, 32))
    comm.cfg.attn_mode = "no_such_mode"
    with pytest.raises(ValueError):
        comm(torch.randn(1, 6, 32))
    comm.cfg.attn_mode = "topk"
    with pytest.raises(RuntimeError, match="CUDA"):
        comm(torch.randn(1, 6, 32))              # no CPU fallback


def test_launch_form_shim_maps_arguments(monkeypatch):
    seen = {}

    def fake_topk(q, k, v, topk, mode="argmax", scale=None, return_indices=False):
        seen.update(shape=tuple(q.shape), stride=q.stride(), topk=topk,
                    mode=mode, scale=scale)
        return torch.ones(q.shape)

    monkeypatch.setattr(fta.ops, "topk_attention", fake_topk)
    B, N, d = 2, 10, 16
    qkv = torch.zeros(B, N, 3 * d)
    q, k, v = qkv.chunk(3, -1)
    o = torch.zeros(B, N, d)
    strides = [*q.stride(), *k.stride(), *v.stride(), *o.stride()]
    fta._fused_topk_tiled_kernel[(1, B)](
        q, k, v, o, *strides, N, 0.25, TOPK=3, BLOCK_M=32, BLOCK_N=16,
        BLOCK_D=16, BLOCK_DC=16, HEAD_D=d, PRECISION="ieee", num_warps=4)
    assert seen == dict(shape=(B, N, d), stride=(N * 3 * d, 3 * d, 1), topk=3,
                        mode="argmax", scale=0.25)
    assert (o == 1).all()


def test_stride_buffer_layout(monkeypatch):
    """The launchers pass q, k, v, out batch and row strides as the int64[8]
    the C ABI reads (include/tarmac_b200.h): packed bytes in that order, out
    contiguous; checked on CPU with the library call captured."""
    import struct

    import torch
    from tarmac_b200 import _lib, ops

    seen = {}
    monkeypatch.setattr(_lib, "call", lambda name, *a: seen.setdefault(name, a))
    monkeypatch.setattr(ops, "_check_qkv", lambda q, k, v: (q, k, v))
    monkeypatch.setattr(ops, "_on", lambda dev: ops._SAME_DEVICE)
    monkeypatch.setattr(ops, "_stream", lambda dev: 0)
    base = torch.randn(3, 5, 3 * 8)
    q, k, v = base.chunk(3, dim=-1)              # row stride 24, batch 120
    out = ops.topk_attention(q, k, v, 2)
    assert out.is_contiguous() and out.shape == (3, 5, 8)
    args = seen["tarmac_topk_attention"]
    strides = struct.unpack("=8q", args[4])
    assert strides == (120, 24, 120, 24, 120, 24, 40, 8)
    assert args[3] == out.data_ptr() and args[0] == q.data_ptr()
    assert struct.unpack("=4q", ops._strides_n(q, out)) == (120, 24, 40, 8)
