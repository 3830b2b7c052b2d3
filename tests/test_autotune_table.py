"""This build's tuned-configuration table (topk-tarmac_b200/results/
autotune_b200.json, written on a B200 by tarmac_b200/autotune.py) in the
reference's wire format (results/autotune*.json rows, read back by
src/kernels/streaming_topk_attention.py:186-203): every row is well formed
and names the kernel and tiling that the library's dispatch chooses for that
shape today (tarmac_kernel_plan, host-only, no GPU needed)."""

from __future__ import annotations

import json

import pytest
import torch

from tarmac_b200 import TarmacError, autotune, ops


@pytest.fixture(scope="module")
def table():
    return json.loads(autotune.DEFAULT_TABLE.read_text())


def test_rows_have_the_wire_format(table):
    assert table["rows"]
    for r in table["rows"]:
        assert r["kind"] in ("dense", "topk", "streaming")
        for key in ("head_dim", "n_agents", "batch", "best", "n_configs", "n_ran", "all"):
            assert key in r
        assert ("k" in r) == (r["kind"] != "dense")
        best = r["best"]
        assert best["name"] == best["cfg"]["kernel"]
        assert best["ms"] > 0
        assert r["n_configs"] == r["n_ran"] == 1 and r["all"] == [best]


def test_table_covers_the_grid(table):
    keys = {autotune.key_of(r) for r in table["rows"]}
    assert keys == {autotune.key_of(r) for r in autotune.grid()}


def test_rows_name_the_current_dispatch(table):
    for r in table["rows"]:
        assert autotune.plan_of(r) == r["best"]["cfg"], autotune.key_of(r)


def test_load_table_indexes_rows():
    t = autotune.load_table()
    row = t[("topk", "fp32", 16, 512, 2, 1024)]
    assert row["best"]["name"] == "topk_ws"
    assert row["best"]["cfg"]["chunks_kept"] == 2


@pytest.mark.parametrize("op,B,N,d,dt,k,want", [
    ("topk", 1024, 512, 16, torch.float32, 2, "topk_ws"),
    ("topk", 256, 512, 16, torch.float32, 2, "topk_tc"),
    ("topk", 1024, 32, 16, torch.float32, 2, "topk_small"),
    ("topk", 1024, 512, 24, torch.float32, 2, "topk_chunk"),
    ("topk", 64, 100, 16, torch.float32, 12, "topk_rows"),
    ("streaming", 256, 1024, 16, torch.bfloat16, 4, "topk_tc"),
    ("dense", 4096, 512, 64, torch.bfloat16, 1, "dense_ws"),
    ("dense", 1024, 512, 16, torch.float32, 1, "dense_tc_f32"),
    ("dense", 64, 40, 16, torch.float32, 1, "dense_ffma")])
def test_kernel_plan_by_shape(op, B, N, d, dt, k, want):
    assert ops.kernel_plan(op, B, N, d, dt, k=k)["kernel"] == want


def test_kernel_plan_rejects_what_the_call_rejects():
    with pytest.raises(TarmacError):
        ops.kernel_plan("topk", 4, 8, 16, torch.float32, k=8)     # k > N - 1
    with pytest.raises(TarmacError):
        ops.kernel_plan("streaming", 4, 64, 16, torch.float32, k=9)  # streaming k <= 8
    with pytest.raises(TarmacError):
        ops.kernel_plan("dense", 4, 1, 16, torch.float32)          # N < 2
