"""This build's tuned-configuration table, in the reference's wire format.

The reference searches Triton tilings per shape (scripts/autotune_kernels.py)
and records the winner of each row in ``results/autotune*.json``: rows of
``{kind, head_dim, n_agents, batch[, k], best: {name, cfg, ms, deviation},
n_configs, n_ran, all}`` that ``_tuned_cfg`` and the bench harness read back
(src/kernels/streaming_topk_attention.py:186-203,
scripts/bench_attention_core.py:120-145). Here the library chooses the kernel
and its tiles from the shape (csrc/abi.cu); ``tarmac_kernel_plan`` reports
that choice. This module times the chosen kernel at each row of the bench
grids on a GPU and writes the rows in the same format, so the table records
which kernel and tiling each shape runs and how long it takes:

    python topk-tarmac_b200/tarmac_b200/autotune.py [--out PATH]

Each row's ``best.name`` is the kernel, ``best.cfg`` its tiling (the plan's
JSON object) and ``best.ms`` the device time per call (a CUDA graph of 10
calls replayed, inputs warm). ``n_configs`` is 1: there is no search, the
plan is the library's. ``deviation`` is null: parity is the test suite's job.
Rows also carry ``dtype``, which the reference's rows leave implicit (fp32).
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

DEFAULT_TABLE = Path(__file__).resolve().parents[1] / "results" / "autotune_b200.json"


def grid() -> list[dict]:
    """The rows: the bench's C2 (fp32, B=1024, N 32-1024, fused top-k k 1/2/4
    and dense), C3 (streaming top-k, B=256, N 512-1024, k 1/2/4, fp32 and
    bf16) and C5 (bf16, B 256/1024/4096, N 128/512, d 16/32/64, dense and
    top-k k 1/2) points."""
    rows = []
    for N in (32, 64, 128, 256, 512, 768, 1024):
        rows.append(dict(kind="dense", dtype="fp32", head_dim=16, n_agents=N, batch=1024))
        for k in (1, 2, 4):
            rows.append(dict(kind="topk", dtype="fp32", head_dim=16, n_agents=N,
                             batch=1024, k=k))
    for N in (512, 768, 1024):
        for dt in ("fp32", "bf16"):
            for k in (1, 2, 4):
                rows.append(dict(kind="streaming", dtype=dt, head_dim=16, n_agents=N,
                                 batch=256, k=k))
    for B in (256, 1024, 4096):
        for N in (128, 512):
            for d in (16, 32, 64):
                rows.append(dict(kind="dense", dtype="bf16", head_dim=d, n_agents=N, batch=B))
                for k in (1, 2):
                    rows.append(dict(kind="topk", dtype="bf16", head_dim=d, n_agents=N,
                                     batch=B, k=k))
    return rows


def _torch_dtype(name: str):
    import torch
    return torch.bfloat16 if name == "bf16" else torch.float32


def plan_of(row: dict) -> dict:
    """The library's kernel plan for a table row (no GPU needed)."""
    from tarmac_b200 import ops
    return ops.kernel_plan(row["kind"], row["batch"], row["n_agents"], row["head_dim"],
                           _torch_dtype(row["dtype"]), k=row.get("k", 1))


def key_of(row: dict) -> tuple:
    return (row["kind"], row["dtype"], row["head_dim"], row["n_agents"],
            row.get("k"), row["batch"])


def load_table(path: Path = DEFAULT_TABLE) -> dict:
    """{(kind, dtype, head_dim, n_agents, k, batch): row} from a table file."""
    rows = json.loads(Path(path).read_text()).get("rows", [])
    return {key_of(r): r for r in rows}


def _time_row(row: dict, dev) -> float:
    import torch
    from tarmac_b200 import ops
    B, N, d = row["batch"], row["n_agents"], row["head_dim"]
    g = torch.Generator().manual_seed(1234 + 7 * N + d)
    q, k, v = (torch.randn(B, N, d, generator=g).to(_torch_dtype(row["dtype"])).to(dev)
               for _ in range(3))
    if row["kind"] == "dense":
        fn = lambda: ops.dense_attention(q, k, v)  # noqa: E731
    elif row["kind"] == "streaming":
        fn = lambda: ops.streaming_topk_attention(q, k, v, row["k"])  # noqa: E731
    else:
        fn = lambda: ops.topk_attention(q, k, v, row["k"])  # noqa: E731
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(10):
            fn()
    graph.replay()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        graph.replay()
    e1.record()
    e1.synchronize()
    del graph
    return e0.elapsed_time(e1) / 100.0


def build_table() -> dict:
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    rows = []
    for row in grid():
        plan = plan_of(row)
        ms = _time_row(row, dev)
        best = {"name": plan["kernel"], "cfg": plan, "ms": ms, "deviation": None}
        rows.append(dict(row, best=best, n_configs=1, n_ran=1, all=[best]))
        print(json.dumps({k: rows[-1][k] for k in ("kind", "dtype", "head_dim",
                                                    "n_agents", "batch")}
                         | {"k": row.get("k"), "kernel": plan["kernel"],
                            "ms": round(ms, 5)}), flush=True)
    return {"device_name": torch.cuda.get_device_name(dev), "torch": torch.__version__,
            "note": ("kernel and tiling chosen by the library from the shape "
                     "(tarmac_kernel_plan); ms = device time per call from a CUDA "
                     "graph of 10 calls, inputs warm"),
            "rows": rows}


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--out", type=Path, default=DEFAULT_TABLE)
    a = ap.parse_args()
    table = build_table()
    a.out.parent.mkdir(parents=True, exist_ok=True)
    a.out.write_text(json.dumps(table, indent=1) + "\n")
    print(f"wrote {len(table['rows'])} rows to {a.out}", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    raise SystemExit(main())
