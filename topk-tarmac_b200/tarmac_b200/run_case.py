"""Run one attention-core case on cuda:0 a few times (for profilers).

    python topk-tarmac_b200/tarmac_b200/run_case.py --op topk --B 1024 \\
        --N 512 --d 16 --k 2 --dtype bf16 --reps 3

Inputs are seeded i.i.d. N(0, 1) Q, K, V (positions U[0, 1)^2 for the
Morton ops; for the comm module, x rows of width --in_dim and its
weights with message width --d; for the gradient ops dense_bwd and
topk_bwd, an N(0, 1) dO and the forward's output or retained peers), drawn
on the CPU and copied to the device once; every repetition is one call of
the selected operation on the current stream.
Prints "ok" and the mean per-call time (CUDA events) on success.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--op", default="topk",
                    choices=("topk", "topk_sort", "topk_threshold", "stream",
                             "dense", "morton_prescore", "morton_select",
                             "prescore", "comm", "dense_bwd", "topk_bwd"))
    ap.add_argument("--B", type=int, default=1024)
    ap.add_argument("--N", type=int, default=512)
    ap.add_argument("--d", type=int, default=16)
    ap.add_argument("--k", type=int, default=2)
    ap.add_argument("--bits", type=int, default=16)
    ap.add_argument("--in_dim", type=int, default=64,
                    help="comm op: input width (d is the message width)")
    ap.add_argument("--dtype", default="fp32", choices=("fp32", "bf16"))
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--seed", type=int, default=1)
    a = ap.parse_args()

    import torch

    from tarmac_b200 import ops

    dt = torch.bfloat16 if a.dtype == "bf16" else torch.float32
    g = torch.Generator().manual_seed(a.seed)
    q, k, v = (torch.randn(a.B, a.N, a.d, generator=g).to(dt).cuda()
               for _ in range(3))
    pos = torch.rand(a.B, a.N, 2, generator=g).cuda()
    # the Z-order window indices, for the stand-alone prescore op
    widx = ops.morton_select(pos, a.k, bits=a.bits) if a.op == "prescore" else None
    # the comm module's input rows and weights (Linear-style scaling)
    if a.op == "comm":
        x = torch.randn(a.B, a.N, a.in_dim, generator=g).cuda()
        wq = (torch.randn(3 * a.d, a.in_dim, generator=g) / a.in_dim ** 0.5).cuda()
        bq = (0.1 * torch.randn(3 * a.d, generator=g)).cuda()
        wp = (torch.randn(a.d, a.d, generator=g) / a.d ** 0.5).cuda()
        bp = (0.1 * torch.randn(a.d, generator=g)).cuda()
    # gradient ops: dO and the forward's output (dense) or retained peers
    # (top-k), computed once before the timed calls
    if a.op in ("dense_bwd", "topk_bwd"):
        go = torch.randn(a.B, a.N, a.d, generator=g).to(dt).cuda()
        o_d = ops.dense_attention(q, k, v) if a.op == "dense_bwd" else None
        idx = (ops.topk_attention(q, k, v, a.k, return_indices=True)[1]
               if a.op == "topk_bwd" else None)
    calls = {
        "topk": lambda: ops.topk_attention(q, k, v, a.k),
        "topk_sort": lambda: ops.topk_attention(q, k, v, a.k, mode="sort"),
        "topk_threshold": lambda: ops.topk_attention(q, k, v, a.k,
                                                     mode="threshold"),
        "stream": lambda: ops.streaming_topk_attention(q, k, v, a.k),
        "dense": lambda: ops.dense_attention(q, k, v),
        "morton_prescore": lambda: ops.morton_prescore_attention(
            q, k, v, pos, a.k, bits=a.bits),
        "morton_select": lambda: ops.morton_select(pos, a.k, bits=a.bits),
        "prescore": lambda: ops.prescore_attention(q, k, v, widx),
        "comm": lambda: ops.comm_forward(x, wq, bq, wp, bp, a.k),
        "dense_bwd": lambda: ops.dense_attention_backward(q, k, v, o_d, go),
        "topk_bwd": lambda: ops.gather_attention_backward(q, k, v, go, idx),
    }
    fn = calls[a.op]
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.reps):
        fn()
    e1.record()
    e1.synchronize()
    print(f"ok {a.op} B={a.B} N={a.N} d={a.d} k={a.k} {a.dtype}: "
          f"{1e3 * e0.elapsed_time(e1) / max(1, a.reps):.2f} us per call")
    return 0


if __name__ == "__main__":
    sys.exit(main())
