"""Streaming exact top-k attention — drop-in for the reference module
``src/kernels/streaming_topk_attention.py`` (MHHamdan/TopK-TarMAC), running
the sm_100a streaming kernel of ``tarmac_b200`` through the C ABI.

``streaming_topk_attention`` keeps the reference's signature, clamping,
``topk <= 8`` assertion and ``return_indices`` output
(streaming_topk_attention.py:206-258). An exact tie at the k-th score keeps
the lower index (streaming_topk_attention.py:37-44). The retained indices
come back as int32 [B, N, k] in rank order (score descending, then index).

Tiling arguments and the tuned-configuration table are accepted for call
compatibility: ``_tuned_cfg`` reads the same ``results/autotune_streaming.json``
rows (``rows[].{kind, head_dim, n_agents, k, batch, best.cfg}``) when the
file is present next to this tree, but the CUDA kernel chooses its own tiles.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from tarmac_b200 import ops

from ._shim import KernelShim, as_view

_INT64_MIN = -(2 ** 63)
_INT64_MAX = 2 ** 63 - 1

_TUNED: dict | None = None


def _next_pow2(x: int) -> int:
    """Smallest power of two >= x (streaming_topk_attention.py:182-183)."""
    return 1 << (x - 1).bit_length()


def _tuned_cfg(d: int, N: int, topk: int, batch: int):
    """The tuned tiling row for (d, N, k, B) from
    ``results/autotune_streaming.json`` if that file exists beside this tree
    (same keys as streaming_topk_attention.py:191-203), else None."""
    global _TUNED
    if _TUNED is None:
        f = Path(__file__).resolve().parents[2] / "results" / "autotune_streaming.json"
        table: dict = {}
        if f.exists():
            for r in json.loads(f.read_text()).get("rows", []):
                if r.get("kind") == "streaming":
                    table[(r["head_dim"], r["n_agents"], r["k"],
                           r["batch"])] = r["best"]["cfg"]
        _TUNED = table
    return _TUNED.get((d, N, topk, batch))


def streaming_topk_attention(q: torch.Tensor, k: torch.Tensor,
                             v: torch.Tensor, topk: int,
                             block_m: int | None = None,
                             block_n: int | None = None,
                             num_warps: int | None = None,
                             num_stages: int | None = None,
                             tuned: bool = True,
                             bitonic: bool | None = None,
                             early_exit: bool | None = None,
                             precision: str = "ieee",
                             return_indices: bool = False):
    """Exact top-k attention with streamed keys. q, k, v: (B, N, d)."""
    B, N, d = q.shape
    assert k.shape == v.shape == q.shape
    topk = max(1, min(topk, N - 1))
    assert topk <= 8, "register candidate buffer is sized for small k"
    if N < 2:
        out = torch.full_like(q, float("nan"))
        if return_indices:
            return out, torch.zeros(B, N, topk, device=q.device,
                                    dtype=torch.int32)
        return out
    return ops.streaming_topk_attention(q, k, v, topk,
                                        return_indices=return_indices)


def _stream_launch(args, meta):
    q, k, v, o, idx = args[:5]
    st = args[5:17]
    N, scale = args[17], args[18]
    B = q.shape[0]
    d = meta.get("HEAD_D", q.shape[-1])
    topk = max(1, min(meta["TOPK"], N - 1))
    shape = (B, N, d)
    want_idx = bool(meta.get("WRITE_IDX", False))
    res = ops.streaming_topk_attention(as_view(q, shape, st[0:3]),
                                       as_view(k, shape, st[3:6]),
                                       as_view(v, shape, st[6:9]), topk,
                                       scale=scale, return_indices=want_idx)
    if want_idx:
        res, ix = res
        idx.view(-1)[: ix.numel()].copy_(ix.view(-1))
    as_view(o, shape, st[9:12]).copy_(res)


_streaming_topk_kernel = KernelShim("_streaming_topk_kernel", _stream_launch)
