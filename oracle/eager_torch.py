"""The reference's eager PyTorch attention core, restated for CPU timing.

TEST AND MEASUREMENT INFRASTRUCTURE. Only ``tests/`` and the CPU legs of
``bench.py`` (``cpu_baseline`` and ``--impl reference``) import this module;
the product path never does.

The reference's CPU baseline is its eager path: a handful of ATen calls
(batched matmul, masked fill, ``topk``, ``softmax``, ``gather``, matmul). Its
sources cannot travel to the GPU box, so the timed baseline there is this
restatement, which issues the same ATen operations on the same shapes in the
same order, so that it costs what the reference costs on the same host
threads. Each function names the reference lines it follows:

* ``topk_gather``   reference_topk_attention
                    (src/kernels/fused_topk_attention.py:388-402; also
                    topk_gather, scripts/bench_attention_core.py:94-101)
* ``dense``         dense_unfused (scripts/bench_attention_core.py:69-75)
* ``morton_window`` _morton_code + select_morton_window
                    (src/kernels/prescore_selection.py:51-84)
* ``prescore``      prescore_attention (src/kernels/prescore_selection.py:184-195)

Numerically these are fp32 ATen arithmetic; the float64 numpy oracle
(``tarmac_oracle``) stays the parity checker.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def _masked_scores(q: torch.Tensor, k: torch.Tensor) -> torch.Tensor:
    """q k^T / sqrt(d) with the diagonal at -inf (one bmm, one masked fill)."""
    n, d = q.shape[1], q.shape[2]
    s = torch.matmul(q, k.transpose(-1, -2)) / (d ** 0.5)
    diag = torch.eye(n, dtype=torch.bool, device=q.device)[None]
    return s.masked_fill(diag, float("-inf"))


def topk_gather(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                topk: int) -> torch.Tensor:
    """Score every pair, keep ``topk`` per row (clamped to [1, N-1]), softmax
    over the kept scores, gather their V rows and contract."""
    B, N, d = q.shape
    kk = min(max(topk, 1), N - 1)
    vals, idx = _masked_scores(q, k).topk(kk, dim=-1, sorted=False)
    w = torch.softmax(vals, dim=-1)
    rows = idx.reshape(B, N * kk, 1).expand(B, N * kk, d)
    v_sel = v.gather(1, rows).view(B, N, kk, d)
    return torch.matmul(w.unsqueeze(-2), v_sel).squeeze(-2)


def dense(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
    """softmax over all peers (diagonal excluded), then P V."""
    return torch.matmul(F.softmax(_masked_scores(q, k), dim=-1), v)


def _spread(x: torch.Tensor) -> torch.Tensor:
    for sh, mask in ((16, 0x0000FFFF), (8, 0x00FF00FF), (4, 0x0F0F0F0F),
                     (2, 0x33333333), (1, 0x55555555)):
        x = (x | (x << sh)) & mask
    return x


def morton_window(pos: torch.Tensor, k: int, bits: int = 10) -> torch.Tensor:
    """Per-episode Morton codes at ``bits`` per axis, the curve order by
    argsort, and the peers at ranks r+1..r+h, r-1..r-(k-h) (mod N),
    h = (k+1)//2; int64 [B, N, k]."""
    B, N, _ = pos.shape
    lo = pos.amin(dim=1, keepdim=True)
    span = (pos.amax(dim=1, keepdim=True) - lo).clamp_min(1e-6)
    top = 2 ** bits - 1
    cell = ((pos - lo) / span * top).long().clamp_(0, top)
    code = _spread(cell[..., 0]) | (_spread(cell[..., 1]) << 1)
    order = code.argsort(dim=-1)
    rank = torch.empty_like(order)
    rank.scatter_(-1, order, torch.arange(N, device=pos.device).expand(B, N))
    h = (k + 1) // 2
    offs = torch.cat([torch.arange(1, h + 1, device=pos.device),
                      -torch.arange(1, k - h + 1, device=pos.device)])
    peer_rank = (rank.unsqueeze(-1) + offs.view(1, 1, -1)) % N
    return order.gather(1, peer_rank.reshape(B, N * k)).view(B, N, k)


def prescore(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
             idx: torch.Tensor) -> torch.Tensor:
    """Attention over the given peers only: gather K and V rows, kk scores
    per query, softmax over them, contract."""
    B, N, d = q.shape
    kk = idx.shape[-1]
    rows = idx.reshape(B, N * kk, 1).expand(B, N * kk, d)
    k_sel = k.gather(1, rows).view(B, N, kk, d)
    v_sel = v.gather(1, rows).view(B, N, kk, d)
    s = torch.matmul(q.unsqueeze(-2), k_sel.transpose(-1, -2)) / (d ** 0.5)
    return torch.matmul(F.softmax(s, dim=-1), v_sel).squeeze(-2)
