"""Select-before-scoring — drop-in for the reference module
``src/kernels/prescore_selection.py`` (MHHamdan/TopK-TarMAC).

On the sm_100a kernels of ``tarmac_b200``:

``_morton_code(pos, bits=10)``     per-episode Morton codes (lines 51-68)
``select_morton_window(pos, k)``   Z-order window peers (lines 71-84); the
                                   curve order is the stable one (equal codes
                                   keep agent-index order), the deterministic
                                   member of the reference's unstable argsort
``prescore_attention(q,k,v,idx)``  attention over the given peers (184-195)
``prescore_full(...)``             selector + attention; ``morton_window`` runs
                                   as one fused kernel (198-200)

``select_radius_knn(pos, k)``      exact k nearest peers (lines 35-42)
``select_grid_knn(pos, k)``        grid kNN with the reference's sizing and
                                   capacity (lines 87-164); the cell order is
                                   the stable one
``grid_knn_recall(pos, k)``        membership recall of the grid selector
                                   (lines 167-172)
``analytic_flops(...)``            the selector cost ledger, delegated to the
                                   reference's ``src.analysis.selector_costs``
                                   as the reference does (lines 203-212)
"""

from __future__ import annotations

import torch

from tarmac_b200 import ops

MORTON_BITS = 10  # the reference's _morton_code default


def _spread_bits(v: torch.Tensor) -> torch.Tensor:
    """Insert a zero between consecutive bits of values below 2^16
    (prescore_selection.py:51-59); elementwise torch on the input's device,
    kept for callers of the private helper."""
    for shift, mask in ((8, 0x00FF00FF), (4, 0x0F0F0F0F), (2, 0x33333333),
                        (1, 0x55555555)):
        v = (v | (v << shift)) & mask
    return v


def _morton_code(pos: torch.Tensor, bits: int = MORTON_BITS) -> torch.Tensor:
    """Interleave the bits of quantised 2-D coordinates. pos: (B, N, 2)."""
    return ops.morton_code(pos, bits)


def select_morton_window(pos: torch.Tensor, k: int,
                         bits: int = MORTON_BITS) -> torch.Tensor:
    """k peers adjacent along a Z-order curve, int64 (B, N, k)."""
    return ops.morton_select(pos, k, bits)


def select_radius_knn(pos: torch.Tensor, k: int) -> torch.Tensor:
    """k spatially nearest peers per agent, int64 (B, N, k)
    (prescore_selection.py:35-42): squared distances in fp32, self excluded,
    peers by increasing (distance, index)."""
    return ops.knn_select(pos, k)


def grid_knn_shape(N: int, k: int) -> tuple[int, int]:
    """Grid side G and per-cell capacity M (prescore_selection.py:87-101):
    cells sized for about max(2, k) agents, capacity mean + 3 sd + 2."""
    occ = max(2, k)
    G = max(1, int((N / occ) ** 0.5))
    mean = N / (G * G)
    return G, int(mean + 3 * mean ** 0.5 + 2)


def select_grid_knn(pos: torch.Tensor, k: int) -> torch.Tensor:
    """k nearest peers among the 3x3 grid cells around each agent
    (prescore_selection.py:107-164): the reference's grid and capacity, cells
    sorted stably, the exact selector where the neighbourhood would hold N or
    more candidates."""
    return ops.grid_knn_select(pos, k)


def grid_knn_recall(pos: torch.Tensor, k: int) -> float:
    """Fraction of retained peers that exact kNN would also retain
    (prescore_selection.py:167-172)."""
    got = select_grid_knn(pos, k)
    ref = select_radius_knn(pos, k)
    hit = (got.unsqueeze(-1) == ref.unsqueeze(-2)).any(-1)
    return hit.float().mean().item()


def analytic_flops(selector: str, B: int, N: int, d: int, kk: int) -> dict:
    """Partial scalar charge of a selector plus its attention (not an
    executed FLOP count), as the reference defines it
    (prescore_selection.py:203-212): a delegation to the reference's
    ``src.analysis.selector_costs.partial_counts``. The ledger is analytic
    bookkeeping, not part of the attention core, so this build does not
    carry it; once these modules sit in the reference tree (the merge the
    integration notes describe) the import resolves and the call returns the
    reference's own dict. Without that tree it raises NotImplementedError."""
    try:
        from src.analysis.selector_costs import partial_counts
    except ImportError as e:
        raise NotImplementedError(
            "analytic_flops needs the reference's src.analysis.selector_costs "
            "(merge these modules into the reference tree)") from e
    return partial_counts(selector, B, N, d, kk)


SELECTORS = {"radius_knn": select_radius_knn,
             "grid_knn": select_grid_knn,
             "morton_window": select_morton_window}


def prescore_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       idx: torch.Tensor) -> torch.Tensor:
    """Score only the retained pairs. q,k,v: (B,N,d); idx: (B,N,kk)."""
    return ops.prescore_attention(q, k, v, idx)


def prescore_full(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                  pos: torch.Tensor, kk: int, selector: str) -> torch.Tensor:
    if selector == "morton_window":
        return ops.morton_prescore_attention(q, k, v, pos, kk, MORTON_BITS)
    return prescore_attention(q, k, v, SELECTORS[selector](pos, kk))
