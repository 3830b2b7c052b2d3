"""Attention over a pre-chosen peer set — drop-in for the reference module
``src/kernels/fused_prescore_attention.py`` (MHHamdan/TopK-TarMAC), running
the sm_100a prescore kernel of ``tarmac_b200`` through the C ABI.

``fused_prescore_attention(q, k, v, idx, block_m=None)`` keeps the reference
signature (fused_prescore_attention.py:88-90): idx is (B, N, kk) int64 or
int32, walked in order with an online softmax; nothing intermediate is
written. ``block_m`` is accepted and ignored. A row naming a peer outside
[0, N) is returned as NaN instead of reading out of bounds.
"""

from __future__ import annotations

import torch

from tarmac_b200 import ops

from ._shim import KernelShim, as_view


def _next_pow2(x: int) -> int:
    """Smallest power of two >= x (fused_prescore_attention.py:84-85)."""
    return 1 << (x - 1).bit_length()


def fused_prescore_attention(q: torch.Tensor, k: torch.Tensor,
                             v: torch.Tensor, idx: torch.Tensor,
                             block_m: int | None = None) -> torch.Tensor:
    """Attention over the peers named by ``idx``. q, k, v: (B, N, d)."""
    return ops.prescore_attention(q, k, v, idx)


def _prescore_launch(args, meta):
    q, k, v, idx, o = args[:5]
    st = args[5:20]
    N, scale = args[20], args[21]
    B = q.shape[0]
    d = meta.get("HEAD_D", q.shape[-1])
    kk = meta["KK"]
    shape = (B, N, d)
    iv = idx.as_strided((B, N, kk), st[9:12])
    res = ops.prescore_attention(as_view(q, shape, st[0:3]),
                                 as_view(k, shape, st[3:6]),
                                 as_view(v, shape, st[6:9]), iv, scale=scale)
    as_view(o, shape, st[12:15]).copy_(res)


_fused_prescore_kernel = KernelShim("_fused_prescore_kernel", _prescore_launch)
