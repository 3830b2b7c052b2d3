"""Dense masked-diagonal attention — drop-in for the reference module
``src/kernels/fused_dense_attention.py`` (MHHamdan/TopK-TarMAC), running the
sm_100a dense kernel of ``tarmac_b200`` through the C ABI.

``fused_dense_attention`` keeps the reference's signature
(fused_dense_attention.py:106-111). Tile arguments (``block_m``,
``block_kn``, ``num_warps``, ``num_stages``) are accepted and ignored: the
CUDA kernel picks its own tiling. Scores are always IEEE fp32 (``precision``
is accepted for call compatibility only).
"""

from __future__ import annotations

import torch

from tarmac_b200 import ops

from ._shim import KernelShim, as_view


def _next_pow2(x: int) -> int:
    """Smallest power of two >= x (fused_dense_attention.py:102-103)."""
    return 1 << (x - 1).bit_length()


def fused_dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                          block_m: int | None = None,
                          block_kn: int | None = None,
                          num_warps: int | None = None,
                          num_stages: int | None = None,
                          precision: str = "ieee") -> torch.Tensor:
    """Streaming dense self-attention with the diagonal masked."""
    return ops.dense_attention(q, k, v)


def _dense_launch(args, meta):
    q, k, v, o = args[:4]
    st = args[4:16]
    N, scale = args[16], args[17]
    B = q.shape[0]
    d = meta.get("HEAD_D", q.shape[-1])
    shape = (B, N, d)
    res = ops.dense_attention(as_view(q, shape, st[0:3]),
                              as_view(k, shape, st[3:6]),
                              as_view(v, shape, st[6:9]), scale=scale)
    as_view(o, shape, st[9:12]).copy_(res)


_flash_dense_kernel = KernelShim("_flash_dense_kernel", _dense_launch)
