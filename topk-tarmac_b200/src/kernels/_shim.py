"""Launch-form shims for the reference's private kernel objects.

Harness scripts of the reference launch Triton kernels directly, e.g.
``fta._fused_topk_tiled_kernel[grid](q, k, v, o, *12 strides, N, scale,
TOPK=..., BLOCK_M=..., ...)`` (scripts/bench_precision.py:115-125,
scripts/autotune_kernels.py:87-119). :class:`KernelShim` gives that call form
to the CUDA kernels: ``shim[grid]`` returns a callable that maps the
positional tensors, strides and keyword meta-parameters onto the C ABI. Tile
meta-parameters (BLOCK_*, num_warps, num_stages) are accepted and ignored —
the CUDA kernels choose their own tiling. No Triton is involved.
"""

from __future__ import annotations

from typing import Callable

import torch

_TILE_KEYS = {"BLOCK_M", "BLOCK_N", "BLOCK_KN", "BLOCK_D", "BLOCK_DC",
              "BLOCK_K", "HEAD_D", "KP", "num_warps", "num_stages",
              "PRECISION", "BITONIC", "EARLY_EXIT", "WRITE_IDX", "BISECT"}


def as_view(t: torch.Tensor, shape, strides) -> torch.Tensor:
    """``t`` re-viewed with the [B, N, d] shape and element strides given by
    the caller of a launch-form kernel."""
    return t.as_strided(shape, strides)


class KernelShim:
    """``kernel[grid](*args, **meta)`` call form over a Python launcher.

    ``launch(args, meta)`` receives the positional arguments and the
    keyword meta-parameters (tile keys removed) and performs the work.
    """

    def __init__(self, name: str, launch: Callable):
        self.__name__ = name
        self._launch = launch

    def __getitem__(self, grid):
        def run(*args, **meta):
            meta = {k: v for k, v in meta.items() if k not in _TILE_KEYS or
                    k in ("HEAD_D", "PRECISION", "BISECT", "WRITE_IDX")}
            return self._launch(args, meta)
        return run

    def __repr__(self) -> str:
        return f"<tarmac_b200 kernel shim {self.__name__}>"
