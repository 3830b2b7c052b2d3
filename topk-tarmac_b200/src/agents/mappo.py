"""Attention-communication module — drop-in for the attention-core part of the
reference module ``src/agents/mappo.py`` (MHHamdan/TopK-TarMAC).

``MAPPOConfig`` and ``AttentionComm`` keep the reference's names, fields,
parameters (``qkv``, ``proj``, ``k_gate`` — so reference state dicts load)
and forward signature ``forward(x, pos=None) -> (msg, info)``
(mappo.py:31-86, 138-420). The attention core between the qkv projection and
``proj(gelu(.))`` runs on the sm_100a kernels of ``tarmac_b200``:

``dense``, ``dense_sdpa``   dense masked-diagonal attention (mappo.py:174-190,
                            361-373)
``topk``, ``topk_gather``   fused score-then-select top-k, lowest index on a
                            tie; the two modes compute the same function
                            (mappo.py:192-231, 374-382)
``zorder_k``                fused Z-order selection + attention over the
                            selected peers, 10-bit codes (mappo.py:265-292)
``random_k``                k peers uniform at random (self excluded), then
                            attention over them (mappo.py:233-263)

In inference (no gradient needed), fp32, the dense and top-k modes run the
whole module (qkv projection, attention core, GELU, output projection) as one
kernel in which Q, K and V never leave the SM. Otherwise the q, k, v chunks
of the qkv output are passed to the kernels as strided views (no copies). Training works: the attention core's backward runs the
gradient kernels (tarmac_b200.autograd), giving the gradients autograd forms
through the reference's eager path (the peer selection carries none).
Gradients of the top-k modes need k <= 8. The ``entmax`` and ``adaptive_topk``
study arms and the MAPPO actor/critic are outside this build.
The weight-based diagnostics of ``collect_info`` (attention entropy) need the
weight matrix, which the fused kernels never form; ``info`` carries
``effective_k`` where the reference reports it.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

from tarmac_b200 import autograd as tgrad
from tarmac_b200 import ops

#: Slice of a simple_spread observation holding the agent's own position
#: (mappo.py:24-28).
SELF_POS = slice(2, 4)
MORTON_BITS = 10


@dataclass
class MAPPOConfig:
    obs_dim: int
    n_actions: int
    n_agents: int
    hidden: int = 64
    use_orthogonal_init: bool = True
    use_comm: bool = False
    msg_dim: int = 16
    n_heads: int = 1
    attn_mode: str = "dense"
    topk: int = 0
    entmax_alpha: float = 1.5


def _ortho_init(layer: nn.Linear, gain: float = float(np.sqrt(2.0))) -> None:
    nn.init.orthogonal_(layer.weight, gain=gain)
    nn.init.zeros_(layer.bias)


class AttentionComm(nn.Module):
    """Inter-agent attention communication block: (B, N, D_in) -> (B, N, msg_dim)."""

    _MODES = ("dense", "dense_sdpa", "topk", "topk_gather", "zorder_k",
              "random_k")

    def __init__(self, cfg: MAPPOConfig, in_dim: int) -> None:
        super().__init__()
        self.cfg = cfg
        self.collect_info = True
        self.qkv = nn.Linear(in_dim, 3 * cfg.msg_dim)
        self.proj = nn.Linear(cfg.msg_dim, cfg.msg_dim)
        self.k_bins = max(cfg.n_agents - 1, 1)
        self.k_gate = nn.Linear(in_dim, self.k_bins)
        if cfg.use_orthogonal_init:
            for layer in (self.qkv, self.proj, self.k_gate):
                _ortho_init(layer)

    def _k_eff(self, N: int) -> int:
        return min(max(self.cfg.topk, 1), N - 1)

    #: largest episode the fused module kernel takes (its K and V rows sit in
    #: shared memory)
    FUSED_MAX_N = 1024

    def _fused_ok(self, x: torch.Tensor, mode: str, N: int) -> bool:
        if torch.is_grad_enabled() and (
                x.requires_grad or any(p.requires_grad for p in self.parameters())):
            return False
        if mode not in ("dense", "dense_sdpa", "topk", "topk_gather"):
            return False
        if mode in ("topk", "topk_gather") and self._k_eff(N) > 8:
            return False
        m, D = self.cfg.msg_dim, x.shape[-1]
        return (x.is_cuda and x.dtype == torch.float32 and 2 <= N and
                m <= 64 and D <= 256 and N * m <= 16384 and N <= self.FUSED_MAX_N)

    def forward(self, x: torch.Tensor,
                pos: torch.Tensor | None = None) -> tuple[torch.Tensor, dict]:
        B, N, _ = x.shape
        mode = self.cfg.attn_mode
        if mode not in self._MODES:
            if mode in ("entmax", "adaptive_topk"):
                raise NotImplementedError(
                    f"attn_mode={mode!r} is outside the tarmac_b200 build")
            raise ValueError(f"unknown attn_mode {mode!r}")
        info: dict = {}
        if self._fused_ok(x, mode, N):
            # inference: the whole module (qkv, core, gelu, proj) is one kernel
            k_eff = 0 if mode in ("dense", "dense_sdpa") else self._k_eff(N)
            if k_eff:
                info["effective_k"] = float(k_eff)
            return ops.comm_forward(x, self.qkv.weight, self.qkv.bias,
                                    self.proj.weight, self.proj.bias,
                                    k_eff), info
        q, k, v = self.qkv(x).chunk(3, dim=-1)
        if mode == "zorder_k":
            if pos is None:
                raise ValueError("attn_mode='zorder_k' needs agent positions")
            k_eff = self._k_eff(N)
            msg = tgrad.morton_prescore_attention(q, k, v, pos.float(), k_eff,
                                                  MORTON_BITS)
            info["effective_k"] = float(k_eff)
        elif mode in ("dense", "dense_sdpa"):
            msg = tgrad.dense_attention(q, k, v)
        elif mode == "random_k":
            # k peers uniform at random, self excluded (mappo.py:233-263);
            # same gather-path aggregation as topk_gather
            k_eff = self._k_eff(N)
            idx = ops.random_select(B, N, k_eff, x.device)
            msg = tgrad.prescore_attention(q, k, v, idx)
            info["effective_k"] = float(k_eff)
        else:
            k_eff = self._k_eff(N)
            msg = tgrad.topk_attention(q, k, v, k_eff, "argmax")
            info["effective_k"] = float(k_eff)
        return self.proj(F.gelu(msg)), info
