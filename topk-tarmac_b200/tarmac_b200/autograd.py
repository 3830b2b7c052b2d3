"""Differentiable attention-core operations (torch.autograd.Function).

Forward runs the sm_100a kernels of :mod:`tarmac_b200.ops`; backward runs the
gradient kernels (csrc/backward.cu) through the same C ABI. These give the
gradients autograd forms through the reference's eager path
(src/agents/mappo.py:192-231 topk_gather, 265-292 zorder_k, 361-373 dense):
the peer selection itself carries no gradient. Gradients come back in the
dtype of q.
"""

from __future__ import annotations

import torch

from . import ops


class DenseAttention(torch.autograd.Function):
    """softmax(q k^T * scale, diagonal excluded) v."""

    @staticmethod
    def forward(ctx, q, k, v, scale=None):
        out = ops.dense_attention(q, k, v, scale)
        ctx.save_for_backward(q, k, v, out)
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out = ctx.saved_tensors
        dq, dk, dv = ops.dense_attention_backward(q, k, v, out, dout, ctx.scale)
        t = q.dtype
        return dq.to(t), dk.to(t), dv.to(t), None


class TopkAttention(torch.autograd.Function):
    """Fused score-then-select top-k attention (k <= 8; "argmax" keeps the
    lowest index on a tie, "sort" the highest)."""

    @staticmethod
    def forward(ctx, q, k, v, topk, mode="argmax", scale=None):
        if topk > ops.STREAM_MAX_K or mode == "threshold":
            raise NotImplementedError(
                "gradients of top-k attention need k <= 8 and the argmax or "
                "sort tie rule (the retained set must be a list of k peers)")
        out, idx = ops.topk_attention(q, k, v, topk, mode, scale,
                                      return_indices=True)
        ctx.save_for_backward(q, k, v, idx)
        ctx.scale = scale
        ctx.mark_non_differentiable(idx)
        return out, idx

    @staticmethod
    def backward(ctx, dout, _didx):
        q, k, v, idx = ctx.saved_tensors
        dq, dk, dv = ops.gather_attention_backward(q, k, v, dout, idx,
                                                   ctx.scale)
        t = q.dtype
        return dq.to(t), dk.to(t), dv.to(t), None, None, None


class PrescoreAttention(torch.autograd.Function):
    """Attention over the given peers idx ([B, N, kk])."""

    @staticmethod
    def forward(ctx, q, k, v, idx, scale=None):
        out = ops.prescore_attention(q, k, v, idx, scale)
        ctx.save_for_backward(q, k, v, idx)
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, idx = ctx.saved_tensors
        dq, dk, dv = ops.gather_attention_backward(q, k, v, dout, idx,
                                                   ctx.scale)
        t = q.dtype
        return dq.to(t), dk.to(t), dv.to(t), None, None


class MortonPrescoreAttention(torch.autograd.Function):
    """Fused Z-order window selection + attention over the selected peers."""

    @staticmethod
    def forward(ctx, q, k, v, pos, topk, bits=10, scale=None):
        out, idx = ops.morton_prescore_attention(q, k, v, pos, topk, bits,
                                                 scale, return_indices=True)
        ctx.save_for_backward(q, k, v, idx)
        ctx.scale = scale
        ctx.mark_non_differentiable(idx)
        return out, idx

    @staticmethod
    def backward(ctx, dout, _didx):
        q, k, v, idx = ctx.saved_tensors
        dq, dk, dv = ops.gather_attention_backward(q, k, v, dout, idx,
                                                   ctx.scale)
        t = q.dtype
        return dq.to(t), dk.to(t), dv.to(t), None, None, None, None


def _needs_grad(*ts) -> bool:
    return torch.is_grad_enabled() and any(t.requires_grad for t in ts)


# The functions below take the differentiable form only when autograd will
# need it; otherwise they call the forward kernels directly (same results).

def dense_attention(q, k, v, scale=None):
    if _needs_grad(q, k, v):
        return DenseAttention.apply(q, k, v, scale)
    return ops.dense_attention(q, k, v, scale)


def topk_attention(q, k, v, topk, mode="argmax", scale=None):
    if _needs_grad(q, k, v):
        return TopkAttention.apply(q, k, v, topk, mode, scale)[0]
    return ops.topk_attention(q, k, v, topk, mode, scale)


def prescore_attention(q, k, v, idx, scale=None):
    if _needs_grad(q, k, v):
        return PrescoreAttention.apply(q, k, v, idx, scale)
    return ops.prescore_attention(q, k, v, idx, scale)


def morton_prescore_attention(q, k, v, pos, topk, bits=10, scale=None):
    if _needs_grad(q, k, v):
        return MortonPrescoreAttention.apply(q, k, v, pos, topk, bits,
                                             scale)[0]
    return ops.morton_prescore_attention(q, k, v, pos, topk, bits, scale)
