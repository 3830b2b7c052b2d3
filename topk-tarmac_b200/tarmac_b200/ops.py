"""Torch-facing launchers over the C ABI.

Each function takes CUDA tensors, checks them, allocates the output
(``torch.empty_like`` / ``torch.empty``; the C ABI itself never allocates) and
launches on the current stream of the tensors' device. Q, K, V are ``[B, N, d]`` fp32 or bf16 tensors
with a unit innermost stride; other strides (e.g. the ``qkv.chunk(3, -1)``
views of the comm module) are passed through without a copy. Nothing here
computes on the CPU: a CPU tensor or a missing library is an error.

The semantics are those of the reference's eager path
(src/kernels/fused_topk_attention.py:390-402): scores q.k * scale with the
diagonal excluded, softmax over the retained peers, weighted sum of V rows.
"""

from __future__ import annotations

import contextlib
import struct

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16}
_MODES = {"argmax": _lib.SELECT_ARGMAX, "threshold": _lib.SELECT_THRESHOLD,
          "sort": _lib.SELECT_SORT}

RESIDENT_MAX_N = 1024
STREAM_MAX_K = 8
MORTON_MAX_N = 4096


def default_scale(d: int) -> float:
    """1/sqrt(d), as the reference kernels pass it (fused_topk_attention.py:327)."""
    return 1.0 / (d ** 0.5)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# the raw current-stream handle without building a Stream object (falls back
# to the public call on a torch without the accessor)
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)
_SAME_DEVICE = contextlib.nullcontext()


def _index(dev: torch.device) -> int:
    """The device's ordinal (a bare "cuda" device means the current one)."""
    return torch.cuda.current_device() if dev.index is None else dev.index


def _stream(dev: torch.device) -> int:
    if _RAW_STREAM is not None:
        return _RAW_STREAM(_index(dev))
    return torch.cuda.current_stream(dev).cuda_stream


def _on(dev: torch.device):
    """Device context for a launch: the library launches on the current
    device, so switch only when the tensors live on another one."""
    if dev.index is None or dev.index == torch.cuda.current_device():
        return _SAME_DEVICE
    return torch.cuda.device(dev)


def _unit_inner(t: torch.Tensor) -> torch.Tensor:
    return t if (t.shape[-1] == 1 or t.stride(-1) == 1) else t.contiguous()


def _check_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
    if q.dim() != 3 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q, k, v must share one [B, N, d] shape; got "
                         f"{tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    if not (q.is_cuda and k.is_cuda and v.is_cuda):
        raise RuntimeError("tarmac_b200 kernels need CUDA tensors (there is no "
                           "CPU implementation)")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be on one device")
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in _DTYPES:
        raise TypeError(f"q, k, v must all be float32 or bfloat16; got "
                        f"{q.dtype}, {k.dtype}, {v.dtype}")
    return _unit_inner(q), _unit_inner(k), _unit_inner(v)


def _strides(q, k, v, o) -> bytes:
    """Batch and row strides of q, k, v, o as the int64[8] the C ABI reads.
    A bytes object passes as a pointer to its buffer and lives as long as
    the call's arguments; packing costs well under the eight-element ctypes
    array it replaces (host cost per call matters for small problems)."""
    sq, sk, sv, so = q.stride(), k.stride(), v.stride(), o.stride()
    return _PACK8(sq[0], sq[1], sk[0], sk[1], sv[0], sv[1], so[0], so[1])


_PACK8 = struct.Struct("=8q").pack
_CONTIG = torch.contiguous_format


def _empty_as(q: torch.Tensor) -> torch.Tensor:
    """A contiguous output of q's shape, dtype and device."""
    return torch.empty_like(q, memory_format=_CONTIG)


def _scale(d: int, scale: float | None) -> float:
    return default_scale(d) if scale is None else float(scale)


def dense_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                    scale: float | None = None) -> torch.Tensor:
    """softmax(q k^T * scale, diagonal excluded) v."""
    q, k, v = _check_qkv(q, k, v)
    B, N, d = q.shape
    out = _empty_as(q)
    if N < 2:
        return out.fill_(float("nan"))
    strides = _strides(q, k, v, out)
    with _on(q.device):
        _lib.call("tarmac_dense_attention", _ptr(q), _ptr(k), _ptr(v),
                  _ptr(out), strides, B, N, d,
                  _DTYPES[q.dtype], _scale(d, scale), _stream(q.device))
    return out


def topk_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   topk: int, mode: str = "argmax", scale: float | None = None,
                   return_indices: bool = False):
    """Fused score-then-select top-k attention.

    ``mode``: ``"argmax"`` (lowest index wins a tie at the k-th score),
    ``"sort"`` (highest index wins) or ``"threshold"`` (every tied peer kept).
    ``topk`` must already lie in [1, N-1]. With ``return_indices`` also returns
    the retained peers, int32 ``[B, N, topk]`` in rank order (k <= 8,
    argmax/sort only).
    """
    q, k, v = _check_qkv(q, k, v)
    B, N, d = q.shape
    if mode not in _MODES:
        raise ValueError(f"unknown selection mode {mode!r}")
    out = _empty_as(q)
    idx = (torch.empty((B, N, topk), device=q.device, dtype=torch.int32)
           if return_indices else None)
    strides = _strides(q, k, v, out)
    with _on(q.device):
        _lib.call("tarmac_topk_attention", _ptr(q), _ptr(k), _ptr(v),
                  _ptr(out), strides, B, N, d,
                  _DTYPES[q.dtype], _scale(d, scale), int(topk), _MODES[mode],
                  _ptr(idx), _stream(q.device))
    return (out, idx) if return_indices else out


def streaming_topk_attention(q: torch.Tensor, k: torch.Tensor,
                             v: torch.Tensor, topk: int,
                             scale: float | None = None,
                             return_indices: bool = False):
    """Exact top-k (k <= 8, lowest index wins a tie) with keys streamed
    through shared memory; no cap on N."""
    q, k, v = _check_qkv(q, k, v)
    B, N, d = q.shape
    out = _empty_as(q)
    idx = (torch.empty((B, N, topk), device=q.device, dtype=torch.int32)
           if return_indices else None)
    strides = _strides(q, k, v, out)
    with _on(q.device):
        _lib.call("tarmac_streaming_topk_attention", _ptr(q), _ptr(k), _ptr(v),
                  _ptr(out), strides, B, N, d,
                  _DTYPES[q.dtype], _scale(d, scale), int(topk), _ptr(idx),
                  _stream(q.device))
    return (out, idx) if return_indices else out


def prescore_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       idx: torch.Tensor,
                       scale: float | None = None) -> torch.Tensor:
    """Attention over the peers named by ``idx`` ([B, N, kk], int64 or int32).
    Rows naming a peer outside [0, N) come back as NaN."""
    q, k, v = _check_qkv(q, k, v)
    B, N, d = q.shape
    if idx.dim() != 3 or tuple(idx.shape[:2]) != (B, N):
        raise ValueError(f"idx must be [B, N, kk]; got {tuple(idx.shape)}")
    if idx.dtype not in (torch.int64, torch.int32):
        raise TypeError(f"idx must be int64 or int32; got {idx.dtype}")
    if idx.device != q.device:
        raise ValueError("idx must be on the device of q")
    idx = idx.contiguous()
    kk = idx.shape[-1]
    out = _empty_as(q)
    if kk == 0:
        return out.fill_(float("nan"))
    strides = _strides(q, k, v, out)
    with _on(q.device):
        _lib.call("tarmac_prescore_attention", _ptr(q), _ptr(k), _ptr(v),
                  _ptr(out), strides, _ptr(idx),
                  int(idx.dtype == torch.int64), kk, B, N, d,
                  _DTYPES[q.dtype], _scale(d, scale), _stream(q.device))
    return out


def _check_pos(pos: torch.Tensor) -> torch.Tensor:
    if pos.dim() != 3 or pos.shape[-1] != 2:
        raise ValueError(f"pos must be [B, N, 2]; got {tuple(pos.shape)}")
    if not pos.is_cuda:
        raise RuntimeError("tarmac_b200 kernels need CUDA tensors")
    if pos.dtype != torch.float32:
        raise TypeError(f"pos must be float32; got {pos.dtype}")
    return pos.contiguous()


def morton_code(pos: torch.Tensor, bits: int = 10) -> torch.Tensor:
    """Per-episode Morton codes, int64 [B, N]."""
    pos = _check_pos(pos)
    B, N, _ = pos.shape
    out = torch.empty((B, N), device=pos.device, dtype=torch.int64)
    with _on(pos.device):
        _lib.call("tarmac_morton_code", _ptr(pos), B, N, int(bits), _ptr(out),
                  _stream(pos.device))
    return out


def morton_select(pos: torch.Tensor, k: int, bits: int = 10) -> torch.Tensor:
    """Z-order window peers, int64 [B, N, k] (stable order on equal codes)."""
    pos = _check_pos(pos)
    B, N, _ = pos.shape
    out = torch.empty((B, N, k), device=pos.device, dtype=torch.int64)
    with _on(pos.device):
        _lib.call("tarmac_morton_select", _ptr(pos), B, N, int(k), int(bits),
                  _ptr(out), _stream(pos.device))
    return out


def morton_prescore_attention(q: torch.Tensor, k: torch.Tensor,
                              v: torch.Tensor, pos: torch.Tensor, topk: int,
                              bits: int = 10, scale: float | None = None,
                              return_indices: bool = False):
    """Fused Z-order selection + attention over the selected peers."""
    q, k, v = _check_qkv(q, k, v)
    pos = _check_pos(pos)
    B, N, d = q.shape
    if tuple(pos.shape[:2]) != (B, N):
        raise ValueError("pos must be [B, N, 2] matching q")
    out = _empty_as(q)
    idx = (torch.empty((B, N, topk), device=q.device, dtype=torch.int64)
           if return_indices else None)
    strides = _strides(q, k, v, out)
    with _on(q.device):
        _lib.call("tarmac_morton_prescore_attention", _ptr(q), _ptr(k),
                  _ptr(v), _ptr(out), strides, _ptr(pos),
                  B, N, d, _DTYPES[q.dtype], _scale(d, scale), int(topk),
                  int(bits), _ptr(idx), _stream(q.device))
    return (out, idx) if return_indices else out


# ---------------------------------------------------------------------------
# gradients (training path)
# ---------------------------------------------------------------------------

def _strides_n(*ts) -> bytes:
    vals = []
    for t in ts:
        st = t.stride()
        vals += [st[0], st[1]]
    return struct.pack(f"={len(vals)}q", *vals)


def gather_attention_backward(q: torch.Tensor, k: torch.Tensor,
                              v: torch.Tensor, dout: torch.Tensor,
                              idx: torch.Tensor, scale: float | None = None):
    """Gradients (dq, dk, dv), fp32 [B, N, d], of attention over the fixed
    peer set ``idx`` ([B, N, kk], int32 or int64): the peers a top-k call
    retained, the Morton window, or given indices. The selection carries no
    gradient. dk and dv accumulate with atomic adds (summation order not
    fixed)."""
    q, k, v = _check_qkv(q, k, v)
    dout = _unit_inner(dout)
    B, N, d = q.shape
    if dout.shape != q.shape or dout.device != q.device:
        raise ValueError("dout must match q's shape and device")
    if dout.dtype != q.dtype:
        dout = dout.to(q.dtype)
    if idx.dim() != 3 or tuple(idx.shape[:2]) != (B, N):
        raise ValueError(f"idx must be [B, N, kk]; got {tuple(idx.shape)}")
    if idx.dtype not in (torch.int64, torch.int32):
        raise TypeError(f"idx must be int64 or int32; got {idx.dtype}")
    idx = idx.contiguous()
    dq = torch.empty((B, N, d), device=q.device, dtype=torch.float32)
    dk = torch.empty_like(dq)
    dv = torch.empty_like(dq)
    strides = _strides_n(q, k, v, dout)
    with _on(q.device):
        _lib.call("tarmac_gather_attention_backward", _ptr(q), _ptr(k),
                  _ptr(v), _ptr(dout), strides, _ptr(idx),
                  int(idx.dtype == torch.int64), idx.shape[-1], B, N, d,
                  _DTYPES[q.dtype], _scale(d, scale), _ptr(dq), _ptr(dk),
                  _ptr(dv), _stream(q.device))
    return dq, dk, dv


def dense_attention_backward(q: torch.Tensor, k: torch.Tensor,
                             v: torch.Tensor, out: torch.Tensor,
                             dout: torch.Tensor, scale: float | None = None):
    """Gradients (dq, dk, dv), fp32 [B, N, d], of dense masked-diagonal
    attention given its forward output ``out``. P is recomputed, not stored;
    deterministic."""
    q, k, v = _check_qkv(q, k, v)
    out, dout = _unit_inner(out), _unit_inner(dout)
    B, N, d = q.shape
    for t, name in ((out, "out"), (dout, "dout")):
        if t.shape != q.shape or t.device != q.device:
            raise ValueError(f"{name} must match q's shape and device")
    out = out.to(q.dtype)
    dout = dout.to(q.dtype)
    dq = torch.empty((B, N, d), device=q.device, dtype=torch.float32)
    dk = torch.empty_like(dq)
    dv = torch.empty_like(dq)
    work = torch.empty((2, B, N), device=q.device, dtype=torch.float32)
    strides = _strides_n(q, k, v, out, dout)
    with _on(q.device):
        _lib.call("tarmac_dense_attention_backward", _ptr(q), _ptr(k), _ptr(v),
                  _ptr(out), _ptr(dout), strides, B, N, d,
                  _DTYPES[q.dtype], _scale(d, scale), _ptr(dq), _ptr(dk),
                  _ptr(dv), _ptr(work), _stream(q.device))
    return dq, dk, dv


# ---------------------------------------------------------------------------
# positional and random selectors
# ---------------------------------------------------------------------------

SELECT_MAX_N = 8192
SELECT_MAX_K = 32


def knn_select(pos: torch.Tensor, k: int) -> torch.Tensor:
    """Exact k nearest peers (self excluded), int64 [B, N, k], by increasing
    (distance, index)."""
    pos = _check_pos(pos)
    B, N, _ = pos.shape
    out = torch.empty((B, N, k), device=pos.device, dtype=torch.int64)
    with _on(pos.device):
        _lib.call("tarmac_knn_select", _ptr(pos), B, N, int(k), _ptr(out),
                  _stream(pos.device))
    return out


def grid_knn_select(pos: torch.Tensor, k: int) -> torch.Tensor:
    """k nearest among the 3 x 3 grid cells around each agent (the reference's
    grid sizing and per-cell capacity), int64 [B, N, k]."""
    pos = _check_pos(pos)
    B, N, _ = pos.shape
    out = torch.empty((B, N, k), device=pos.device, dtype=torch.int64)
    with _on(pos.device):
        _lib.call("tarmac_grid_knn_select", _ptr(pos), B, N, int(k),
                  _ptr(out), _stream(pos.device))
    return out


def random_select(B: int, N: int, k: int, device,
                  generator: torch.Generator | None = None) -> torch.Tensor:
    """k distinct peers per agent, uniform over the k-subsets of the other
    N - 1 agents, int64 [B, N, k]. The Philox key is drawn from ``generator``
    (torch's default CPU generator when None), so torch.manual_seed fixes
    the selection."""
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("tarmac_b200 kernels need a CUDA device")
    seed, offset = (int(x) for x in torch.randint(
        0, 2 ** 62, (2,), generator=generator))
    out = torch.empty((B, N, k), device=device, dtype=torch.int64)
    with _on(device):
        _lib.call("tarmac_random_select", int(B), int(N), int(k), seed,
                  offset, _ptr(out), _stream(device))
    return out


# ---------------------------------------------------------------------------
# the whole communication module (inference)
# ---------------------------------------------------------------------------

def comm_forward(x: torch.Tensor, w_qkv: torch.Tensor, b_qkv: torch.Tensor,
                 w_proj: torch.Tensor, b_proj: torch.Tensor,
                 topk: int) -> torch.Tensor:
    """gelu(attention(split(x W_qkv^T + b_qkv))) W_proj^T + b_proj in one
    kernel: dense attention for ``topk == 0``, else top-k (k <= 8, lowest
    index on a tie). fp32, inference only (no autograd)."""
    ts = (x, w_qkv, b_qkv, w_proj, b_proj)
    if not x.is_cuda:
        raise RuntimeError("tarmac_b200 kernels need CUDA tensors")
    if any(t.device != x.device for t in ts[1:]):
        raise ValueError("x and the comm weights must be on one device")
    if x.dim() != 3:
        raise ValueError(f"x must be [B, N, in_dim]; got {tuple(x.shape)}")
    x, w_qkv, b_qkv, w_proj, b_proj = (
        t if t.dtype == torch.float32 and t.is_contiguous()
        else t.contiguous().float() for t in ts)
    B, N, D = x.shape
    m = w_proj.shape[0]
    if w_qkv.shape != (3 * m, D) or b_qkv.shape != (3 * m,) or \
            w_proj.shape != (m, m) or b_proj.shape != (m,):
        raise ValueError("weights must be qkv [3m, in_dim], [3m] and proj "
                         "[m, m], [m]")
    out = torch.empty((B, N, m), device=x.device, dtype=torch.float32)
    with _on(x.device):
        _lib.call("tarmac_comm_forward", _ptr(x), _ptr(w_qkv), _ptr(b_qkv),
                  _ptr(w_proj), _ptr(b_proj), B, N, D, m, int(topk),
                  _ptr(out), _stream(x.device))
    return out


_PLAN_OPS = {"dense": 0, "topk": 1, "streaming": 2}
_PLAN_MODES = {"argmax": _lib.SELECT_ARGMAX, "threshold": _lib.SELECT_THRESHOLD,
               "sort": _lib.SELECT_SORT}


def kernel_plan(op: str, B: int, N: int, d: int, dtype: torch.dtype = torch.float32,
                k: int = 1, mode: str = "argmax") -> dict:
    """The kernel and tiling a contiguous call of ``op`` ("dense", "topk" or
    "streaming") with these shapes takes, as the library decides it from the
    shape: e.g. {"kernel": "topk_ws", "query_tile": 128, "key_tile": 128,
    "chunk": 8, "chunks_kept": 2}. Host-only (no GPU needed); raises
    :class:`TarmacError` for arguments the call itself would reject."""
    import ctypes
    import json
    if dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("dtype must be float32 or bfloat16")
    dt = _lib.BF16 if dtype == torch.bfloat16 else _lib.F32
    buf = ctypes.create_string_buffer(256)
    _lib.call("tarmac_kernel_plan", _PLAN_OPS[op], B, N, d, dt, k,
              _PLAN_MODES[mode], None, buf, len(buf))
    return json.loads(buf.value.decode())
