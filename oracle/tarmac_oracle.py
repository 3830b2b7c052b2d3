"""numpy restatement of the reference's attention-core algorithm.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): imported by tests/,
__graft_entry__.smoke() and bench.py's CPU legs, never by the product path.

Every function names the reference lines it restates (paths are within the
MHHamdan/TopK-TarMAC project). Inputs are numpy arrays: q, k, v float32
[B, N, d] (bf16 inputs are passed as the float32 values of the same rounded
numbers), pos float32 [B, N, 2]. Work is done ``CHUNK`` episodes at a time so
large batches stay within host memory.
"""

from __future__ import annotations

import numpy as np

CHUNK = 64
U32 = 2.0 ** -24  # unit roundoff of fp32


def _bmm(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Batched a @ b as one BLAS product per episode (numpy's stacked matmul
    is several times slower than a loop of 2-D products here)."""
    out = np.empty(a.shape[:-1] + b.shape[-1:], dtype=np.result_type(a, b))
    for i in range(a.shape[0]):
        np.matmul(a[i], b[i], out=out[i])
    return out


def _chunks(B: int):
    for b0 in range(0, B, CHUNK):
        yield slice(b0, min(B, b0 + CHUNK))


def scores_f64(q: np.ndarray, k: np.ndarray, d_scale: float | None = None):
    """Exact-as-possible scaled scores in float64 with the diagonal at -inf.

    fused_topk_attention.py:395-397: ``q @ k^T / sqrt(d)``, diagonal masked.
    Products of fp32 values are exact in float64, so this is the true score to
    about 1e-16 relative.
    """
    d = q.shape[-1]
    sc = (1.0 / np.sqrt(d)) if d_scale is None else d_scale
    s = _bmm(q.astype(np.float64), np.swapaxes(k.astype(np.float64), -1, -2))
    s *= sc
    N = q.shape[1]
    s[:, np.arange(N), np.arange(N)] = -np.inf
    return s


def scores_f32(q: np.ndarray, k: np.ndarray):
    """fp32 scores as the reference forms them: the dot product rounded to
    fp32, then divided by fp32(sqrt(d)) (fused_topk_attention.py:395), with the
    diagonal at -inf (fused_topk_attention.py:396-397).

    The dot product is evaluated in float64 and rounded once, so it does not
    depend on a BLAS summation order.
    """
    d = q.shape[-1]
    dot = _bmm(q.astype(np.float64),
               np.swapaxes(k.astype(np.float64), -1, -2)).astype(np.float32)
    s = dot / np.float32(np.sqrt(d))
    N = q.shape[1]
    s[:, np.arange(N), np.arange(N)] = -np.inf
    return s


def select_mask(s: np.ndarray, topk: int, tie: str = "low") -> np.ndarray:
    """Boolean [.., N] mask of the retained peers of each score row.

    Retained = every score above the k-th largest value T, plus the peers
    tied at T chosen by ``tie``:
      "low"  — the lowest indices (k argmax rounds, fused_topk_attention.py:
               275-284; packed (ordkey<<32)|(0x7FFFFFFF-idx) words,
               streaming_topk_attention.py:114-117);
      "high" — the highest indices (descending sort of (key<<32)|idx,
               fused_topk_attention.py:469-479);
      "all"  — all of them (bisection threshold keeps keys >= T,
               fused_topk_attention.py:180-191).
    Exactly k peers are kept for "low"/"high"; "all" keeps k or more.
    """
    if tie not in ("low", "high", "all"):
        raise ValueError(f"unknown tie rule {tie!r}")
    N = s.shape[-1]
    T = np.partition(s, N - topk, axis=-1)[..., N - topk]
    ge = s >= T[..., None]
    if tie == "all":
        return ge
    # rows with more than k peers >= T have surplus ties at T: rank the tied
    # peers by index and keep the first (low) or last (high) ones needed
    extra = ge.sum(-1) > topk
    if extra.any():
        rows = np.nonzero(extra)
        sr, Tr = s[rows], T[rows][:, None]
        eq = sr == Tr
        need = topk - (sr > Tr).sum(-1)
        if tie == "low":
            rank = np.cumsum(eq, axis=-1)
        else:
            rank = np.cumsum(eq[:, ::-1], axis=-1)[:, ::-1]
        ge[rows] = (sr > Tr) | (eq & (rank <= need[:, None]))
    return ge


def topk_indices(s: np.ndarray, topk: int, tie: str = "low") -> np.ndarray:
    """Retained peers, int64 [.., topk], in rank order: score descending,
    ties by index ascending ("low") or descending ("high")."""
    mask = select_mask(s, topk, tie)
    shp = s.shape[:-1]
    flat_s = s.reshape(-1, s.shape[-1])
    flat_m = mask.reshape(-1, s.shape[-1])
    out = np.empty((flat_s.shape[0], topk), dtype=np.int64)
    cols = np.nonzero(flat_m)[1].reshape(-1, topk)  # index-ascending per row
    if tie == "high":
        cols = cols[:, ::-1]
    vals = np.take_along_axis(flat_s, cols, axis=1)
    order = np.argsort(-vals, axis=1, kind="stable")
    out[:] = np.take_along_axis(cols, order, axis=1)
    return out.reshape(*shp, topk)


def topk_attention(q, k, v, topk: int, tie: str = "low", exact: bool = True,
                   want_mask: bool = True):
    """Fused score-then-select top-k attention.

    fused_topk_attention.py:390-402 (reference_topk_attention): scores, mask
    the diagonal, keep k peers, softmax over the retained scores, weighted sum
    of the retained V rows. ``topk`` is clamped to [1, N-1] as the reference's
    launchers do (fused_topk_attention.py:310).

    exact=True (the checker): the selection runs on correctly rounded fp32
    scores (scores_f32) and the softmax and sum in float64.
    exact=False (the timed CPU baseline): every step in fp32 as the
    reference's eager path computes it (fp32 BLAS product, fp32 softmax).

    Returns (out float32 [B, N, d], mask bool [B, N, N] or None).
    """
    B, N, d = q.shape
    topk = max(1, min(topk, N - 1))
    out = np.empty((B, N, d), dtype=np.float32)
    masks = np.empty((B, N, N), dtype=bool) if want_mask else None
    diag = np.arange(N)
    for sl in _chunks(B):
        if exact:
            s = scores_f32(q[sl], k[sl])
        else:
            s = _bmm(q[sl], np.swapaxes(k[sl], -1, -2)) / np.float32(np.sqrt(d))
            s[:, diag, diag] = -np.inf
        m = select_mask(s, topk, tie)
        if exact:
            s64 = np.where(m, s.astype(np.float64), -np.inf)
            mx = s64.max(-1, keepdims=True)
            e = np.exp(s64 - mx)
            w = e / e.sum(-1, keepdims=True)
            out[sl] = _bmm(w, v[sl].astype(np.float64)).astype(np.float32)
        elif tie == "all":
            s32 = np.where(m, s, np.float32(-np.inf))
            e = np.exp(s32 - s32.max(-1, keepdims=True))
            w = e / e.sum(-1, keepdims=True)
            out[sl] = _bmm(w, v[sl])
        else:
            # gathered form (mappo.py:217-223): k scores, k-wide softmax,
            # gather the k value rows, k-term weighted sum
            nb = s.shape[0]
            ind = np.nonzero(m.reshape(-1, N))[1].reshape(nb, N, topk)
            val = np.take_along_axis(s, ind, -1)
            e = np.exp(val - val.max(-1, keepdims=True))
            w = e / e.sum(-1, keepdims=True)
            vg = v[sl][np.arange(nb)[:, None, None], ind]      # [b, N, k, d]
            out[sl] = np.einsum("bnk,bnkd->bnd", w, vg)
        if want_mask:
            masks[sl] = m
    return out, masks


def dense_attention(q, k, v):
    """softmax(q k^T / sqrt(d), diagonal masked) v, float64 arithmetic.

    dense_unfused (scripts/bench_attention_core.py:69-75) and
    _flash_dense_kernel (src/kernels/fused_dense_attention.py:38-99).
    """
    B, N, d = q.shape
    out = np.empty((B, N, d), dtype=np.float32)
    for sl in _chunks(B):
        s = scores_f64(q[sl], k[sl])
        mx = s.max(-1, keepdims=True)
        e = np.exp(s - mx)
        w = e / e.sum(-1, keepdims=True)
        out[sl] = _bmm(w, v[sl].astype(np.float64)).astype(np.float32)
    return out


def prescore_attention(q, k, v, idx):
    """Attention over the given peers idx [B, N, kk].

    prescore_attention (src/kernels/prescore_selection.py:184-195): gather the
    kk key and value rows, scores q.k_j / sqrt(d), softmax over the kk, sum.
    float64 arithmetic. Rows naming a peer outside [0, N) are NaN.
    """
    B, N, d = q.shape
    idx = np.asarray(idx, dtype=np.int64)
    bad = ((idx < 0) | (idx >= N)).any(-1)
    safe = np.clip(idx, 0, N - 1)
    bi = np.arange(B)[:, None, None]
    kg = k.astype(np.float64)[bi, safe]            # [B, N, kk, d]
    vg = v.astype(np.float64)[bi, safe]
    s = np.einsum("bnd,bnjd->bnj", q.astype(np.float64), kg) / np.sqrt(d)
    mx = s.max(-1, keepdims=True)
    e = np.exp(s - mx)
    w = e / e.sum(-1, keepdims=True)
    out = np.einsum("bnj,bnjd->bnd", w, vg).astype(np.float32)
    out[bad] = np.nan
    return out


# ---------------------------------------------------------------------------
# gradients: what autograd forms through the reference's eager path
# ---------------------------------------------------------------------------

def gather_attention_grad(q, k, v, idx, g, scale: float | None = None):
    """Gradients (dq, dk, dv) of attention over a fixed peer set, float64.

    The eager path gathers the selected rows and contracts
    (src/agents/mappo.py:211-222 topk_gather, 279-286 zorder_k;
    prescore_selection.py:184-195): s = q.k_j * scale, w = softmax(s),
    out = sum w v_j. The indices come from topk / the Morton selector and
    carry no gradient, so autograd's result is the chain rule through
    gather, softmax and the two contractions, with scatter-adds into dk, dv.
    """
    B, N, d = q.shape
    sc = 1.0 / np.sqrt(d) if scale is None else float(scale)
    idx = np.asarray(idx, dtype=np.int64)
    q64, k64, v64, g64 = (np.asarray(t, dtype=np.float64) for t in (q, k, v, g))
    bi = np.arange(B)[:, None, None]
    kg, vg = k64[bi, idx], v64[bi, idx]              # [B, N, kk, d]
    s = np.einsum("bnd,bnjd->bnj", q64, kg) * sc
    w = np.exp(s - s.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    dw = np.einsum("bnd,bnjd->bnj", g64, vg)
    ds = w * (dw - (w * dw).sum(-1, keepdims=True))
    dq = sc * np.einsum("bnj,bnjd->bnd", ds, kg)
    dk = np.zeros_like(k64)
    dv = np.zeros_like(v64)
    bb = np.broadcast_to(bi, idx.shape)
    np.add.at(dk, (bb, idx), sc * ds[..., None] * q64[:, :, None, :])
    np.add.at(dv, (bb, idx), w[..., None] * g64[:, :, None, :])
    return dq, dk, dv


def dense_attention_grad(q, k, v, g, scale: float | None = None, out=None):
    """Gradients (dq, dk, dv) of dense masked-diagonal attention, float64:
    the chain rule through the eager path's matmul, masked softmax and matmul
    (src/agents/mappo.py:361-373). ``out`` (optional) is the forward output
    that D_i = g_i . out_i is taken from, as a kernel given a stored (e.g.
    bf16-rounded) output forms it; by default the exact output."""
    B, N, d = q.shape
    sc = 1.0 / np.sqrt(d) if scale is None else float(scale)
    q64, k64, v64, g64 = (np.asarray(t, dtype=np.float64) for t in (q, k, v, g))
    s = np.einsum("bid,bjd->bij", q64, k64) * sc
    s[:, np.arange(N), np.arange(N)] = -np.inf
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    o64 = (np.einsum("bij,bjd->bid", p, v64) if out is None
           else np.asarray(out, dtype=np.float64))
    dp = np.einsum("bid,bjd->bij", g64, v64)
    dsc = p * (dp - (g64 * o64).sum(-1)[..., None])
    dq = sc * np.einsum("bij,bjd->bid", dsc, k64)
    dk = sc * np.einsum("bij,bid->bjd", dsc, q64)
    dv = np.einsum("bij,bid->bjd", p, g64)
    return dq, dk, dv


# ---------------------------------------------------------------------------
# positional selectors
# ---------------------------------------------------------------------------

def _dist2(pi: np.ndarray, pj: np.ndarray) -> np.ndarray:
    """fp32 squared distance, each step rounded (no fused multiply-add)."""
    dx = (pj[..., 0] - pi[..., 0]).astype(np.float32)
    dy = (pj[..., 1] - pi[..., 1]).astype(np.float32)
    return (dx * dx).astype(np.float32) + (dy * dy).astype(np.float32)


def knn_exact(pos: np.ndarray, k: int) -> np.ndarray:
    """k nearest peers, self excluded, by increasing (distance, index);
    int64 [B, N, k].

    select_radius_knn (src/kernels/prescore_selection.py:35-42) ranks
    cdist(pos, pos) with the diagonal at +inf and keeps the k smallest; the
    squared distance has the same order, and exact ties go to the lower index.
    """
    pos = np.asarray(pos, dtype=np.float32)
    B, N, _ = pos.shape
    out = np.empty((B, N, k), dtype=np.int64)
    for b in range(B):
        d2 = _dist2(pos[b][:, None, :], pos[b][None, :, :])
        d2[np.arange(N), np.arange(N)] = np.inf
        # candidates: every peer at or below the k-th smallest distance (all
        # of a tie at the boundary), then the first k by (distance, index)
        kth = np.partition(d2, k - 1, axis=-1)[:, k - 1:k]
        rows, cols = np.nonzero(d2 <= kth)
        order = np.lexsort((cols, d2[rows, cols], rows))
        rows, cols = rows[order], cols[order]
        first = np.searchsorted(rows, np.arange(N))
        out[b] = cols[first[:, None] + np.arange(k)[None, :]]
    return out


def knn_ambiguous(pos: np.ndarray, k: int, tol: float = 1e-6) -> np.ndarray:
    """Rows whose k-th and (k+1)-th squared distances differ by less than
    ``tol``: rounding of a distance evaluation (the reference's cdist uses a
    matrix-product form for larger N) may order them either way."""
    pos = np.asarray(pos, dtype=np.float64)
    B, N, _ = pos.shape
    res = np.zeros((B, N), dtype=bool)
    if k >= N - 1:
        return res
    for b in range(B):
        d2 = ((pos[b][:, None, :] - pos[b][None, :, :]) ** 2).sum(-1)
        d2[np.arange(N), np.arange(N)] = np.inf
        srt = np.sort(d2, axis=-1)
        res[b] = (srt[:, k] - srt[:, k - 1]) < tol
    return res


def grid_knn_shape(N: int, k: int) -> tuple[int, int]:
    """Grid side and per-cell capacity (prescore_selection.py:87-101)."""
    occ = max(2, k)
    G = max(1, int((N / occ) ** 0.5))
    mean = N / (G * G)
    return G, int(mean + 3 * mean ** 0.5 + 2)


def grid_knn(pos: np.ndarray, k: int) -> np.ndarray:
    """Grid kNN, int64 [B, N, k] by increasing (distance, index).

    select_grid_knn (src/kernels/prescore_selection.py:107-164): cells of a
    G x G grid over the episode's bounding box (normalise, scale by G,
    truncate, clamp), agents sorted by cell id x*G + y (stably: equal cells
    keep agent order), and for each agent the three sorted runs from cell
    (x', max(y-1, 0)) to the end of cell (x', min(y+1, G-1)) for
    x' = x-1..x+1, each cut at 3M entries; the k nearest among them. The
    exact selector when 9M >= N; an agent with fewer than k candidates takes
    its exact k nearest.
    """
    pos = np.asarray(pos, dtype=np.float32)
    B, N, _ = pos.shape
    G, M = grid_knn_shape(N, k)
    L = 3 * M
    if 3 * L >= N:
        return knn_exact(pos, k)
    out = np.empty((B, N, k), dtype=np.int64)
    exact = knn_exact(pos, k)
    for b in range(B):
        p = pos[b]
        lo = p.min(0)
        span = np.maximum((p.max(0) - lo).astype(np.float32), np.float32(1e-6))
        g = (((p - lo).astype(np.float32) / span).astype(np.float32)
             * np.float32(G)).astype(np.float32)
        cxy = np.clip(np.trunc(g).astype(np.int64), 0, G - 1)
        cell = cxy[:, 0] * G + cxy[:, 1]
        order = np.argsort(cell, kind="stable")
        start = np.searchsorted(cell[order], np.arange(G * G + 1), side="left")
        for i in range(N):
            x, y = cxy[i]
            cand = []
            for xx in (x - 1, x, x + 1):
                if xx < 0 or xx >= G:
                    continue
                s_lo = start[xx * G + max(y - 1, 0)]
                s_hi = min(start[xx * G + min(y + 1, G - 1) + 1], s_lo + L)
                cand.extend(int(j) for j in order[s_lo:s_hi] if j != i)
            if len(cand) < k:
                out[b, i] = exact[b, i]
                continue
            cand = np.array(sorted(cand))
            d2 = _dist2(p[i][None, :], p[cand])
            out[b, i] = cand[np.argsort(d2, kind="stable")[:k]]
    return out


# ---------------------------------------------------------------------------
# the communication module forward
# ---------------------------------------------------------------------------

def _gelu_erf(x: np.ndarray) -> np.ndarray:
    from scipy.special import erf
    return 0.5 * x * (1.0 + erf(x / np.sqrt(2.0)))


def comm_forward(x, w_qkv, b_qkv, w_proj, b_proj, topk: int):
    """AttentionComm.forward, float64 (src/agents/mappo.py:332-353, 361-373,
    419-420): q, k, v = split(x W_qkv^T + b_qkv); dense softmax (topk == 0)
    or the top-k gathered softmax with the lowest index on a tie; then
    gelu(msg) W_proj^T + b_proj with the exact GELU. Returns (out, q, k) so
    callers can classify near-tie rows on the same q, k."""
    x = np.asarray(x, dtype=np.float64)
    qkv = x @ np.asarray(w_qkv, np.float64).T + np.asarray(b_qkv, np.float64)
    m = qkv.shape[-1] // 3
    q, k, v = qkv[..., :m], qkv[..., m:2 * m], qkv[..., 2 * m:]
    B, N, _ = q.shape
    s = np.einsum("bid,bjd->bij", q, k) / np.sqrt(m)
    s[:, np.arange(N), np.arange(N)] = -np.inf
    if topk:
        keep = np.zeros_like(s, dtype=bool)
        idx = np.argsort(-s, axis=-1, kind="stable")[..., :topk]
        np.put_along_axis(keep, idx, True, axis=-1)
        s = np.where(keep, s, -np.inf)
    w = np.exp(s - s.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    msg = np.einsum("bij,bjd->bid", w, v)
    out = _gelu_erf(msg) @ np.asarray(w_proj, np.float64).T + \
        np.asarray(b_proj, np.float64)
    return out, q, k


_SPREAD = ((8, 0x00FF00FF), (4, 0x0F0F0F0F), (2, 0x33333333), (1, 0x55555555))


def _spread_bits(x: np.ndarray) -> np.ndarray:
    """Insert a zero between consecutive bits of a value below 2^16
    (prescore_selection.py:51-59; its first (16, 0x0000FFFF) step is the
    identity for such values)."""
    x = x.astype(np.int64)
    for sh, mask in _SPREAD:
        x = (x | (x << sh)) & mask
    return x


def morton_code(pos: np.ndarray, bits: int = 10) -> np.ndarray:
    """int64 [B, N] Morton codes (prescore_selection.py:62-68).

    Per episode and axis: lo/hi = min/max, span = max(hi - lo, 1e-6),
    g = trunc((pos - lo) / span * (2^bits - 1)) clamped to [0, 2^bits - 1],
    code = spread(gx) | spread(gy) << 1. Every step is a single rounded fp32
    operation, as the reference's elementwise tensor ops are.
    """
    pos = np.asarray(pos, dtype=np.float32)
    lo = pos.min(axis=1, keepdims=True)
    hi = pos.max(axis=1, keepdims=True)
    span = np.maximum(hi - lo, np.float32(1e-6))
    g = ((pos - lo) / span) * np.float32(2 ** bits - 1)
    gi = np.clip(np.trunc(g).astype(np.int64), 0, 2 ** bits - 1)
    return _spread_bits(gi[..., 0]) | (_spread_bits(gi[..., 1]) << 1)


def morton_window(pos: np.ndarray, k: int, bits: int = 10) -> np.ndarray:
    """int64 [B, N, k] Z-order window peers (prescore_selection.py:71-84).

    Agents sorted by code (stable: equal codes keep index order); the agent at
    rank r keeps the agents at ranks r+1..r+h and r-1..r-(k-h), modulo N,
    h = (k+1)//2, in that order. The reference sorts with an unstable argsort
    (line 75); the stable order is the deterministic member of its outcomes.
    """
    code = morton_code(pos, bits)
    B, N = code.shape
    order = np.argsort(code, axis=-1, kind="stable")
    rank = np.empty_like(order)
    np.put_along_axis(rank, order, np.broadcast_to(np.arange(N), (B, N)), -1)
    half = (k + 1) // 2
    offs = np.array(list(range(1, half + 1)) + [-o for o in range(1, k - half + 1)],
                    dtype=np.int64)
    nr = (rank[..., None] + offs) % N
    return np.take_along_axis(order, nr.reshape(B, N * k), -1).reshape(B, N, k)


def ambiguous_rows(q, k, topk: int, ulps: float = 2.0) -> np.ndarray:
    """Rows whose retained set is not determined by fp32 arithmetic.

    A row is ambiguous when its k-th and (k+1)-th exact scores differ, but by
    no more than the error bound of an fp32 dot product of length d
    (``ulps * (d + 2) * u * sum_c |q_c k_c| * scale`` for either candidate,
    u = 2^-24): two correct fp32 evaluations of the scores may then order the
    pair differently. Exact ties (difference 0) are not ambiguous: the tie rule
    decides them. The reference counts such rows instead of failing on them
    (scripts/bench_attention_core.py:386-395).
    """
    B, N, d = q.shape
    topk = max(1, min(topk, N - 1))
    if topk >= N - 1:
        return np.zeros((B, N), dtype=bool)
    res = np.empty((B, N), dtype=bool)
    sc = 1.0 / np.sqrt(d)
    for sl in _chunks(B):
        s = scores_f64(q[sl], k[sl])
        mag = _bmm(np.abs(q[sl].astype(np.float64)),
                        np.swapaxes(np.abs(k[sl].astype(np.float64)), -1, -2)) * sc
        srt = np.sort(s, axis=-1)[..., ::-1]
        a, b = srt[..., topk - 1], srt[..., topk]
        tol = ulps * (d + 2) * U32 * mag.max(-1)
        gap = a - b
        res[sl] = (gap > 0) & (gap <= tol)
    return res
