"""Generate the golden vectors that pin the oracle to the reference.

Runs the UNMODIFIED reference (MHHamdan/TopK-TarMAC) on small seeded inputs,
on the CPU, and stores inputs and outputs as ``tests/golden/*.npz``:

* the reference's eager functions: ``reference_topk_attention``
  (src/kernels/fused_topk_attention.py:390-402), ``dense_unfused``
  (scripts/bench_attention_core.py:74-75), ``_morton_code`` and
  ``select_morton_window`` (src/kernels/prescore_selection.py:51-84),
  ``prescore_attention`` (src/kernels/prescore_selection.py:184-195),
  ``select_radius_knn``, ``select_grid_knn``, ``grid_knn_recall``
  (src/kernels/prescore_selection.py:35-172);
* the reference's Triton kernels run by Triton's CPU interpreter
  (``TRITON_INTERPRET=1``), which pin the kernel-specific tie rules:
  ``fused_topk_attention_tiled`` (lowest index), ``fused_topk_attention_sort``
  (highest index), ``fused_topk_attention_masked`` (all ties kept),
  ``streaming_topk_attention(return_indices=True)`` (lowest index, indices),
  ``fused_prescore_attention``, ``fused_dense_attention``.

Usage (needs the reference tree; it is not needed afterwards):
    python tests/golden/make_golden.py --reference /path/to/TopK-TarMAC
The fixtures are committed; tests only read them.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def _setup(ref: Path):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(ref))
    import torch  # noqa: F401
    from src.kernels import fused_dense_attention as fda
    from src.kernels import fused_prescore_attention as fpa
    from src.kernels import fused_topk_attention as fta
    from src.kernels import prescore_selection as ps
    from src.kernels import streaming_topk_attention as sta
    from scripts import bench_attention_core as bac
    return fta, fda, fpa, ps, sta, bac


def _qkv(gen, B, N, d):
    import torch
    q = torch.randn(B, N, d, generator=gen)
    k = torch.randn(B, N, d, generator=gen)
    v = torch.randn(B, N, d, generator=gen)
    return q, k, v


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", required=True, type=Path)
    ap.add_argument("--only", default=None,
                    help="comma-separated fixture groups to (re)write: "
                         "topk,dense,morton,selectors (default: all)")
    args = ap.parse_args()
    only = set(args.only.split(",")) if args.only else None

    def want(group):
        return only is None or group in only
    fta, fda, fpa, ps, sta, bac = _setup(args.reference.resolve())
    import numpy as np
    import torch

    def save(name, **arrs):
        out = {k: (v.detach().cpu().numpy() if torch.is_tensor(v) else np.asarray(v))
               for k, v in arrs.items()}
        np.savez_compressed(HERE / f"{name}.npz", **out)
        print("wrote", name, {k: v.shape for k, v in out.items()})

    # -- fused top-k: eager reference + interpreted kernels ------------------
    if want("topk"):
        _topk_fixtures(fta, sta, save)
    if want("dense"):
        _dense_fixtures(fda, bac, save)
    if want("morton"):
        _morton_fixtures(ps, fpa, save)
    if want("selectors"):
        _selector_fixtures(ps, save)
    return 0


def _topk_fixtures(fta, sta, save):
    import numpy as np
    import torch
    cases = [("topk_c1", 8, 6, 16, (1, 2, 4)),
             ("topk_n40", 4, 40, 16, (1, 2, 4, 7)),
             ("topk_n64_d32", 2, 64, 32, (1, 3, 8)),
             ("topk_n33_d8", 3, 33, 8, (2, 5))]
    for name, B, N, d, ks in cases:
        gen = torch.Generator().manual_seed(1234 + 7 * N + d)
        q, k, v = _qkv(gen, B, N, d)
        rec = {"q": q, "k": k, "v": v, "ks": np.array(ks)}
        for kk in ks:
            rec[f"eager_k{kk}"] = fta.reference_topk_attention(q, k, v, kk)
            rec[f"tiled_k{kk}"] = fta.fused_topk_attention_tiled(q, k, v, kk)
            if kk <= 8:
                o, ix = sta.streaming_topk_attention(q, k, v, kk,
                                                     return_indices=True)
                rec[f"stream_k{kk}"] = o
                rec[f"stream_idx_k{kk}"] = ix
        save(name, **rec)

    # -- exact ties: duplicated key rows ------------------------------------
    gen = torch.Generator().manual_seed(77)
    B, N, d = 3, 16, 16
    q, k, v = _qkv(gen, B, N, d)
    k[0] = k[0, 3]                   # episode 0: every key identical
    k[1, 9] = k[1, 4]                # episode 1: pairs and a triple
    k[1, 12] = k[1, 2]
    k[1, 15] = k[1, 2]
    k[2, :, :] = k[2, :, :].round()  # episode 2: coarse keys, many ties
    q[2] = q[2].round()
    rec = {"q": q, "k": k, "v": v, "ks": np.array((1, 2, 3, 5))}
    for kk in (1, 2, 3, 5):
        rec[f"tiled_k{kk}"] = fta.fused_topk_attention_tiled(q, k, v, kk)
        rec[f"sort_k{kk}"] = fta.fused_topk_attention_sort(q, k, v, kk)
        rec[f"masked_k{kk}"] = fta.fused_topk_attention_masked(q, k, v, kk)
        o, ix = sta.streaming_topk_attention(q, k, v, kk, return_indices=True)
        rec[f"stream_k{kk}"] = o
        rec[f"stream_idx_k{kk}"] = ix
    save("topk_ties", **rec)

    # -- masked (threshold) and sort kernels on random inputs ----------------
    gen = torch.Generator().manual_seed(4321)
    B, N, d = 3, 48, 16
    q, k, v = _qkv(gen, B, N, d)
    rec = {"q": q, "k": k, "v": v, "ks": np.array((1, 3, 12))}
    for kk in (1, 3, 12):
        rec[f"masked_k{kk}"] = fta.fused_topk_attention_masked(q, k, v, kk)
        rec[f"sort_k{kk}"] = fta.fused_topk_attention_sort(q, k, v, kk)
        rec[f"rowwise_k{kk}"] = fta.fused_topk_attention(q, k, v, kk)
        rec[f"eager_k{kk}"] = fta.reference_topk_attention(q, k, v, kk)
    save("topk_modes", **rec)



def _dense_fixtures(fda, bac, save):
    import torch
    for name, B, N, d in (("dense_n40", 4, 40, 16), ("dense_c1", 8, 6, 16),
                          ("dense_n70_d32", 2, 70, 32)):
        gen = torch.Generator().manual_seed(1234 + 7 * N + d)
        q, k, v = _qkv(gen, B, N, d)
        eye = torch.eye(N, dtype=torch.bool).unsqueeze(0)
        save(name, q=q, k=k, v=v,
             eager=bac.dense_unfused(q, k, v, eye, N - 1),
             flash=fda.fused_dense_attention(q, k, v))



def _morton_fixtures(ps, fpa, save):
    import numpy as np
    import torch
    gen = torch.Generator().manual_seed(4242 + 50)
    B, N, d = 6, 50, 16
    q, k, v = _qkv(gen, B, N, d)
    pos = torch.rand(B, N, 2, generator=gen)
    code10 = ps._morton_code(pos)
    code16 = ps._morton_code(pos, bits=16)
    dup10 = torch.tensor([len(set(c.tolist())) < N for c in code10])
    rec = {"q": q, "k": k, "v": v, "pos": pos, "code10": code10,
           "code16": code16, "dup10": dup10, "ks": np.array((1, 2, 3, 4))}
    for kk in (1, 2, 3, 4):
        idx = ps.select_morton_window(pos, kk)
        rec[f"win_k{kk}"] = idx
        rec[f"prescore_k{kk}"] = ps.prescore_attention(q, k, v, idx)
        rec[f"fused_prescore_k{kk}"] = fpa.fused_prescore_attention(q, k, v, idx)
    save("morton_n50", **rec)

    # positions with deliberate duplicate cells and a degenerate axis
    gen = torch.Generator().manual_seed(99)
    pos = torch.rand(4, 24, 2, generator=gen)
    pos[0, :, 1] = 0.5                          # zero span on one axis
    pos[1] = (pos[1] * 4).floor() / 4           # many equal codes
    pos[2, 5] = pos[2, 7]                       # one duplicate position
    pos[3] = pos[3] * 1e-7                      # span below the 1e-6 clamp
    save("morton_edge", pos=pos, code10=ps._morton_code(pos),
         code16=ps._morton_code(pos, bits=16),
         code4=ps._morton_code(pos, bits=4))


def _selector_fixtures(ps, save):
    """select_radius_knn, select_grid_knn (grid path at N >= 600, the exact
    fallback at N = 50) and grid_knn_recall on seeded uniform positions."""
    import numpy as np
    import torch
    for name, B, N, ks in (("knn_n50", 4, 50, (1, 2, 5)),
                           ("knn_n600", 3, 600, (2, 4)),
                           ("knn_n3000", 1, 3000, (2,))):
        gen = torch.Generator().manual_seed(4242 + N)
        pos = torch.rand(B, N, 2, generator=gen)
        rec = {"pos": pos, "ks": np.array(ks)}
        for kk in ks:
            rec[f"radius_k{kk}"] = ps.select_radius_knn(pos, kk)
            rec[f"grid_k{kk}"] = ps.select_grid_knn(pos, kk)
            rec[f"shape_k{kk}"] = np.array(ps.grid_knn_shape(N, kk))
            rec[f"recall_k{kk}"] = np.array(ps.grid_knn_recall(pos, kk))
        save(name, **rec)


if __name__ == "__main__":
    raise SystemExit(main())
