"""CPU oracle for the TarMAC attention core — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference's algorithm for the hot path
(MHHamdan/TopK-TarMAC: src/kernels/fused_topk_attention.py,
src/kernels/streaming_topk_attention.py, src/kernels/fused_dense_attention.py,
src/kernels/prescore_selection.py, src/kernels/fused_prescore_attention.py).
It is the checker for the CUDA kernels and the timed CPU baseline; it is
pinned against golden vectors produced by the reference itself
(tests/golden/make_golden.py).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
and ``--impl reference`` legs may import it. The product path
(``tarmac_b200``, ``src.kernels``, ``src.agents``) never does.
"""

from .tarmac_oracle import (  # noqa: F401
    ambiguous_rows, comm_forward, dense_attention, dense_attention_grad,
    gather_attention_grad, grid_knn, grid_knn_shape, knn_ambiguous,
    knn_exact, morton_code, morton_window, prescore_attention, scores_f32,
    scores_f64, select_mask, topk_attention, topk_indices)
