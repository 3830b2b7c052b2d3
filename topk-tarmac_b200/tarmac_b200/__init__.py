"""tarmac_b200 — B200-native (sm_100a) TarMAC attention core.

Host-side package over the C ABI of ``include/tarmac_b200.h``
(``libtarmac_b200.so``, built by ``topk-tarmac_b200/build.py``):

* :mod:`tarmac_b200.ops` — torch-facing launchers (dense, fused top-k in three
  tie modes, streaming top-k, attention over a given peer set, Morton codes,
  Morton window selection, fused Morton selection + attention);
* :mod:`tarmac_b200.autograd` — differentiable forms (torch.autograd.Function)
  whose backward runs the gradient kernels;
* :mod:`tarmac_b200._lib` — the ctypes binding itself.

The drop-in modules with the reference's import paths (``src.kernels.*``,
``src.agents.mappo``) live beside this package and call these launchers.
"""

from __future__ import annotations

from . import _lib, autograd, ops  # noqa: F401
from ._lib import TarmacError, lib  # noqa: F401

__all__ = ["ops", "autograd", "lib", "TarmacError", "load"]


def load():
    """Load the shared library now (raises ImportError if it is missing)."""
    return _lib.lib()
