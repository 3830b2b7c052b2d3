"""ctypes binding of the C ABI in ``include/tarmac_b200.h``.

The shared library ``libtarmac_b200.so`` sits next to this file (built by
``topk-tarmac_b200/build.py``). There is no fallback: if the library is
missing or does not export the expected ABI version, :func:`lib` raises
:class:`ImportError`, so no caller can silently run some other path.
"""

from __future__ import annotations

import ctypes
import threading
from ctypes import c_char_p, c_float, c_int, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().with_name("libtarmac_b200.so")
ABI_VERSION = 2

# status codes (include/tarmac_b200.h)
OK = 0
ERR_NULL = 1
ERR_SHAPE = 2
ERR_DTYPE = 3
ERR_TOPK = 4
ERR_N_TOO_LARGE = 5
ERR_ALIGN = 6
ERR_MODE = 7
ERR_LAUNCH = 8
ERR_BITS = 9
ERR_SCRATCH = 10

F32 = 0
BF16 = 1

SELECT_ARGMAX = 0
SELECT_THRESHOLD = 1
SELECT_SORT = 2

# name -> (restype, argtypes); the order follows the header's declarations
SIGNATURES: dict[str, tuple] = {
    "tarmac_abi_version": (c_int, []),
    "tarmac_strerror": (c_char_p, [c_int]),
    "tarmac_dense_attention": (c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int, c_int, c_int, c_int, c_float, c_void_p]),
    "tarmac_topk_attention": (c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int, c_int, c_int, c_int, c_float, c_int, c_int, c_void_p,
        c_void_p]),
    "tarmac_streaming_topk_attention": (c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int, c_int, c_int, c_int, c_float, c_int, c_void_p, c_void_p]),
    "tarmac_prescore_attention": (c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_void_p, c_int, c_int, c_int, c_int, c_int, c_int, c_float,
        c_void_p]),
    "tarmac_morton_code": (c_int, [
        c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "tarmac_morton_select": (c_int, [
        c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "tarmac_morton_prescore_attention": (c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int, c_int, c_int, c_int, c_float, c_int, c_int, c_void_p,
        c_void_p]),
    "tarmac_knn_select": (c_int, [
        c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "tarmac_grid_knn_select": (c_int, [
        c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    "tarmac_random_select": (c_int, [
        c_int, c_int, c_int, c_uint64, c_uint64, c_void_p, c_void_p]),
    "tarmac_comm_forward": (c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    "tarmac_gather_attention_backward": (c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int, c_int, c_int, c_int, c_int, c_int, c_float,
        c_void_p, c_void_p, c_void_p, c_void_p]),
    "tarmac_dense_attention_backward": (c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int, c_int, c_int, c_int, c_float,
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    "tarmac_dense_attention_backward_noalloc": (c_int, [
        c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
        c_int, c_int, c_int, c_int, c_float,
        c_void_p, c_void_p, c_void_p, c_void_p]),
    "tarmac_kernel_plan": (c_int, [
        c_int, c_int, c_int, c_int, c_int, c_int, c_int, c_void_p,
        c_char_p, c_int]),
}

_LOCK = threading.Lock()
_LIB: ctypes.CDLL | None = None


class TarmacError(RuntimeError):
    """A non-zero status returned by the C ABI."""

    def __init__(self, fn: str, status: int, text: str):
        super().__init__(f"{fn}: {text} (status {status})")
        self.status = status


def lib() -> ctypes.CDLL:
    """The loaded library (loaded once per process)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is not None:
            return _LIB
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with "
                "`python topk-tarmac_b200/build.py` (nvcc, sm_100a). "
                "There is no fallback implementation.")
        so = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(so, name)
            fn.restype = res
            fn.argtypes = args
        ver = so.tarmac_abi_version()
        if ver != ABI_VERSION:
            raise ImportError(f"{LIB_PATH} has ABI version {ver}, "
                              f"expected {ABI_VERSION}")
        _LIB = so
        return so


def strerror(status: int) -> str:
    return lib().tarmac_strerror(status).decode()


_FNS: dict = {}


def call(name: str, *args) -> None:
    """Call an entry point and raise :class:`TarmacError` on a non-zero
    status. The function objects are looked up once (a per-call attribute
    lookup on the library costs more than the launch at small sizes)."""
    fn = _FNS.get(name)
    if fn is None:
        fn = getattr(lib(), name)
        _FNS[name] = fn
    st = fn(*args)
    if st != OK:
        raise TarmacError(name, st, strerror(st))
