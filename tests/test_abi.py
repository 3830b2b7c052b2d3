"""The C-ABI library loads and exports every entry point include/*.h declares;
argument validation returns the documented status codes. No kernel is
launched here (every call fails validation or has B = 0), so no GPU is
needed."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from tarmac_b200 import _lib

HEADER_DIR = Path(__file__).resolve().parents[1] / "include"
FAKE = 1 << 20  # a non-null, 16-byte aligned address that is never touched


def _declared() -> set[str]:
    names = set()
    for h in HEADER_DIR.glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(tarmac_\w+)\s*\(", text))
    return names


def test_every_declared_symbol_is_exported():
    so = _lib.lib()
    declared = _declared()
    assert len(declared) >= 9
    for name in declared:
        assert hasattr(so, name), f"{name} not exported"
    assert declared == set(_lib.SIGNATURES), "ctypes table out of sync"


def test_abi_version_and_strerror():
    assert _lib.lib().tarmac_abi_version() == _lib.ABI_VERSION
    for st in range(0, 10):
        assert _lib.strerror(st)
    assert _lib.strerror(12345) == "unknown status"


def _topk(**kw):
    a = dict(q=FAKE, k=FAKE, v=FAKE, o=FAKE, strides=None, B=4, N=64, d=16,
             dtype=_lib.F32, scale=0.25, topk=2, mode=_lib.SELECT_ARGMAX,
             idx=None, stream=None)
    a.update(kw)
    return _lib.lib().tarmac_topk_attention(
        a["q"], a["k"], a["v"], a["o"], a["strides"], a["B"], a["N"], a["d"],
        a["dtype"], a["scale"], a["topk"], a["mode"], a["idx"], a["stream"])


@pytest.mark.parametrize("kw,status", [
    (dict(q=None), _lib.ERR_NULL),
    (dict(dtype=7), _lib.ERR_DTYPE),
    (dict(N=1, topk=1), _lib.ERR_SHAPE),
    (dict(d=0), _lib.ERR_SHAPE),
    (dict(d=129), _lib.ERR_SHAPE),
    (dict(B=-1), _lib.ERR_SHAPE),
    (dict(topk=0), _lib.ERR_TOPK),
    (dict(topk=64), _lib.ERR_TOPK),
    (dict(mode=5), _lib.ERR_MODE),
    (dict(mode=_lib.SELECT_THRESHOLD, idx=FAKE), _lib.ERR_MODE),
    (dict(topk=9, idx=FAKE), _lib.ERR_MODE),
    (dict(N=2000, topk=20), _lib.ERR_N_TOO_LARGE),
    (dict(N=2000, topk=5, mode=_lib.SELECT_THRESHOLD), _lib.ERR_N_TOO_LARGE),
    (dict(q=FAKE + 2), _lib.ERR_ALIGN),
    (dict(B=0), _lib.OK),
])
def test_topk_validation(kw, status):
    assert _topk(**kw) == status


def test_other_entry_points_validate():
    so = _lib.lib()
    assert so.tarmac_streaming_topk_attention(
        FAKE, FAKE, FAKE, FAKE, None, 4, 64, 16, 0, 0.25, 9, None, None) == _lib.ERR_TOPK
    assert so.tarmac_dense_attention(
        FAKE, FAKE, FAKE, None, None, 4, 64, 16, 0, 0.25, None) == _lib.ERR_NULL
    assert so.tarmac_dense_attention(
        FAKE, FAKE, FAKE, FAKE, None, 0, 64, 16, 0, 0.25, None) == _lib.OK
    assert so.tarmac_prescore_attention(
        FAKE, FAKE, FAKE, FAKE, None, None, 1, 2, 4, 64, 16, 0, 0.25,
        None) == _lib.ERR_NULL
    assert so.tarmac_prescore_attention(
        FAKE, FAKE, FAKE, FAKE, None, FAKE + 4, 1, 2, 4, 64, 16, 0, 0.25,
        None) == _lib.ERR_ALIGN
    assert so.tarmac_morton_code(FAKE, 4, 64, 17, FAKE, None) == _lib.ERR_BITS
    assert so.tarmac_morton_code(FAKE, 4, 64, 0, FAKE, None) == _lib.ERR_BITS
    assert so.tarmac_morton_select(FAKE, 4, 5000, 2, 16, FAKE, None) == _lib.ERR_N_TOO_LARGE
    assert so.tarmac_morton_select(FAKE, 4, 64, 64, 16, FAKE, None) == _lib.ERR_TOPK
    assert so.tarmac_morton_prescore_attention(
        FAKE, FAKE, FAKE, FAKE, None, FAKE, 4, 64, 16, 0, 0.25, 2, 16, FAKE + 4,
        None) == _lib.ERR_ALIGN


def test_strides_argument_is_read():
    """A strides array is accepted (validation passes; B = 0, no launch)."""
    st = (ctypes.c_int64 * 8)(*([64 * 48, 48] * 4))
    assert _topk(strides=ctypes.addressof(st), B=0) == _lib.OK
