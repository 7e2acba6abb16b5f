"""Per-shape kernel selection for matrix_mul on B200.

B200 counterpart of the reference's config picker (tilec/tune.py:135-151, ``pick``),
which predicts the best launch config of a shape from a model trained on per-machine
timings.  Here the trained artefact is a JSON table (never a pickle) of log2-size boxes:

    {"device": "NVIDIA B200", "rows": [[lm0, lm1, ln0, ln1, lk0, lk1, "3xtf32", 0], ...]}

Row r matches an [M,K]x[K,N] product when lm0 <= floor(log2 M) < lm1 (same for N and K);
the first matching row gives (variant, split_k).  The table is installed into the C
library (tilec_mm_set_table) on first use; shapes no row matches use the library's
built-in rules.  ``tilec_b200.tune`` measures the sweep and writes the table.
"""
import ctypes
import json
import os
import threading

from . import _native

TABLE_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "mm_select.json")
_ENV_TABLE = "TILEC_MM_TABLE"

_installed = False
_lock = threading.Lock()


def load_table(path=None):
    """Parse a selection table into int32 rows (raises ValueError on malformed input)."""
    path = path or os.environ.get(_ENV_TABLE) or TABLE_PATH
    if not os.path.exists(path):
        return []
    with open(path) as f:
        doc = json.load(f)
    rows = []
    for i, r in enumerate(doc.get("rows", [])):
        if len(r) != 8:
            raise ValueError(f"{path}: row {i} has {len(r)} fields, expected 8")
        v = r[6]
        if isinstance(v, str):
            if v not in _native.VARIANTS or v == "auto":
                raise ValueError(f"{path}: row {i}: unknown variant {v!r}")
            v = _native.VARIANTS[v]
        lo_hi = [int(x) for x in r[:6]]
        if any(lo_hi[j] > lo_hi[j + 1] for j in (0, 2, 4)):
            raise ValueError(f"{path}: row {i}: empty range {lo_hi}")
        split = int(r[7])
        if split < 0:
            raise ValueError(f"{path}: row {i}: negative split_k")
        rows.append(lo_hi + [int(v), split])
    return rows


def install(rows):
    """Install int32 rows into the C library (an empty list restores the built-in rules)."""
    lib = _native.load()
    from . import ext
    ext._WS_BYTES.clear()  # cached workspace sizes depend on the plans the table selects
    flat = [x for r in rows for x in r]
    arr = (ctypes.c_int32 * max(len(flat), 1))(*flat)
    _native.check(lib.tilec_mm_set_table(arr, len(rows)), "tilec_mm_set_table")


def ensure_installed():
    global _installed
    if _installed:
        return
    with _lock:
        if not _installed:
            install(load_table())
            _installed = True


def lookup(rows, M, N, K):
    """Pure-Python mirror of the library's table match (for tests and reports)."""
    def lg(v):
        return max(int(v), 1).bit_length() - 1
    lm, ln, lk = lg(M), lg(N), lg(K)
    for r in rows:
        if r[0] <= lm < r[1] and r[2] <= ln < r[3] and r[4] <= lk < r[5]:
            return _native.VARIANT_NAMES[r[6]], r[7]
    return None
