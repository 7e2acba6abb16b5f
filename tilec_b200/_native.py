"""ctypes binding of the C ABI in include/tilec_mm.h (libtilec_mm.so, built in-tree).

This is the binding a maintainer of the reference would add on the Python side; the
same symbols bind from any other FFI.  There is no fallback: if the library is missing
or cannot load, every call raises.
"""
import ctypes
import os
import threading

from . import build as _build

TILEC_OK = 0
TILEC_ERR_DEVICE = 5
STATUS_NAMES = {
    0: "TILEC_OK", 1: "TILEC_ERR_BAD_ARG", 2: "TILEC_ERR_MISALIGNED", 3: "TILEC_ERR_NO_DEVICE",
    4: "TILEC_ERR_LAUNCH", 5: "TILEC_ERR_DEVICE", 6: "TILEC_ERR_WORKSPACE", 7: "TILEC_ERR_UNSUPPORTED",
    8: "TILEC_ERR_TOO_LARGE",
}

VARIANTS = {"auto": 0, "simt": 1, "splitk": 2, "tf32": 3, "3xtf32": 4, "3xtf32_masked": 5, "3xmixed": 6}
VARIANT_NAMES = {v: k for k, v in VARIANTS.items()}

# Every function the header declares (tests check the library exports exactly these).
EXPORTS = [
    "tilec_mm_f32", "tilec_mm_workspace_bytes", "tilec_mm_plan", "tilec_mm_set_table",
    "tilec_mm_device_status", "tilec_strerror", "tilec_mm_abi_version", "tilec_mm_built_arch",
    "tilec_mm_f32_splitk_noalloc", "tilec_mm_selftest_wait", "tilec_mm_f32_ex", "tilec_mm_workspace_bytes_ex",
    "tilec_mm_set_wait_limit",
]

# Bits of the device status word (TILEC_DEV_STATUS_* in include/tilec_mm.h).
DEV_STATUS_BITS = {1: "TIMEOUT", 2: "TMEM", 4: "BAD_LAUNCH"}


def status_bits(word):
    """Names of the bits set in a device status word, e.g. 'TIMEOUT|TMEM'."""
    names = [n for b, n in DEV_STATUS_BITS.items() if word & b]
    rest = word & ~sum(DEV_STATUS_BITS)
    if rest:
        names.append(hex(rest))
    return "|".join(names) or "clean"


class MMConfig(ctypes.Structure):
    _fields_ = [("variant", ctypes.c_int32), ("split_k", ctypes.c_int32), ("flags", ctypes.c_int32),
                ("activation", ctypes.c_int32), ("reserved", ctypes.c_int32 * 4)]


TRANS_A = 1   # TILEC_MM_TRANS_A: A stored K x M (x1 is a column view, e.g. y.t())
TRANS_B = 2   # TILEC_MM_TRANS_B: B stored N x K
STREAM_K = 4  # TILEC_MM_STREAM_K: CTA-pair kernel as one wave of pairs sharing out K blocks
TILE_M64 = 8     # TILEC_MM_TILE_M64: 1-CTA tensor-core kernel with 64-row tiles
TILE_M128 = 16   # TILEC_MM_TILE_M128: 1-CTA tensor-core kernel with 128-row tiles
ACTIVATIONS = {None: 0, "none": 0, "relu": 1, "gelu": 2}   # TILEC_MM_ACT_*


class TilecError(RuntimeError):
    """A C-ABI call returned a non-zero tilec_status."""

    def __init__(self, code, where):
        self.code = code
        try:
            text = strerror(code)
        except Exception:  # noqa: BLE001  (the library itself may be what failed to load)
            text = "?"
        super().__init__(f"{where}: {STATUS_NAMES.get(code, code)}: {text}")


_lib = None
_fast = None     # the CPython fast-call module, once loaded and installed
_fast_error = None
_lock = threading.Lock()


def lib_path():
    return _build.LIB


def load():
    """Load libtilec_mm.so (building it first if the sources are newer and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not _build.up_to_date():
            try:
                _build.build()
            except Exception as e:  # noqa: BLE001
                if not os.path.exists(_build.LIB):
                    raise RuntimeError(f"tilec_b200: kernel library {_build.LIB} is missing and could not "
                                       f"be built ({e})") from e
        lib = ctypes.CDLL(_build.LIB)
        vp, i64, sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_size_t
        cfgp = ctypes.POINTER(MMConfig)
        lib.tilec_mm_f32.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, cfgp, vp, sz, vp]
        lib.tilec_mm_f32.restype = ctypes.c_int
        lib.tilec_mm_workspace_bytes.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, cfgp]
        lib.tilec_mm_workspace_bytes.restype = sz
        lib.tilec_mm_plan.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, cfgp, cfgp]
        lib.tilec_mm_plan.restype = ctypes.c_int
        lib.tilec_mm_set_table.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.c_int32]
        lib.tilec_mm_set_table.restype = ctypes.c_int
        lib.tilec_mm_device_status.argtypes = [vp, ctypes.POINTER(ctypes.c_int32)]
        lib.tilec_mm_device_status.restype = ctypes.c_int
        lib.tilec_strerror.argtypes = [ctypes.c_int]
        lib.tilec_strerror.restype = ctypes.c_char_p
        lib.tilec_mm_abi_version.restype = ctypes.c_int
        lib.tilec_mm_built_arch.restype = ctypes.c_int
        lib.tilec_mm_f32_splitk_noalloc.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, ctypes.c_int32, vp]
        lib.tilec_mm_f32_splitk_noalloc.restype = ctypes.c_int
        lib.tilec_mm_selftest_wait.argtypes = [i64, vp]
        lib.tilec_mm_selftest_wait.restype = ctypes.c_int
        lib.tilec_mm_set_wait_limit.argtypes = [i64, vp]
        lib.tilec_mm_set_wait_limit.restype = ctypes.c_int
        lib.tilec_mm_f32_ex.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, i64, i64, i64, cfgp, vp,
                                        sz, vp]
        lib.tilec_mm_f32_ex.restype = ctypes.c_int
        lib.tilec_mm_workspace_bytes_ex.argtypes = [vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, i64, i64, i64,
                                                    cfgp]
        lib.tilec_mm_workspace_bytes_ex.restype = sz
        _load_fast(lib)
        _lib = lib
        return _lib


def _load_fast(lib):
    """Load _tilec_fast (csrc/fastcall.c; rebuilt first when stale and gcc exists) and give
    it the addresses of this library's tilec_mm_f32 and tilec_mm_workspace_bytes.  When it
    cannot be had, the binding makes the same calls through ctypes (`fast_error()` says
    why); the kernels that run are the same either way."""
    global _fast, _fast_error
    try:
        import importlib.util
        if not _build.fast_up_to_date():
            try:
                _build.build_fast()
            except Exception:  # noqa: BLE001  (no compiler here: use the module if one exists)
                if not os.path.exists(_build.FAST):
                    raise
        spec = importlib.util.spec_from_file_location("_tilec_fast", _build.FAST)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.install(ctypes.cast(lib.tilec_mm_f32, ctypes.c_void_p).value,
                    ctypes.cast(lib.tilec_mm_workspace_bytes, ctypes.c_void_p).value)
        _fast = mod
    except Exception as e:  # noqa: BLE001
        _fast, _fast_error = None, f"{type(e).__name__}: {e}"


def fast():
    """The fast-call module, or None when the binding uses ctypes for every call."""
    if _lib is None:
        load()
    return _fast


def fast_error():
    """Why the fast-call module is not in use (None when it is)."""
    return _fast_error


def strerror(code):
    return load().tilec_strerror(int(code)).decode()


def check(code, where):
    if code != TILEC_OK:
        raise TilecError(code, where)


_CFG_CACHE = {}


def make_cfg(variant="auto", split_k=0, flags=0, activation=0):
    key = (variant, split_k, flags, activation)
    cfg = _CFG_CACHE.get(key)
    if cfg is None:
        cfg = _make_cfg(variant, split_k, flags, activation)
        _CFG_CACHE[key] = cfg
    return cfg


def _make_cfg(variant, split_k, flags=0, activation=0):
    if isinstance(variant, str):
        try:
            v = VARIANTS[variant.lower()]
        except KeyError:
            raise ValueError(f"unknown matrix_mul variant {variant!r}; expected one of {sorted(VARIANTS)}")
    else:
        v = int(variant)
    return MMConfig(v, int(split_k), int(flags), int(activation))
