"""The C-ABI library: it builds for sm_100a, loads, and exports what include/tilec_mm.h declares.

No compute call runs here (this host has no GPU): only symbol, string and error-path
checks.
"""
import ctypes
import os
import re
import subprocess

import pytest
import torch

from tilec_b200 import _native, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "tilec_mm.h")


def _header():
    with open(HEADER) as f:
        return f.read()


def _declared_functions():
    return re.findall(r"TILEC_API\s+[\w\s\*]+?\b(tilec_\w+)\s*\(", _header())


def test_header_declares_the_binding_list():
    assert sorted(_declared_functions()) == sorted(_native.EXPORTS)


def test_library_builds_and_exports_every_declared_symbol():
    path = build.build()
    out = subprocess.run(["nm", "-D", "--defined-only", path], check=True, capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (tilec_\w+)", out))
    assert set(_declared_functions()) <= exported
    # Nothing else leaks: only the ABI is visible.
    assert exported == set(_declared_functions())
    lib = _native.load()
    for name in _declared_functions():
        assert getattr(lib, name) is not None


def test_abi_constants_match_header():
    h = _header()
    lib = _native.load()
    ver = int(re.search(r"#define TILEC_MM_ABI_VERSION (\d+)", h).group(1))
    assert lib.tilec_mm_abi_version() == ver
    assert lib.tilec_mm_built_arch() == 100
    for name, code in re.findall(r"(TILEC_(?:OK|ERR_\w+))\s*=\s*(\d+)", h):
        assert _native.STATUS_NAMES[int(code)] == name
    found = re.findall(r"TILEC_MM_(AUTO|SIMT|SPLITK|TF32|3XTF32|3XTF32_MASKED|3XMIXED)\s*=\s*(\d+)", h)
    assert {name.lower() for name, _ in found} == set(_native.VARIANTS), "header and binding list the same variants"
    for name, code in found:
        assert _native.VARIANTS[name.lower()] == int(code)
    assert ctypes.sizeof(_native.MMConfig) == 32


def test_strerror_names_every_code():
    for code in _native.STATUS_NAMES:
        assert _native.strerror(code)
    assert "unknown" in _native.strerror(99)


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device error path")
def test_no_device_is_an_error_not_a_fallback():
    lib = _native.load()
    cfg = _native.make_cfg("auto")
    res = _native.MMConfig()
    rc = lib.tilec_mm_plan(16, 16, 16, 4, 4, 4, 4, 4, 4, ctypes.byref(cfg), ctypes.byref(res))
    assert rc == 3  # TILEC_ERR_NO_DEVICE
    rc = lib.tilec_mm_f32(16, 16, 16, 4, 4, 4, 4, 4, 4, None, None, 0, None)
    assert rc == 3


def test_bad_arguments_rejected_before_device():
    lib = _native.load()
    # negative size / too-small leading dimension / null output
    assert lib.tilec_mm_f32(16, 16, 16, -1, 4, 4, 4, 4, 4, None, None, 0, None) == 1
    assert lib.tilec_mm_f32(16, 16, 16, 4, 4, 4, 3, 4, 4, None, None, 0, None) == 1
    assert lib.tilec_mm_f32(16, 16, None, 4, 4, 4, 4, 4, 4, None, None, 0, None) == 1
    # empty problems are a no-op even without a device
    assert lib.tilec_mm_f32(None, None, None, 0, 4, 4, 4, 4, 4, None, None, 0, None) == 0
    rows = (ctypes.c_int32 * 8)(0, 1, 0, 1, 0, 1, 9, 0)
    assert lib.tilec_mm_set_table(rows, 1) == 1  # unknown variant
    assert lib.tilec_mm_set_table(None, 0) == 0


def test_transposed_operand_leading_dimensions():
    """TILEC_MM_TRANS_A / _B change which extent the leading dimension must cover (A stored
    K x M needs lda >= M, B stored N x K needs ldb >= K); checked before the device."""
    h = _header()
    assert int(re.search(r"#define TILEC_MM_TRANS_A (\d+)", h).group(1)) == _native.TRANS_A == 1
    assert int(re.search(r"#define TILEC_MM_TRANS_B (\d+)", h).group(1)) == _native.TRANS_B == 2
    lib = _native.load()
    M, N, K = 8, 6, 20
    ta = _native.make_cfg("auto", 0, _native.TRANS_A)
    tb = _native.make_cfg("auto", 0, _native.TRANS_B)
    # row-major A needs lda >= K = 20; transposed A needs lda >= M = 8
    assert lib.tilec_mm_f32(16, 16, 16, M, N, K, 8, N, N, None, None, 0, None) == 1
    assert lib.tilec_mm_f32(16, 16, 16, M, N, K, 7, N, N, ctypes.byref(ta), None, 0, None) == 1
    # row-major B needs ldb >= N = 6; transposed B needs ldb >= K = 20
    assert lib.tilec_mm_f32(16, 16, 16, M, N, K, K, 19, N, ctypes.byref(tb), None, 0, None) == 1
    if not torch.cuda.is_available():
        # valid for the transposed layouts: gets past the argument checks to the device
        assert lib.tilec_mm_f32(16, 16, 16, M, N, K, 8, N, N, ctypes.byref(ta), None, 0, None) == 3
        assert lib.tilec_mm_f32(16, 16, 16, M, N, K, K, K, N, ctypes.byref(tb), None, 0, None) == 3


def test_wait_limit_rejects_negative_before_device():
    lib = _native.load()
    assert lib.tilec_mm_set_wait_limit(-1, None) == 1  # TILEC_ERR_BAD_ARG
    assert _native.status_bits(0) == "clean"
    assert _native.status_bits(1) == "TIMEOUT" and _native.status_bits(5) == "TIMEOUT|BAD_LAUNCH"


def test_fast_call_module_matches_ctypes():
    """The CPython fast-call module (csrc/fastcall.c) builds, is installed with the loaded
    library's entry points, and returns exactly what the ctypes calls return (argument
    errors caught before any device work; a size query with no device)."""
    build.build_fast()
    lib = _native.load()
    fast = _native.fast()
    assert fast is not None, _native.fast_error()
    cfg = _native.make_cfg("auto", 0, 0)
    cases = [(0, 0, 0, -1, 4, 4, 4, 4, 4), (0, 0, 0, 4, 4, 4, 2, 4, 4), (16, 32, 48, 4, 4, 4, 4, 4, 4),
             (16, 32, 48, 4, 4, 4, 4, 4, 2)]
    for args in cases:
        assert fast.mm(*args, cfg.variant, cfg.split_k, cfg.flags, None, 0, None) == \
            lib.tilec_mm_f32(*args, ctypes.byref(cfg), None, 0, None), args
        assert fast.ws_bytes(*args, cfg.variant, cfg.split_k, cfg.flags) == \
            lib.tilec_mm_workspace_bytes(*args, ctypes.byref(cfg)), args
    with pytest.raises(TypeError):
        fast.mm(0, 0, 0)
    with pytest.raises(ValueError):
        fast.mm(*cases[0], 0, 0, 0, None, -1, None)
