"""CPU: libkq.so builds, loads and exports every entry point include/kq.h
declares (no compute call: there is no GPU here)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "kq.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b(kq_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def libkq():
    from kq import build as kqbuild  # noqa: F401  (k-search_b200/kq/build.py)
    path = kqbuild.build()
    return ctypes.CDLL(path)


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("kq_gemm_f32act", "kq_mul_mat_q", "kq_quantize_q8_1", "kq_fa_decode_q8_0_mha",
              "kq_fa_decode_q8_0_ragged", "kq_w4a32c8_q4_0_fp32_int8", "kq_flash_attn_q8_0"):
        assert s in syms


def test_library_exports_all_declared(libkq):
    missing = [s for s in declared_symbols() if not hasattr(libkq, s)]
    assert not missing, missing


def test_python_binding_covers_header(libkq):
    from kq import _lib
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_host_only_entry_points(libkq):
    """Calls that do not touch a device: ABI version, block sizes, argument checks."""
    from kq import _lib
    L = _lib.lib()
    assert L.kq_abi_version() == 1
    assert [L.kq_block_bytes(t) for t in (0, 1, 2, 7)] == [18, 20, 34, 0]
    # invalid arguments are rejected before any CUDA call
    assert L.kq_mul_mat_q(9, None, None, None, 1, 1, 32, None) == 1
    assert "unknown weight type" in _lib.last_error()
    assert L.kq_gemm_f32act(0, None, None, None, 1, 1, 33, 2, None) == 1
    assert "multiple of 32" in _lib.last_error()
    assert L.kq_quantize_q8_1(None, None, 1, 31, 0, None) == 1
    assert L.kq_fa_decode_q8_0_mha(None, None, None, None, 1, 1, 1, 48, None) == 1
    # empty problems are no-ops
    assert L.kq_gemm_f32act(0, None, None, None, 0, 16, 64, 2, None) == 0
