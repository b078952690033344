"""ctypes binding of libkq.so (the C ABI declared in include/kq.h).

The library is built in-tree (``python k-search_b200/kq/build.py``) and loaded
from this package directory. There is no fallback: if the library is missing
or fails to load, every operator raises.
"""
from __future__ import annotations

import ctypes
import os

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG_DIR, "libkq.so")

KQ_OK = 0
STATUS_NAMES = {
    0: "KQ_OK", 1: "KQ_ERR_INVALID", 2: "KQ_ERR_UNSUPPORTED", 3: "KQ_ERR_CUDA",
    4: "KQ_ERR_NOMEM", 5: "KQ_ERR_TIMEOUT", 6: "KQ_ERR_DEVICE",
}

# (name, restype, argtypes) of every symbol include/kq.h declares.
_vp, _i, _i64, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "kq_abi_version": (_i, []),
    "kq_last_error": (ctypes.c_char_p, []),
    "kq_block_bytes": (_sz, [_i]),
    "kq_device_error": (_i, [_vp, _vp]),
    "kq_selftest_wait_timeout": (_i, [_i64, _vp]),
    "kq_w4a32c8_q4_0_fp32_int8": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "kq_w4a32c8_q4_1_fp32_int8": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "kq_w8a32c8_q8_0_fp32_int8": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "kq_w4a8_q4_0_q8_1": (None, [_vp, _vp, _vp, _i, _i, _i]),
    "kq_flash_attn_q8_0": (None, [_vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    "kq_flash_attn_q4_0": (None, [_vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    "kq_flash_attn_f16": (None, [_vp, _vp, _vp, _vp, _i, _i, _i, _i]),
    "kq_rms_norm": (None, [_vp, _vp, _vp, _i, _i]),
    "kq_rms_norm_f32": (_i, [_vp, _vp, _vp, _i, _i, _f, _vp]),
    "kq_rms_norm_quantize_q8_1": (_i, [_vp, _vp, _vp, _i, _i, _f, _i, _vp]),
    "kq_gemm_f32act_rmsnorm": (_i, [_i, _vp, _vp, _vp, _f, _vp, _i, _i, _i, _i, _vp]),
    "kq_quantize_q8_1": (_i, [_vp, _vp, _i64, _i64, _i, _vp]),
    "kq_quantize_rows": (_i, [_i, _vp, _vp, _i64, _i64, _vp]),
    "kq_mul_mat_q": (_i, [_i, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "kq_gemm_f32act": (_i, [_i, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "kq_gemm_f32act_noalloc": (_i, [_i, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "kq_noalloc_device_error": (_i, [_vp, _vp]),
    "kq_mul_mat_q8x": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "kq_moe_q4_0": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp]),
    "kq_gemm_f32act_scatter": (_i, [_i, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "kq_peer_alloc": (_i, [ctypes.c_size_t, _vp, _vp]),
    "kq_peer_open": (_i, [_vp, _vp]),
    "kq_peer_close": (_i, [_vp]),
    "kq_peer_free": (_i, [_vp]),
    "kq_copy_2d": (_i, [_vp, ctypes.c_size_t, _vp, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_size_t, _vp]),
    "kq_moe_route": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp]),
    "kq_moe_experts_q4_0": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp]),
    "kq_moe_experts_q4_0_q8_1": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp]),
    "kq_moe_experts_stages_q4_0": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp,
                                        _vp]),
    "kq_moe_combine": (_i, [_vp, _vp, _i, _i, _i, _vp, _vp]),
    "kq_block_sums_i32": (_i, [_i, _vp, _vp, _vp, _i, _i, _i, _vp]),
    "kq_fa_decode_q8_0_mha": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "kq_fa_decode_mha": (_i, [_i, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "kq_fa_decode_q8_0_ragged": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _f, _vp, _vp]),
}

_lib: ctypes.CDLL | None = None


class KQError(RuntimeError):
    """A libkq entry point returned a non-zero status."""

    def __init__(self, status: int, what: str, msg: str):
        self.status = status
        super().__init__(f"{what}: {STATUS_NAMES.get(status, status)}: {msg}")


def lib() -> ctypes.CDLL:
    """Load libkq.so (once). Raises if it is absent: there is no CPU path."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"libkq.so not built: {LIB_PATH} (run k-search_b200/kq/build.py)")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    v = lib().kq_last_error()
    return v.decode() if v else ""


def check(status: int, what: str) -> None:
    if status != KQ_OK:
        raise KQError(status, what, last_error())
