"""kq: B200 (sm_100a) kernels for the GGML block-quantized inference path of
KernelEvalPlus (qhy991/K-Search), behind the C ABI in include/kq.h.

    import kq
    out = kq.gemm_f32act(weight_u8, act_f32, M, N, K, wtype="q4_0")

``kq.harness`` mirrors the KernelEvalPlus operator interface (module.forward
signatures, test configurations, performance accounting).
"""
from ._lib import KQError, lib, LIB_PATH  # noqa: F401
from . import harness  # noqa: F401
from .ops import (  # noqa: F401
    ACT_MODES, BLOCK_BYTES, WTYPES, block_sums_i32, device_error, flash_attn, flash_attn_q8_0, flash_decode_ragged,
    gemm_f32act, gemm_f32act_rmsnorm, gemm_f32act_scatter, moe_combine, moe_experts_q4_0, moe_experts_q4_0_q8_1, moe_q4_0,
    moe_route, mul_mat_q,
    mul_mat_q8x, quantize_q8_1, quantize_rows, rms_norm, rms_norm_quantize_q8_1,
)
