"""PyTorch-facing operators over libkq (device tensors in, device tensors out).

Every function runs on the current CUDA stream of its input's device and
raises ``KQError`` on a non-zero status. Tensors must be contiguous CUDA
tensors; nothing here falls back to a CPU path.

Byte layouts are the reference's (kernelevalplus-main/include/quant_types.h):
weights are uint8 tensors holding N rows of K/32 blocks (any shape whose
element count is N * K/32 * block_bytes), q8_1 activations likewise.
"""
from __future__ import annotations

import ctypes
import math

import torch

from ._lib import check, lib

WTYPES = {"q4_0": 0, "q4_1": 1, "q8_0": 2}
BLOCK_BYTES = {"q4_0": 18, "q4_1": 20, "q8_0": 34, "q8_1": 36}
# Activation-quantisation modes (include/kq.h KQ_ACT_*).
ACT_MODES = {"sum_x": 0, "sum_dq": 1, "f32": 2}


def _wtype(wtype) -> int:
    if isinstance(wtype, int):
        return wtype
    w = str(wtype).replace("block_", "")
    if w not in WTYPES:
        raise ValueError(f"unsupported weight type {wtype!r}")
    return WTYPES[w]


def _act_mode(mode) -> int:
    return mode if isinstance(mode, int) else ACT_MODES[mode]


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(t: torch.Tensor, name: str, dtype=None, numel=None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if numel is not None and t.numel() != numel:
        raise ValueError(f"{name} has {t.numel()} elements, expected {numel}")
    return t


def quantize_q8_1(x: torch.Tensor, sum_mode: str = "sum_x") -> torch.Tensor:
    """fp32 [M, K] -> q8_1 bytes uint8 [M, K/32, 36] (quantize.py:165-214)."""
    _cuda(x, "x", torch.float32)
    M, K = x.shape
    y = torch.empty((M, K // 32, 36), dtype=torch.uint8, device=x.device)
    check(lib().kq_quantize_q8_1(x.data_ptr(), y.data_ptr(), M, K, _act_mode(sum_mode), _stream(x)),
          "kq_quantize_q8_1")
    return y


def quantize_rows(x: torch.Tensor, wtype="q8_0") -> torch.Tensor:
    """fp32 [rows, K] -> q4_0 / q4_1 / q8_0 bytes uint8 [rows, K/32, block_bytes]
    (quantize.py:12-162: weights and KV caches)."""
    _cuda(x, "x", torch.float32)
    wt = _wtype(wtype)
    rows, K = x.shape
    y = torch.empty((rows, K // 32, lib().kq_block_bytes(wt)), dtype=torch.uint8, device=x.device)
    check(lib().kq_quantize_rows(wt, x.data_ptr(), y.data_ptr(), rows, K, _stream(x)), "kq_quantize_rows")
    return y


def mul_mat_q(weight: torch.Tensor, a_q8_1: torch.Tensor, M: int, N: int, K: int, wtype="q4_0",
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Weights x pre-quantised q8_1 activations -> fp32 [M, N]."""
    wt = _wtype(wtype)
    nb = K // 32
    _cuda(weight, "weight", torch.uint8, N * nb * lib().kq_block_bytes(wt))
    _cuda(a_q8_1, "a_q8_1", torch.uint8, M * nb * 36)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=weight.device)
    check(lib().kq_mul_mat_q(wt, weight.data_ptr(), a_q8_1.data_ptr(), out.data_ptr(), M, N, K, _stream(weight)),
          "kq_mul_mat_q")
    return out


def gemm_f32act(weight: torch.Tensor, activation: torch.Tensor, M: int, N: int, K: int, wtype="q4_0",
                act_mode="f32", out: torch.Tensor | None = None) -> torch.Tensor:
    """Weights x fp32 activations quantised on the fly -> fp32 [M, N]
    (the harness quant_gemm operator; act_mode 'f32' is its semantics)."""
    wt = _wtype(wtype)
    nb = K // 32
    _cuda(weight, "weight", torch.uint8, N * nb * lib().kq_block_bytes(wt))
    _cuda(activation, "activation", torch.float32, M * K)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=weight.device)
    check(lib().kq_gemm_f32act(wt, weight.data_ptr(), activation.data_ptr(), out.data_ptr(), M, N, K,
                               _act_mode(act_mode), _stream(weight)), "kq_gemm_f32act")
    return out


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6, out: torch.Tensor | None = None) -> torch.Tensor:
    """x fp32 [M, K], weight fp32 [K] -> x / sqrt(mean(x^2) + eps) * weight
    (the harness rms_norm operator, op_test_handler.py:641-690)."""
    _cuda(x, "x", torch.float32)
    if x.dim() != 2:
        raise ValueError(f"x must be [M, K], got {tuple(x.shape)}")
    M, K = x.shape
    _cuda(weight, "weight", torch.float32, K)
    if out is None:
        out = torch.empty_like(x)
    check(lib().kq_rms_norm_f32(x.data_ptr(), weight.data_ptr(), out.data_ptr(), M, K, float(eps), _stream(x)),
          "kq_rms_norm_f32")
    return out


def rms_norm_quantize_q8_1(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6,
                           sum_mode: str = "sum_x") -> torch.Tensor:
    """RMSNorm fused into quantize_q8_1: fp32 [M, K] -> q8_1 bytes uint8
    [M, K/32, 36] of the normalised rows."""
    _cuda(x, "x", torch.float32)
    M, K = x.shape
    _cuda(weight, "weight", torch.float32, K)
    y = torch.empty((M, K // 32, 36), dtype=torch.uint8, device=x.device)
    check(lib().kq_rms_norm_quantize_q8_1(x.data_ptr(), weight.data_ptr(), y.data_ptr(), M, K, float(eps),
                                          _act_mode(sum_mode), _stream(x)), "kq_rms_norm_quantize_q8_1")
    return y


def gemm_f32act_rmsnorm(weight: torch.Tensor, activation: torch.Tensor, norm_weight: torch.Tensor, M: int, N: int,
                        K: int, wtype="q4_0", act_mode="f32", eps: float = 1e-6,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """gemm_f32act on rms_norm(activation, norm_weight, eps), the RMSNorm
    fused into the on-the-fly quantisation -> fp32 [M, N]."""
    wt = _wtype(wtype)
    _cuda(weight, "weight", torch.uint8, N * (K // 32) * lib().kq_block_bytes(wt))
    _cuda(activation, "activation", torch.float32, M * K)
    _cuda(norm_weight, "norm_weight", torch.float32, K)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=weight.device)
    check(lib().kq_gemm_f32act_rmsnorm(wt, weight.data_ptr(), activation.data_ptr(), norm_weight.data_ptr(),
                                       float(eps), out.data_ptr(), M, N, K, _act_mode(act_mode), _stream(weight)),
          "kq_gemm_f32act_rmsnorm")
    return out


def gemm_f32act_scatter(weight: torch.Tensor, activation: torch.Tensor, outs: list[int], ldo: int, col0: int, M: int,
                        N: int, K: int, wtype="q4_0", act_mode="sum_dq", stream_of: torch.Tensor | None = None) -> None:
    """kq_gemm_f32act_scatter: the fused GEMM writing element (m, n) to
    outs[d] + (m * ldo + col0 + n) * 4 bytes for every destination address d
    (device pointers, e.g. peer mappings from kq.dist.PeerBuffer)."""
    wt = _wtype(wtype)
    _cuda(weight, "weight", torch.uint8, N * (K // 32) * lib().kq_block_bytes(wt))
    _cuda(activation, "activation", torch.float32, M * K)
    if not 1 <= len(outs) <= 8:
        raise ValueError("1 to 8 destinations")
    arr = (ctypes.c_void_p * len(outs))(*[int(o) for o in outs])
    check(lib().kq_gemm_f32act_scatter(wt, weight.data_ptr(), activation.data_ptr(), arr, len(outs), ldo, col0, M, N,
                                       K, _act_mode(act_mode), _stream(stream_of if stream_of is not None else weight)),
          "kq_gemm_f32act_scatter")


def mul_mat_q8x(weight: torch.Tensor, a_qs: torch.Tensor, a_ds: torch.Tensor, M: int, N: int, K: int, wtype="q4_0",
                out: torch.Tensor | None = None) -> torch.Tensor:
    """Weights x staged activations (int8 codes [M, K], fp32 (d, s) [M, K/32, 2]) -> fp32 [M, N]."""
    wt = _wtype(wtype)
    nb = K // 32
    _cuda(weight, "weight", torch.uint8, N * nb * lib().kq_block_bytes(wt))
    _cuda(a_qs, "a_qs", torch.int8, M * K)
    _cuda(a_ds, "a_ds", torch.float32, M * nb * 2)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=weight.device)
    check(lib().kq_mul_mat_q8x(wt, weight.data_ptr(), a_qs.data_ptr(), a_ds.data_ptr(), out.data_ptr(), M, N, K,
                               _stream(weight)), "kq_mul_mat_q8x")
    return out


def moe_q4_0(x: torch.Tensor, router_logits: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
             w_down: torch.Tensor, topk: int = 2, act_mode="sum_dq", out: torch.Tensor | None = None) -> torch.Tensor:
    """Grouped q4_0 MoE FFN: x fp32 [T, H], logits fp32 [T, E]; w_gate / w_up uint8
    [E, I, H/32, 18], w_down uint8 [E, H, I/32, 18]. Returns fp32 [T, H]."""
    _cuda(x, "x", torch.float32)
    T, H = x.shape
    _cuda(router_logits, "router_logits", torch.float32)
    E = router_logits.shape[1]
    _cuda(w_gate, "w_gate", torch.uint8)
    _cuda(w_up, "w_up", torch.uint8)
    _cuda(w_down, "w_down", torch.uint8)
    I = w_gate.numel() // (E * (H // 32) * 18)
    if w_gate.numel() != E * I * (H // 32) * 18 or w_up.numel() != w_gate.numel() or w_down.numel() != E * H * (I // 32) * 18:
        raise ValueError("expert weight sizes do not match [E, I, H/32, 18] / [E, H, I/32, 18]")
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=x.device)
    check(lib().kq_moe_q4_0(x.data_ptr(), router_logits.data_ptr(), w_gate.data_ptr(), w_up.data_ptr(),
                            w_down.data_ptr(), E, topk, T, H, I, _act_mode(act_mode), out.data_ptr(), _stream(x)),
          "kq_moe_q4_0")
    return out


def moe_route(router_logits: torch.Tensor, topk: int = 2) -> tuple[torch.Tensor, torch.Tensor]:
    """Router: (idx int32 [T, topk], wts fp32 [T, topk]) from logits fp32 [T, E]."""
    _cuda(router_logits, "router_logits", torch.float32)
    T, E = router_logits.shape
    idx = torch.empty((T, topk), dtype=torch.int32, device=router_logits.device)
    wts = torch.empty((T, topk), dtype=torch.float32, device=router_logits.device)
    check(lib().kq_moe_route(router_logits.data_ptr(), T, E, topk, idx.data_ptr(), wts.data_ptr(),
                             _stream(router_logits)), "kq_moe_route")
    return idx, wts


def moe_experts_q4_0(x_rows: torch.Tensor, expert_of_row: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                     w_down: torch.Tensor, act_mode="sum_dq", out: torch.Tensor | None = None) -> torch.Tensor:
    """Expert FFNs of routed rows: x_rows fp32 [P, H], expert_of_row int32 [P]
    (indices into this call's experts); weights as in moe_q4_0. fp32 [P, H]."""
    _cuda(x_rows, "x_rows", torch.float32)
    P, H = x_rows.shape
    _cuda(expert_of_row, "expert_of_row", torch.int32, P)
    _cuda(w_gate, "w_gate", torch.uint8)
    _cuda(w_up, "w_up", torch.uint8)
    _cuda(w_down, "w_down", torch.uint8)
    E = w_gate.shape[0]
    I = w_gate.numel() // (E * (H // 32) * 18)
    if w_gate.numel() != E * I * (H // 32) * 18 or w_up.numel() != w_gate.numel() or w_down.numel() != E * H * (I // 32) * 18:
        raise ValueError("expert weight sizes do not match [E, I, H/32, 18] / [E, H, I/32, 18]")
    if out is None:
        out = torch.empty((P, H), dtype=torch.float32, device=x_rows.device)
    check(lib().kq_moe_experts_q4_0(x_rows.data_ptr(), expert_of_row.data_ptr(), w_gate.data_ptr(), w_up.data_ptr(),
                                    w_down.data_ptr(), E, P, H, I, _act_mode(act_mode), out.data_ptr(),
                                    _stream(x_rows)), "kq_moe_experts_q4_0")
    return out


def moe_experts_q4_0_q8_1(a_rows: torch.Tensor, expert_of_row: torch.Tensor, w_gate: torch.Tensor,
                          w_up: torch.Tensor, w_down: torch.Tensor, act_mode="sum_dq",
                          out: torch.Tensor | None = None) -> torch.Tensor:
    """moe_experts_q4_0 on pre-quantised rows: a_rows uint8 [P, H/32, 36] (or
    [P, H/32 * 36]) q8_1 blocks as quantize_q8_1 writes them; act_mode is the
    re-quantisation mode of silu(gate) * up. fp32 [P, H]."""
    _cuda(a_rows, "a_rows", torch.uint8)
    P = a_rows.shape[0]
    H = a_rows.numel() // max(P, 1) // 36 * 32
    if a_rows.numel() != P * (H // 32) * 36:
        raise ValueError("a_rows must hold P rows of q8_1 blocks (36 bytes per 32 values)")
    _cuda(expert_of_row, "expert_of_row", torch.int32, P)
    _cuda(w_gate, "w_gate", torch.uint8)
    _cuda(w_up, "w_up", torch.uint8)
    _cuda(w_down, "w_down", torch.uint8)
    E = w_gate.shape[0]
    I = w_gate.numel() // (E * (H // 32) * 18)
    if w_gate.numel() != E * I * (H // 32) * 18 or w_up.numel() != w_gate.numel() or w_down.numel() != E * H * (I // 32) * 18:
        raise ValueError("expert weight sizes do not match [E, I, H/32, 18] / [E, H, I/32, 18]")
    if out is None:
        out = torch.empty((P, H), dtype=torch.float32, device=a_rows.device)
    check(lib().kq_moe_experts_q4_0_q8_1(a_rows.data_ptr(), expert_of_row.data_ptr(), w_gate.data_ptr(),
                                         w_up.data_ptr(), w_down.data_ptr(), E, P, H, I, _act_mode(act_mode),
                                         out.data_ptr(), _stream(a_rows)), "kq_moe_experts_q4_0_q8_1")
    return out


def moe_combine(y: torch.Tensor, wts: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum_k wts[t, k] * y[t * topk + k]; y fp32 [T * topk, H]."""
    _cuda(wts, "wts", torch.float32)
    T, topk = wts.shape
    _cuda(y, "y", torch.float32)
    if y.dim() != 2 or y.shape[0] != T * topk:
        raise ValueError(f"y must be [T * topk, H] = [{T * topk}, H], got {tuple(y.shape)}")
    H = y.shape[1]
    if out is None:
        out = torch.empty((T, H), dtype=torch.float32, device=y.device)
    check(lib().kq_moe_combine(y.data_ptr(), wts.data_ptr(), T, topk, H, out.data_ptr(), _stream(y)), "kq_moe_combine")
    return out


def block_sums_i32(weight: torch.Tensor, a_q8_1: torch.Tensor, M: int, N: int, K: int, wtype="q4_0") -> torch.Tensor:
    """int32 sumi [M, N, K/32] (the bit-exact parity quantity)."""
    wt = _wtype(wtype)
    nb = K // 32
    _cuda(weight, "weight", torch.uint8, N * nb * lib().kq_block_bytes(wt))
    _cuda(a_q8_1, "a_q8_1", torch.uint8, M * nb * 36)
    out = torch.empty((M, N, nb), dtype=torch.int32, device=weight.device)
    check(lib().kq_block_sums_i32(wt, weight.data_ptr(), a_q8_1.data_ptr(), out.data_ptr(), M, N, K, _stream(weight)),
          "kq_block_sums_i32")
    return out


# KV cache formats of the flash_attention definitions (include/kq.h KQ_KV_*)
# and the bytes of one 32-element group of a cache row in each.
KV_FORMATS = {"q8_0": 0, "q4_0": 1, "f16": 2}
KV_GROUP_BYTES = {"q8_0": 34, "q4_0": 18, "f16": 64}


def flash_attn(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor, batch_size: int,
               seq_len: int, num_heads: int, head_dim: int, kv_format: str = "q8_0") -> torch.Tensor:
    """Harness flash_attention -> fp32 [B, H, D]. query fp32 [B, H, D]; the
    caches are the [S, H, D] rows as q8_0 blocks, q4_0 blocks or fp16."""
    if kv_format not in KV_FORMATS:
        raise ValueError(f"unknown KV format {kv_format!r} (expected one of {sorted(KV_FORMATS)})")
    _cuda(query, "query", torch.float32, batch_size * num_heads * head_dim)
    nbytes = seq_len * num_heads * (head_dim // 32) * KV_GROUP_BYTES[kv_format]
    _cuda(key_cache, "key_cache", None, None)
    _cuda(value_cache, "value_cache", None, None)
    if key_cache.numel() * key_cache.element_size() != nbytes or value_cache.numel() * value_cache.element_size() != nbytes:
        raise ValueError(f"{kv_format} cache size does not match seq_len * num_heads * head_dim/32 * "
                         f"{KV_GROUP_BYTES[kv_format]} bytes")
    out = torch.empty((batch_size, num_heads, head_dim), dtype=torch.float32, device=query.device)
    check(lib().kq_fa_decode_mha(KV_FORMATS[kv_format], query.data_ptr(), key_cache.data_ptr(),
                                 value_cache.data_ptr(), out.data_ptr(), batch_size, seq_len, num_heads, head_dim,
                                 _stream(query)),
          "kq_fa_decode_mha")
    return out


def flash_attn_q8_0(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor, batch_size: int,
                    seq_len: int, num_heads: int, head_dim: int) -> torch.Tensor:
    """Harness flash_attention with q8_0 caches -> fp32 [B, H, D]."""
    return flash_attn(query, key_cache, value_cache, batch_size, seq_len, num_heads, head_dim, "q8_0")


def flash_decode_ragged(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens: torch.Tensor, num_kv_heads: int,
                        max_seqlen: int | None = None, scale: float | None = None,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """Ragged GQA decode: q fp16 [B, Hq, D]; k, v q8_0 bytes of [T, Hkv, D]
    (T cache rows); cu_seqlens int32 [B+1] (device). Returns fp16 [B, Hq, D]."""
    _cuda(q, "q", torch.float16)
    B, Hq, D = q.shape
    _cuda(cu_seqlens, "cu_seqlens", torch.int32, B + 1)
    _cuda(k, "k")
    _cuda(v, "v")
    row_bytes = num_kv_heads * (D // 32) * 34
    nbytes = k.numel() * k.element_size()
    if nbytes % row_bytes or v.numel() * v.element_size() != nbytes:
        raise ValueError("k/v must hold whole cache rows of num_kv_heads * D/32 q8_0 blocks")
    total_rows = nbytes // row_bytes
    if max_seqlen is None:
        max_seqlen = int((cu_seqlens[1:] - cu_seqlens[:-1]).max().item()) if B else 0
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    check(lib().kq_fa_decode_q8_0_ragged(q.data_ptr(), k.data_ptr(), v.data_ptr(), cu_seqlens.data_ptr(), B, Hq,
                                         num_kv_heads, D, int(max_seqlen), int(total_rows), float(scale),
                                         out.data_ptr(), _stream(q)),
          "kq_fa_decode_q8_0_ragged")
    return out


def device_error(stream: torch.cuda.Stream | None = None) -> int:
    """Read and clear the device error word (0 = no device-side error)."""
    import ctypes

    s = (stream or torch.cuda.current_stream()).cuda_stream
    code = ctypes.c_int(0)
    check(lib().kq_device_error(ctypes.byref(code), s), "kq_device_error")
    return code.value
