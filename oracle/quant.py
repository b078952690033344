"""NumPy restatement of the KernelEvalPlus quantized-inference reference.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the shipped library
never imports this module.

Every function cites the reference it restates. Paths are relative to
``kernelevalplus-main/`` inside qhy991/K-Search.

Block layouts (``include/quant_types.h:59-152``):

=========  =====  ================================================
type       bytes  layout
=========  =====  ================================================
q4_0       18     fp16 d | 16 B nibbles (low = elem i, high = i+16)
q4_1       20     fp16 d | fp16 m | 16 B nibbles
q8_0       34     fp16 d | 32 x int8
q8_1       36     fp16 d | fp16 s | 32 x int8
=========  =====  ================================================
"""
from __future__ import annotations

import numpy as np

QK = 32
BLOCK_BYTES = {"q4_0": 18, "q4_1": 20, "q8_0": 34, "q8_1": 36}
WTYPES = ("q4_0", "q4_1", "q8_0")

# Activation-quantisation modes (the int8 codes are identical in all three;
# only the per-block scale d and sum s differ):
#   SUM_X   q8_1 as the reference stores it (quantize.py:165-214): fp16 d,
#           fp16 s = sum of the original fp32 values.
#   SUM_DQ  fp16 d, fp16 s = fp16(d) * sum(q) (the benchmark configurations'
#           convention; under it the q4_0 x q8_1 formula equals the
#           dequantise-then-matmul product exactly).
#   ACT_F32 fp32 d and fp32 s = sum of x, never rounded to fp16: the
#           per-definition W4A32C8 / W8A8C8 references
#           (core/operators/quant_gemm/variants/deepseek_v2/w4a32c8_q4_0_fp32_int8/reference.py:50-73,
#           .../deepseek_v3/w8a8c8_q8_0_q8_1/reference.py:43-59) quantise this way.
SUM_X = 0
SUM_DQ = 1
ACT_F32 = 2


def _f16_to_bytes(a: np.ndarray) -> np.ndarray:
    """fp32 array [...] -> uint8 [..., 2] holding the IEEE binary16 (RNE) bits."""
    h = np.ascontiguousarray(a.astype(np.float16))
    return h.view(np.uint8).reshape(a.shape + (2,))


def _bytes_to_f32(b: np.ndarray) -> np.ndarray:
    """uint8 [..., 2] little-endian binary16 -> fp32 [...]."""
    b = np.ascontiguousarray(b)
    return b.view(np.float16).reshape(b.shape[:-1]).astype(np.float32)


# ---------------------------------------------------------------------------
# Quantizers
# ---------------------------------------------------------------------------

def quantize_act(x: np.ndarray, mode: int = SUM_X):
    """fp32 [M, K] -> (q int8 [M, nb, 32], d fp32 [M, nb], s fp32 [M, nb]).

    Restates llm_kernel_test/reference/quantize.py:181-194: d = amax/127 in fp32
    (1.0 when amax == 0), q = round_half_even(x / d) clipped to [-128, 127],
    s = fp32 sum of x (numpy's pairwise order). ``mode`` selects whether d and
    s are rounded to fp16 (SUM_X, SUM_DQ) or kept in fp32 (ACT_F32)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    assert K % QK == 0
    nb = K // QK
    xb = x.reshape(M, nb, QK)
    amax = np.max(np.abs(xb), axis=2)
    d = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.round(xb / d[:, :, None]).clip(-128, 127).astype(np.int8)
    if mode == SUM_X:
        s = np.sum(xb, axis=2).astype(np.float16).astype(np.float32)
        d = d.astype(np.float16).astype(np.float32)
    elif mode == SUM_DQ:
        d = d.astype(np.float16).astype(np.float32)
        s = (d * q.astype(np.int32).sum(axis=2).astype(np.float32)).astype(np.float32)
        s = s.astype(np.float16).astype(np.float32)
    elif mode == ACT_F32:
        s = np.sum(xb, axis=2).astype(np.float32)
    else:
        raise ValueError(f"bad activation mode {mode}")
    return q, d, s


def quantize_q8_1(x: np.ndarray, sum_mode: int = SUM_X) -> np.ndarray:
    """fp32 [M, K] -> q8_1 bytes [M, K/32, 36] (quantize.py:165-214):
    ds = (fp16(d), fp16(s)) with s per ``sum_mode`` (SUM_X or SUM_DQ)."""
    if sum_mode not in (SUM_X, SUM_DQ):
        raise ValueError("q8_1 bytes hold fp16 d and s: use SUM_X or SUM_DQ")
    q, d, s = quantize_act(x, sum_mode)
    M, nb, _ = q.shape
    out = np.zeros((M, nb, 36), dtype=np.uint8)
    out[:, :, 0:2] = _f16_to_bytes(d)
    out[:, :, 2:4] = _f16_to_bytes(s)
    out[:, :, 4:] = q.view(np.uint8)
    return out


def quantize_q8_0(w: np.ndarray) -> np.ndarray:
    """fp32 [N, K] -> q8_0 bytes [N, K/32, 34]. Restates quantize.py:12-53."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    nb = K // QK
    wb = w.reshape(N, nb, QK)
    amax = np.max(np.abs(wb), axis=2)
    d = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.round(wb / d[:, :, None]).clip(-128, 127).astype(np.int8)
    out = np.zeros((N, nb, 34), dtype=np.uint8)
    out[:, :, 0:2] = _f16_to_bytes(d)
    out[:, :, 2:] = q.view(np.uint8)
    return out


def quantize_q4_0(w: np.ndarray) -> np.ndarray:
    """fp32 [N, K] -> q4_0 bytes [N, K/32, 18]. Restates quantize.py:56-102
    (d = amax/7, q = clip(round(x/d + 8), 0, 15), byte i = q[i] | q[i+16] << 4)."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    nb = K // QK
    wb = w.reshape(N, nb, QK)
    amax = np.max(np.abs(wb), axis=2)
    d = np.where(amax > 0, amax / np.float32(7.0), np.float32(1.0)).astype(np.float32)
    q = np.round(wb / d[:, :, None] + np.float32(8.0)).clip(0, 15).astype(np.uint8)
    out = np.zeros((N, nb, 18), dtype=np.uint8)
    out[:, :, 0:2] = _f16_to_bytes(d)
    out[:, :, 2:] = (q[:, :, :16] & 0x0F) | ((q[:, :, 16:] & 0x0F) << 4)
    return out


def quantize_q4_1(w: np.ndarray) -> np.ndarray:
    """fp32 [N, K] -> q4_1 bytes [N, K/32, 20]. Restates quantize.py:105-162
    (d = (max-min)/15, m = min, q = clip(round((x-m)/d), 0, 15))."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    N, K = w.shape
    nb = K // QK
    wb = w.reshape(N, nb, QK)
    mn = np.min(wb, axis=2)
    mx = np.max(wb, axis=2)
    d = np.where(mx > mn, (mx - mn) / np.float32(15.0), np.float32(1.0)).astype(np.float32)
    q = np.round((wb - mn[:, :, None]) / d[:, :, None]).clip(0, 15).astype(np.uint8)
    out = np.zeros((N, nb, 20), dtype=np.uint8)
    out[:, :, 0:2] = _f16_to_bytes(d)
    out[:, :, 2:4] = _f16_to_bytes(mn)
    out[:, :, 4:] = (q[:, :, :16] & 0x0F) | ((q[:, :, 16:] & 0x0F) << 4)
    return out


def quantize_weights(wtype: str, w: np.ndarray) -> np.ndarray:
    return {"q4_0": quantize_q4_0, "q4_1": quantize_q4_1, "q8_0": quantize_q8_0}[wtype](w)


# ---------------------------------------------------------------------------
# Synthetic weight generators of the benchmark configurations
# ---------------------------------------------------------------------------

def make_q4_0_blocks(rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    """q4_0 blocks drawn directly: d = fp16(|N(0, 0.02)| / 8), 16 nibble bytes
    uniform in 0..255 (both nibbles uniform in 0..15). Returns [N, K/32, 18]."""
    nb = K // QK
    d = (np.abs(rng.standard_normal((N, nb), dtype=np.float32) * np.float32(0.02)) / np.float32(8.0))
    out = np.empty((N, nb, 18), dtype=np.uint8)
    out[:, :, 0:2] = _f16_to_bytes(d.astype(np.float32))
    out[:, :, 2:] = rng.integers(0, 256, size=(N, nb, 16), dtype=np.uint8)
    return out


def make_q4_1_blocks(rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    """q4_1 blocks drawn directly: d as q4_0, m = fp16(-8 d), nibbles uniform."""
    nb = K // QK
    d = (np.abs(rng.standard_normal((N, nb), dtype=np.float32) * np.float32(0.02)) / np.float32(8.0))
    out = np.empty((N, nb, 20), dtype=np.uint8)
    out[:, :, 0:2] = _f16_to_bytes(d.astype(np.float32))
    out[:, :, 2:4] = _f16_to_bytes((-8.0 * d).astype(np.float32))
    out[:, :, 4:] = rng.integers(0, 256, size=(N, nb, 16), dtype=np.uint8)
    return out


def make_q8_0_blocks(rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    """q8_0 blocks: int8 = clamp(round(N(0,1) * 40), +-127), d = fp16(0.02/40)."""
    nb = K // QK
    q = np.clip(np.round(rng.standard_normal((N, nb, QK), dtype=np.float32) * np.float32(40.0)), -127, 127).astype(np.int8)
    out = np.empty((N, nb, 34), dtype=np.uint8)
    out[:, :, 0:2] = _f16_to_bytes(np.full((N, nb), 0.02 / 40.0, dtype=np.float32))
    out[:, :, 2:] = q.view(np.uint8)
    return out


def make_blocks(wtype: str, rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    return {"q4_0": make_q4_0_blocks, "q4_1": make_q4_1_blocks, "q8_0": make_q8_0_blocks}[wtype](rng, N, K)


# ---------------------------------------------------------------------------
# Unpacking
# ---------------------------------------------------------------------------

def unpack_weights(wtype: str, w: np.ndarray, N: int, K: int):
    """Return (d [N,nb] f32, m [N,nb] f32 or None, q [N,nb,32] int32).

    q is the stored code: 0..15 for q4_0 / q4_1 (no -8 applied, as in
    gemm_ref.py:84-88), the signed int8 for q8_0 (gemm_ref.py:39-40)."""
    nb = K // QK
    blk = np.ascontiguousarray(w, dtype=np.uint8).reshape(N, nb, BLOCK_BYTES[wtype])
    d = _bytes_to_f32(blk[:, :, 0:2])
    if wtype == "q4_0":
        p = blk[:, :, 2:]
        q = np.concatenate([p & 0x0F, p >> 4], axis=-1).astype(np.int32)
        return d, None, q
    if wtype == "q4_1":
        m = _bytes_to_f32(blk[:, :, 2:4])
        p = blk[:, :, 4:]
        q = np.concatenate([p & 0x0F, p >> 4], axis=-1).astype(np.int32)
        return d, m, q
    if wtype == "q8_0":
        q = np.ascontiguousarray(blk[:, :, 2:]).view(np.int8).astype(np.int32)
        return d, None, q
    raise ValueError(wtype)


def unpack_q8_1(a: np.ndarray, M: int, K: int):
    """q8_1 bytes -> (d [M,nb] f32, s [M,nb] f32, q [M,nb,32] int32); gemm_ref.py:132-140."""
    nb = K // QK
    blk = np.ascontiguousarray(a, dtype=np.uint8).reshape(M, nb, 36)
    d = _bytes_to_f32(blk[:, :, 0:2])
    s = _bytes_to_f32(blk[:, :, 2:4])
    q = np.ascontiguousarray(blk[:, :, 4:]).view(np.int8).astype(np.int32)
    return d, s, q


def dequantize(wtype: str, w: np.ndarray, N: int, K: int) -> np.ndarray:
    """Weights -> fp32 [N, K]. q4_0: d*(q-8) (gemm_ref.py:92); q4_1: d*q+m
    (gemm_ref.py:191); q8_0: q*d (gemm_ref.py:43)."""
    d, m, q = unpack_weights(wtype, w, N, K)
    if wtype == "q4_0":
        x = d[:, :, None] * (q.astype(np.float32) - np.float32(8.0))
    elif wtype == "q4_1":
        x = d[:, :, None] * q.astype(np.float32) + m[:, :, None]
    else:
        x = q.astype(np.float32) * d[:, :, None]
    return x.reshape(N, K).astype(np.float32)


# ---------------------------------------------------------------------------
# GEMM formulas
# ---------------------------------------------------------------------------

def block_sums_i32(wtype: str, w: np.ndarray, a: np.ndarray, M: int, N: int, K: int) -> np.ndarray:
    """int32 sumi[m, n, b] = sum_i q_w[n,b,i] * q_a[m,b,i] (gemm_ref.py:146,
    include/gemm_reference.h:200-211). Computed exactly through fp64 BLAS
    (all partial sums are integers far below 2**53)."""
    _, _, qw = unpack_weights(wtype, w, N, K)
    _, _, qa = unpack_q8_1(a, M, K)
    A = qa.transpose(1, 0, 2).astype(np.float64)          # [nb, M, 32]
    B = qw.transpose(1, 2, 0).astype(np.float64)          # [nb, 32, N]
    s = np.matmul(A, B)                                   # [nb, M, N]
    return np.ascontiguousarray(s.transpose(1, 2, 0)).astype(np.int32)


def _formula(wtype, dw, mw, da, sa, sumi, M, N, nb):
    out = np.zeros((M, N), dtype=np.float64)
    for b in range(nb):
        sb = sumi[:, :, b]
        if wtype == "q4_0":
            out += dw[None, :, b] * (da[:, b:b + 1] * sb - np.float32(8.0) * sa[:, b:b + 1])
        elif wtype == "q4_1":
            out += dw[None, :, b] * da[:, b:b + 1] * sb + mw[None, :, b] * sa[:, b:b + 1]
        else:
            out += (dw[None, :, b].astype(np.float64) * da[:, b:b + 1].astype(np.float64)) * sb
    return out.astype(np.float32)


def gemm_q8_1(wtype: str, w: np.ndarray, a: np.ndarray, M: int, N: int, K: int) -> np.ndarray:
    """Weights x pre-quantized q8_1 activations -> fp32 [M, N], fp64 accumulation.

    q4_0: sum_b d_w*(d_a*sumi - 8*s_a)   gemm_ref.py:100-153
    q4_1: sum_b d_w*d_a*sumi + m_w*s_a    gemm_ref.py:274-331
    q8_0: sum_b d_w*d_a*sumi             include/gemm_reference.h:311-336,
          core/operators/quant_gemm/variants/deepseek_v3/w8a8c8_q8_0_q8_1/reference.py:61-68
    """
    dw, mw, _ = unpack_weights(wtype, w, N, K)
    da, sa, _ = unpack_q8_1(a, M, K)
    sumi = block_sums_i32(wtype, w, a, M, N, K)
    return _formula(wtype, dw, mw, da, sa, sumi, M, N, K // QK)


def block_sums_codes(wtype: str, w: np.ndarray, qa: np.ndarray, N: int, K: int) -> np.ndarray:
    """int32 block sums from int8 activation codes qa [M, nb, 32]."""
    _, _, qw = unpack_weights(wtype, w, N, K)
    A = qa.transpose(1, 0, 2).astype(np.float64)
    B = qw.transpose(1, 2, 0).astype(np.float64)
    return np.ascontiguousarray(np.matmul(A, B).transpose(1, 2, 0)).astype(np.int32)


def gemm_codes(wtype: str, w: np.ndarray, qa: np.ndarray, da: np.ndarray, sa: np.ndarray, M: int, N: int,
               K: int) -> np.ndarray:
    """The per-block formula on given activation codes qa int8 [M, K/32, 32]
    and block scales / sums da, sa [M, K/32] (fp32): the GEMM a kernel runs on
    activations it quantised itself (gemm_ref.py:100-153, 274-331;
    gemm_reference.h:311-336)."""
    dw, mw, _ = unpack_weights(wtype, w, N, K)
    sumi = block_sums_codes(wtype, w, np.asarray(qa, dtype=np.int8).reshape(M, K // QK, QK), N, K)
    return _formula(wtype, dw, mw, np.asarray(da, dtype=np.float32), np.asarray(sa, dtype=np.float32), sumi, M, N,
                    K // QK)


def gemm_f32act(wtype: str, w: np.ndarray, x: np.ndarray, M: int, N: int, K: int,
                mode: int = ACT_F32) -> np.ndarray:
    """The harness operator: fp32 activations quantised on the fly, then the
    same per-block formula. ACT_F32 is the per-definition W4A32C8 semantics
    (core/operators/quant_gemm/variants/deepseek_v2/w4a32c8_q4_0_fp32_int8/reference.py:5-95);
    SUM_X / SUM_DQ equal gemm_q8_1(quantize_q8_1(x)) bit for bit."""
    qa, da, sa = quantize_act(x, mode)
    dw, mw, _ = unpack_weights(wtype, w, N, K)
    sumi = block_sums_codes(wtype, w, qa, N, K)
    return _formula(wtype, dw, mw, da, sa, sumi, M, N, K // QK)


def gemm_dequant_f32(wtype: str, w: np.ndarray, x: np.ndarray, M: int, N: int, K: int) -> np.ndarray:
    """The harness's own correctness gate: dequantise the weights and do an fp32
    matmul with the fp32 activations (gemm_ref.py:13-48, 51-97, 156-199)."""
    W = dequantize(wtype, w, N, K)
    return (np.asarray(x, dtype=np.float32) @ W.T).astype(np.float32)


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """RMSNormHandler.get_reference_output (llm_kernel_test/op_test_handler.py:662-673):
    rms = sqrt(mean(x^2) + eps) per row, out = x / rms * weight. The mean and
    square root here are fp64 rounded once to fp32; the divide and the
    multiply are fp32, as torch does them. x fp32 [M, K], w fp32 [K]."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    ms = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    rms = np.sqrt(ms + eps).astype(np.float32)
    return ((x / rms).astype(np.float32) * w).astype(np.float32)


def nmse(out: np.ndarray, ref: np.ndarray) -> float:
    """NMSE as the harness computes it (llm_kernel_test/unified_test_runner.py:426-428)."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.mean((out - ref) ** 2) / (np.mean(ref ** 2) + 1e-10))


def rel_l2(out: np.ndarray, ref: np.ndarray) -> float:
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.linalg.norm(out - ref) / max(np.linalg.norm(ref), 1e-300))


def check_close(out: np.ndarray, ref: np.ndarray, rel_l2_tol: float = 1e-3,
                elem_rel: float = 1e-2, elem_abs_rms: float = 1e-3) -> tuple[bool, str]:
    """The fp32 parity bar: rel-L2 <= 1e-3 and per element
    |out - ref| <= 1e-2 |ref| + 1e-3 rms(ref)."""
    out = np.asarray(out, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    if out.shape != ref.shape:
        return False, f"shape {out.shape} != {ref.shape}"
    if not np.all(np.isfinite(out)):
        return False, "non-finite output"
    r = rel_l2(out, ref)
    rms = float(np.sqrt(np.mean(ref ** 2))) if ref.size else 0.0
    bad = np.abs(out - ref) > elem_rel * np.abs(ref) + elem_abs_rms * rms
    nbad = int(np.count_nonzero(bad))
    ok = (r <= rel_l2_tol) and nbad == 0
    return ok, f"rel_l2={r:.3e} bad_elems={nbad}/{out.size}"


def dequant_q8_0_rows(kv: np.ndarray, rows: int, D: int) -> np.ndarray:
    """q8_0 bytes [rows, D/32, 34] -> fp32 [rows, D] (x = q * d)."""
    return dequantize("q8_0", kv, rows, D)


def dequant_q4_0_rows(kv: np.ndarray, rows: int, D: int) -> np.ndarray:
    """q4_0 bytes of [rows, D] -> fp32 [rows, D] (value d (q - 8); low nibbles
    are elements 0-15 of a block, high nibbles 16-31: quantize.py:56-102)."""
    return dequantize("q4_0", np.asarray(kv, dtype=np.uint8).reshape(rows, -1), rows, D)


def dequant_kv_rows(kv_format: str, kv: np.ndarray, rows: int, D: int) -> np.ndarray:
    """A KV cache of one of the flash_attention definitions' formats
    (op_test_handler.py:489-534: q8_0 or q4_0 blocks of each D-long row, or
    fp16) -> fp32 [rows, D]."""
    if kv_format == "q8_0":
        return dequant_q8_0_rows(kv, rows, D)
    if kv_format == "q4_0":
        return dequant_q4_0_rows(kv, rows, D)
    if kv_format == "f16":
        return np.asarray(kv).view(np.float16).reshape(rows, D).astype(np.float32)
    raise ValueError(f"unknown KV format {kv_format!r}")


def flash_decode_mha(q: np.ndarray, k: np.ndarray, v: np.ndarray, S: int, H: int, D: int,
                     kv_format: str = "q8_0") -> np.ndarray:
    """Harness flash_attention op (llm_kernel_test/op_test_handler.py:489-534
    builds the cache from fp32 [S, H, D] as q8_0 / q4_0 blocks of the [S*H, D]
    rows or as fp16; :543-563 is the attention). K/V are dequantised from the
    cache bytes; scores, softmax and the weighted sum are in fp64.
    q: fp32 [B, H, D]; k, v: cache bytes. Returns fp32 [B, H, D]."""
    K_ = dequant_kv_rows(kv_format, k, S * H, D).reshape(S, H, D).astype(np.float64)
    V_ = dequant_kv_rows(kv_format, v, S * H, D).reshape(S, H, D).astype(np.float64)
    qq = np.asarray(q, dtype=np.float64)
    sc = np.einsum("bhd,shd->bhs", qq, K_) / np.sqrt(D)
    sc -= sc.max(axis=-1, keepdims=True)
    p = np.exp(sc)
    p /= p.sum(axis=-1, keepdims=True)
    return np.einsum("bhs,shd->bhd", p, V_).astype(np.float32)


def flash_decode_ragged(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_seqlens: np.ndarray,
                        Hq: int, Hkv: int, D: int, scale: float) -> np.ndarray:
    """Ragged GQA decode (benchmark configuration 3): query head h reads KV head
    h // (Hq / Hkv); sequence b owns cache rows cu_seqlens[b]:cu_seqlens[b+1].
    Same restated semantics as ``flash_decode_mha`` (fp64). q: fp16/fp32
    [B, Hq, D]; k, v: bytes of [T, Hkv, D/32, 34]. Returns fp64 [B, Hq, D]."""
    T = int(cu_seqlens[-1])
    B = len(cu_seqlens) - 1
    g = Hq // Hkv
    K_ = dequant_q8_0_rows(k, T * Hkv, D).reshape(T, Hkv, D).astype(np.float64)
    V_ = dequant_q8_0_rows(v, T * Hkv, D).reshape(T, Hkv, D).astype(np.float64)
    qq = np.asarray(q, dtype=np.float64)
    out = np.zeros((B, Hq, D), dtype=np.float64)
    for b in range(B):
        s0, s1 = int(cu_seqlens[b]), int(cu_seqlens[b + 1])
        if s1 == s0:
            continue
        for hk in range(Hkv):
            Kb = K_[s0:s1, hk, :]
            Vb = V_[s0:s1, hk, :]
            qh = qq[b, hk * g:(hk + 1) * g, :]           # [g, D]
            sc = (qh @ Kb.T) * scale
            sc -= sc.max(axis=-1, keepdims=True)
            p = np.exp(sc)
            p /= p.sum(axis=-1, keepdims=True)
            out[b, hk * g:(hk + 1) * g, :] = p @ Vb
    return out


# ---------------------------------------------------------------------------
# q4_0 MoE expert FFN (benchmark configuration 4)
# ---------------------------------------------------------------------------

def moe_route(logits: np.ndarray, topk: int):
    """softmax over experts, top-k (ties -> lower expert index), renormalised
    weights. Returns (idx [T, topk] int32, w [T, topk] fp64)."""
    l = np.asarray(logits, dtype=np.float64)
    T, E = l.shape
    order = np.argsort(-l, axis=1, kind="stable")[:, :topk]
    p = np.exp(l - l.max(axis=1, keepdims=True))
    p /= p.sum(axis=1, keepdims=True)
    pw = np.take_along_axis(p, order, axis=1)
    pw /= pw.sum(axis=1, keepdims=True)
    return order.astype(np.int32), pw


def silu(x: np.ndarray) -> np.ndarray:
    """x * sigmoid(x) (semantics of kernels/activation/silu.cuh:97 silu_mul)."""
    x = np.asarray(x, dtype=np.float64)
    return x / (1.0 + np.exp(-x))


def moe_forward(x: np.ndarray, logits: np.ndarray, w_gate, w_up, w_down, topk: int,
                H: int, I: int, sum_mode: int = SUM_DQ, tokens=None):
    """Grouped q4_0 expert FFN: route, then per expert
    y = W_down * q8_1( silu(W_gate * q8_1(x)) * (W_up * q8_1(x)) ),
    combined with the renormalised routing weights. w_gate/w_up/w_down are
    per-expert byte arrays ([I, H/32, 18] and [H, I/32, 18]). ``tokens``
    optionally restricts the output to a subset of token rows (the routing
    is still computed for all). Returns fp64 [len(tokens), H]."""
    T = x.shape[0]
    idx, wts = moe_route(logits, topk)
    rows = np.arange(T) if tokens is None else np.asarray(tokens)
    out = np.zeros((len(rows), H), dtype=np.float64)
    E = len(w_gate)
    for e in range(E):
        sel_t, sel_k = np.nonzero(idx[rows] == e)
        if len(sel_t) == 0:
            continue
        xt = np.ascontiguousarray(x[rows[sel_t]], dtype=np.float32)
        m = xt.shape[0]
        g = gemm_f32act("q4_0", w_gate[e], xt, m, I, H, sum_mode)
        u = gemm_f32act("q4_0", w_up[e], xt, m, I, H, sum_mode)
        h = (silu(g) * u.astype(np.float64)).astype(np.float32)
        y = gemm_f32act("q4_0", w_down[e], h, m, H, I, sum_mode)
        out[sel_t] += wts[rows[sel_t], sel_k][:, None] * y.astype(np.float64)
    return out
