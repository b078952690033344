"""CPU: the oracle against the reference's own outputs (golden fixtures made
by tests/golden/make_golden.py from the reference's Python functions)."""
import os

import numpy as np
import pytest

from oracle import quant as Q

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_quantizers_bit_exact():
    g = _load("quantize.npz")
    assert np.array_equal(Q.quantize_q8_1(g["x"]).reshape(-1), g["q8_1"])
    for t in ("q8_0", "q4_0", "q4_1"):
        assert np.array_equal(Q.quantize_weights(t, g["w"]).reshape(-1), g[t]), t


def test_q8_1_edge_rows():
    g = _load("quantize.npz")
    q = Q.quantize_q8_1(g["x"])
    # amax == 0 -> d = 1.0 (fp16 0x3C00), all codes 0, s = +0
    assert q[1, 0, 0] == 0x00 and q[1, 0, 1] == 0x3C and not q[1, :, 4:].any()
    # a block of -0.0 sums to +0.0 (numpy adds the pairwise sum to +0)
    assert q[5, 0, 2] == 0 and q[5, 0, 3] == 0


@pytest.mark.parametrize("wtype,key", [("q4_0", "ref_q4_0_q8_1"), ("q4_1", "ref_q4_1_q8_1")])
def test_q8_1_gemm_matches_reference(wtype, key):
    g = _load("gemm.npz")
    M, N, K = int(g["M"]), int(g["N"]), int(g["K"])
    out = Q.gemm_q8_1(wtype, g["w_" + wtype], g["a_q8_1"], M, N, K)
    assert np.array_equal(out, g[key])


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
def test_harness_gate_matches_reference(wtype):
    g = _load("gemm.npz")
    M, N, K = int(g["M"]), int(g["N"]), int(g["K"])
    out = Q.gemm_dequant_f32(wtype, g["w_" + wtype], g["act"], M, N, K)
    assert np.array_equal(out, g[f"ref_{wtype}_fp32"])
    # the quantised-activation operator passes the harness's NMSE <= 0.05 gate
    for mode in (Q.SUM_X, Q.SUM_DQ, Q.ACT_F32):
        assert Q.nmse(Q.gemm_f32act(wtype, g["w_" + wtype], g["act"], M, N, K, mode), out) < 0.05


def test_variant_references():
    """ACT_F32 is the per-definition W4A32C8 / W8A8C8 semantics (fp32 d, s)."""
    g = _load("variants.npz")
    M, N, K = int(g["M"]), int(g["N"]), int(g["K"])
    ok, msg = Q.check_close(Q.gemm_f32act("q4_0", g["w_q4_0"], g["act"], M, N, K, Q.ACT_F32), g["ref_w4a32c8"],
                            1e-5, 1e-4, 1e-6)
    assert ok, msg
    ok, msg = Q.check_close(Q.gemm_f32act("q8_0", g["w_q8_0"], g["act"], M, N, K, Q.ACT_F32), g["ref_w8a8c8"],
                            1e-5, 1e-4, 1e-6)
    assert ok, msg
    assert np.array_equal(Q.gemm_q8_1("q4_0", g["w_q4_0"], g["a_q8_1"], M, N, K), g["ref_w4a8"])


def test_sum_modes_equal_two_step_path():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((7, 256)).astype(np.float32)
    for t in Q.WTYPES:
        w = Q.make_blocks(t, rng, 16, 256)
        for mode in (Q.SUM_X, Q.SUM_DQ):
            assert np.array_equal(Q.gemm_f32act(t, w, x, 7, 16, 256, mode),
                                  Q.gemm_q8_1(t, w, Q.quantize_q8_1(x, mode), 7, 16, 256))


def test_sum_dq_equals_dequant_matmul():
    """Under s = d * sum(q) the q4_0 formula is the dequantise-both-then-matmul product."""
    rng = np.random.default_rng(4)
    M, N, K = 3, 32, 512
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = Q.make_q4_0_blocks(rng, N, K)
    a = Q.quantize_q8_1(x, Q.SUM_DQ)
    da, sa, qa = Q.unpack_q8_1(a, M, K)
    xa = (qa * da[:, :, None].astype(np.float64)).reshape(M, K)
    ref = xa @ Q.dequantize("q4_0", w, N, K).astype(np.float64).T
    ok, msg = Q.check_close(Q.gemm_q8_1("q4_0", w, a, M, N, K), ref, 2e-3, 5e-2, 2e-3)
    assert ok, msg


def test_gemm_codes_equals_gemm_f32act():
    """gemm_codes on the oracle quantiser's own codes and scales is the
    quant_gemm formula bit for bit (the MoE down projection check uses it on
    codes the GPU formed)."""
    rng = np.random.default_rng(21)
    M, N, K = 5, 64, 256
    x = rng.standard_normal((M, K)).astype(np.float32)
    for wtype in ("q4_0", "q4_1", "q8_0"):
        w = Q.make_blocks(wtype, rng, N, K)
        for mode in (Q.SUM_X, Q.SUM_DQ, Q.ACT_F32):
            qa, da, sa = Q.quantize_act(x, mode)
            assert np.array_equal(Q.gemm_codes(wtype, w, qa, da, sa, M, N, K), Q.gemm_f32act(wtype, w, x, M, N, K, mode))


def test_block_sums_direct():
    rng = np.random.default_rng(5)
    M, N, K = 2, 5, 96
    for t in Q.WTYPES:
        w = Q.make_blocks(t, rng, N, K)
        a = Q.quantize_q8_1(rng.standard_normal((M, K)).astype(np.float32))
        s = Q.block_sums_i32(t, w, a, M, N, K)
        _, _, qw = Q.unpack_weights(t, w, N, K)
        _, _, qa = Q.unpack_q8_1(a, M, K)
        for m in range(M):
            for n in range(N):
                for b in range(K // 32):
                    assert s[m, n, b] == int(np.dot(qw[n, b].astype(np.int64), qa[m, b].astype(np.int64)))


def test_flash_attention_matches_reference():
    g = _load("flash_attn.npz")
    B, S, H, D = (int(g[k]) for k in "BSHD")
    out = Q.flash_decode_mha(g["q"], g["k_q8_0"], g["v_q8_0"], S, H, D)
    np.testing.assert_allclose(out, g["ref_on_q8_0"], rtol=1e-5, atol=1e-6)
    assert Q.nmse(out, g["ref_on_fp32"]) < 0.05


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0", "f16"])
def test_flash_attention_kv_formats_match_reference(fmt):
    """Cache bytes from the harness's own input builder (format chosen from the
    spec, fp32 caches quantised by the reference): the oracle's quantiser
    reproduces them bit for bit and its attention on them matches the
    harness's attention on the dequantised cache."""
    g = _load("flash_attn_kv.npz")
    B, S, H, D = (int(g[k]) for k in "BSHD")
    k, v = g[f"{fmt}_k"], g[f"{fmt}_v"]
    if fmt == "f16":
        assert np.array_equal(g[f"{fmt}_k_fp32"].astype(np.float16), k)
    else:
        quant = Q.quantize_q8_0 if fmt == "q8_0" else Q.quantize_q4_0
        assert np.array_equal(quant(g[f"{fmt}_k_fp32"].reshape(-1, D)).reshape(-1), k.reshape(-1))
        assert np.array_equal(quant(g[f"{fmt}_v_fp32"].reshape(-1, D)).reshape(-1), v.reshape(-1))
    out = Q.flash_decode_mha(g[f"{fmt}_q"], k, v, S, H, D, fmt)
    np.testing.assert_allclose(out, g[f"{fmt}_ref_on_cache"], rtol=1e-5, atol=1e-6)
    assert Q.nmse(out, g[f"{fmt}_ref_on_fp32"]) < 0.05


def test_ragged_decode_reduces_to_mha():
    g = _load("flash_attn.npz")
    B, S, H, D = (int(g[k]) for k in "BSHD")
    # one sequence per query row, each the whole cache, Hq == Hkv
    ref = Q.flash_decode_mha(g["q"], g["k_q8_0"], g["v_q8_0"], S, H, D)
    k = np.concatenate([g["k_q8_0"]] * B)
    v = np.concatenate([g["v_q8_0"]] * B)
    cu = np.arange(B + 1, dtype=np.int32) * S
    out = Q.flash_decode_ragged(g["q"], k, v, cu, H, H, D, 1.0 / np.sqrt(D))
    np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-6)


def test_moe_route():
    l = np.array([[0.1, 2.0, -1.0, 2.0], [3.0, 0.0, 1.0, -2.0]])
    idx, w = Q.moe_route(l, 2)
    assert idx.tolist() == [[1, 3], [0, 2]]   # tie -> lower expert first
    np.testing.assert_allclose(w.sum(1), 1.0)
    np.testing.assert_allclose(w[1, 0], 1 / (1 + np.exp(-2.0)))


@pytest.mark.parametrize("hs", [128, 4096])
def test_rms_norm_matches_reference(hs):
    """The oracle against the harness's RMSNormHandler on its own inputs."""
    g = _load("rms_norm.npz")
    out = Q.rms_norm(g[f"x{hs}"], g[f"w{hs}"], 1e-6)
    ref = g[f"out{hs}"]
    np.testing.assert_allclose(out, ref, rtol=2e-6, atol=1e-6 * float(np.sqrt(np.mean(ref ** 2))))


def test_kv_dequant_round_trip_bounds():
    """q4_0 / q8_0 caches dequantise to within half a step of the fp32 rows
    (q4_0 step d = amax/7, q8_0 step d = amax/127) plus the fp16 rounding of
    the stored scale (|code| * 2^-11 * d); fp16 to fp16 rounding."""
    rng = np.random.default_rng(21)
    D = 128
    x = (rng.standard_normal((64, D)) * rng.uniform(0.01, 10.0, (64, 1))).astype(np.float32)
    for fmt, steps, qmax, quant in (("q4_0", 7.0, 8.0, Q.quantize_q4_0), ("q8_0", 127.0, 127.0, Q.quantize_q8_0)):
        back = Q.dequant_kv_rows(fmt, quant(x), 64, D)
        amax = np.abs(x.reshape(64, D // 32, 32)).max(-1, keepdims=True)
        step = np.broadcast_to(amax / steps, (64, D // 32, 32)).reshape(64, D)
        err = np.abs(back.astype(np.float64) - x)
        assert np.all(err <= step * (0.5 + qmax * 2.0 ** -11) * (1 + 1e-6) + 1e-6), (fmt, float((err / step).max()))
    h = x.astype(np.float16)
    np.testing.assert_array_equal(Q.dequant_kv_rows("f16", h, 64, D), h.astype(np.float32))


def test_rms_norm_properties():
    """Unit weights give rows of unit root mean square (eps aside); the result
    is invariant to scaling a row by c > 0 (eps aside) and linear in the weight."""
    rng = np.random.default_rng(22)
    x = rng.standard_normal((5, 256)).astype(np.float32) * 3.0
    ones = np.ones(256, dtype=np.float32)
    y = Q.rms_norm(x, ones, 0.0)
    np.testing.assert_allclose(np.sqrt(np.mean(y.astype(np.float64) ** 2, axis=-1)), 1.0, rtol=1e-5)
    np.testing.assert_allclose(Q.rms_norm(np.float32(7.5) * x, ones, 0.0), y, rtol=1e-5, atol=1e-6)
    w = rng.standard_normal(256).astype(np.float32)
    np.testing.assert_allclose(Q.rms_norm(x, w, 1e-6), Q.rms_norm(x, ones, 1e-6) * w, rtol=1e-6, atol=1e-6)
