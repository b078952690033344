"""GPU parity of the quantised GEMV/GEMM path against the oracle.

Bars: int32 block sums and q8_1 bytes bit-exact; fp32 outputs rel-L2 <= 1e-3
and per element |out - ref| <= 1e-2 |ref| + 1e-3 rms(ref) (oracle.quant.check_close),
plus the harness's own NMSE <= 0.05 gate against the fp32 dequant matmul.
"""
import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu
MODES = {"sum_x": Q.SUM_X, "sum_dq": Q.SUM_DQ, "f32": Q.ACT_F32}


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _x(rng, M, K):
    return rng.standard_normal((M, K)).astype(np.float32)


def test_quantize_q8_1_bit_exact(cuda):
    import kq
    rng = np.random.default_rng(10)
    x = _x(rng, 33, 4096)
    x[1] = 0.0
    x[2, :64] = -0.0
    x[3] *= np.float32(1e-6)
    x[4] *= np.float32(1e4)
    x[5, :32] = np.float32(0.5) * (np.arange(32) % 5 - 2)   # exact .5 ties
    x[6, :32] = np.float32(1.0) * (np.arange(32) - 16)
    for mode in ("sum_x", "sum_dq"):
        got = kq.quantize_q8_1(_t(x, cuda), mode).cpu().numpy()
        ref = Q.quantize_q8_1(x, MODES[mode])
        assert np.array_equal(got, ref), (mode, np.argwhere(got != ref)[:5])


def test_quantize_q8_1_golden(cuda):
    import kq
    g = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "quantize.npz"))
    got = kq.quantize_q8_1(_t(g["x"], cuda)).cpu().numpy().reshape(-1)
    assert np.array_equal(got, g["q8_1"])


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
@pytest.mark.parametrize("M,N,K", [(1, 96, 256), (3, 200, 512), (8, 64, 4096), (5, 130, 96), (40, 72, 320)])
def test_block_sums_bit_exact(cuda, wtype, M, N, K):
    import kq
    rng = np.random.default_rng(M * 1000 + N + K)
    w = Q.make_blocks(wtype, rng, N, K)
    a = Q.quantize_q8_1(_x(rng, M, K))
    got = kq.block_sums_i32(_t(w, cuda), _t(a, cuda), M, N, K, wtype).cpu().numpy()
    assert np.array_equal(got, Q.block_sums_i32(wtype, w, a, M, N, K))


SHAPES = [
    (1, 4096, 4096),    # configuration 0 (GEMV)
    (1, 257, 512),      # ragged row split
    (2, 1000, 1024),
    (3, 333, 768),
    (4, 512, 4352),     # K slices with a partial tail (nb = 136)
    (5, 96, 256),
    (8, 1024, 2048),
    (8, 77, 14336),     # long rows
    (1, 64, 96),        # K % 256 != 0 -> generic path
    (16, 256, 512),     # tensor-core path from here on (M > 8, K % 256 == 0)
    (64, 320, 1024),
    (9, 128, 256),
    (33, 130, 2048),    # partial weight tile
    (129, 200, 512),    # partial token tile
    (256, 384, 4096),
    (24, 64, 256),      # one raw stage: a single 8-block extra group
    (40, 256, 2304),    # 36 K-chunks: second extra group partial
    (130, 136, 14336),  # 7 extra groups (down-projection K)
]


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
@pytest.mark.parametrize("M,N,K", SHAPES)
def test_gemm_f32act_parity(cuda, wtype, M, N, K):
    import kq
    rng = np.random.default_rng(7 * M + N + 3 * K)
    w = Q.make_blocks(wtype, rng, N, K)
    x = _x(rng, M, K)
    wd, xd = _t(w, cuda), _t(x, cuda)
    for mode in ("f32", "sum_x", "sum_dq"):
        got = kq.gemm_f32act(wd, xd, M, N, K, wtype, mode).cpu().numpy()
        ref = Q.gemm_f32act(wtype, w, x, M, N, K, MODES[mode])
        ok, msg = Q.check_close(got, ref)
        assert ok, f"{mode}: {msg}"


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
def test_gemm_row_magnitudes(cuda, wtype):
    """Rows spanning 1e-7 .. 1e5 in magnitude and zero rows. The q8_1 modes
    store s in fp16, so their rows stop where a block sum would overflow it
    (|sum x| > 65504 is inf in the reference's format too)."""
    import kq
    M, N, K = 48, 256, 1024
    rng = np.random.default_rng(99)
    w = Q.make_blocks(wtype, rng, N, K)
    wd = _t(w, cuda)
    for mode, top in (("f32", 5), ("sum_x", 3), ("sum_dq", 3)):
        x = _x(rng, M, K)
        scales = np.float32(10.0) ** np.linspace(-7, top, M).astype(np.float32)
        x *= scales[:, None]
        x[5] = 0.0
        x[17, :300] *= np.float32(1e-3)   # mixed magnitudes inside one row
        got = kq.gemm_f32act(wd, _t(x, cuda), M, N, K, wtype, mode).cpu().numpy()
        ref = Q.gemm_f32act(wtype, w, x, M, N, K, MODES[mode])
        for m in range(M):   # per row: rows differ by up to 12 orders of magnitude
            ok, msg = Q.check_close(got[m:m + 1], ref[m:m + 1])
            assert ok, f"{mode} row {m}: {msg}"


def test_skinny_path_opt_in(cuda):
    """KQ_GEMM_PATH=skinny (the warp-MMA kernel for 8 < M <= 128; the
    split-fp16 tcgen05 kernel takes those shapes by default), in a child
    process: the full parity bar on every row."""
    import os
    import subprocess
    import sys
    code = (
        "import sys, numpy as np, torch; sys.path[:0] = %r\n"
        "import kq; from oracle import quant as Q\n"
        "for wt in ('q4_0', 'q4_1', 'q8_0'):\n"
        "  for (M, N, K) in ((16, 256, 512), (129, 200, 512), (100, 384, 4096), (40, 256, 2304)):\n"
        "    rng = np.random.default_rng(M + N + K)\n"
        "    w = Q.make_blocks(wt, rng, N, K); x = rng.standard_normal((M, K)).astype(np.float32)\n"
        "    x[3] *= np.float32(1e-6); x[5] *= np.float32(1e3)\n"
        "    for mode in ('f32', 'sum_x', 'sum_dq'):\n"
        "      got = kq.gemm_f32act(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda(), M, N, K, wt, mode)\n"
        "      ref = Q.gemm_f32act(wt, w, x, M, N, K, {'f32': Q.ACT_F32, 'sum_x': Q.SUM_X, 'sum_dq': Q.SUM_DQ}[mode])\n"
        "      g = got.cpu().numpy().astype(np.float64)\n"
        "      for m in range(M):\n"
        "        ok, msg = Q.check_close(g[m:m + 1], ref[m:m + 1])\n"
        "        assert ok, (wt, M, N, K, mode, m, msg)\n"
        "print('ok')\n" % ([p for p in sys.path if p],))
    env = dict(os.environ, KQ_GEMM_PATH="skinny")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


def test_int8_path_opt_in(cuda):
    """KQ_GEMM_PATH=int8 (int8 tcgen05 MMA per 32-block, int32 block sums
    rescaled on the FP32 pipe), in a child process: the full parity bar on
    every row, including rows of very small and very large magnitude."""
    import os
    import subprocess
    import sys
    code = (
        "import sys, numpy as np, torch; sys.path[:0] = %r\n"
        "import kq; from oracle import quant as Q\n"
        "for wt in ('q4_0', 'q4_1', 'q8_0'):\n"
        "  for (M, N, K) in ((16, 256, 512), (129, 200, 512), (256, 384, 4096), (40, 256, 2304)):\n"
        "    rng = np.random.default_rng(M + N + K)\n"
        "    w = Q.make_blocks(wt, rng, N, K); x = rng.standard_normal((M, K)).astype(np.float32)\n"
        "    x[3] *= np.float32(1e-6); x[5] *= np.float32(1e3)\n"
        "    for mode in ('f32', 'sum_x', 'sum_dq'):\n"
        "      got = kq.gemm_f32act(torch.from_numpy(w).cuda(), torch.from_numpy(x).cuda(), M, N, K, wt, mode)\n"
        "      ref = Q.gemm_f32act(wt, w, x, M, N, K, {'f32': Q.ACT_F32, 'sum_x': Q.SUM_X, 'sum_dq': Q.SUM_DQ}[mode])\n"
        "      g = got.cpu().numpy().astype(np.float64)\n"
        "      for m in range(M):\n"
        "        ok, msg = Q.check_close(g[m:m + 1], ref[m:m + 1])\n"
        "        assert ok, (wt, M, N, K, mode, m, msg)\n"
        "print('ok')\n" % ([p for p in sys.path if p],))
    env = dict(os.environ, KQ_GEMM_PATH="int8")
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
@pytest.mark.parametrize("M,N,K", [(1, 4096, 4096), (4, 300, 1024), (8, 128, 256), (12, 64, 512)])
def test_mul_mat_q_parity(cuda, wtype, M, N, K):
    import kq
    rng = np.random.default_rng(M + N + K)
    w = Q.make_blocks(wtype, rng, N, K)
    a = Q.quantize_q8_1(_x(rng, M, K))
    got = kq.mul_mat_q(_t(w, cuda), _t(a, cuda), M, N, K, wtype).cpu().numpy()
    ok, msg = Q.check_close(got, Q.gemm_q8_1(wtype, w, a, M, N, K))
    assert ok, msg


def test_golden_reference_outputs(cuda):
    """The fixtures hold the reference's own gemm_ref.py outputs."""
    import kq
    import os
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "gemm.npz"))
    M, N, K = int(g["M"]), int(g["N"]), int(g["K"])
    for wtype, key in (("q4_0", "ref_q4_0_q8_1"), ("q4_1", "ref_q4_1_q8_1")):
        got = kq.mul_mat_q(_t(g["w_" + wtype], cuda), _t(g["a_q8_1"], cuda), M, N, K, wtype).cpu().numpy()
        ok, msg = Q.check_close(got, g[key])
        assert ok, msg
    for wtype in ("q4_0", "q4_1", "q8_0"):
        got = kq.gemm_f32act(_t(g["w_" + wtype], cuda), _t(g["act"], cuda), M, N, K, wtype).cpu().numpy()
        assert Q.nmse(got, g[f"ref_{wtype}_fp32"]) < 0.05
    v = np.load(os.path.join(os.path.dirname(__file__), "golden", "variants.npz"))
    M, N, K = int(v["M"]), int(v["N"]), int(v["K"])
    got = kq.gemm_f32act(_t(v["w_q4_0"], cuda), _t(v["act"], cuda), M, N, K, "q4_0", "f32").cpu().numpy()
    ok, msg = Q.check_close(got, v["ref_w4a32c8"])
    assert ok, msg
    got = kq.gemm_f32act(_t(v["w_q8_0"], cuda), _t(v["act"], cuda), M, N, K, "q8_0", "f32").cpu().numpy()
    ok, msg = Q.check_close(got, v["ref_w8a8c8"])
    assert ok, msg


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
@pytest.mark.parametrize("M", [1, 8, 512])
def test_harness_configs(cuda, wtype, M):
    """The harness's own test configurations (op_test_handler.py:449-458: M in
    {1, 8, 512}) on weights quantised from N(0,1) as the harness makes them,
    against the fp32 dequant-matmul gate (NMSE <= 0.05) and the oracle."""
    import kq
    N, K = 512, 4096
    rng = np.random.default_rng(M)
    wf = rng.standard_normal((N, K)).astype(np.float32)
    w = Q.quantize_weights(wtype, wf)
    x = _x(rng, M, K)
    got = kq.gemm_f32act(_t(w, cuda), _t(x, cuda), M, N, K, wtype).cpu().numpy()
    assert not np.isnan(got).any() and not np.isinf(got).any()
    assert Q.nmse(got, Q.gemm_dequant_f32(wtype, w, x, M, N, K)) < 0.05
    ok, msg = Q.check_close(got, Q.gemm_f32act(wtype, w, x, M, N, K, Q.ACT_F32))
    assert ok, msg


def test_void_harness_entry_points(cuda):
    """The signature-for-signature KernelEvalPlus entries (legacy stream)."""
    import kq
    L = kq.lib()
    rng = np.random.default_rng(11)
    M, N, K = 3, 256, 1024
    x = _x(rng, M, K)
    for wtype, fn in (("q4_0", L.kq_w4a32c8_q4_0_fp32_int8), ("q4_1", L.kq_w4a32c8_q4_1_fp32_int8),
                      ("q8_0", L.kq_w8a32c8_q8_0_fp32_int8)):
        w = Q.make_blocks(wtype, rng, N, K)
        wd, xd = _t(w, cuda), _t(x, cuda)
        out = torch.empty((M, N), dtype=torch.float32, device=cuda)
        torch.cuda.synchronize()
        fn(wd.data_ptr(), xd.data_ptr(), out.data_ptr(), M, N, K)
        torch.cuda.synchronize()
        ok, msg = Q.check_close(out.cpu().numpy(), Q.gemm_f32act(wtype, w, x, M, N, K, Q.ACT_F32))
        assert ok, f"{wtype}: {msg}"
    w = Q.make_q4_0_blocks(rng, N, K)
    a = Q.quantize_q8_1(x)
    out = torch.empty((M, N), dtype=torch.float32, device=cuda)
    wd, ad = _t(w, cuda), _t(a, cuda)   # keep the device buffers alive across the raw call
    torch.cuda.synchronize()
    L.kq_w4a8_q4_0_q8_1(wd.data_ptr(), ad.data_ptr(), out.data_ptr(), M, N, K)
    torch.cuda.synchronize()
    ok, msg = Q.check_close(out.cpu().numpy(), Q.gemm_q8_1("q4_0", w, a, M, N, K))
    assert ok, msg


def test_errors_raise(cuda):
    import kq
    w = torch.zeros(18 * 4, dtype=torch.uint8, device=cuda)
    x = torch.zeros((1, 100), dtype=torch.float32, device=cuda)
    with pytest.raises((kq.KQError, ValueError)):
        kq.gemm_f32act(w, x, 1, 1, 100, "q4_0")
    with pytest.raises(ValueError):
        kq.gemm_f32act(w.cpu(), x, 1, 1, 128, "q4_0")
    assert kq.device_error() == 0


def test_stream_and_repeat_determinism(cuda):
    """Same inputs on a side stream give the identical bits (no atomics)."""
    import kq
    rng = np.random.default_rng(12)
    M, N, K = 4, 2048, 4096
    w, x = _t(Q.make_q4_0_blocks(rng, N, K), cuda), _t(_x(rng, M, K), cuda)
    a = kq.gemm_f32act(w, x, M, N, K)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        b = kq.gemm_f32act(w, x, M, N, K)
    s.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
def test_quantize_rows_bit_exact(cuda, wtype):
    import kq
    rng = np.random.default_rng(21)
    w = rng.standard_normal((37, 512)).astype(np.float32)
    w[1] = 0.0
    w[2, 32:64] = 3.0          # constant block (q4_1: max == min)
    w[3] *= np.float32(1e-5)
    got = kq.quantize_rows(_t(w, cuda), wtype).cpu().numpy()
    assert np.array_equal(got, Q.quantize_weights(wtype, w))
    g = np.load(__import__("os").path.join(__import__("os").path.dirname(__file__), "golden", "quantize.npz"))
    got = kq.quantize_rows(_t(g["w"], cuda), wtype).cpu().numpy().reshape(-1)
    assert np.array_equal(got, g[wtype])


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
def test_full_size_config_sampled_rows(cuda, wtype):
    """BASELINE configuration 1 shape (M=512, N=11008, K=4096): rows of the
    output are independent, so the oracle checks a sample of token rows that
    covers every 128-row tile boundary; the whole output is checked for
    finiteness and against the harness's NMSE gate on the same rows."""
    import kq
    M, N, K = 512, 11008, 4096
    rng = np.random.default_rng(2026)
    w = Q.make_blocks(wtype, rng, N, K)
    x = _x(rng, M, K)
    got = kq.gemm_f32act(_t(w, cuda), _t(x, cuda), M, N, K, wtype, "sum_dq").cpu().numpy()
    assert np.isfinite(got).all()
    rows = np.array([0, 1, 126, 127, 128, 255, 256, 383, 384, 510, 511])
    ref = Q.gemm_f32act(wtype, w, x[rows], len(rows), N, K, Q.SUM_DQ)
    ok, msg = Q.check_close(got[rows], ref)
    assert ok, msg
    assert Q.nmse(got[rows], Q.gemm_dequant_f32(wtype, w, x[rows], len(rows), N, K)) < 0.05


@pytest.mark.parametrize("M", [16, 128, 2048])
def test_full_size_config2_sampled_rows(cuda, M):
    """BASELINE configuration 2 at full size (q4_0, N=14336, K=4096) for
    M = 16 and 128 (the weight-streaming kernel) and 2048 (the split-fp16
    kernel, 16 token tiles): the whole product runs in one call and the
    oracle checks sampled token rows, including every 128-row tile edge for
    M = 2048 (output rows are independent)."""
    import kq
    N, K = 14336, 4096
    rng = np.random.default_rng(14336 + M)
    w = Q.make_q4_0_blocks(rng, N, K)
    x = _x(rng, M, K)
    got = kq.gemm_f32act(_t(w, cuda), _t(x, cuda), M, N, K, "q4_0", "sum_dq").cpu().numpy()
    assert np.isfinite(got).all()
    if M <= 128:
        rows = np.array(sorted({0, 1, 7, 8, 9, M // 2, M - 2, M - 1}))
    else:
        rows = np.array(sorted({0, 1} | {t * 128 + o for t in range(M // 128) for o in (0, 127)} | {M - 1}))
    ref = Q.gemm_f32act("q4_0", w, x[rows], len(rows), N, K, Q.SUM_DQ)
    ok, msg = Q.check_close(got[rows], ref)
    assert ok, msg
    # int32 block sums of one sampled row, bit-exact against the oracle's
    a = Q.quantize_q8_1(x[rows[:1]])
    sumi = kq.block_sums_i32(_t(w, cuda), _t(a, cuda), 1, N, K, "q4_0").cpu().numpy()
    assert np.array_equal(sumi, Q.block_sums_i32("q4_0", w, a, 1, N, K))


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
def test_gemm_several_tiles_per_cta(cuda, wtype):
    """More output tiles than SMs (each persistent CTA runs two or three, so
    both TMEM accumulator pairs and every ring wrap around), a partial last
    tile in N and a partial last group of extra columns in K; every row is
    checked, three calls in a row."""
    import kq
    M, N, K = 256, 10000, 2304   # 180 tiles of 128 x 112 on 148 SMs; K: 36 chunks, groups of 32 + 4
    rng = np.random.default_rng(77)
    w = Q.make_blocks(wtype, rng, N, K)
    x = _x(rng, M, K)
    ref = Q.gemm_f32act(wtype, w, x, M, N, K, Q.SUM_DQ)
    wd, xd = _t(w, cuda), _t(x, cuda)
    for rep in range(3):
        got = kq.gemm_f32act(wd, xd, M, N, K, wtype, "sum_dq").cpu().numpy()
        ok, msg = Q.check_close(got, ref)
        assert ok, f"call {rep}: {msg}"


def test_harness_mirror(cuda):
    """kq.harness.quant_gemm_forward has the harness module.forward signature."""
    import kq
    rng = np.random.default_rng(31)
    M, N, K = 8, 256, 1024
    w = Q.make_q4_1_blocks(rng, N, K)
    x = _x(rng, M, K)
    got = kq.harness.quant_gemm_forward(_t(w, cuda).reshape(-1), _t(x, cuda), M, N, K, "block_q4_1", "float32")
    ok, msg = Q.check_close(got.cpu().numpy(), Q.gemm_f32act("q4_1", w, x, M, N, K, Q.ACT_F32))
    assert ok, msg
    a = Q.quantize_q8_1(x)
    got = kq.harness.quant_gemm_forward(_t(Q.make_q4_0_blocks(rng, N, K), cuda), _t(a, cuda), M, N, K,
                                        "block_q4_0", "block_q8_1")
    assert got.shape == (M, N)
    perf = kq.harness.quant_gemm_performance(0.01, M, N, K)
    assert perf["tflops"] == round(2 * M * N * K / 1e-5 / 1e12, 3)


@pytest.mark.parametrize("wtype", ["q4_0", "q4_1", "q8_0"])
@pytest.mark.parametrize("N,K", [(1, 256), (7, 3584), (33, 4096), (4096, 4096), (300, 11008), (129, 14336),
                                 (1000, 2048), (5, 65536)])
def test_single_launch_gemv(cuda, wtype, N, K):
    """M = 1 runs one kernel that quantises the row itself (gemv1.cu). K
    sets the lanes per row (4-bit chunk counts 1, 14, 16, 43, 56, 8, 256,
    twice as many for q8_0's 4-block chunks: idle lanes, several chunks per
    lane, the 32-lane cap) and N the ragged
    last warp. Checked against the oracle in every activation mode, and
    against the two-launch path on the same q8_1 bytes (kq_quantize_q8_1 then
    kq_mul_mat_q, the staged GEMV): both read identical codes and scales, so
    they differ only in summation order."""
    import kq
    rng = np.random.default_rng(N + K)
    w = Q.make_blocks(wtype, rng, N, K)
    x = _x(rng, 1, K)
    x[0, :32] = 0.0                                         # zero block: d = 1
    x[0, 32:64] = np.float32(0.5) * (np.arange(32) % 5 - 2)  # exact .5 ties
    if K >= 512:
        x[0, 256:512] *= np.float32(1e-4)                    # mixed magnitudes
    wd, xd = _t(w, cuda), _t(x, cuda)
    for mode in ("f32", "sum_x", "sum_dq"):
        got = kq.gemm_f32act(wd, xd, 1, N, K, wtype, mode).cpu().numpy()
        ok, msg = Q.check_close(got, Q.gemm_f32act(wtype, w, x, 1, N, K, MODES[mode]))
        assert ok, f"{mode}: {msg}"
        if mode != "f32":
            staged = kq.mul_mat_q(wd, kq.quantize_q8_1(xd, mode), 1, N, K, wtype).cpu().numpy()
            scale = float(np.sqrt(np.mean(staged.astype(np.float64) ** 2))) + 1e-30
            assert np.max(np.abs(got - staged)) <= 1e-5 * scale, f"{mode}: differs from the staged GEMV"
    assert kq.device_error() == 0


def test_single_launch_gemv_unaligned_falls_back(cuda):
    """Weights off the 16-byte grid (2-byte aligned, as the block fields
    allow) take the two-launch path (quantiser + generic kernel), with the
    same result to the parity bar."""
    import kq
    rng = np.random.default_rng(5)
    N, K = 64, 1024
    w = Q.make_q4_0_blocks(rng, N, K).reshape(-1)
    x = _x(rng, 1, K)
    wbuf = torch.zeros(w.size + 16, dtype=torch.uint8, device=cuda)
    wbuf[2:2 + w.size] = _t(w, cuda)
    got = kq.gemm_f32act(wbuf[2:2 + w.size], _t(x, cuda), 1, N, K, "q4_0", "f32")
    ok, msg = Q.check_close(got.cpu().numpy(), Q.gemm_f32act("q4_0", w.reshape(N, -1), x, 1, N, K, Q.ACT_F32))
    assert ok, msg


def test_single_launch_gemv_after_producer(cuda):
    """The single-launch GEMV is a programmatic dependent of whatever kernel
    precedes it: it must not read the activation row or the weights before
    that kernel ends. Here each call directly follows a device kernel that
    rewrites its input (torch's copy of a new row, then the library's own
    weight quantiser), with fresh values every time."""
    import kq
    rng = np.random.default_rng(31)
    N, K = 2048, 4096
    xd = torch.empty((1, K), dtype=torch.float32, device=cuda)
    wf_d = torch.empty((N, K), dtype=torch.float32, device=cuda)
    for it in range(4):
        x = _x(rng, 1, K) * np.float32(1 + it)
        wf = rng.standard_normal((N, K)).astype(np.float32)
        wf_d.copy_(_t(wf, cuda))
        w = kq.quantize_rows(wf_d, "q4_0")           # producer of the weights
        xd.copy_(_t(x, cuda))                         # producer of the row, directly before the GEMV
        got = kq.gemm_f32act(w.reshape(-1), xd, 1, N, K, "q4_0", "sum_x").cpu().numpy()
        ref = Q.gemm_f32act("q4_0", Q.quantize_weights("q4_0", wf), x, 1, N, K, Q.SUM_X)
        ok, msg = Q.check_close(got, ref)
        assert ok, f"iteration {it}: {msg}"
