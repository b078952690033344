"""GPU parity of RMSNorm (the harness rms_norm operator) and of its fusion
into the on-the-fly q8_1 quantisation of the GEMM.

rms_norm: every shipped definition (hidden size, each batch size) against the
oracle; the bar is fp32 rounding (per element <= 2e-6 |ref| + 1e-6 rms(ref):
the row's mean of squares is summed in a different order).
RMSNorm -> q8_1: scales within 1e-5 relative of the oracle's quantisation of
the oracle's normalised rows, codes equal except a step of 1 where a
normalised value sits within rounding of a code boundary (<= 0.1% of codes).
Fused GEMM: the usual GEMM bar against the oracle GEMM on the library's
normalised rows, rel-L2 against the oracle's own normalisation.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu

_DEFS = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "rms_norm_definitions.json")))["definitions"]


def _t(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def _check_norm(got, ref):
    tol = 2e-6 * np.abs(ref) + 1e-6 * float(np.sqrt(np.mean(ref.astype(np.float64) ** 2)))
    bad = np.abs(got.astype(np.float64) - ref) > tol
    assert not bad.any(), f"{int(bad.sum())} elements outside the bar, max err {np.abs(got - ref).max():.3e}"


def test_golden_fixture(cuda):
    import kq
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "rms_norm.npz"))
    for hs in (128, 4096):
        got = kq.rms_norm(_t(g[f"x{hs}"], cuda), _t(g[f"w{hs}"], cuda), 1e-6).cpu().numpy()
        _check_norm(got, g[f"out{hs}"])


@pytest.mark.parametrize("defn", _DEFS, ids=lambda d: os.path.basename(d["definition"])[:-5])
def test_definition_rms_norm(cuda, defn):
    import kq
    K, eps = defn["hidden_size"], defn["epsilon"]
    rng = np.random.default_rng(K)
    w = rng.standard_normal(K).astype(np.float32)
    wd = _t(w, cuda)
    for B in defn["B"]:
        x = rng.standard_normal((B, K)).astype(np.float32)
        got = kq.harness.rms_norm_forward(_t(x, cuda), wd, eps).cpu().numpy()
        _check_norm(got, Q.rms_norm(x, w, eps))


@pytest.mark.parametrize("B,K", [(3, 100), (1, 7), (5, 4098)])
def test_rms_norm_scalar_path(cuda, B, K):
    """Hidden sizes that are not a multiple of 4 (element loads)."""
    import kq
    rng = np.random.default_rng(B + K)
    x = rng.standard_normal((B, K)).astype(np.float32)
    w = rng.standard_normal(K).astype(np.float32)
    _check_norm(kq.rms_norm(_t(x, cuda), _t(w, cuda)).cpu().numpy(), Q.rms_norm(x, w))


def test_harness_void_entry(cuda):
    import kq
    rng = np.random.default_rng(9)
    B, K = 8, 3584
    x = rng.standard_normal((B, K)).astype(np.float32)
    w = rng.standard_normal(K).astype(np.float32)
    xd, wd = _t(x, cuda), _t(w, cuda)
    out = torch.empty((B, K), dtype=torch.float32, device=cuda)
    torch.cuda.synchronize()
    kq.lib().kq_rms_norm(xd.data_ptr(), wd.data_ptr(), out.data_ptr(), B, K)
    torch.cuda.synchronize()
    assert kq.lib().kq_last_error() == b""
    _check_norm(out.cpu().numpy(), Q.rms_norm(x, w, 1e-6))


@pytest.mark.parametrize("sum_mode", ["sum_x", "sum_dq"])
@pytest.mark.parametrize("M,K", [(1, 4096), (8, 7168), (512, 2048), (3, 32)])
def test_rms_norm_quantize_q8_1(cuda, sum_mode, M, K):
    import kq
    rng = np.random.default_rng(M * K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    w = rng.standard_normal(K).astype(np.float32)
    got = kq.rms_norm_quantize_q8_1(_t(x, cuda), _t(w, cuda), 1e-6, sum_mode).cpu().numpy()
    ref = Q.quantize_q8_1(Q.rms_norm(x, w), Q.SUM_X if sum_mode == "sum_x" else Q.SUM_DQ)
    dg, sg, qg = Q.unpack_q8_1(got, M, K)
    dr, sr, qr = Q.unpack_q8_1(ref, M, K)
    np.testing.assert_allclose(dg, dr, rtol=1e-3)  # fp16 scales: at most one fp16 step apart
    diff = np.abs(qg.astype(np.int32) - qr.astype(np.int32))
    assert diff.max() <= 1 and (diff > 0).mean() <= 1e-3, f"{int((diff > 0).sum())} codes differ"
    np.testing.assert_allclose(sg, sr, rtol=2e-3, atol=2e-3 * float(np.abs(sr).max()))


@pytest.mark.parametrize("wtype", ["q4_0", "q8_0", "q4_1"])
@pytest.mark.parametrize("M", [1, 5, 512])
def test_gemm_f32act_rmsnorm(cuda, wtype, M):
    """The fused call against the oracle GEMM on the library's normalised rows
    (themselves pinned to the oracle's RMSNorm to fp32 rounding), with the
    usual bar; against the oracle's own normalisation the bar is rel-L2 only,
    since a normalised value an ulp away can move its q8_1 code by one."""
    import kq
    N, K = 1024, 4096
    rng = np.random.default_rng(M + N + len(wtype))
    x = rng.standard_normal((M, K)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, K).astype(np.float32)
    wq = Q.quantize_weights(wtype, (rng.standard_normal((N, K)) * 0.02).astype(np.float32))
    xd, gd = _t(x, cuda), _t(g, cuda)
    got = kq.gemm_f32act_rmsnorm(_t(wq, cuda), xd, gd, M, N, K, wtype, "f32").cpu().numpy()
    xn = kq.rms_norm(xd, gd).cpu().numpy()
    _check_norm(xn, Q.rms_norm(x, g))
    ok, msg = Q.check_close(got, Q.gemm_f32act(wtype, wq, xn, M, N, K, Q.ACT_F32))
    assert ok, msg
    ref = Q.gemm_f32act(wtype, wq, Q.rms_norm(x, g), M, N, K, Q.ACT_F32)
    rel = float(np.linalg.norm(got.astype(np.float64) - ref) / np.linalg.norm(ref.astype(np.float64)))
    assert rel <= 1e-3, rel
