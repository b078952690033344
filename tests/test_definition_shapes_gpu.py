"""Parity at every quant_gemm definition shape the reference ships.

The reference's harness runs each definition JSON (weight type, N, K, and
M in {1, 2, 3, 4, 5, 8, 512}) through the W4A32C8 / W8A32C8 operator;
tests/golden/definition_shapes.json lists the distinct (weight type, N, K)
(written by tests/golden/make_definition_shapes.py from the reference's
definitions). For each shape this calls the fused fp32-activation GEMM at
M = 1 and 5 (the GEMV kernel) and M = 512 (the tensor-core kernel) with the
per-definition activation semantics (ACT_F32), and checks a sample of output
rows and up to 2048 evenly spaced output columns (edges included) against
the oracle with the usual bar. Weights are random bytes with their fp16
scale fields set to sane values (every code pattern occurs)."""
import json
import os

import numpy as np
import pytest
import torch

from oracle import quant as Q

pytestmark = pytest.mark.gpu

_SHAPES = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "definition_shapes.json")))["shapes"]


def _blocks(wtype: str, rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    bb = Q.BLOCK_BYTES[wtype]
    nb = K // 32
    w = rng.integers(0, 256, size=(N, nb, bb), dtype=np.uint8)
    d = (rng.uniform(0.002, 0.02, size=(N, nb)) * rng.choice([-1.0, 1.0], size=(N, nb))).astype(np.float16)
    w[:, :, 0:2] = d.view(np.uint8).reshape(N, nb, 2)
    if wtype == "q4_1":
        m = rng.uniform(-0.16, 0.0, size=(N, nb)).astype(np.float16)
        w[:, :, 2:4] = m.view(np.uint8).reshape(N, nb, 2)
    return w.reshape(N, nb * bb)


@pytest.mark.parametrize("shape", _SHAPES, ids=lambda s: f"{s['wtype']}-n{s['N']}-k{s['K']}")
def test_definition_shape(cuda, shape):
    import kq
    wt, N, K = shape["wtype"], shape["N"], shape["K"]
    rng = np.random.default_rng(7 * N + K + {"q4_0": 0, "q4_1": 1, "q8_0": 2}[wt])
    w = _blocks(wt, rng, N, K)
    wd = torch.from_numpy(w).to(cuda)
    cols = np.unique(np.linspace(0, N - 1, min(N, 2048)).astype(np.int64))
    wsub = np.ascontiguousarray(w[cols])
    cols_t = torch.from_numpy(cols).to(cuda)
    for M in (1, 5, 512):
        x = rng.standard_normal((M, K)).astype(np.float32)
        got = kq.gemm_f32act(wd, torch.from_numpy(x).to(cuda), M, N, K, wt, "f32")
        rows = np.unique(np.array([0, M // 2, M - 1]))
        g = got[torch.from_numpy(rows).to(cuda)][:, cols_t].cpu().numpy()
        ref = Q.gemm_f32act(wt, wsub, x[rows], len(rows), len(cols), K, Q.ACT_F32)
        ok, msg = Q.check_close(g, ref)
        assert ok, f"M={M}: {msg}"
