"""Seeded synthetic inputs of the benchmark configurations (host-side numpy).

Weights are drawn directly as GGML blocks:
  q4_0: d = fp16(|N(0, 0.02)| / 8), 16 nibble bytes uniform in 0..255
  q4_1: d as q4_0, m = fp16(-8 d), nibble bytes uniform
  q8_0: codes clamp(round(N(0,1) * 40), +-127), d = fp16(0.02 / 40)
"""
from __future__ import annotations

import numpy as np


def _f16_bytes(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a.astype(np.float16)).view(np.uint8).reshape(a.shape + (2,))


def q4_0_blocks(rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    nb = K // 32
    d = np.abs(rng.standard_normal((N, nb), dtype=np.float32) * np.float32(0.02)) / np.float32(8.0)
    out = np.empty((N, nb, 18), dtype=np.uint8)
    out[:, :, 0:2] = _f16_bytes(d)
    out[:, :, 2:] = rng.integers(0, 256, size=(N, nb, 16), dtype=np.uint8)
    return out


def q4_1_blocks(rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    nb = K // 32
    d = np.abs(rng.standard_normal((N, nb), dtype=np.float32) * np.float32(0.02)) / np.float32(8.0)
    out = np.empty((N, nb, 20), dtype=np.uint8)
    out[:, :, 0:2] = _f16_bytes(d)
    out[:, :, 2:4] = _f16_bytes((-8.0 * d).astype(np.float32))
    out[:, :, 4:] = rng.integers(0, 256, size=(N, nb, 16), dtype=np.uint8)
    return out


def q8_0_blocks(rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    nb = K // 32
    q = np.clip(np.round(rng.standard_normal((N, nb, 32), dtype=np.float32) * np.float32(40.0)), -127, 127)
    out = np.empty((N, nb, 34), dtype=np.uint8)
    out[:, :, 0:2] = _f16_bytes(np.full((N, nb), 0.02 / 40.0, dtype=np.float32))
    out[:, :, 2:] = q.astype(np.int8).view(np.uint8)
    return out


def blocks(wtype: str, rng: np.random.Generator, N: int, K: int) -> np.ndarray:
    return {"q4_0": q4_0_blocks, "q4_1": q4_1_blocks, "q8_0": q8_0_blocks}[wtype](rng, N, K)
