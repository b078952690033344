"""Run one operator of the path on seeded synthetic device inputs, a few
times, for profilers (ncu) and quick timing:

    python bench_cases.py gemm --wtype q8_0 --M 512 --N 11008 --K 4096 --reps 3
    python bench_cases.py gemv --wtype q4_0 --N 14336 --K 4096
    python bench_cases.py decode --B 32 --Lmax 8192
    python bench_cases.py mha --B 512 --S 8192 --fmt q4_0
    python bench_cases.py moe --T 1024

Inputs are generated on the GPU (weights drawn as q-blocks with the
benchmark configurations' distributions), then the operator runs --warmup
untimed and --reps timed calls; the mean CUDA-event time per call is
printed. The activation quantisation kernel runs inside each GEMM call, as
in the operator itself; ``--staged`` times the GEMM on pre-staged
activations alone (kq_mul_mat_q8x).
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "k-search_b200"))
import kq  # noqa: E402
from kq import synth  # noqa: E402


def _time(fn, warmup: int, reps: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / max(1, reps)


def _stage(x: torch.Tensor, M: int, K: int):
    a8 = kq.quantize_q8_1(x, "sum_dq")
    nb = K // 32
    ds = torch.stack([a8[:, :, 0:2].contiguous().view(torch.float16).float().squeeze(-1),
                      a8[:, :, 2:4].contiguous().view(torch.float16).float().squeeze(-1)], dim=-1).contiguous()
    qs = a8[:, :, 4:].contiguous().view(torch.int8).reshape(M, K).contiguous()
    assert ds.shape == (M, nb, 2)
    return qs, ds


def run_gemm(a) -> str:
    dev = torch.device("cuda")
    rng = np.random.default_rng(a.seed)
    w = torch.from_numpy(synth.blocks(a.wtype, rng, a.N, a.K)).to(dev)
    x = torch.randn((a.M, a.K), generator=torch.Generator().manual_seed(a.seed)).to(dev)
    out = torch.empty((a.M, a.N), dtype=torch.float32, device=dev)
    if a.staged:
        qs, ds = _stage(x, a.M, a.K)
        fn = lambda: kq.mul_mat_q8x(w, qs, ds, a.M, a.N, a.K, a.wtype, out=out)
    else:
        fn = lambda: kq.gemm_f32act(w, x, a.M, a.N, a.K, a.wtype, a.act, out=out)
    ms = _time(fn, a.warmup, a.reps)
    tops = 2.0 * a.M * a.N * a.K / (ms * 1e-3) / 1e12
    return f"gemm {a.wtype} M={a.M} N={a.N} K={a.K} staged={a.staged}: {ms * 1e3:.2f} us/call, {tops:.1f} TOPS"


def run_decode(a) -> str:
    dev = torch.device("cuda")
    rng = np.random.default_rng(a.seed)
    lens = rng.integers(a.Lmin, a.Lmax + 1, size=a.B).astype(np.int32)
    cu = torch.from_numpy(np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)).to(dev)
    T = int(lens.sum())
    gd = torch.Generator(device=dev).manual_seed(a.seed)
    k = kq.quantize_rows(torch.randn((T * a.Hkv, a.D), generator=gd, device=dev), "q8_0")
    v = kq.quantize_rows(torch.randn((T * a.Hkv, a.D), generator=gd, device=dev), "q8_0")
    q = torch.randn((a.B, a.Hq, a.D), generator=gd, device=dev).half()
    out = torch.empty_like(q)
    fn = lambda: kq.flash_decode_ragged(q, k, v, cu, a.Hkv, int(lens.max()), out=out)
    ms = _time(fn, a.warmup, a.reps)
    kv = 2 * T * a.Hkv * (a.D // 32) * 34
    return f"decode B={a.B} sum_L={T}: {ms * 1e3:.2f} us/call, {kv / (ms * 1e-3) / 1e9:.0f} GB/s of KV"


def run_mha(a) -> str:
    """The harness flash_attention form: fp32 queries [B, H, 128] over one
    shared [S, H, 128] cache (--fmt q8_0, q4_0 or f16)."""
    dev = torch.device("cuda")
    gd = torch.Generator(device=dev).manual_seed(a.seed)
    D = 128
    kf = torch.randn((a.S * a.H, D), generator=gd, device=dev)
    vf = torch.randn((a.S * a.H, D), generator=gd, device=dev)
    if a.fmt == "f16":
        k, v = kf.half(), vf.half()
    else:
        k, v = kq.quantize_rows(kf, a.fmt), kq.quantize_rows(vf, a.fmt)
    q = torch.randn((a.B, a.H, D), generator=gd, device=dev)
    fn = lambda: kq.flash_attn(q, k, v, a.B, a.S, a.H, D, a.fmt)
    ms = _time(fn, a.warmup, a.reps)
    flop = 4.0 * a.B * a.H * a.S * D
    kv = 2 * k.numel() * k.element_size()
    return (f"mha {a.fmt} B={a.B} S={a.S} H={a.H}: {ms * 1e3:.2f} us/call, {flop / (ms * 1e-3) / 1e12:.1f} TFLOP/s, "
            f"{kv / (ms * 1e-3) / 1e9:.0f} GB/s of KV")


def run_moe(a) -> str:
    dev = torch.device("cuda")
    rng = np.random.default_rng(a.seed)
    E, H, I = a.E, a.H, a.I
    wg = torch.from_numpy(np.stack([synth.q4_0_blocks(rng, I, H) for _ in range(E)])).to(dev)
    wu = torch.from_numpy(np.stack([synth.q4_0_blocks(rng, I, H) for _ in range(E)])).to(dev)
    wd = torch.from_numpy(np.stack([synth.q4_0_blocks(rng, H, I) for _ in range(E)])).to(dev)
    g = torch.Generator().manual_seed(a.seed)
    x = torch.randn((a.T, H), generator=g).to(dev)
    logits = torch.randn((a.T, E), generator=g).to(dev)
    out = torch.empty((a.T, H), dtype=torch.float32, device=dev)
    fn = lambda: kq.moe_q4_0(x, logits, wg, wu, wd, a.topk, "sum_dq", out=out)
    ms = _time(fn, a.warmup, a.reps)
    ops = 2.0 * a.T * a.topk * 3 * H * I
    return f"moe T={a.T} E={E} top{a.topk} H={H} I={I}: {ms:.3f} ms/call, {ops / (ms * 1e-3) / 1e12:.1f} TOPS"


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="op", required=True)
    for name in ("gemm", "gemv"):
        p = sub.add_parser(name)
        p.add_argument("--wtype", default="q8_0" if name == "gemm" else "q4_0")
        p.add_argument("--M", type=int, default=512 if name == "gemm" else 1)
        p.add_argument("--N", type=int, default=11008 if name == "gemm" else 4096)
        p.add_argument("--K", type=int, default=4096)
        p.add_argument("--act", default="sum_dq")
        p.add_argument("--staged", action="store_true")
    p = sub.add_parser("decode")
    for k, v in dict(B=32, Hq=32, Hkv=8, D=128, Lmin=64, Lmax=8192).items():
        p.add_argument(f"--{k}", type=int, default=v)
    p = sub.add_parser("mha")
    for k, v in dict(B=512, S=8192, H=32).items():
        p.add_argument(f"--{k}", type=int, default=v)
    p.add_argument("--fmt", default="q8_0", choices=["q8_0", "q4_0", "f16"])
    p = sub.add_parser("moe")
    for k, v in dict(T=4096, E=8, topk=2, H=4096, I=14336).items():
        p.add_argument(f"--{k}", type=int, default=v)
    for p in sub.choices.values():
        p.add_argument("--reps", type=int, default=3)
        p.add_argument("--warmup", type=int, default=2)
        p.add_argument("--seed", type=int, default=0)
    a = ap.parse_args(argv)
    kq.lib()
    fn = {"gemm": run_gemm, "gemv": run_gemm, "decode": run_decode, "mha": run_mha, "moe": run_moe}[a.op]
    print(fn(a), flush=True)


if __name__ == "__main__":
    main()
