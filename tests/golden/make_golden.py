"""Generate the golden fixtures in this directory from the reference itself.

Runs ONLY where the qhy991/K-Search checkout is present (pass its path as
argv[1] or set KSEARCH_REF). It imports the reference's own Python functions
(kernelevalplus-main/llm_kernel_test/reference, the harness's
FlashAttentionHandler and the per-variant reference.py files) and records
their outputs on small seeded inputs as .npz files. The tests never import the
reference; they only read these files.

    python tests/golden/make_golden.py /path/to/K-Search
"""
from __future__ import annotations

import importlib.util
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _load_module(path: str, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main() -> None:
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KSEARCH_REF", "")
    kep = os.path.join(root, "kernelevalplus-main")
    if not os.path.isdir(kep):
        raise SystemExit(f"reference checkout not found under {root!r}")
    sys.path.insert(0, kep)
    import torch
    from llm_kernel_test.reference import (  # noqa: E402
        quantize_to_q8_0, quantize_to_q4_0, quantize_to_q4_1, quantize_to_q8_1,
        reference_q8_0_gemm, reference_q4_0_fp32_gemm, reference_q4_0_q8_1_gemm,
        reference_q4_1_fp32_gemm, reference_q4_1_q8_1_gemm,
    )
    from llm_kernel_test.op_test_handler import FlashAttentionHandler  # noqa: E402

    rng = np.random.default_rng(20261201)

    # --- quantizers ---------------------------------------------------------
    x = rng.standard_normal((6, 256)).astype(np.float32)
    x[1] = 0.0                                      # amax == 0 -> d = 1.0
    x[2] *= np.float32(1e-3)                        # small scale
    x[3, :32] = np.float32(0.5) * (np.arange(32) % 5 - 2)  # exact .5 ties after /d
    x[4] *= np.float32(300.0)                       # large values (fp16 s overflow stays finite)
    x[5, :32] = -0.0                                # negative zeros
    w = rng.standard_normal((8, 256)).astype(np.float32)
    w[1, 32:64] = 0.0
    np.savez_compressed(
        os.path.join(HERE, "quantize.npz"),
        x=x, w=w,
        q8_1=quantize_to_q8_1(x), q8_0=quantize_to_q8_0(w),
        q4_0=quantize_to_q4_0(w), q4_1=quantize_to_q4_1(w),
    )

    # --- GEMM formulas (llm_kernel_test/reference/gemm_ref.py) --------------
    M, N, K = 5, 24, 512
    act = rng.standard_normal((M, K)).astype(np.float32)
    wf = rng.standard_normal((N, K)).astype(np.float32)
    w40 = quantize_to_q4_0(wf)
    w41 = quantize_to_q4_1(wf)
    w80 = quantize_to_q8_0(wf)
    a81 = quantize_to_q8_1(act)
    T = torch.from_numpy
    np.savez_compressed(
        os.path.join(HERE, "gemm.npz"),
        M=M, N=N, K=K, act=act, w_q4_0=w40, w_q4_1=w41, w_q8_0=w80, a_q8_1=a81,
        ref_q4_0_q8_1=reference_q4_0_q8_1_gemm(T(w40), T(a81), M, N, K).numpy(),
        ref_q4_1_q8_1=reference_q4_1_q8_1_gemm(T(w41), T(a81), M, N, K).numpy(),
        ref_q4_0_fp32=reference_q4_0_fp32_gemm(T(w40), T(act), M, N, K).numpy(),
        ref_q4_1_fp32=reference_q4_1_fp32_gemm(T(w41), T(act), M, N, K).numpy(),
        ref_q8_0_fp32=reference_q8_0_gemm(T(w80), T(act), M, N, K).numpy(),
    )

    # --- per-variant per-element references (core/operators/quant_gemm) -----
    vdir = os.path.join(kep, "core", "operators", "quant_gemm", "variants")
    v2 = _load_module(os.path.join(vdir, "deepseek_v2", "w4a32c8_q4_0_fp32_int8", "reference.py"), "ref_v2")
    v3 = _load_module(os.path.join(vdir, "deepseek_v3", "w8a8c8_q8_0_q8_1", "reference.py"), "ref_v3")
    w48 = _load_module(os.path.join(vdir, "w4a8_q4_0_fp32_int8", "reference.py"), "ref_w4a8")
    Ms, Ns, Ks = 2, 6, 128
    act_s = rng.standard_normal((Ms, Ks)).astype(np.float32)
    wf_s = rng.standard_normal((Ns, Ks)).astype(np.float32)
    w40_s = quantize_to_q4_0(wf_s).reshape(Ns, Ks // 32, 18)
    w80_s = quantize_to_q8_0(wf_s).reshape(Ns, Ks // 32, 34)
    a81_s = quantize_to_q8_1(act_s).reshape(Ms, Ks // 32, 36)
    np.savez_compressed(
        os.path.join(HERE, "variants.npz"),
        M=Ms, N=Ns, K=Ks, act=act_s, w_q4_0=w40_s, w_q8_0=w80_s, a_q8_1=a81_s,
        ref_w4a32c8=v2.run(T(act_s), T(w40_s)).numpy(),
        ref_w8a8c8=v3.run(T(act_s), T(w80_s)).numpy(),
        ref_w4a8=w48.run(T(w40_s), T(a81_s)).numpy(),
    )

    # --- flash-attention decode (llm_kernel_test/op_test_handler.py) -------
    B, S, H, D = 3, 40, 4, 64
    q = rng.standard_normal((B, H, D)).astype(np.float32)
    kf = rng.standard_normal((S, H, D)).astype(np.float32)
    vf = rng.standard_normal((S, H, D)).astype(np.float32)
    kq = quantize_to_q8_0(kf.reshape(-1, D))      # op_test_handler.py:500-505
    vq = quantize_to_q8_0(vf.reshape(-1, D))
    # The harness oracle attends over the fp32 caches it is given; giving it
    # the dequantised q8_0 rows pins the attention arithmetic on q8_0 data.
    def deq(b):
        blk = b.reshape(S * H, D // 32, 34)
        d = blk[:, :, 0:2].copy().view(np.float16).astype(np.float32)
        qs = blk[:, :, 2:].copy().view(np.int8).astype(np.float32)
        return (qs * d).reshape(S, H, D)
    spec = {"axes": {"seq_len": {"value": S}, "num_heads": {"value": H}, "head_dim": {"value": D}}}
    h = FlashAttentionHandler()
    inputs_deq = {"query": T(q), "key_cache_fp32": T(deq(kq)), "value_cache_fp32": T(deq(vq))}
    inputs_raw = {"query": T(q), "key_cache_fp32": T(kf), "value_cache_fp32": T(vf)}
    np.savez_compressed(
        os.path.join(HERE, "flash_attn.npz"),
        B=B, S=S, H=H, D=D, q=q, k_fp32=kf, v_fp32=vf, k_q8_0=kq, v_q8_0=vq,
        ref_on_q8_0=h.get_reference_output(spec, inputs_deq).numpy(),
        ref_on_fp32=h.get_reference_output(spec, inputs_raw).numpy(),
    )

    # --- flash-attention decode, every KV format: the harness's own input
    # builder (op_test_handler.py:472-541) picks the format from the spec
    # fields and quantises the fp32 caches; the attention is then its oracle
    # (:543-563) on the dequantised cache (q4_0 dequantised by the reference's
    # q4_0 GEMM against an identity, gemm_ref.py:51-99, exact in fp32; fp16
    # through the handler's key_cache path) and on the fp32 caches.
    B, S, H, D = 2, 48, 3, 64
    specs = {
        "q8_0": ("int8", "FP32_Q8_0", ["kv_cache:q8_0"]),
        "q4_0": ("int8", "FP32_Q4_0", ["kv_cache:q4_0"]),
        "f16": ("float16", "FP32", ["kv_cache:f16"]),
    }
    fa = {"B": B, "S": S, "H": H, "D": D}
    for i, (fmt, (dtype, variant, tags)) in enumerate(specs.items()):
        spec = {"axes": {"seq_len": {"value": S}, "num_heads": {"value": H}, "head_dim": {"value": D}},
                "inputs": {"key_cache": {"dtype": dtype}}, "variant": variant, "tags": tags}
        torch.manual_seed(1000 + i)
        inp = h.generate_inputs(spec, {"batch_size": B}, "cpu")
        kc, vc = inp["key_cache"].numpy(), inp["value_cache"].numpy()
        if fmt == "q8_0":
            kd, vd = deq(kc.reshape(-1)), deq(vc.reshape(-1))
        elif fmt == "q4_0":
            eye = torch.eye(D, dtype=torch.float32)
            kd = reference_q4_0_fp32_gemm(T(kc), eye, D, S * H, D).numpy().T.reshape(S, H, D)
            vd = reference_q4_0_fp32_gemm(T(vc), eye, D, S * H, D).numpy().T.reshape(S, H, D)
        else:
            kd, vd = kc.astype(np.float32), vc.astype(np.float32)
        on_cache = {"query": inp["query"], "key_cache_fp32": T(np.ascontiguousarray(kd)),
                    "value_cache_fp32": T(np.ascontiguousarray(vd))}
        fa.update({f"{fmt}_spec_dtype": dtype, f"{fmt}_spec_variant": variant,
                   f"{fmt}_q": inp["query"].numpy(),
                   f"{fmt}_k_fp32": inp["key_cache_fp32"].numpy(), f"{fmt}_v_fp32": inp["value_cache_fp32"].numpy(),
                   f"{fmt}_k": kc, f"{fmt}_v": vc,
                   f"{fmt}_ref_on_cache": h.get_reference_output(spec, on_cache).numpy(),
                   f"{fmt}_ref_on_fp32": h.get_reference_output(spec, inp).numpy()})
    np.savez_compressed(os.path.join(HERE, "flash_attn_kv.npz"), **fa)

    # --- rms_norm (op_test_handler.py:641-690): the handler's own inputs and
    # reference output at two hidden sizes of the shipped definitions.
    from llm_kernel_test.op_test_handler import RMSNormHandler  # noqa: E402
    rh = RMSNormHandler()
    rn = {}
    for i, (hs, bs) in enumerate([(128, 3), (4096, 2)]):
        spec = {"axes": {"hidden_size": {"value": hs}, "epsilon": {"value": 1e-6}}}
        torch.manual_seed(2000 + i)
        inp = rh.generate_inputs(spec, {"batch_size": bs}, "cpu")
        rn.update({f"x{hs}": inp["hidden_states"].numpy(), f"w{hs}": inp["weight"].numpy(),
                   f"out{hs}": rh.get_reference_output(spec, inp).numpy()})
    np.savez_compressed(os.path.join(HERE, "rms_norm.npz"), **rn)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
