"""Mirror of the KernelEvalPlus operator interface for this path.

``quant_gemm_forward``, ``flash_attention_forward`` and ``rms_norm_forward``
have the signatures of the ``module.forward`` the harness calls
(kernelevalplus-main/llm_kernel_test/op_test_handler.py:251-256, :565-579 and
:677-679);
``quant_gemm_test_configs`` / ``*_performance`` restate the harness's test
configurations and FLOP accounting (op_test_handler.py:258-266, :449-458,
:581-596) so runs here report the same numbers the harness would.
"""
from __future__ import annotations

import torch

from . import ops

# definition dtype -> weight type; activation dtype "float32" = on-the-fly q8_1
_WEIGHT = {"block_q4_0": "q4_0", "q4_0": "q4_0", "block_q4_1": "q4_1", "q4_1": "q4_1",
           "block_q8_0": "q8_0", "q8_0": "q8_0"}


def quant_gemm_forward(weight: torch.Tensor, activation: torch.Tensor, M: int, N: int, K: int,
                       weight_dtype: str = "block_q4_0", activation_dtype: str = "float32") -> torch.Tensor:
    """forward(weight, activation, M, N, K) -> fp32 [M, N] (op_test_handler.py:251-256).
    fp32 activations use the per-definition W4A32C8 semantics (fp32 block
    scale and sum); ``block_q8_1`` activations are pre-quantised bytes."""
    wt = _WEIGHT[weight_dtype]
    if activation_dtype in ("float32", "fp32"):
        return ops.gemm_f32act(weight, activation, M, N, K, wt, "f32")
    if activation_dtype in ("q8_1", "block_q8_1"):
        return ops.mul_mat_q(weight, activation, M, N, K, wt)
    raise ValueError(f"unsupported activation dtype {activation_dtype!r}")


def flash_attention_kv_format(spec: dict) -> str:
    """KV cache format of a flash_attention definition, decided as the harness
    decides it (op_test_handler.py:483-534): key_cache dtype "int8" means q8_0
    when the variant or a tag names q8, else q4_0; "float16" (and any other
    dtype but "float32") means fp16. fp32 caches are not a format of any
    shipped definition and are rejected."""
    dtype = spec.get("inputs", {}).get("key_cache", {}).get("dtype", "float16")
    if dtype == "int8":
        variant = spec.get("variant", "").lower()
        tags = spec.get("tags", [])
        return "q8_0" if ("q8" in variant or any("q8" in t for t in tags)) else "q4_0"
    if dtype == "float32":
        raise ValueError("fp32 KV caches are not supported (no flash_attention definition uses them)")
    return "f16"


def flash_attention_forward(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                            batch_size: int, seq_len: int, num_heads: int, head_dim: int,
                            kv_format: str = "q8_0") -> torch.Tensor:
    """forward(q, k, v, B, S, H, D) -> fp32 [B, H, D] (op_test_handler.py:565-579);
    ``kv_format`` is ``flash_attention_kv_format(spec)`` of the definition."""
    return ops.flash_attn(query, key_cache, value_cache, batch_size, seq_len, num_heads, head_dim, kv_format)


def rms_norm_forward(hidden_states: torch.Tensor, weight: torch.Tensor, epsilon: float = 1e-6) -> torch.Tensor:
    """forward(hidden_states, weight) -> fp32 [batch, hidden] (op_test_handler.py:677-679;
    every rms_norm definition has epsilon 1e-6)."""
    return ops.rms_norm(hidden_states, weight, epsilon)


def rms_norm_performance(latency_ms: float, batch_size: int, hidden_size: int) -> dict:
    """GB/s as the harness reports them: (2 B H + H + B H) * 4 bytes / latency
    (op_test_handler.py:681-690: the input is counted twice)."""
    nbytes = (batch_size * hidden_size * 2 + hidden_size + batch_size * hidden_size) * 4
    return {"gbps": round(nbytes / (latency_ms / 1000) / 1e9, 2)}


# GPUs with a GGML baseline table in the reference (unified_test_runner.py:593-604).
_BASELINE_GPUS = ("RTX4090", "RTX4070", "A100", "RTX5090")


def baseline_hardware(gpu_name: str) -> str | None:
    """The baseline table for a GPU, or None when the reference has none.
    The harness strips "NVIDIA", spaces, "Laptop" and "Mobile" from the name
    and falls back to RTX4090 for any GPU it does not list, so a B200 run
    would be compared with RTX 4090 numbers; this returns None instead."""
    key = gpu_name.replace(" ", "").replace("NVIDIA", "").replace("Laptop", "").replace("Mobile", "")
    for hw in _BASELINE_GPUS:
        if hw in key:
            return hw
    return None


def quant_gemm_baseline_case(weight_dtype: str, M: int, N: int, K: int, activation: str = "f32") -> str:
    """Case id of the GGML baseline table for a quant_gemm call. GGML's m is
    the output features (our N) and its n the batch (our M)
    (op_test_handler.py:274-281); the id format is BaselineAPI.get_gemm's
    (core/tools/baseline_api.py:121-123). The handler calls a method the API
    does not have (`get_baseline`), so its lookups always fail; this is the
    key `get_gemm` reads."""
    wt = _WEIGHT[weight_dtype]
    return f"w{4 if 'q4' in wt else 8}a32c8_{wt}_{activation.replace('float', 'f')}_m{N}_n{M}_k{K}"


# GGML (llama.cpp) timings the reference ships as its quant_gemm baseline,
# microseconds per run, for the cases that share a shape with the benchmark
# configurations (kernelevalplus-main/data/baseline/baseline_data_compact.json:
# entries at lines 2, 41, 15346, 18407, 1996, 20362, 20401; GGML's m is our N
# and its n our M). There are no B200 entries.
GGML_GEMM_US = {
    "w4a32c8_q4_0_f32_m4096_n1_k4096": {"H800": 8.83, "A100": 13.2, "RTX4090": 6.77},
    "w4a32c8_q4_0_f32_m14336_n1_k4096": {"H800": 19.57, "A100": 30.08, "RTX4090": 14.26},
    "w4a32c8_q4_0_f32_m14336_n8_k4096": {"H800": 42.8, "A100": 69.44, "RTX4090": 47.09},
    "w4a32c8_q4_0_f32_m14336_n512_k4096": {"H800": 325.27, "A100": 718.44, "RTX4090": 266.66},
    "w8a32c8_q8_0_f32_m4096_n1_k4096": {"H800": 10.35},
    "w8a32c8_q8_0_f32_m4096_n512_k4096": {"H800": 106.13, "A100": 235.47, "RTX4090": 77.58},
    "w8a32c8_q8_0_f32_m14336_n512_k4096": {"H800": 320.25, "A100": 743.74, "RTX4090": 291.89},
}


def ggml_gemm_us(weight_dtype: str, M: int, N: int, K: int) -> dict | None:
    """GGML's published time per run (us, by GPU) for a quant_gemm call with
    fp32 activations, or None when the baseline data has no such case."""
    return GGML_GEMM_US.get(quant_gemm_baseline_case(weight_dtype, M, N, K))


def definition_test_configs(spec: dict) -> list[dict]:
    """The test configurations a definition lists itself. The harness's
    quant_gemm handler ignores them and always runs M = 1, 8, 512
    (op_test_handler.py:449-458); this returns the definition's own list
    (its M values for quant_gemm, batch sizes for flash_attention and
    rms_norm), falling back to the handler's fixed list."""
    cfgs = [dict(c) for c in spec.get("test_configs", [])]
    if cfgs:
        return cfgs
    if spec.get("op_type") == "quant_gemm":
        return quant_gemm_test_configs(spec["axes"]["N"]["value"], spec["axes"]["K"]["value"])
    return [{"name": "batch_1", "batch_size": 1}]


def quant_gemm_test_configs(N: int, K: int) -> list[dict]:
    """The harness's fixed configurations (op_test_handler.py:449-458)."""
    return [{"M": 1, "N": N, "K": K, "name": "single_token"},
            {"M": 8, "N": N, "K": K, "name": "small_batch"},
            {"M": 512, "N": N, "K": K, "name": "large_batch"}]


def quant_gemm_performance(latency_ms: float, M: int, N: int, K: int) -> dict:
    """TFLOPS as the harness reports them: 2 M N K / latency (op_test_handler.py:258-266)."""
    flops = 2 * M * N * K / (latency_ms / 1000)
    return {"tflops": round(flops / 1e12, 3), "gflops": round(flops / 1e9, 1)}


def flash_attention_performance(latency_ms: float, batch_size: int, seq_len: int, num_heads: int,
                                head_dim: int) -> dict:
    """4 B H S D / latency (op_test_handler.py:581-596)."""
    return {"tflops": round(4 * batch_size * num_heads * seq_len * head_dim / (latency_ms / 1000) / 1e12, 3)}
