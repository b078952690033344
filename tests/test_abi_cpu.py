"""CPU: libkq.so builds, loads and exports every entry point include/kq.h
declares (no compute call: there is no GPU here)."""
import ctypes
import os
import re

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "kq.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:[A-Za-z_][\w\s\*]*?)\b(kq_\w+)\s*\(", src, flags=re.M)))


@pytest.fixture(scope="module")
def libkq():
    from kq import build as kqbuild  # noqa: F401  (k-search_b200/kq/build.py)
    path = kqbuild.build()
    return ctypes.CDLL(path)


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("kq_gemm_f32act", "kq_mul_mat_q", "kq_quantize_q8_1", "kq_fa_decode_q8_0_mha",
              "kq_fa_decode_q8_0_ragged", "kq_w4a32c8_q4_0_fp32_int8", "kq_flash_attn_q8_0"):
        assert s in syms


def test_library_exports_all_declared(libkq):
    missing = [s for s in declared_symbols() if not hasattr(libkq, s)]
    assert not missing, missing


def test_python_binding_covers_header(libkq):
    from kq import _lib
    assert set(declared_symbols()) == set(_lib.SIGNATURES)


def test_host_only_entry_points(libkq):
    """Calls that do not touch a device: ABI version, block sizes, argument checks."""
    from kq import _lib
    L = _lib.lib()
    assert L.kq_abi_version() == 1
    assert [L.kq_block_bytes(t) for t in (0, 1, 2, 7)] == [18, 20, 34, 0]
    # invalid arguments are rejected before any CUDA call
    assert L.kq_mul_mat_q(9, None, None, None, 1, 1, 32, None) == 1
    assert "unknown weight type" in _lib.last_error()
    assert L.kq_gemm_f32act(0, None, None, None, 1, 1, 33, 2, None) == 1
    assert "multiple of 32" in _lib.last_error()
    assert L.kq_quantize_q8_1(None, None, 1, 31, 0, None) == 1
    assert L.kq_fa_decode_q8_0_mha(None, None, None, None, 1, 1, 1, 48, None) == 1
    assert L.kq_fa_decode_mha(3, None, None, None, None, 1, 1, 1, 32, None) == 1
    assert "unknown KV format" in _lib.last_error()
    assert L.kq_fa_decode_mha(1, None, None, None, None, 1, 1, 1, 48, None) == 1
    assert L.kq_rms_norm_quantize_q8_1(None, None, None, 2, 48, ctypes.c_float(1e-6), 0, None) == 1
    assert "K % 32" in _lib.last_error()
    assert L.kq_rms_norm_quantize_q8_1(None, None, None, 2, 64, ctypes.c_float(1e-6), 2, None) == 1
    assert L.kq_rms_norm_f32(None, None, None, -1, 64, ctypes.c_float(1e-6), None) == 1
    assert L.kq_rms_norm_f32(None, None, None, 0, 64, ctypes.c_float(1e-6), None) == 0
    assert L.kq_gemm_f32act_rmsnorm(0, None, None, None, ctypes.c_float(1e-6), None, 1, 1, 33, 2, None) == 1
    # empty problems are no-ops
    assert L.kq_gemm_f32act(0, None, None, None, 0, 16, 64, 2, None) == 0


def test_harness_kv_format_of_every_definition():
    """The harness mirror picks each flash_attention definition's KV format
    as the harness does (key_cache dtype, then q8 in variant or tags); the
    shipped definitions name their format in the file name."""
    import json
    from kq import harness
    here = os.path.join(REPO, "tests", "golden")
    defs = json.load(open(os.path.join(here, "flash_attention_definitions.json")))["definitions"]
    assert len(defs) == 18
    seen = set()
    for d in defs:
        spec = {"inputs": {"key_cache": {"dtype": d["key_cache_dtype"]}}, "variant": d["variant"], "tags": d["tags"]}
        fmt = harness.flash_attention_kv_format(spec)
        assert f"_{fmt}_cache" in d["definition"], d["definition"]
        seen.add(fmt)
    assert seen == {"q8_0", "q4_0", "f16"}
    import numpy as np
    g = np.load(os.path.join(here, "flash_attn_kv.npz"))
    for fmt in ("q8_0", "q4_0", "f16"):
        spec = {"inputs": {"key_cache": {"dtype": str(g[f"{fmt}_spec_dtype"])}},
                "variant": str(g[f"{fmt}_spec_variant"]), "tags": []}
        assert harness.flash_attention_kv_format(spec) == fmt


@pytest.mark.parametrize("name", ["kernel_quant_gemm_q4_0.cu", "kernel_quant_gemm_q4_1.cu",
                                  "kernel_quant_gemm_q8_0.cu", "kernel_quant_gemm_w4a8_q8_1.cu",
                                  "kernel_flash_attn.cu", "kernel_flash_attn_q4_0.cu",
                                  "kernel_flash_attn_f16.cu", "kernel_rms_norm.cu"])
def test_harness_forwarders_build(name, tmp_path):
    """The attempt files are host-only C++: they compile with g++ and export
    the entry the harness binds."""
    import shutil
    import subprocess
    if not shutil.which("g++"):
        pytest.skip("g++ not available")
    src = os.path.join(REPO, "k-search_b200", "harness", name)
    so = str(tmp_path / "attempt.so")
    subprocess.run(["g++", "-x", "c++", "-std=c++17", "-O1", "-fPIC", "-shared", src, "-o", so, "-ldl"], check=True)
    entry = re.search(r'extern "C" void (\w+)\(', open(src).read()).group(1)
    assert hasattr(ctypes.CDLL(so), entry)


def test_definition_test_configs():
    """The harness mirror returns a definition's own test configurations
    (the quant_gemm handler's fixed M = 1, 8, 512 only when it lists none)."""
    import json
    from kq import harness
    here = os.path.join(REPO, "tests", "golden")
    rdefs = json.load(open(os.path.join(here, "rms_norm_definitions.json")))["definitions"]
    assert len(rdefs) == 9 and all(d["epsilon"] == 1e-6 for d in rdefs)
    spec = {"op_type": "rms_norm", "test_configs": [{"name": f"batch_{b}", "batch_size": b} for b in (1, 8, 32, 512)]}
    assert [c["batch_size"] for c in harness.definition_test_configs(spec)] == [1, 8, 32, 512]
    qspec = {"op_type": "quant_gemm", "axes": {"N": {"value": 4096}, "K": {"value": 4096}}}
    assert [c["M"] for c in harness.definition_test_configs(qspec)] == [1, 8, 512]
    assert harness.rms_norm_performance(1.0, 512, 4096)["gbps"] == round((512 * 4096 * 3 + 4096) * 4 / 1e-3 / 1e9, 2)


def test_baseline_lookup_fixups():
    """Baseline reporting as the harness means it: no RTX 4090 fallback for
    GPUs without a table, and the GGML case id with m = N, n = M."""
    from kq import harness
    assert harness.baseline_hardware("NVIDIA GeForce RTX 4090") == "RTX4090"
    assert harness.baseline_hardware("NVIDIA A100-SXM4-80GB") == "A100"
    assert harness.baseline_hardware("NVIDIA B200") is None
    assert harness.quant_gemm_baseline_case("block_q4_0", 1, 4096, 14336) == "w4a32c8_q4_0_f32_m4096_n1_k14336"
    assert harness.quant_gemm_baseline_case("block_q8_0", 512, 11008, 4096) == "w8a32c8_q8_0_f32_m11008_n512_k4096"
