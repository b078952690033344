"""Record the shapes of the reference's quant_gemm and flash_attention
definitions as fixtures.

Runs ONLY where the qhy991/K-Search checkout is present (pass its path as
argv[1] or set KSEARCH_REF). Reads every JSON under
kernelevalplus-main/definitions/quant_gemm*/ (the harness's operator
definitions: weight type, the constant N and K axes, the test_configs' M
values) and writes definition_shapes.json next to this script, one entry per
distinct (weight type, N, K) with the definition names that use it. The
sweep test (tests/test_definition_shapes_gpu.py) reads only that file.
Also writes flash_attention_definitions.json: for every JSON under
definitions/flash_attention/, the fields the harness reads to build the
inputs (key_cache dtype, variant, tags, the S / H / D axes, the test_configs'
batch sizes) and rms_norm_definitions.json (hidden size, epsilon, batch
sizes); tests/test_flash_decode_gpu.py, tests/test_rms_norm_gpu.py and
tests/test_abi_cpu.py read them.

    python tests/golden/make_definition_shapes.py /path/to/K-Search
"""
from __future__ import annotations

import glob
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
WTYPES = {"q4_0": "q4_0", "block_q4_0": "q4_0", "q4_1": "q4_1", "block_q4_1": "q4_1", "q8_0": "q8_0",
          "block_q8_0": "q8_0"}


def main() -> None:
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("KSEARCH_REF")
    if not root:
        raise SystemExit("usage: make_definition_shapes.py /path/to/K-Search")
    pattern = os.path.join(root, "kernelevalplus-main", "definitions", "quant_gemm*", "**", "*.json")
    shapes: dict[tuple, dict] = {}
    skipped = []
    for f in sorted(glob.glob(pattern, recursive=True)):
        rel = os.path.relpath(f, os.path.join(root, "kernelevalplus-main", "definitions"))
        try:
            d = json.load(open(f))
        except (json.JSONDecodeError, OSError):
            skipped.append(rel)
            continue
        wt = WTYPES.get(d["inputs"]["weight"]["dtype"])
        N, K = d["axes"]["N"]["value"], d["axes"]["K"]["value"]
        ms = sorted({int(t["M"]) for t in d.get("test_configs", [])})
        e = shapes.setdefault((wt, N, K), {"wtype": wt, "N": N, "K": K, "M": [], "definitions": []})
        e["M"] = sorted(set(e["M"]) | set(ms))
        e["definitions"].append(rel)
    out = {"source": "kernelevalplus-main/definitions/quant_gemm*/ (read by make_definition_shapes.py)",
           "skipped_unparsable": skipped,
           "shapes": [shapes[k] for k in sorted(shapes)]}
    with open(os.path.join(HERE, "definition_shapes.json"), "w") as fh:
        json.dump(out, fh, indent=1)
    print(f"{len(out['shapes'])} shapes from {sum(len(s['definitions']) for s in out['shapes'])} definitions; "
          f"skipped {len(skipped)}")
    fa_defs(root)


def fa_defs(root: str) -> None:
    base = os.path.join(root, "kernelevalplus-main", "definitions")
    defs = []
    for f in sorted(glob.glob(os.path.join(base, "flash_attention", "**", "*.json"), recursive=True)):
        d = json.load(open(f))
        defs.append({"definition": os.path.relpath(f, base),
                     "key_cache_dtype": d["inputs"]["key_cache"]["dtype"],
                     "variant": d.get("variant", ""), "tags": d.get("tags", []),
                     "S": d["axes"]["seq_len"]["value"], "H": d["axes"]["num_heads"]["value"],
                     "D": d["axes"]["head_dim"]["value"],
                     "B": sorted({int(t["batch_size"]) for t in d.get("test_configs", [])})})
    with open(os.path.join(HERE, "flash_attention_definitions.json"), "w") as fh:
        json.dump({"source": "kernelevalplus-main/definitions/flash_attention/ (read by make_definition_shapes.py)",
                   "definitions": defs}, fh, indent=1)
    print(f"{len(defs)} flash_attention definitions")
    rdefs = []
    for f in sorted(glob.glob(os.path.join(base, "rms_norm", "**", "*.json"), recursive=True)):
        d = json.load(open(f))
        rdefs.append({"definition": os.path.relpath(f, base), "hidden_size": d["axes"]["hidden_size"]["value"],
                      "epsilon": d["axes"].get("epsilon", {}).get("value", 1e-6),
                      "B": sorted({int(t["batch_size"]) for t in d.get("test_configs", [])})})
    with open(os.path.join(HERE, "rms_norm_definitions.json"), "w") as fh:
        json.dump({"source": "kernelevalplus-main/definitions/rms_norm/ (read by make_definition_shapes.py)",
                   "definitions": rdefs}, fh, indent=1)
    print(f"{len(rdefs)} rms_norm definitions")


if __name__ == "__main__":
    main()
