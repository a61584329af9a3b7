"""Regenerate tests/golden/reference_known_answers.json.

The reference (khulnasoft-research/kyro, all Rust) cannot be built here, so
its own unit tests, read as text, are the only known answers on the verify
path.  This script extracts the sample_token cases from the test module of
src/worker.rs (the inputs, temperature, top_p, top_k and expected token)
and records the BlockManager and PagedAttention cases of
src/scheduler/block_manager.rs and src/model/attention_kernel.rs, each with
the file:line it came from.

Run in the development container (where the reference is mounted):
    python tests/golden/make_golden.py /path/to/reference
Nothing at test time reads the reference; tests load the JSON.
"""
from __future__ import annotations

import json
import os
import re
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def _line_of(text: str, pos: int) -> int:
    return text.count("\n", 0, pos) + 1


def sample_token_cases(ref: str):
    path = "src/worker.rs"
    src = open(os.path.join(ref, path)).read()
    tests = src[src.index("mod tests"):]
    base = src.index("mod tests")
    cases = []
    pat = re.compile(
        r"fn (test_\w+)\(\)\s*\{(?P<body>.*?)\n    \}", re.S)
    for m in pat.finditer(tests):
        name, body = m.group(1), m.group("body")
        arr = re.search(r"from_slice\(\s*&\[(.*?)\]", body, re.S)
        call = re.search(r"sample_token\(&logits,\s*([-\d.]+),\s*([-\d.]+),\s*(None|Some\((\d+)\))\)",
                         body)
        if not arr or not call:
            continue
        raw = arr.group(1).strip()
        values = [] if raw.startswith("]") or "as &[f32]" in arr.group(0) or raw == "" else [
            float(v.replace("_f32", "")) for v in raw.split(",") if v.strip()]
        eq = re.search(r"assert_eq!\(token,\s*(\d+)\)", body)
        contains = re.search(r"assert!\(\[(.*?)\]\.contains", body)
        lt = re.search(r"assert!\(token < (\d+)\)", body)
        case = {
            "name": name,
            "source": f"{path}:{_line_of(src, base + m.start())}",
            "logits": values,
            "temperature": float(call.group(1)),
            "top_p": float(call.group(2)),
            "top_k": int(call.group(4)) if call.group(4) else None,
        }
        if eq:
            case["expect_token"] = int(eq.group(1))
        elif contains:
            case["expect_one_of"] = [int(v.replace("u32", "")) for v in contains.group(1).split(",")]
        elif lt:
            case["expect_below"] = int(lt.group(1))
        cases.append(case)
    return cases


def main(argv):
    ref = argv[1] if len(argv) > 1 else os.environ.get("KYRO_REFERENCE", "")
    if not ref or not os.path.isdir(ref):
        raise SystemExit("usage: make_golden.py <reference checkout>")
    data = {
        "about": "Known answers from the reference's own unit tests (read as text).",
        "sample_token": sample_token_cases(ref),
        "block_manager": [
            {"name": "test_allocate_with_prefix_no_cache",
             "source": "src/scheduler/block_manager.rs:165-175",
             "block_size": 4, "num_gpu_blocks": 10, "tokens": 5,
             "expect_blocks": 2, "expect_free_after": 8},
            {"name": "test_oom_returns_none", "source": "src/scheduler/block_manager.rs:208-213",
             "block_size": 4, "num_gpu_blocks": 1, "tokens": 5, "expect_ok": False},
            {"name": "test_multiple_requests_unique_block_tables",
             "source": "src/scheduler/block_manager.rs:228-235",
             "block_size": 4, "num_gpu_blocks": 20, "requests": [4, 4],
             "expect_distinct_tables": True},
        ],
        "paged_attention": [
            {"name": "test_paged_attention_zero_context",
             "source": "src/model/attention_kernel.rs:164-183",
             "block_size": 16, "num_heads": 8, "head_dim": 64, "num_kv_heads": 2,
             "num_blocks": 4, "context_len": 0, "fill": 0.0, "expect_shape": [1, 8, 64],
             "expect_value": 0.0},
            {"name": "test_paged_attention_mha_single_block",
             "source": "src/model/attention_kernel.rs:186-205",
             "block_size": 16, "num_heads": 8, "head_dim": 64, "num_kv_heads": 8,
             "num_blocks": 4, "context_len": 8, "fill": 1.0, "expect_shape": [1, 8, 64],
             "expect_value": 1.0},
            {"name": "test_paged_attention_mha_multi_block",
             "source": "src/model/attention_kernel.rs:208-227",
             "block_size": 16, "num_heads": 8, "head_dim": 64, "num_kv_heads": 8,
             "num_blocks": 4, "context_len": 24, "fill": 1.0, "expect_shape": [1, 8, 64],
             "expect_value": 1.0},
        ],
        "ngram": [
            {"name": "test_ngram_table_building", "source": "src/speculative.rs:405-414",
             "corpus": [[1, 2, 3, 4, 5]], "order": 2,
             "expect": {"1": 2, "2": 3, "3": 4}},
        ],
    }
    out = os.path.join(HERE, "reference_known_answers.json")
    with open(out, "w") as f:
        json.dump(data, f, indent=1)
    print(out, len(data["sample_token"]), "sample_token cases")


if __name__ == "__main__":
    main(sys.argv)
