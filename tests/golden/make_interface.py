"""Record the call signatures of the reference's hot-path interface.

Run in the build container, where the reference source tree is present::

    python tests/golden/make_interface.py --reference-src <reference>/src

Writes ``interface.json``: for every function and KV-manager method that the
reference's request and speculative loops
(``experiments/models/qwen_explicit_runtime_loop.py:11-39``) and stack drivers
reach on the semantic path, its parameter names and defaults, read with
``inspect.signature`` from the reference modules.  ``tests/test_interface.py``
checks ``leanstack_b200``'s drop-in modules against it.
"""

from __future__ import annotations

import argparse
import inspect
import json
import os
import sys
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
HERE = Path(__file__).resolve().parent

MODULES = {
    "runtime.qwen_explicit": [
        "build_qwen_position_cache", "slice_qwen_position_embeddings", "build_decode_attention_mask",
        "build_qwen_kv_cache", "qwen_rmsnorm", "qwen_rmsnorm_vector", "last_hidden_vector",
        "normalize_stop_token_ids", "resolve_semantic_logits_backend",
        "_semantic_attention_qkv_vector", "_semantic_attention_qkv", "_semantic_decode_attention_output_vector",
        "_semantic_decode_attention_output", "_semantic_mlp_epilogue_vector", "_semantic_mlp_epilogue",
        "_semantic_post_attention_mlp", "sdpa_qwen_attention_forward", "semantic_qwen_decode_layer_forward",
        "semantic_qwen_layer_forward", "run_semantic_stack_prefill", "run_semantic_stack_prefill_from_hidden",
        "run_semantic_stack_decode", "run_semantic_stack_decode_from_hidden",
        "run_semantic_stack_verify_tokens", "run_semantic_stack_verify_from_hidden",
        "select_semantic_greedy_token",
    ],
    "runtime.kv_cache": [
        "StaticKVBlockManager.append", "StaticKVBlockManager.get", "StaticKVBlockManager.append_and_get",
        "StaticKVBlockManager.get_seq_length", "StaticKVBlockManager.get_layer_seq_length",
        "StaticKVBlockManager.page_table", "StaticKVBlockManager.summary", "StaticKVBlockManager.snapshot_cursor",
        "StaticKVBlockManager.restore_cursor", "StaticKVBlockManager.cursor_after_tokens",
    ],
    "leanserve": [
        "materialize_qwen_full_semantic_runtime_from_leanpack", "materialize_qwen_semantic_stack_from_leanpack",
    ],
}


def describe(fn) -> list:
    out = []
    for name, par in inspect.signature(fn).parameters.items():
        default = None if par.default is inspect.Parameter.empty else repr(par.default)
        out.append([name, par.kind.name, default])
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    import importlib

    record = {}
    for mod_name, names in MODULES.items():
        mod = importlib.import_module(f"leanstack.{mod_name}")
        for name in names:
            obj = mod
            for part in name.split("."):
                obj = getattr(obj, part)
            sig = describe(obj)
            if [p[1] for p in sig] == ["VAR_POSITIONAL", "VAR_KEYWORD"] and hasattr(mod, name + "_eager"):
                # the dispatch-table entries are torch.compile wrappers (qwen_explicit.py:963-971)
                # around <name>_eager: record the wrapped function's parameters
                sig = describe(getattr(mod, name + "_eager"))
            record[f"{mod_name}:{name}"] = sig
    (HERE / "interface.json").write_text(json.dumps(record, indent=1) + "\n")
    print(f"{len(record)} signatures")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
