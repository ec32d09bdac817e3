"""The drop-in modules expose the reference's hot-path interface.

``tests/golden/interface.json`` (made by ``tests/golden/make_interface.py``
from the reference's own modules) lists, for every function and KV-manager
method that the reference's request / speculative loops and stack drivers
reach on the semantic path, its parameter names, kinds and defaults.  The
``leanstack_b200`` counterpart must take the same parameters in the same order
with the same defaults; it may add trailing parameters only if they have
defaults (so every reference call site still binds).  CPU only: signatures,
no kernels.
"""

from __future__ import annotations

import importlib
import inspect
import json

import pytest

OURS = {
    "runtime.qwen_explicit": "leanstack_b200.qwen_explicit",
    "runtime.kv_cache": "leanstack_b200.kv_cache",
    "leanserve": "leanstack_b200.leanserve",
}


def _entries(golden_dir):
    return json.loads((golden_dir / "interface.json").read_text())


def _resolve(key):
    mod_name, name = key.split(":")
    obj = importlib.import_module(OURS[mod_name])
    for part in name.split("."):
        obj = getattr(obj, part)
    return obj


def test_every_reference_entry_point_exists(golden_dir):
    missing = []
    for key in _entries(golden_dir):
        try:
            _resolve(key)
        except AttributeError:
            missing.append(key)
    assert not missing, missing


def test_signatures_bind_like_the_reference(golden_dir):
    bad = []
    for key, ref in _entries(golden_dir).items():
        ours = [[n, p.kind.name, None if p.default is inspect.Parameter.empty else repr(p.default)]
                for n, p in inspect.signature(_resolve(key)).parameters.items()]
        if [r[0] for r in ref] != [o[0] for o in ours[:len(ref)]]:
            bad.append((key, "names", [r[0] for r in ref], [o[0] for o in ours]))
            continue
        for r, o in zip(ref, ours):
            # keyword-only where the reference allows positional would break positional call sites
            if r[1] != o[1] and not (r[1] == "POSITIONAL_OR_KEYWORD" and o[1] == "POSITIONAL_OR_KEYWORD"):
                if not (r[1] == "KEYWORD_ONLY" and o[1] == "POSITIONAL_OR_KEYWORD"):
                    bad.append((key, "kind", r, o))
            if r[2] is not None and r[2] != o[2]:
                bad.append((key, "default", r, o))
        for extra in ours[len(ref):]:
            if extra[2] is None and extra[1] not in ("VAR_POSITIONAL", "VAR_KEYWORD"):
                bad.append((key, "extra parameter without a default", extra))
    assert not bad, bad


@pytest.mark.parametrize("value,want", [(None, ()), (7, (7,)), ([1, 2], (1, 2)), ((3,), (3,))])
def test_normalize_stop_token_ids(value, want):
    from leanstack_b200.qwen_explicit import normalize_stop_token_ids

    assert normalize_stop_token_ids(value) == want
