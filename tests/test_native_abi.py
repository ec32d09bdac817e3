"""The C-ABI library loads on a machine without a GPU and exports every
symbol that include/leanb200.h declares.  No kernel is launched here."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from leanstack_b200 import _native as nat

HEADER = Path(__file__).resolve().parents[1] / "include" / "leanb200.h"


def _declared(text: str) -> list[str]:
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(ls_\w+)\s*\(", text, flags=re.M)))


def _split_header() -> tuple[str, str]:
    """(release part, LEANB200_PROFILING part) of the header."""
    text = HEADER.read_text()
    start = text.index("#ifdef LEANB200_PROFILING")
    end = text.index("#endif /* LEANB200_PROFILING */")
    return text[:start] + text[end:], text[start:end]


def declared_symbols() -> list[str]:
    return _declared(_split_header()[0])


@pytest.fixture(scope="module")
def lib():
    if not nat.LIB_PATH.exists():
        from leanstack_b200 import build

        build.build()
    return nat.load()


def test_header_declares_the_hot_path_entry_points():
    syms = declared_symbols()
    for name in ("ls_rmsnorm_qkv_rope_kvappend", "ls_decode_attention", "ls_oproj_residual",
                 "ls_rmsnorm_gateup_silu", "ls_down_residual", "ls_lmhead_argmax", "ls_version", "ls_last_error"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in leanb200.h but not exported"
    assert set(declared_symbols()) <= set(nat.exported_symbols()), "ctypes signature table is incomplete"


def test_release_library_has_no_measurement_hooks(lib):
    """The per-CTA trace hooks and the NVLink probe exist only in a library built
    with LEANB200_PROFILING; the default build exports none of them."""
    hooks = _declared(_split_header()[1])
    assert set(hooks) == set(nat.PROFILING_SIGNATURES)
    stamp = nat.LIB_PATH.parent / "build_flags.txt"
    if stamp.exists() and "LEANB200_PROFILING" in stamp.read_text():
        pytest.skip("library built with --profiling")
    for name in hooks:
        assert not hasattr(lib, name), f"{name} exported by the release library"


def test_version_and_argument_errors_without_gpu(lib):
    assert lib.ls_version() == 1
    # argument validation happens before any CUDA call and returns a code
    rc = lib.ls_linear_bf16(None, 1, 2560, None, ctypes.c_float(1e-6), None, 4096, 0, None, None, None)
    assert rc == 1  # LS_ERR_INVALID_ARGUMENT
    assert "null" in nat.last_error()
    rc = lib.ls_rmsnorm_qkv_rope_kvappend(*([None] + [1, 1, 2560, None, ctypes.c_float(1e-6), None, 32, 8, 64]
                                            + [None] * 4 + [16, 0, None, 0, None, None, 16, None, None, None, None,
                                                            None]))
    assert rc != 0
    with pytest.raises(nat.LeanB200Error):
        nat.call("ls_embed_gather", None, 1, None, 10, 8, None, None)


def test_split_and_fused_entry_points_validate_before_any_cuda_call(lib):
    """The split-partial consumers and the one-launch bs1 attention reject bad
    arguments with a status code before touching the device (the addresses
    below are never dereferenced)."""
    f = ctypes.c_float(1e-6)
    p = 256  # a 16-byte aligned stand-in address
    # one-launch attention: null qkv; head_dim 64; 32 query heads per kv head (at most 16)
    args = [p, 1, 32, 8, 128, p, p, f, p, p, 4096, 0, p, 0, p, p, 4096, ctypes.c_float(0.088), p, None]
    for i, v, code in ((0, None, 1), (4, 64, 2), (3, 1, 1)):
        a = list(args)
        a[i] = v
        assert lib.ls_decode_attention_qkv(*a) == code
    # a host cursor outside the cache
    a = list(args)
    a[12], a[13] = None, 4096
    assert lib.ls_decode_attention_qkv(*a) == 6
    assert "outside" in nat.last_error()
    # residual + norm over split partials: the norm needs both weight and output
    assert lib.ls_residual_rmsnorm_splits(p, 4, 2, 2560, p, p, f, p, None, None) == 1
    # rows that are not a multiple of 8
    assert lib.ls_residual_rmsnorm_splits(p, 4, 2, 2564, p, None, f, p, None, None) == 3
    # zero splits
    assert lib.ls_sum_splits_f32(p, 0, 16, p, None) == 1


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    monkeypatch.setattr(nat, "LIB_PATH", tmp_path / "nope.so")
    monkeypatch.setattr(nat, "_LIB", None)
    with pytest.raises(nat.NativeLibraryMissing):
        nat.load()


def test_kernel_wrappers_refuse_cpu_tensors():
    import torch

    from leanstack_b200 import kernels as K

    x = torch.zeros(1, 256, dtype=torch.bfloat16)
    w = torch.zeros(256, 256, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="no CPU path"):
        K.linear(x, w)
