"""ctypes binding of libleanb200.so (the C ABI declared in include/leanb200.h).

The library is built in-tree (``python -m leanstack_b200.build``).  There is no
fallback: if the library is missing or a call fails, the caller gets an
exception with the library's own error message.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libleanb200.so"

LS_OK = 0
STATUS_NAMES = {
    1: "LS_ERR_INVALID_ARGUMENT",
    2: "LS_ERR_UNSUPPORTED_SHAPE",
    3: "LS_ERR_MISALIGNED",
    4: "LS_ERR_WORKSPACE",
    5: "LS_ERR_CUDA",
    6: "LS_ERR_KV_OVERFLOW",
    7: "LS_ERR_TIMEOUT",
    8: "LS_ERR_NOT_SUPPORTED",
}

EPI_STORE, EPI_RESIDUAL, EPI_SILU_MUL, EPI_STORE_F32, EPI_SPLIT_F32 = 0, 1, 2, 4, 8


class NativeLibraryMissing(RuntimeError):
    """libleanb200.so has not been built; there is no CPU fallback."""


class LeanB200Error(RuntimeError):
    def __init__(self, fn: str, code: int, message: str):
        super().__init__(f"{fn} failed with {STATUS_NAMES.get(code, code)}: {message}")
        self.fn = fn
        self.code = code


_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_f32 = ctypes.c_float

MAX_TP_RANKS = 8


class P2PExchangeDesc(ctypes.Structure):
    """``ls_p2p_exchange`` of include/leanb200.h."""

    _fields_ = [("peer", ctypes.c_void_p * MAX_TP_RANKS), ("rank", ctypes.c_int32), ("world", ctypes.c_int32),
                ("max_ctas", ctypes.c_int32), ("max_rows", ctypes.c_int32), ("width", ctypes.c_int64),
                ("trace", ctypes.c_void_p)]
_int = ctypes.c_int

# name -> argtypes (all return int status unless listed in _RESTYPES)
SIGNATURES: dict[str, list] = {
    "ls_version": [],
    "ls_last_error": [],
    "ls_get_device_error": [ctypes.POINTER(_int), _int],
    "ls_set_wait_limit_ns": [_i64],
    "ls_get_wait_limit_ns": [ctypes.POINTER(_i64)],
    "ls_sm_count": [ctypes.POINTER(_int)],
    "ls_embed_gather": [_p, _i64, _p, _i64, _i64, _p, _p],
    "ls_linear_bf16": [_p, _i64, _i64, _p, _f32, _p, _i64, _int, _p, _p, _p],
    "ls_rmsnorm_qkv_rope_kvappend": [_p, _i64, _i64, _i64, _p, _f32, _p, _i64, _i64, _i64, _p, _p, _p, _p, _i64,
                                     _i64, _p, _i64, _p, _p, _i64, _p, _p, _p, _p, _p],
    "ls_decode_attention": [_p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _f32, _p, _p, _i64, _p],
    "ls_decode_attention_workspace_bytes": [_i64, _i64, _i64, _i64, _i64, _i64, ctypes.POINTER(_i64)],
    "ls_decode_attention_qkv": [_p, _i64, _i64, _i64, _i64, _p, _p, _f32, _p, _p, _i64, _i64, _p, _i64, _p, _p,
                                _i64, _f32, _p, _p],
    "ls_oproj_residual": [_p, _i64, _i64, _p, _i64, _p, _p, _p],
    "ls_rmsnorm_gateup_silu": [_p, _i64, _i64, _p, _f32, _p, _i64, _p, _p],
    "ls_down_residual": [_p, _i64, _i64, _p, _i64, _p, _p, _p],
    "ls_lmhead_argmax": [_p, _i64, _i64, _p, _f32, _p, _i64, _p, _p, _i64, _p],
    "ls_lmhead_argmax_noalloc": [_p, _i64, _i64, _p, _f32, _p, _i64, _p, _p],
    "ls_lmhead_workspace_bytes": [_i64, _i64, ctypes.POINTER(_i64)],
    "ls_rmsnorm": [_p, _i64, _i64, _p, _f32, _p, _p],
    "ls_residual_add_f32": [_p, _p, _i64, _p, _p],
    "ls_spec_accept": [_p, _p, _i64, _i64, _p, _p, _p, _p, _p, _p, _i64, _p],
    "ls_gemm_bf16_tcgen05_big": [_p, _i64, _i64, _p, _i64, ctypes.c_int, _p, _p, _p],
    "ls_gemm_tc_tiled_bytes": [_i64, _i64, ctypes.c_int, _p],
    "ls_gemm_tc_tile_weight": [_p, _i64, _i64, ctypes.c_int, _p, _p],
    "ls_gemm_bf16_tcgen05_tiled": [_p, _i64, _i64, _p, _i64, ctypes.c_int, _p, _p, _p, _i64, _p],
    "ls_p2p_region_bytes": [_i64, _i64, _i64, _p],
    "ls_p2p_alloc": [_i64, _p],
    "ls_p2p_free": [_p],
    "ls_ipc_get_handle": [_p, _p],
    "ls_ipc_open": [_p, _p],
    "ls_ipc_close": [_p],
    "ls_linear_allreduce_residual": [_p, _i64, _i64, _p, _i64, _p, _p, _p, _p],
    "ls_allreduce_residual_f32": [_p, _i64, _i64, _p, _p, _p, _p],
    "ls_lmhead_argmax_keys": [_p, _i64, _i64, _p, _f32, _p, _i64, _i64, _p, _p, _i64, _p],
    "ls_argmax_rows_keys": [_p, _i64, _i64, _i64, _p, _p, _i64, _p],
    "ls_argmax_keys_to_ids": [_p, _i64, _p, _p],
    "ls_qk_norm_rope_kvappend": [_p, _i64, _i64, _i64, _i64, _i64, _p, _p, _f32, _p, _p, _i64, _i64, _p, _i64, _p,
                                 _p, _i64, _p, _p, _p, _p],
    "ls_argmax_rows": [_p, _i64, _i64, _p, _p, _i64, _p],
    "ls_argmax_rows_workspace_bytes": [_i64, _i64, ctypes.POINTER(_i64)],
    "ls_gemm_bf16_tcgen05": [_p, _i64, _i64, _p, _i64, _int, _p, _p, _p, _i64, _p],
    "ls_gemm_bf16_tcgen05_workspace_bytes": [_i64, _i64, _i64, _int, ctypes.POINTER(_i64)],
    "ls_gemm_bf16_tcgen05_splits": [_i64, _i64, _i64, ctypes.POINTER(_i64)],
    "ls_qk_norm_rope_kvappend_splits": [_p, _i64, _i64, _i64, _i64, _i64, _i64, _p, _p, _f32, _p, _p, _i64, _i64, _p,
                                        _i64, _p, _p, _i64, _p, _p, _p, _p],
    "ls_residual_rmsnorm_splits": [_p, _i64, _i64, _i64, _p, _p, _f32, _p, _p, _p],
    "ls_silu_mul_splits": [_p, _i64, _i64, _i64, _p, _p],
    "ls_allreduce_residual_splits": [_p, _i64, _i64, _i64, _p, _p, _p, _p],
    "ls_sum_splits_f32": [_p, _i64, _i64, _p, _p],
    "ls_advance_cursors": [_p, _p, _i64, _i64, _p],
}
_RESTYPES = {"ls_last_error": ctypes.c_char_p}
# Measurement hooks, present only in a library built with --profiling (LEANB200_PROFILING).
PROFILING_SIGNATURES: dict[str, list] = {
    "ls_linear_set_trace": [_p],
    "ls_gemm_tc_set_trace": [_p],
    "ls_p2p_pingpong": [_p, _p, ctypes.c_int, ctypes.c_int, _p, _p],
}

_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once (after torch, so it binds torch's CUDA runtime)."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise NativeLibraryMissing(
            f"{LIB_PATH} is missing: build it with `python -m leanstack_b200.build` (sm_100a, needs nvcc)")
    import torch  # noqa: F401  (loads libcudart.so.12 first)

    lib = ctypes.CDLL(str(LIB_PATH))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _RESTYPES.get(name, ctypes.c_int)
    for name, argtypes in PROFILING_SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is not None:
            fn.argtypes = argtypes
            fn.restype = ctypes.c_int
    _LIB = lib
    return lib


def last_error() -> str:
    msg = load().ls_last_error()
    return msg.decode("utf-8", "replace") if msg else ""


def call(name: str, *args) -> None:
    rc = getattr(load(), name)(*args)
    if rc != LS_OK:
        raise LeanB200Error(name, rc, last_error())


def exported_symbols() -> list[str]:
    return list(SIGNATURES)
