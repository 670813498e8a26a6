"""ctypes binding of libpk.so (C ABI in include/pk.h).

The library is built in-tree by ``python -m parakeet_b200.build``.  There is
no fallback: if the shared object is missing or a call fails, an exception
is raised.
"""
from __future__ import annotations

import ctypes
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libpk.so")
HEADER = os.path.join(os.path.dirname(os.path.dirname(_HERE)), "include", "pk.h")

PK_OK, PK_EINVAL, PK_ECUDA, PK_ENOTSUP = 0, 1, 2, 3
PK_DTYPE_F32, PK_DTYPE_BF16 = 0, 1
PK_DEV_POOL_EXHAUSTED, PK_DEV_BAD_PAGE, PK_DEV_TIMEOUT, PK_DEV_BAD_SLOT = 1, 2, 4, 8
PK_DEV_BAD_COUNT = 16
PK_GEMM_STORE, PK_GEMM_SILU, PK_GEMM_RESIDUAL, PK_GEMM_RESIDUAL_RELU, PK_GEMM_BIAS = 0, 1, 2, 3, 4
PK_FE_HIST, PK_FE_META_STRIDE, PK_FE_FIRST, PK_FE_FINAL = 512, 4, 1, 2
PK_NOALLOC_SCRATCH_BYTES = 32 * 1024 * 1024   # pk_paged_attention_noalloc's static scratch
META_FIRST, META_NEXT, META_WRITTEN, META_PROCESSED, META_CACHE_LEN = 0, 1, 2, 3, 4
META_STRIDE = 8
WIN_STRIDE = 128
PK_MAX_BATCH = 6144   # most rows of one step (pk_pages_begin_step)


class PKError(RuntimeError):
    """A libpk entry point returned a non-zero status."""


class PagedKVDesc(ctypes.Structure):
    _fields_ = [
        ("kv", ctypes.c_void_p),
        ("page_table", ctypes.c_void_p),
        ("free_ring", ctypes.c_void_p),
        ("ring_ctr", ctypes.c_void_p),
        ("meta", ctypes.c_void_p),
        ("error", ctypes.c_void_p),
        ("window", ctypes.c_void_p),
        ("num_pages", ctypes.c_int32),
        ("num_slots", ctypes.c_int32),
        ("num_layers", ctypes.c_int32),
        ("dim", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("left", ctypes.c_int32),
        ("chunk", ctypes.c_int32),
        ("page_size", ctypes.c_int32),
        ("ring", ctypes.c_int32),
        ("dtype", ctypes.c_int32),
    ]


class FeaturesDesc(ctypes.Structure):
    _fields_ = [
        ("tables", ctypes.c_void_p),
        ("history", ctypes.c_void_p),
        ("meta", ctypes.c_void_p),
        ("error", ctypes.c_void_p),
        ("num_slots", ctypes.c_int32),
        ("n_fft", ctypes.c_int32),
        ("hop", ctypes.c_int32),
        ("n_mels", ctypes.c_int32),
        ("mel_nnz", ctypes.c_int32),
        ("preemph", ctypes.c_float),
        ("dither", ctypes.c_float),
        ("mag_power", ctypes.c_float),
        ("log_guard", ctypes.c_float),
        ("pad_value", ctypes.c_float),
        ("seed", ctypes.c_uint64),
    ]


_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64

SIGNATURES = {
    "pk_paged_kv_create": [ctypes.POINTER(PagedKVDesc), ctypes.POINTER(ctypes.c_void_p)],
    "pk_paged_kv_destroy": [_P],
    "pk_pages_per_stream": [_I32, _I32, _I32],
    "pk_ring_size": [_I32, _I32, _I32],
    "pk_pages_reset": [_P, _P, _P],
    "pk_pages_begin_step": [_P, _P, _P, _I32, _P, _I32, _P],
    "pk_pages_end_step": [_P, _P, _P, _I32, _P],
    "pk_append_kv": [_P, _I32, _I32, _P, _P, _I64, _I64, _I64, _P, _I32, _P],
    "pk_gather_window": [_P, _I32, _P, _I32, _P, _P, _P],
    "pk_gather_windows": [_P, _I32, _I32, _P, _I32, _P, _P, _I64, _P],
    "pk_rnnt_pick": [_P, _I64, _I32, _I32, _I32, _I32, _P, _I32, _I32, _I32, _I32, _P, _P, _P, _P,
                     _P, _P],
    "pk_lstm_cell": [_P, _I64, _P, _I64, _P, _P, _P, _I64, _P, _I32, _I32, _I32, _P],
    "pk_pre_encode_window": [_P, _I32, _P, _P, _I32, _I32, _I32, _I32, _I32, _P, _I32, _P, _P],
    "pk_paged_attention": [_P, _I32, _I32, _P, _I64, _I64, _I64, _P, _P, _P, _I64, _P, _P,
                           _I64, _P, _P, _I32, _P, _I64, _I64, _I64, _P],
    "pk_relpos_bd_cols": [_P],
    "pk_relpos_bd": [_P, _I32, _I32, _P, _I64, _I64, _I64, _P, _I64, _P, _I64, _I32, _P, _P],
    "pk_pages_begin_step_relpos": [_P, _P, _P, _I32, _P, _I32, _I32, _I32, _P, _I64, _I64, _I64,
                                   _P, _I64, _P, _I64, _P, _P],
    "pk_paged_attention_bd": [_P, _I32, _I32, _P, _I64, _I64, _I64, _P, _P, _P, _P, _I64, _P, _P,
                              _I32, _P, _I64, _I64, _I64, _P],
    "pk_paged_attention_noalloc": [_P, _I32, _I32, _P, _I64, _I64, _I64, _P, _P, _P, _I64, _P,
                                   _P, _I64, _P, _P, _I32, _P, _I64, _I64, _I64, _P],
    "pk_conv_step": [_P, _I32, _I32, _I32, _I32, _I32, _I32, _I32, _P, _I64, _I64, _P, _P, _P,
                     ctypes.c_float, _P, _P, _I32, _P, _P, _P],
    "pk_gemm_bf16": [_P, _I64, _P, _I64, _I32, _I32, _I32, _P, _I64, _I32, _P, _I64, _P,
                     ctypes.c_float, _P, _P],
    "pk_subsample_stage12": [_P, _I64, _I64, _I64, _I32, _I32, _I32, _P, _P, _P, _P, _I32,
                             _I32, _P, _I32, _P],
    "pk_subsample_dw": [_P, _I32, _I32, _I32, _I32, _P, _P, _I32, _I32, _P, _I32, _P],
    "pk_layer_norm": [_P, _I64, _I32, _I32, _P, _P, ctypes.c_float, _P, _I64, _P, _P,
                      ctypes.c_float, _P, _I64, _I32, _P],
    "pk_features_tables": [_I32, _I32, _I32, _I32, ctypes.c_double, ctypes.c_double, _I32, _P,
                           ctypes.POINTER(_I64), ctypes.POINTER(_I32)],
    "pk_features_push": [ctypes.POINTER(FeaturesDesc), _P, _I64, _P, _P, _P, _I32, _P, _I32, _I32,
                         _P, _P],
    "pk_selftest_bounded_wait": [_P, _I32, _I64, _P, _P],
    "pk_last_error": [],
}
RESTYPES = {"pk_last_error": ctypes.c_char_p}

_lib = None


def lib():
    """The loaded libpk.so, with argument types set.  Raises if not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise PKError(f"{LIB_PATH} is missing: build it with "
                          "`python -m parakeet_b200.build` (needs nvcc)")
        l = ctypes.CDLL(LIB_PATH)
        for name, args in SIGNATURES.items():
            fn = getattr(l, name)
            fn.argtypes = args
            fn.restype = RESTYPES.get(name, ctypes.c_int)
        _lib = l
    return _lib


def check(status: int, what: str = "") -> None:
    if status != PK_OK:
        msg = lib().pk_last_error().decode(errors="replace")
        kind = {PK_EINVAL: "invalid argument", PK_ECUDA: "CUDA error",
                PK_ENOTSUP: "not supported"}.get(status, f"status {status}")
        raise PKError(f"{what}: {kind}: {msg}")


def declared_functions(header: str = HEADER) -> list[str]:
    """Names of the functions include/pk.h declares."""
    text = open(header).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\**\s*(pk_[a-z_0-9]+)\s*\(",
                                 text, flags=re.M)))
