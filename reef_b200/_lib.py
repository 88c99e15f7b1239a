"""ctypes binding of libreef_b200.so (the C ABI in include/reef_b200.h).

This is the binding a Python host of reef's operator API would add.  Loading
fails loudly when the library has not been built: there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os
import re

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_PATH = os.path.join(PKG, "libreef_b200.so")
HEADER = os.path.join(ROOT, "include", "reef_b200.h")

_lib = None

_sz = C.c_size_t
_p = C.c_void_p
_u = C.c_uint
_i = C.c_int

# argument types per entry point (all pointers as void*)
SIGNATURES = {
    "reef_b200_status_string": ([_i], C.c_char_p),
    "reef_b200_version": ([], _i),
    "reef_b200_kpad": ([_sz], _sz),
    "reef_b200_check_device": ([], _i),
    "reef_b200_device_error": ([_p], _i),
    "reef_b200_quantize_rows": ([_sz, _sz, _p, _p, _p, _p], _i),
    "reef_b200_pack_weight_i8": ([_sz, _sz, _p, _p, _p], _i),
    "reef_b200_pad_rows_i8": ([_sz, _sz, _p, _p, _p], _i),
    "reef_b200_linear_w8a8": ([_sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p], _i),
    "reef_b200_linear_w8a8_bias": ([_sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p, _p], _i),
    "reef_b200_gemm_w8a8": ([_sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p], _i),
    "reef_b200_linear_int8": ([_sz, _sz, _sz, _p, _p, _u, _p, _p], _i),
    "reef_b200_linear_bias_int8": ([_sz, _sz, _sz, _p, _p, _p, _u, _p, _p], _i),
    "reef_b200_gemm_i8_i32": ([_sz, _sz, _sz, _p, _p, _p, _p], _i),
    "reef_b200_softmax_int8": ([_sz, _sz, _p, _u, _p, _p, _p], _i),
    "reef_b200_attention_head_int8": ([_sz, _sz, _sz, _sz, _sz, _p, _sz, _p, _p, _u, _p,
                                       _u, _p, _p, _p, _sz, _p], _i),
    "reef_b200_attention_head_f32": ([_sz, _sz, _sz, _sz, _sz, _p, _sz, _p, _p, _p, _p,
                                      _sz, _p], _i),
    "reef_b200_attention_heads_f32": ([_sz] * 6 + [_p, _sz, _sz, _p, _p, _sz, _sz, _p, _sz,
                                                   _sz, _p], _i),
    "reef_b200_attention_heads_int8": ([_sz] * 6 + [_p, _sz, _sz, _p, _p, _sz, _sz, _u, _p,
                                                    _u, _p, _sz, _sz, _p], _i),
    "reef_b200_rope_qkv_quant": ([_sz, _sz, _sz, _sz, C.c_float] + [_p] * 9, _i),
    "reef_b200_flash_attn_i8": ([_sz, _sz, _sz, _sz, _sz, _i, C.c_float] + [_p] * 8, _i),
}


class ReefError(RuntimeError):
    def __init__(self, fn: str, status: int):
        name = lib().reef_b200_status_string(status).decode()
        super().__init__(f"{fn} failed: status {status} ({name})")
        self.status = status


def header_functions() -> list[str]:
    """Every function the public header declares."""
    with open(HEADER) as fh:
        text = fh.read()
    return sorted(set(re.findall(r"\b(reef_b200_\w+)\s*\(", text)))


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m reef_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (args, res) in SIGNATURES.items():
            f = getattr(L, name)
            f.argtypes = args
            f.restype = res
        _lib = L
    return _lib


def call(name: str, *args) -> None:
    """Call an entry point that returns a status; raise ReefError on failure."""
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise ReefError(name, rc)
