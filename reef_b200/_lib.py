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
    "reef_b200_matvec_rows_f32": ([_sz, _sz, _p, _p, _p, _p], _i),
    "reef_b200_argmax_f32": ([_sz, _p, _p, _p], _i),
    "reef_b200_blob_read_info": ([_p, _sz, _p], _i),
    "reef_b200_blob_layer_bytes": ([_p], _sz),
    "reef_b200_blob_load_layer": ([_p, _sz, _sz, _p, _sz, _p, _p], _i),
    "reef_b200_blob_model_bytes": ([_p], _sz),
    "reef_b200_blob_load_model": ([_p, _sz, _p, _sz, _p, _p, _p, _p], _i),
    "reef_b200_embedding_f32": ([_sz, _sz, _p, _sz, _sz, _sz, _p, _p, _p, _p], _i),
    "reef_b200_embedding_int8": ([_sz, _sz, _p, _sz, _sz, _sz, _p, _p, _p, _p], _i),
    "reef_b200_linear_f32": ([_sz, _sz, _sz, _p, _p, _p, _p], _i),
    "reef_b200_linear_bias_f32": ([_sz, _sz, _sz, _p, _p, _p, _p, _p], _i),
    "reef_b200_layernorm_f32": ([_sz, _sz, _p, _p, _p, C.c_float, _p, _p], _i),
    "reef_b200_gelu_f32": ([_sz, _p, _p, _p], _i),
    "reef_b200_exp_nonpositive_f32": ([_sz, _p, _p, _p], _i),
    "reef_b200_tanh_f32": ([_sz, _p, _p, _p], _i),
    "reef_b200_add_f32": ([_sz, _p, _p, _p, _p], _i),
    "reef_b200_gelu_int8": ([_sz, _p, _p, _p, _p], _i),
    "reef_b200_layernorm_int8": ([_sz, _sz, _p, _p, _p, _p, _p], _i),
    "reef_b200_add_int8": ([_sz, _p, _p, _p, _p], _i),
    "reef_b200_gptneo_block_forward_cached": ([_p, _p, _p, _sz, _p, _p, _sz, _p, _sz, _p], _i),
    "reef_b200_gptneo_step_workspace_bytes": ([_p, _sz], _sz),
    "reef_b200_gptneo_step": ([_p, _p, _sz, _sz, _p, _p, _sz, _p, _p, _p, _sz, _p], _i),
    "reef_b200_pack_weight_i8": ([_sz, _sz, _p, _p, _p], _i),
    "reef_b200_pad_rows_i8": ([_sz, _sz, _p, _p, _p], _i),
    "reef_b200_linear_w8a8": ([_sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p], _i),
    "reef_b200_linear_w8a8_bias": ([_sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p, _p], _i),
    "reef_b200_gemm_w8a8": ([_sz, _sz, _sz, _p, _p, _p, _p, _p, _p, _p], _i),
    "reef_b200_linear_w8a8_swiglu": ([_sz, _sz, _sz] + [_p] * 7, _i),
    "reef_b200_rmsnorm_quant": ([_sz, _sz, C.c_float] + [_p] * 5, _i),
    "reef_b200_selftest_wait_timeout": ([C.c_uint, _p, _p], _i),
    "reef_b200_selftest_peer_wait_timeout": ([C.c_uint, _p, C.c_uint, _p], _i),
    "reef_b200_weight_tiles_bytes": ([_sz, _sz], _sz),
    "reef_b200_pack_weight_tiles": ([_sz, _sz, _p, _p, _p], _i),
    "reef_b200_linear_w8a8_qkv_rope": ([_sz] * 5 + [C.c_float] + [_p] * 13, _i),
    "reef_b200_gemm_skinny_workspace_bytes": ([_sz, _sz, _sz], _sz),
    "reef_b200_gemm_w8a8_skinny": ([_sz, _sz, _sz] + [_p] * 6 + [_sz, _p, _p], _i),
    "reef_b200_linear_w8a8_noalloc": ([_sz, _sz, _sz, _p, _p, _p, _p, _p, _p], _i),
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
    "reef_b200_flash_attn_i8": ([_sz, _sz, _sz, _sz, _sz, _i, C.c_float] + [_p] * 7, _i),
    "reef_b200_decode_attn_workspace_bytes": ([_sz, _sz, _sz], _sz),
    "reef_b200_decode_attn_i8": ([_sz, _sz, _sz, _sz, _sz, _p, _sz, C.c_float] + [_p] * 7
                                 + [_sz, _p, _p], _i),
    "reef_b200_comm_unique_id_bytes": ([], _sz),
    "reef_b200_comm_unique_id": ([_p, _sz], _i),
    "reef_b200_comm_init": ([_i, _i, _p, C.c_double, _p], _i),
    "reef_b200_comm_destroy": ([_p], _i),
    "reef_b200_comm_abort": ([_p], _i),
    "reef_b200_linear_w8a8_rowpar": ([_p, _sz, _sz, _sz] + [_p] * 9 + [_p], _i),
    "reef_b200_llama_layer_workspace_bytes": ([_p], _sz),
    "reef_b200_llama_layer_forward": ([_p, _p, _p, _p, _sz, _p], _i),
    "reef_b200_llama_layer_kernel_launches": ([_p], _sz),
    "reef_b200_llama_layer_forward_events": ([_p, _p, _p, _p, _sz, _p, _p], _i),
    "reef_b200_llama_decode_workspace_bytes": ([_p, _sz], _sz),
    "reef_b200_llama_decode_forward": ([_p] * 8 + [_sz, _p, _sz, _p], _i),
    "reef_b200_gptneo_block_workspace_bytes": ([_p], _sz),
    "reef_b200_gptneo_block_forward": ([_p, _p, _p, _p, _sz, _p], _i),
}


class LlamaLayerDesc(C.Structure):
    """reef_b200_llama_layer (include/reef_b200.h)."""
    _fields_ = [("batch", _sz), ("seq", _sz), ("hidden", _sz), ("heads_q", _sz),
                ("heads_kv", _sz), ("head_dim", _sz), ("ffn", _sz), ("rms_eps", C.c_float),
                ("rope_base", C.c_float), ("attn_norm", _p), ("w_qkv", _p), ("s_qkv", _p),
                ("w_o", _p), ("s_o", _p), ("mlp_norm", _p), ("w_gu", _p), ("s_gu", _p),
                ("w_down", _p), ("s_down", _p), ("comm", _p), ("tp_mode", _i),
                ("t_qkv", _p), ("t_o", _p), ("t_gu", _p), ("t_down", _p)]


class GptNeoBlockDesc(C.Structure):
    """reef_b200_gptneo_block (include/reef_b200.h)."""
    _fields_ = [("seq", _sz), ("hidden", _sz), ("heads", _sz), ("head_dim", _sz), ("ffn", _sz),
                ("window", _sz), ("eps", C.c_float), ("ln1_g", _p), ("ln1_b", _p),
                ("wq", _p), ("sq", _p), ("wk", _p), ("sk", _p), ("wv", _p), ("sv", _p),
                ("wo", _p), ("so", _p), ("bo", _p), ("ln2_g", _p), ("ln2_b", _p),
                ("wfc", _p), ("sfc", _p), ("bfc", _p), ("wproj", _p), ("sproj", _p),
                ("bproj", _p), ("comm", _p)]


class GptNeoBlockF32Desc(C.Structure):
    """reef_b200_gptneo_block_f32 (include/reef_b200.h)."""
    _fields_ = [("seq", _sz), ("hidden", _sz), ("heads", _sz), ("head_dim", _sz), ("ffn", _sz),
                ("window", _sz), ("eps", C.c_float), ("ln1_g", _p), ("ln1_b", _p),
                ("wq", _p), ("wk", _p), ("wv", _p), ("wo", _p), ("bo", _p), ("ln2_g", _p),
                ("ln2_b", _p), ("wfc", _p), ("bfc", _p), ("wproj", _p), ("bproj", _p)]


class GptNeoModelDesc(C.Structure):
    """reef_b200_gptneo_model (include/reef_b200.h)."""
    _fields_ = [("vocab", _sz), ("max_positions", _sz), ("hidden", _sz), ("layers", _sz),
                ("eps", C.c_float), ("wte", _p), ("wpe", _p), ("ln_f_g", _p), ("ln_f_b", _p),
                ("blocks", _p), ("blocks_f32", _p)]


class BlobInfo(C.Structure):
    """reef_b200_blob_info (include/reef_b200.h)."""
    _fields_ = [("precision", C.c_uint32), ("vocab", _sz), ("max_positions", _sz),
                ("hidden", _sz), ("layers", _sz), ("heads", _sz), ("inner", _sz),
                ("window", _sz), ("eps", C.c_float), ("wte", _sz), ("wpe", _sz),
                ("ln_f_weight", _sz), ("ln_f_bias", _sz)]


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
