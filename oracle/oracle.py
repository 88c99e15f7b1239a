"""numpy-facing wrappers over the parity checkers.

TEST INFRASTRUCTURE ONLY.  Only tests/, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference arm import this module, and only as
the checker (or the timed CPU baseline), never as the product path.

Two libraries sit behind it:

* ``libreef_oracle.so`` -- the C restatement of reef's engine arithmetic
  (``reef_oracle.c``; each function cites the engine file:line it follows).
* ``_ref/libreef_ref.so`` -- reef's own header-only engine compiled in place
  (``ref_shim.cpp``).  It exists only where the reference checkout was present
  at build time; :func:`ref_available` says whether it was built.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_ORACLE_SO = os.path.join(_HERE, "libreef_oracle.so")
_REF_SO = os.path.join(_HERE, "_ref", "libreef_ref.so")

_lib = None
_ref = None

_f32p = C.POINTER(C.c_float)
_i8p = C.POINTER(C.c_int8)
_u8p = C.POINTER(C.c_uint8)
_i32p = C.POINTER(C.c_int32)
_u16p = C.POINTER(C.c_uint16)
_sz = C.c_size_t


def reference_root() -> str | None:
    """The reef checkout the in-place reference builds from: $REEF_REFERENCE,
    else a checkout named ``reference`` beside this repository; None when
    neither holds reef's engine headers."""
    cands = [os.environ.get("REEF_REFERENCE", "")]
    cands.append(os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference"))
    for c in cands:
        if c and os.path.isdir(os.path.join(c, "inference-engine", "reference", "cpp",
                                            "include")):
            return c
    return None


def build(reference: bool = True) -> None:
    """Compile the restatement (and the in-place reference when the reef
    checkout is found; an existing _ref build is kept otherwise)."""
    subprocess.run(["make", "-s", "-C", _HERE, "all"], check=True)
    ref_root = reference_root()
    if reference and ref_root is not None:
        subprocess.run(["make", "-s", "-C", _HERE, "ref",
                        f"REEF_REFERENCE={ref_root}"], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_ORACLE_SO):
            build(reference=False)
        _lib = C.CDLL(_ORACLE_SO)
        L = _lib
        L.ro_fill_uniform.argtypes = [C.c_uint32, _sz, C.c_float, C.c_float, _f32p]
        L.ro_fill_int8.argtypes = [C.c_uint32, _sz, C.c_int32, C.c_int32, _i8p]
        L.ro_fill_int32.argtypes = [C.c_uint32, _sz, C.c_int32, C.c_int32, _i32p]
        L.ro_fill_normal.argtypes = [C.c_uint32, _sz, C.c_float, C.c_float, _f32p]
        L.ro_int8_scale.argtypes = [C.c_float]
        L.ro_int8_scale.restype = C.c_float
        L.ro_quantize_rows.argtypes = [_sz, _sz, _f32p, _i8p, _sz, _f32p]
        L.ro_quantize_rows.restype = C.c_int
        L.ro_gemm_i8_i32.argtypes = [_sz, _sz, _sz, _i8p, _sz, _i8p, _sz,
                                     _i32p, _sz, C.c_int]
        L.ro_linear_w8a8.argtypes = [_sz, _sz, _sz, _f32p, _i8p, _sz, _f32p,
                                     _f32p, _f32p, C.c_int]
        L.ro_linear_w8a8.restype = C.c_int
        L.ro_w8a8_epilogue.argtypes = [_sz, _sz, _i32p, _f32p, _f32p, _f32p,
                                       _f32p]
        L.ro_rounding_shift.argtypes = [C.c_int32, C.c_uint]
        L.ro_rounding_shift.restype = C.c_int32
        L.ro_saturate_int8.argtypes = [C.c_int32]
        L.ro_saturate_int8.restype = C.c_int8
        L.ro_linear_int8.argtypes = [_sz, _sz, _sz, _i8p, _sz, _i8p, _sz,
                                     C.c_uint, _i32p, _i8p, C.c_int]
        L.ro_exp_nonpositive.argtypes = [C.c_float]
        L.ro_exp_nonpositive.restype = C.c_float
        L.ro_tanh_float.argtypes = [C.c_float]
        L.ro_tanh_float.restype = C.c_float
        L.ro_exp_table.argtypes = [C.c_float, _u16p]
        L.ro_softmax_int8_row.argtypes = [_sz, _i32p, C.c_uint, _u16p, _u8p]
        L.ro_attention_head_int8.argtypes = [_sz, _sz, _sz, _sz, _sz, _i8p,
                                             _sz, _i8p, _i8p, C.c_uint, _u16p,
                                             C.c_uint, _i8p, _sz]
        L.ro_attention_head_int8.restype = C.c_int
        L.ro_attention_head_f32.argtypes = [_sz, _sz, _sz, _sz, _sz, _f32p,
                                            _sz, _f32p, _f32p, _sz, _f32p, _sz]
        L.ro_attention_head_f32.restype = C.c_int
        L.ro_layernorm_f32.argtypes = [_sz, _sz, _f32p, _f32p, _f32p, C.c_float,
                                       _f32p]
        L.ro_gelu_f32.argtypes = [_sz, _f32p, _f32p]
        L.ro_matvec_rows_f32.argtypes = [_sz, _sz, _f32p, _f32p, _f32p]
        L.ro_matvec_rows_f32.restype = C.c_int
        L.ro_argmax_f32.argtypes = [_sz, _f32p]
        L.ro_argmax_f32.restype = _sz
        L.ro_gptneo_block_w8a8.argtypes = (
            [_sz, _sz, _sz, _sz, _sz, C.c_float, _f32p, _f32p, _f32p]
            + [_i8p, _f32p] * 3 + [_i8p, _f32p, _f32p, _f32p, _f32p]
            + [_i8p, _f32p, _f32p, _i8p, _f32p, _f32p, _f32p, C.c_int])
        L.ro_gptneo_block_w8a8.restype = C.c_int
    return _lib


def ref_available() -> bool:
    return os.path.exists(_REF_SO)


def ref() -> C.CDLL:
    """reef's own engine compiled in place (raises when it was not built)."""
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(
                f"{_REF_SO} not built (needs the reference checkout)")
        _ref = C.CDLL(_REF_SO)
        R = _ref
        R.ref_quantize_rows.argtypes = [_sz, _sz, _f32p, _i8p, _f32p]
        R.ref_linear_w8a8.argtypes = [_sz, _sz, _sz, _f32p, _i8p, _f32p,
                                      _f32p, _f32p]
        R.ref_weight_new.argtypes = [_sz, _sz, _i8p, _f32p]
        R.ref_weight_new.restype = C.c_void_p
        R.ref_weight_free.argtypes = [C.c_void_p]
        R.ref_weight_free.restype = None
        R.ref_linear_w8a8_weight.argtypes = [C.c_void_p, _sz, _sz, _f32p, _f32p]
        R.ref_linear_int8.argtypes = [_sz, _sz, _sz, _i8p, _i8p, C.c_uint,
                                      _i32p, _i8p]
        R.ref_matmul_i8.argtypes = [_sz, _sz, _sz, _i8p, _i8p, _i32p]
        R.ref_exp_table.argtypes = [C.c_float, _u16p]
        R.ref_exp_nonpositive.argtypes = [_sz, _f32p, _f32p]
        R.ref_softmax_int8.argtypes = [_sz, _sz, _i32p, C.c_uint, _u8p]
        R.ref_attend_head_int8.argtypes = [_sz, _sz, _sz, _sz, _sz, _i8p, _i8p,
                                           _i8p, C.c_uint, C.c_uint, _i8p]
        R.ref_attend_head_f32.argtypes = [_sz, _sz, _sz, _sz, _sz, _f32p,
                                          _f32p, _f32p, _f32p]
        R.ref_block_w8a8.argtypes = ([_sz, _sz, _sz, _sz, _sz, C.c_int,
                                      C.c_float] + [_f32p] * 15)
        R.ref_matvec_rows_f32.argtypes = [_sz, _sz, _f32p, _f32p, _f32p]
        R.ref_argmax_f32.argtypes = [_sz, _f32p, C.POINTER(_sz)]
        R.ref_pack_random_gpt_neo.argtypes = ([_sz] * 7 + [C.c_uint32, C.POINTER(C.c_uint8), _sz,
                                               C.POINTER(_sz)])
        R.ref_linear_f32.argtypes = [_sz, _sz, _sz, _f32p, _f32p, _f32p, _f32p]
        R.ref_layernorm_int8.argtypes = [_sz, _sz, _i8p, _i8p, _i8p, _i8p]
        R.ref_add_int8.argtypes = [_sz, _i8p, _i8p, _i8p]
        R.ref_gelu_int8.argtypes = [_sz, _i8p, C.c_float, C.c_float, _i8p, _i8p]
    return _ref


def _p(a: np.ndarray, t):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(t)


# ---- seeded inputs ---------------------------------------------------------

def uniform(seed: int, shape, low: float, high: float) -> np.ndarray:
    out = np.empty(shape, np.float32)
    lib().ro_fill_uniform(seed, out.size, low, high, _p(out, _f32p))
    return out


def normal(seed: int, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    out = np.empty(shape, np.float32)
    lib().ro_fill_normal(seed, out.size, mean, std, _p(out, _f32p))
    return out


def int8_uniform(seed: int, shape, low: int = -128, high: int = 127) -> np.ndarray:
    out = np.empty(shape, np.int8)
    lib().ro_fill_int8(seed, out.size, low, high, _p(out, _i8p))
    return out


def int32_uniform(seed: int, shape, low: int, high: int) -> np.ndarray:
    out = np.empty(shape, np.int32)
    lib().ro_fill_int32(seed, out.size, low, high, _p(out, _i32p))
    return out


# ---- arithmetic ------------------------------------------------------------

def quantize_rows(x: np.ndarray):
    x = np.ascontiguousarray(x, np.float32)
    rows, cols = x.shape
    q = np.empty((rows, cols), np.int8)
    s = np.empty(rows, np.float32)
    rc = lib().ro_quantize_rows(rows, cols, _p(x, _f32p), _p(q, _i8p), cols,
                                _p(s, _f32p))
    if rc != 0:
        raise ValueError("quantize_rows requires finite values")
    return q, s


def gemm_i8(a: np.ndarray, b: np.ndarray, threads: int = 0) -> np.ndarray:
    """a [M,K] int8, b [N,K] int8 -> [M,N] int32 (exact)."""
    a = np.ascontiguousarray(a, np.int8)
    b = np.ascontiguousarray(b, np.int8)
    m, k = a.shape
    n = b.shape[0]
    c = np.empty((m, n), np.int32)
    lib().ro_gemm_i8_i32(m, n, k, _p(a, _i8p), k, _p(b, _i8p), k,
                         _p(c, _i32p), n, threads)
    return c


def linear_w8a8(x, w, w_scale, bias=None, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.int8)
    w_scale = np.ascontiguousarray(w_scale, np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rows, k = x.shape
    n = w.shape[0]
    y = np.empty((rows, n), np.float32)
    rc = lib().ro_linear_w8a8(rows, k, n, _p(x, _f32p), _p(w, _i8p), k,
                              _p(w_scale, _f32p), _p(bias, _f32p),
                              _p(y, _f32p), threads)
    if rc != 0:
        raise ValueError("linear_w8a8 requires finite values")
    return y


def w8a8_epilogue(acc, x_scale, w_scale, bias=None) -> np.ndarray:
    acc = np.ascontiguousarray(acc, np.int32)
    x_scale = np.ascontiguousarray(x_scale, np.float32)
    w_scale = np.ascontiguousarray(w_scale, np.float32)
    bias = None if bias is None else np.ascontiguousarray(bias, np.float32)
    rows, n = acc.shape
    y = np.empty((rows, n), np.float32)
    lib().ro_w8a8_epilogue(rows, n, _p(acc, _i32p), _p(x_scale, _f32p),
                           _p(w_scale, _f32p), _p(bias, _f32p), _p(y, _f32p))
    return y


def linear_int8(x, w, shift: int, bias=None, threads: int = 0) -> np.ndarray:
    x = np.ascontiguousarray(x, np.int8)
    w = np.ascontiguousarray(w, np.int8)
    bias = None if bias is None else np.ascontiguousarray(bias, np.int32)
    rows, k = x.shape
    n = w.shape[0]
    y = np.empty((rows, n), np.int8)
    lib().ro_linear_int8(rows, k, n, _p(x, _i8p), k, _p(w, _i8p), k, shift,
                         _p(bias, _i32p), _p(y, _i8p), threads)
    return y


def rounding_shift(v: int, s: int) -> int:
    return int(lib().ro_rounding_shift(v, s))


def saturate_int8(v: int) -> int:
    return int(lib().ro_saturate_int8(v))


def exp_nonpositive(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    f = lib().ro_exp_nonpositive
    return np.array([f(float(v)) for v in x.ravel()], np.float32).reshape(x.shape)


def exp_table(step: float = 1.0 / 16.0) -> np.ndarray:
    t = np.empty(256, np.uint16)
    lib().ro_exp_table(step, _p(t, _u16p))
    return t


def softmax_int8(scores, shift: int, table=None) -> np.ndarray:
    scores = np.ascontiguousarray(scores, np.int32)
    table = exp_table() if table is None else np.ascontiguousarray(table, np.uint16)
    rows, n = scores.shape
    probs = np.empty((rows, n), np.uint8)
    for r in range(rows):
        lib().ro_softmax_int8_row(n, _p(scores[r], _i32p), shift,
                                  _p(table, _u16p), _p(probs[r], _u8p))
    return probs


def attention_head_int8(q, k, v, query_start: int, window: int,
                        score_shift: int, out_shift: int = 8,
                        table=None) -> np.ndarray:
    q = np.ascontiguousarray(q, np.int8)
    k = np.ascontiguousarray(k, np.int8)
    v = np.ascontiguousarray(v, np.int8)
    table = exp_table() if table is None else np.ascontiguousarray(table, np.uint16)
    ql, d = q.shape
    kl = k.shape[0]
    out = np.empty((ql, d), np.int8)
    rc = lib().ro_attention_head_int8(ql, kl, d, query_start, window,
                                      _p(q, _i8p), d, _p(k, _i8p), _p(v, _i8p),
                                      score_shift, _p(table, _u16p), out_shift,
                                      _p(out, _i8p), d)
    if rc != 0:
        raise ValueError("attention row has no visible key")
    return out


def attention_head_f32(q, k, v, query_start: int, window: int) -> np.ndarray:
    q = np.ascontiguousarray(q, np.float32)
    k = np.ascontiguousarray(k, np.float32)
    v = np.ascontiguousarray(v, np.float32)
    ql, d = q.shape
    kl = k.shape[0]
    out = np.empty((ql, d), np.float32)
    rc = lib().ro_attention_head_f32(ql, kl, d, query_start, window,
                                     _p(q, _f32p), d, _p(k, _f32p),
                                     _p(v, _f32p), d, _p(out, _f32p), d)
    if rc != 0:
        raise ValueError("attention row has no visible key")
    return out


def layernorm(x, gain, shift, eps: float = 1e-5) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    rows, width = x.shape
    y = np.empty_like(x)
    lib().ro_layernorm_f32(rows, width, _p(x, _f32p),
                           _p(np.ascontiguousarray(gain, np.float32), _f32p),
                           _p(np.ascontiguousarray(shift, np.float32), _f32p),
                           eps, _p(y, _f32p))
    return y


def matvec_rows_f32(w, x):
    """reef's lm_head row, linear(x, w) with w [out][in] (model.hpp:107-110):
    returns (y [out] fp32, ok) -- ok False where the engine would throw."""
    w = np.ascontiguousarray(w, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    out, n = w.shape
    y = np.empty(out, np.float32)
    bad = lib().ro_matvec_rows_f32(out, n, _p(w, _f32p), _p(x, _f32p), _p(y, _f32p))
    return y, bad == 0


def linear_f32(x, wt, bias=None) -> np.ndarray:
    """reef's float linear with Coral's transposed weight (kernels.hpp:26-33;
    operator/linear.hpp:75-84): y[r][c] = sum over k, in order, of x[r][k] *
    wt[k][c], then + bias[c] -- each row is matvec_rows_f32 of wt^T."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(np.asarray(wt, np.float32).T)
    y = np.empty((x.shape[0], w.shape[0]), np.float32)
    for r in range(x.shape[0]):
        y[r], ok = matvec_rows_f32(w, x[r])
        if not ok:
            raise ValueError("non-finite product or sum")
    if bias is not None:
        y = (y + np.asarray(bias, np.float32)).astype(np.float32)
    return y


def gelu_int8(x, table) -> np.ndarray:
    """gelu_int8 (int8.hpp:135-147): y = table[x + 128]."""
    return np.asarray(table, np.int8)[np.asarray(x, np.int32) + 128]


def add_int8(a, b) -> np.ndarray:
    """add_int8 (int8.hpp:382-397): saturate(a + b)."""
    return np.clip(np.asarray(a, np.int32) + np.asarray(b, np.int32), -128, 127).astype(np.int8)


def embedding_int8(wte, wpe, ids, first_position: int = 0) -> np.ndarray:
    """embedding_int8 (kernels.hpp:142-145): saturate(wte[id] + wpe[position])."""
    ids = np.asarray(ids, np.int64)
    pos = first_position + np.arange(ids.size)
    return add_int8(np.asarray(wte)[ids], np.asarray(wpe)[pos])


def layernorm_int8(x, gain, shift) -> np.ndarray:
    """layernorm_int8 (int8.hpp:319-374): per row mean = floor(sum / width)
    (floor_div, :311-316), std = isqrt(sum((x - mean)^2) / width) (isqrt,
    :291-303, the floor of the square root), inv = 2^20 / max(std, 1), then
    saturate(rounding_shift(((x - mean) * inv >> 16) * gain + shift * 32, 5))
    with arithmetic right shifts."""
    import math
    x = np.asarray(x, np.int64)
    rows, width = x.shape
    mean = np.floor_divide(x.sum(axis=1), width)
    c = x - mean[:, None]
    dev = np.array([math.isqrt(int(v) // width) for v in (c * c).sum(axis=1)], np.int64)
    inv = (1 << 20) // np.maximum(dev, 1)
    normed = (c * inv[:, None]) >> 16
    scaled = normed * np.asarray(gain, np.int64) + np.asarray(shift, np.int64) * 32
    r = (scaled >> 5) + ((scaled >> 4) & 1)
    return np.clip(r, -128, 127).astype(np.int8)


def argmax_f32(x) -> int:
    """argmax (model.hpp:32-42): the first index of the largest value."""
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().ro_argmax_f32(x.size, _p(x, _f32p)))


def gelu(x) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    y = np.empty_like(x)
    lib().ro_gelu_f32(x.size, _p(x, _f32p), _p(y, _f32p))
    return y


def gptneo_block_w8a8(x, p: dict, heads: int, window: int = 0,
                      eps: float = 1e-5, threads: int = 0) -> np.ndarray:
    """One GPT-Neo W8A8 block; ``p`` holds the quantized weights (see
    :func:`quantize_block`)."""
    x = np.ascontiguousarray(x, np.float32)
    seq, d = x.shape
    ffn = p["wfc"].shape[0]
    y = np.empty_like(x)
    f, i = _f32p, _i8p
    rc = lib().ro_gptneo_block_w8a8(
        seq, d, heads, ffn, window, eps, _p(x, f), _p(p["ln1_g"], f),
        _p(p["ln1_b"], f), _p(p["wq"], i), _p(p["sq"], f), _p(p["wk"], i),
        _p(p["sk"], f), _p(p["wv"], i), _p(p["sv"], f), _p(p["wo"], i),
        _p(p["so"], f), _p(p["bo"], f), _p(p["ln2_g"], f), _p(p["ln2_b"], f),
        _p(p["wfc"], i), _p(p["sfc"], f), _p(p["bfc"], f), _p(p["wproj"], i),
        _p(p["sproj"], f), _p(p["bproj"], f), _p(y, f), threads)
    if rc != 0:
        raise ValueError("block requires finite values")
    return y


def quantize_block(fw: dict) -> dict:
    """quantize_w8a8 (weights.hpp:460-472) of one block's float weights."""
    p = {k: np.ascontiguousarray(v, np.float32) for k, v in fw.items()
         if not k.startswith("w")}
    for name, scale in (("wq", "sq"), ("wk", "sk"), ("wv", "sv"),
                        ("wo", "so"), ("wfc", "sfc"), ("wproj", "sproj")):
        p[name], p[scale] = quantize_rows(fw[name])
    return p
