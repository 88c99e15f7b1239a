"""Host mirror of reef's operator API (namespace reef_kernels,
inference-engine/coral/include/reef_kernels/kernels.hpp) over CUDA tensors.

Same names and argument meaning as the Coral kernels, batched over rows, on
device memory.  Every function calls into libreef_b200.so through the C ABI
(include/reef_b200.h); none has a CPU path.  torch is used only to hold device
memory and the current stream.  Weights are K-major [out][kpad(in)] int8 (see
:func:`pack_weight_i8` for Coral's transposed [in][out] layout).
"""
from __future__ import annotations

import torch

from . import _lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("reef_b200 entry points take CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("reef_b200 entry points take contiguous tensors")
    return t.data_ptr()


def kpad(n: int) -> int:
    return (n + 15) // 16 * 16


def check_device_error() -> None:
    """Raise when a bounded device wait gave up since the last check."""
    import ctypes as C
    code = C.c_int(0)
    _lib.call("reef_b200_device_error", C.addressof(code))
    if code.value != 0:
        raise _lib.ReefError(f"device wait (code {code.value:#x})", 6)


# ---- quantization --------------------------------------------------------------

def quantize_rows(x: torch.Tensor):
    """quantize_rows (quant.hpp:112-133): returns (x_q [rows][kpad], x_scale)."""
    rows, k = x.shape
    x_q = torch.empty((rows, kpad(k)), dtype=torch.int8, device=x.device)
    xs = torch.empty((rows,), dtype=torch.float32, device=x.device)
    _lib.call("reef_b200_quantize_rows", rows, k, _ptr(x), _ptr(x_q), _ptr(xs), _stream())
    return x_q, xs


def matvec_rows_f32(w: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """reef_kernels::matvec_rows_f32 (kernels.hpp:48-52): y[c] = sum over k, in
    order, of x[k] * w[c][k] (GPT-Neo's lm_head), bit-identical to the engine."""
    out, k = w.shape
    y = torch.empty((out,), dtype=torch.float32, device=w.device)
    _lib.call("reef_b200_matvec_rows_f32", out, k, _ptr(w), _ptr(x), _ptr(y), _stream())
    return y


def argmax_f32(x: torch.Tensor) -> torch.Tensor:
    """reef_kernels::argmax_f32 (kernels.hpp:89-90): index of the first largest
    value, as one device int32 element holding the uint32 index."""
    idx = torch.empty((1,), dtype=torch.int32, device=x.device)
    _lib.call("reef_b200_argmax_f32", x.numel(), _ptr(x), _ptr(idx), _stream())
    return idx


def pack_weight_i8(wt: torch.Tensor) -> torch.Tensor:
    """Coral weight [in][out] -> K-major [out][kpad(in)]."""
    k, n = wt.shape
    w = torch.empty((n, kpad(k)), dtype=torch.int8, device=wt.device)
    _lib.call("reef_b200_pack_weight_i8", k, n, _ptr(wt), _ptr(w), _stream())
    return w


def pad_rows_i8(x: torch.Tensor) -> torch.Tensor:
    rows, k = x.shape
    if k == kpad(k):
        return x
    y = torch.empty((rows, kpad(k)), dtype=torch.int8, device=x.device)
    _lib.call("reef_b200_pad_rows_i8", rows, k, _ptr(x), _ptr(y), _stream())
    return y


# ---- linear layers -------------------------------------------------------------

def linear_w8a8(x: torch.Tensor, w: torch.Tensor, w_scale: torch.Tensor,
                bias: torch.Tensor | None = None, in_features: int | None = None):
    """reef_kernels::linear_w8a8 / linear_w8a8_bias (kernels.hpp:38-46)."""
    rows, k = x.shape
    n = w.shape[0]
    x_q = torch.empty((rows, kpad(k)), dtype=torch.int8, device=x.device)
    xs = torch.empty((rows,), dtype=torch.float32, device=x.device)
    y = torch.empty((rows, n), dtype=torch.float32, device=x.device)
    if bias is None:
        _lib.call("reef_b200_linear_w8a8", rows, k, n, _ptr(x), _ptr(w), _ptr(w_scale),
                  _ptr(x_q), _ptr(xs), _ptr(y), _stream())
    else:
        _lib.call("reef_b200_linear_w8a8_bias", rows, k, n, _ptr(x), _ptr(w),
                  _ptr(w_scale), _ptr(bias), _ptr(x_q), _ptr(xs), _ptr(y), _stream())
    return y


def gemm_w8a8(x_q, x_scale, w, w_scale, bias=None, in_features: int | None = None):
    rows = x_q.shape[0]
    k = in_features if in_features is not None else x_q.shape[1]
    n = w.shape[0]
    y = torch.empty((rows, n), dtype=torch.float32, device=x_q.device)
    _lib.call("reef_b200_gemm_w8a8", rows, k, n, _ptr(x_q), _ptr(x_scale), _ptr(w),
              _ptr(w_scale), _ptr(bias), _ptr(y), _stream())
    return y


def linear_w8a8_swiglu(x_q, x_scale, w_gu, w_scale, in_features: int | None = None):
    """Gate/up projection with SwiGLU in the GEMM epilogue: returns
    (h [rows][ffn] = silu(gate) * up, row_max [rows] = max |h|)."""
    rows = x_q.shape[0]
    k = in_features if in_features is not None else x_q.shape[1]
    ffn = w_gu.shape[0] // 2
    h = torch.empty((rows, ffn), dtype=torch.float32, device=x_q.device)
    row_max = torch.empty(rows, dtype=torch.float32, device=x_q.device)
    _lib.call("reef_b200_linear_w8a8_swiglu", rows, k, ffn, _ptr(x_q), _ptr(x_scale), _ptr(w_gu),
              _ptr(w_scale), _ptr(h), _ptr(row_max), _stream())
    return h, row_max


def linear_int8(x: torch.Tensor, w: torch.Tensor, shift: int,
                bias: torch.Tensor | None = None, in_features: int | None = None):
    """reef_kernels::linear_int8 / linear_bias_int8 (kernels.hpp:101-108).
    x is [rows][kpad(in)] (see :func:`pad_rows_i8`)."""
    rows = x.shape[0]
    k = in_features if in_features is not None else x.shape[1]
    n = w.shape[0]
    y = torch.empty((rows, n), dtype=torch.int8, device=x.device)
    if bias is None:
        _lib.call("reef_b200_linear_int8", rows, k, n, _ptr(x), _ptr(w), shift, _ptr(y),
                  _stream())
    else:
        _lib.call("reef_b200_linear_bias_int8", rows, k, n, _ptr(x), _ptr(w), _ptr(bias),
                  shift, _ptr(y), _stream())
    return y


def gemm_i8_i32(a: torch.Tensor, b: torch.Tensor, k: int | None = None) -> torch.Tensor:
    """matmul<int8,int32>(a, b^T); a [m][kpad], b [n][kpad]."""
    m = a.shape[0]
    n = b.shape[0]
    k = k if k is not None else a.shape[1]
    c = torch.empty((m, n), dtype=torch.int32, device=a.device)
    _lib.call("reef_b200_gemm_i8_i32", m, n, k, _ptr(a), _ptr(b), _ptr(c), _stream())
    return c


# ---- integer softmax and attention heads ---------------------------------------

def exp_table_device(table) -> torch.Tensor:
    """A 256-entry exp_table (int8.hpp:156-164, uint16 values) on the device.
    The bits are held in an int16 tensor; the kernels read them as uint16."""
    import numpy as np
    bits16 = np.ascontiguousarray(np.asarray(table, dtype=np.uint16)).view(np.int16)
    return torch.from_numpy(bits16.copy()).cuda()


def softmax_int8(scores: torch.Tensor, shift: int, table: torch.Tensor) -> torch.Tensor:
    """reef_kernels::softmax_int8 (kernels.hpp:114-117), every row of scores."""
    rows, n = scores.shape
    probs = torch.empty((rows, n), dtype=torch.uint8, device=scores.device)
    _lib.call("reef_b200_softmax_int8", rows, n, _ptr(scores), shift, _ptr(table),
              _ptr(probs), _stream())
    return probs


def attention_head_int8(q, k, v, query_start: int, window: int, score_shift: int,
                        table: torch.Tensor, out_shift: int = 8) -> torch.Tensor:
    """reef_kernels::attention_head_int8 (kernels.hpp:122-129), one head."""
    ql, d = q.shape
    kl = k.shape[0]
    out = torch.empty((ql, d), dtype=torch.int8, device=q.device)
    _lib.call("reef_b200_attention_head_int8", ql, kl, d, query_start, window, _ptr(q), d,
              _ptr(k), _ptr(v), score_shift, _ptr(table), out_shift, None, None, _ptr(out),
              d, _stream())
    return out


def attention_head_f32(q, k, v, query_start: int, window: int) -> torch.Tensor:
    """reef_kernels::attention_head_f32 (kernels.hpp:75-79), one head."""
    ql, d = q.shape
    kl = k.shape[0]
    out = torch.empty((ql, d), dtype=torch.float32, device=q.device)
    _lib.call("reef_b200_attention_head_f32", ql, kl, d, query_start, window, _ptr(q), d,
              _ptr(k), _ptr(v), None, _ptr(out), d, _stream())
    return out


def attention_heads_f32(q, k, v, heads: int, query_start: int = 0, window: int = 0):
    """Attention::context over all heads of [len][d_model] q/k/v."""
    ql, dm = q.shape
    kl = k.shape[0]
    hd = dm // heads
    out = torch.empty((ql, dm), dtype=torch.float32, device=q.device)
    _lib.call("reef_b200_attention_heads_f32", heads, ql, kl, hd, query_start, window,
              _ptr(q), dm, hd, _ptr(k), _ptr(v), dm, hd, _ptr(out), dm, hd, _stream())
    return out


def gemm_w8a8_skinny(x_q, x_scale, w, w_scale, bias=None, in_features: int | None = None):
    """The W8A8 GEMM for rows <= 128 (decode), swap-AB + split-K."""
    rows = x_q.shape[0]
    k = in_features if in_features is not None else x_q.shape[1]
    n = w.shape[0]
    nbytes = _lib.lib().reef_b200_gemm_skinny_workspace_bytes(rows, k, n)
    ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=x_q.device)
    y = torch.empty((rows, n), dtype=torch.float32, device=x_q.device)
    _lib.call("reef_b200_gemm_w8a8_skinny", rows, k, n, _ptr(x_q), _ptr(x_scale), _ptr(w),
              _ptr(w_scale), _ptr(bias), _ptr(ws), ws.numel(), _ptr(y), _stream())
    return y
