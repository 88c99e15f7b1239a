"""Single-kernel cases for profiler captures (ncu) of the hot kernels.

    python -m reef_b200.profile_cases gemm  [--m 16384 --n 12288 --k 4096]
    python -m reef_b200.profile_cases flash [--batch 8 --seq 2048 --heads 32]
    python -m reef_b200.profile_cases qkv   [--batch 8 --seq 2048 --heads 32]
    python -m reef_b200.profile_cases decode [--batch 64 --heads 8 --kv-heads 1 --seq 4096]

Each case allocates its seeded inputs once, launches the kernel twice (a
warm-up launch, then the one to capture: ``ncu -k regex:<name> -s 1 -c 1``)
and synchronises.  The default GEMM is the config-3 QKV projection
(A 64 MiB + B 48 MiB of int8 and an 768 MiB fp32 output: larger than L2,
about 1 GiB on the device); the default flash case is config 3's attention.
"""
from __future__ import annotations

import argparse
import math

import torch

from . import _lib
from . import kernels as K


def gemm(m: int, n: int, k: int) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    a = torch.randint(-127, 128, (m, k), generator=g, device="cuda", dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
    xs = torch.rand(m, generator=g, device="cuda") * 1e-3
    ws = torch.rand(n, generator=g, device="cuda") * 1e-3
    for _ in range(2):
        K.gemm_w8a8(a, xs, b, ws)
    torch.cuda.synchronize()


def flash(batch: int, seq: int, heads: int, kv_heads: int) -> None:
    g = torch.Generator(device="cuda").manual_seed(0)
    T = batch * seq
    q8 = torch.randint(-127, 128, (T, heads * 128), generator=g, device="cuda", dtype=torch.int8)
    k8 = torch.randint(-127, 128, (T, kv_heads * 128), generator=g, device="cuda", dtype=torch.int8)
    vt = (torch.randint(-127, 128, (batch, kv_heads, 128, seq), generator=g,
                        device="cuda") * 0.01).to(torch.float16)
    qs = torch.full((batch, heads, seq), 0.01, device="cuda")
    ks = torch.full((batch, kv_heads, seq), 0.01, device="cuda")
    out = torch.empty((T, heads * 128), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        _lib.call("reef_b200_flash_attn_i8", batch, seq, heads, kv_heads, 128, 1,
                  1.0 / math.sqrt(128), q8.data_ptr(), qs.data_ptr(), k8.data_ptr(),
                  ks.data_ptr(), vt.data_ptr(), out.data_ptr(), st)
    torch.cuda.synchronize()


def qkv(batch: int, seq: int, heads: int, kv_heads: int, hidden: int = 4096) -> None:
    """The QKV projection with RoPE + int8 q / k / V^T packing in its epilogue."""
    g = torch.Generator(device="cuda").manual_seed(0)
    T, W = batch * seq, (heads + 2 * kv_heads) * 128
    xq = torch.randint(-127, 128, (T, hidden), generator=g, device="cuda", dtype=torch.int8)
    w = torch.randint(-127, 128, (W, hidden), generator=g, device="cuda", dtype=torch.int8)
    xs = torch.rand(T, generator=g, device="cuda") * 1e-3
    ws = torch.rand(W, generator=g, device="cuda") * 1e-3
    q8 = torch.empty((T, heads * 128), dtype=torch.int8, device="cuda")
    k8 = torch.empty((T, kv_heads * 128), dtype=torch.int8, device="cuda")
    qs = torch.empty((batch, heads, seq), device="cuda")
    ks = torch.empty((batch, kv_heads, seq), device="cuda")
    vt = torch.empty((batch, kv_heads, 128, seq), dtype=torch.float16, device="cuda")
    rope = torch.empty((seq, 64, 2), device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        _lib.call("reef_b200_linear_w8a8_qkv_rope", batch, seq, hidden, heads, kv_heads, 10000.0,
                  xq.data_ptr(), xs.data_ptr(), w.data_ptr(), ws.data_ptr(), q8.data_ptr(),
                  k8.data_ptr(), None, qs.data_ptr(), ks.data_ptr(), None, vt.data_ptr(),
                  rope.data_ptr(), st)
    torch.cuda.synchronize()


def decode(batch: int, heads: int, kv_heads: int, cache_len: int) -> None:
    """Decode attention over a full int8 KV cache (config 4's TP=8 shard by default)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    q8 = torch.randint(-127, 128, (batch, heads, 128), generator=g, device="cuda", dtype=torch.int8)
    qs = torch.rand((batch, heads), generator=g, device="cuda") * 0.02
    shp = (batch, kv_heads, cache_len)
    k8 = torch.randint(-127, 128, shp + (128,), generator=g, device="cuda", dtype=torch.int8)
    v8 = torch.randint(-127, 128, shp + (128,), generator=g, device="cuda", dtype=torch.int8)
    ks = torch.rand(shp, generator=g, device="cuda") * 0.02
    vs = torch.rand(shp, generator=g, device="cuda") * 0.02
    out = torch.empty((batch, heads, 128), device="cuda")
    n = _lib.lib().reef_b200_decode_attn_workspace_bytes(batch, heads, cache_len)
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        _lib.call("reef_b200_decode_attn_i8", batch, heads, kv_heads, 128, cache_len, None,
                  cache_len, 1.0 / math.sqrt(128), q8.data_ptr(), qs.data_ptr(), k8.data_ptr(),
                  ks.data_ptr(), v8.data_ptr(), vs.data_ptr(), ws.data_ptr(), n, out.data_ptr(),
                  st)
    torch.cuda.synchronize()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "flash", "qkv", "decode"])
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=12288)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=32)
    a = ap.parse_args()
    if a.case == "gemm":
        gemm(a.m, a.n, a.k)
    elif a.case == "qkv":
        qkv(a.batch, a.seq, a.heads, a.kv_heads)
    elif a.case == "decode":
        decode(a.batch, a.heads, a.kv_heads, a.seq)
    else:
        flash(a.batch, a.seq, a.heads, a.kv_heads)
    K.check_device_error()
    print("ok")


if __name__ == "__main__":
    main()
