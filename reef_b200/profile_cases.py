"""Single-kernel cases for profiler captures (ncu) of the hot kernels.

    python -m reef_b200.profile_cases gemm  [--m 16384 --n 12288 --k 4096]
    python -m reef_b200.profile_cases flash [--batch 8 --seq 2048 --heads 32]

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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "flash"])
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
    else:
        flash(a.batch, a.seq, a.heads, a.kv_heads)
    K.check_device_error()
    print("ok")


if __name__ == "__main__":
    main()
