"""Cases for profiler captures (ncu) of the hot kernels, and the config-5
GEMM sweep.  The recipe behind the summaries in profiles/.

    python profile_cases.py gemm  [--m 16384 --n 12288 --k 4096]
    python profile_cases.py flash [--batch 8 --seq 2048 --heads 32]
    python profile_cases.py qkv   [--batch 8 --seq 2048 --heads 32]
    python profile_cases.py decode [--batch 64 --heads 8 --kv-heads 1 --seq 4096]
    python profile_cases.py decode_step [--steps 3]
    python profile_cases.py layer [--batch 8 --steps 2]
    python profile_cases.py layer_timing [--batch 8 --steps 10]
    python profile_cases.py sweep [--out sweep.json] [--tp 1]
    torchrun --nproc-per-node N profile_cases.py tp [--chunks 1,2,4 --steps 20]
    python profile_cases.py stream [--sizes 35,69,138,276]

Each single-kernel case allocates its seeded inputs once, launches the kernel
twice (a warm-up launch, then the one to capture: ``ncu -k regex:<name> -s 1
-c 1``) and synchronises.  ``decode_step`` runs config 4's whole decode step
(the TP=8 shard of rank 0: 64 sequences at position 4095 of a 4096-row int8
cache) `--steps` times, and ``layer`` config 3's prefill layer at TP=1
(`--batch` sequences of 2048), each launch by launch, for the launch list.  The default GEMM is the config-3 QKV projection
(A 64 MiB + B 48 MiB of int8 and an 768 MiB fp32 output: larger than L2,
about 1 GiB on the device); the default flash case is config 3's attention.

``sweep`` is not a capture case: it times the W8A8 GEMM at every point of the
config-5 sweep (M in {1, 16, 128, 1024, 8192, 16384} x five (N, K) shapes)
through the C ABI -- ``reef_b200_gemm_w8a8`` for M > 128, the swap-AB split-K
``reef_b200_gemm_w8a8_skinny`` for M <= 128 -- replayed from a CUDA graph and
timed with CUDA events, and prints
one JSON line per point with its roofline fraction (tensor-bound against twice
the measured burst bf16 rate for M >= 1024, HBM-bound against the measured
copy bandwidth below).  Operands rotate through enough copies that every call
reads them from DRAM, not L2.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from reef_b200 import _lib
from reef_b200 import kernels as K


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


def decode_step(steps: int) -> None:
    """Config 4's decode layer, the TP=8 shard of rank 0 (no collectives)."""
    from reef_b200.layer import LLAMA_70B, LlamaLayer
    B, Lmax = 64, 4096
    L = LlamaLayer(LLAMA_70B, B, 8, seed=11, world=8, rank=0)
    cache = L.alloc_cache(Lmax)
    g = torch.Generator(device="cuda").manual_seed(7)
    cache["k"].random_(-127, 128, generator=g)
    cache["v"].random_(-127, 128, generator=g)
    cache["ks"].uniform_(0.005, 0.015, generator=g)
    cache["vs"].uniform_(0.005, 0.015, generator=g)
    x = torch.randn((B, LLAMA_70B.hidden), generator=g, device="cuda")
    y = torch.empty_like(x)
    pos = torch.full((B,), Lmax - 1, dtype=torch.int32, device="cuda")
    for _ in range(steps):
        L.decode(x, pos, cache, out=y)
    torch.cuda.synchronize()


def layer_timing(batch: int, steps: int) -> None:
    """Config 3's prefill layer at TP=1: the plain forward timed over `steps`
    calls (CUDA events around the whole run), then the instrumented forward
    (reef_b200_llama_layer_forward_events: an event pair around the QKV GEMM,
    flash, o-proj, gate/up and down) with its spans, the time between them and
    its total.  One JSON line."""
    import ctypes as C

    from reef_b200.layer import LLAMA_7B, LlamaLayer
    L = LlamaLayer(LLAMA_7B, batch, 2048, seed=1)
    g = torch.Generator(device="cuda").manual_seed(1234)
    x = torch.randn((batch * 2048, LLAMA_7B.hidden), generator=g, device="cuda")
    y = torch.empty_like(x)
    for _ in range(3):
        L.forward(x, y)
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        L.forward(x, y)
    e1.record()
    torch.cuda.synchronize()
    plain = e0.elapsed_time(e1) / steps
    st = torch.cuda.current_stream().cuda_stream
    rows = []
    for _ in range(steps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(10)]
        for e in ev:  # torch makes the CUDA event at its first record
            e.record()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record()
        handles = (C.c_void_p * 10)(*[e.cuda_event for e in ev])
        _lib.call("reef_b200_llama_layer_forward_events", C.byref(L.desc), x.data_ptr(),
                  y.data_ptr(), L.workspace.data_ptr(), L.workspace.numel(), handles, st)
        end.record()
        torch.cuda.synchronize()
        spans = [ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(5)]
        gaps = [ev[2 * i + 1].elapsed_time(ev[2 * i + 2]) for i in range(4)]
        rows.append((start.elapsed_time(end), start.elapsed_time(ev[0]), spans, gaps,
                     ev[9].elapsed_time(end)))
    K.check_device_error()
    n = len(rows)
    avg = lambda f: sum(f(r) for r in rows) / n
    names = ["qkv", "flash", "o_proj", "gate_up", "down"]
    print(json.dumps({
        "plain_ms": plain,
        "instrumented_total_ms": avg(lambda r: r[0]),
        "before_qkv_ms": avg(lambda r: r[1]),
        "spans_ms": {nm: avg(lambda r, i=i: r[2][i]) for i, nm in enumerate(names)},
        "between_ms": {f"{names[i]}->{names[i + 1]}": avg(lambda r, i=i: r[3][i])
                       for i in range(4)},
        "after_down_ms": avg(lambda r: r[4]),
    }), flush=True)


def layer(batch: int, steps: int) -> None:
    """Config 3's prefill layer at TP=1: `batch` sequences of 2048 tokens."""
    from reef_b200.layer import LLAMA_7B, LlamaLayer
    L = LlamaLayer(LLAMA_7B, batch, 2048, seed=1)
    g = torch.Generator(device="cuda").manual_seed(1234)
    x = torch.randn((batch * 2048, LLAMA_7B.hidden), generator=g, device="cuda")
    y = torch.empty_like(x)
    for _ in range(steps):
        L.forward(x, y)
    torch.cuda.synchronize()


def tp_forward(chunk_list, steps: int = 20) -> None:
    """Config 3's layer under tensor parallelism, one rank per GPU (launched
    by torchrun): the pipelined all-gather plan at each chunk count in
    `chunk_list` and the all-reduce plan, timed over `steps` forwards with
    CUDA events (max over ranks), beside the host's time to issue one
    forward.  Rank 0 prints one JSON line."""
    import datetime
    import time

    import torch.distributed as dist

    from reef_b200 import tp
    from reef_b200.layer import LLAMA_7B, TP_ALLGATHER, TP_ALLREDUCE, LlamaLayer
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    comm = tp.Comm(rank, world, timeout_s=60.0)
    s, B, S = LLAMA_7B, 8, 2048
    res = {"world": world}
    for name, mode in (("allgather", TP_ALLGATHER), ("allreduce", TP_ALLREDUCE)):
        L = LlamaLayer(s, B, S, seed=1, world=world, rank=rank, comm=comm, device=dev,
                       tp_mode=mode)
        g = torch.Generator(device=dev).manual_seed(1234)
        x = torch.randn((B * S, s.hidden), generator=g, device=dev)
        if mode == TP_ALLGATHER:
            x = x[:, tp.col_slice(s.hidden, world, rank)].contiguous()
        y = torch.empty_like(x)
        for chunks in (chunk_list if mode == TP_ALLGATHER else (1,)):
            os.environ["REEF_B200_TP_CHUNKS"] = str(chunks)
            for _ in range(5):
                L.forward(x, y)
            torch.cuda.synchronize(dev)
            dist.barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            h0 = time.perf_counter()
            for _ in range(steps):
                L.forward(x, y)
            h1 = time.perf_counter()
            e1.record()
            torch.cuda.synchronize(dev)
            K.check_device_error()
            t = torch.tensor([e0.elapsed_time(e1) / steps, (h1 - h0) * 1e3 / steps], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            res[f"{name}_chunks{chunks}"] = {"gpu_ms": t[0].item(), "host_issue_ms": t[1].item()}
            dist.barrier()
        del L
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()
    if rank == 0:
        print(json.dumps(res), flush=True)
    comm.close()
    dist.barrier()
    dist.destroy_process_group()


def stream(sizes_mb, reps: int = 20) -> None:
    """The practical ceiling for a read of a given working set: torch's
    float32 sum over the bytes (one read, a few bytes written), a CUDA graph
    of calls over enough rotating copies that every call reads DRAM, timed
    with CUDA events.  One JSON line per size."""
    peaks = _peaks()
    for mb in sizes_mb:
        n = int(mb * 1e6) // 4
        copies = max(2, -(-2 * L2_BYTES // (4 * n)))
        bufs = [torch.rand((n,), device="cuda") for _ in range(copies)]
        out = torch.empty((1,), device="cuda")
        calls = copies * 3
        for b in bufs:
            torch.sum(b, 0, keepdim=True, out=out)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        with torch.cuda.stream(cap), torch.cuda.graph(graph, stream=cap):
            for i in range(calls):
                torch.sum(bufs[i % copies], 0, keepdim=True, out=out)
        graph.replay()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            graph.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * calls)
        gbs = 4 * n / (us * 1e-6) / 1e9
        print(json.dumps({"mb": 4 * n / 1e6, "us": us, "gbs": gbs,
                          "frac": gbs / peaks["hbm_gbs"], "peak_source": peaks["source"],
                          "copies": copies}), flush=True)
        del bufs, graph
        torch.cuda.empty_cache()


SWEEP_M = (1, 16, 128, 1024, 8192, 16384)
SWEEP_NK = ((4096, 4096), (11008, 4096), (4096, 11008), (28672, 8192), (8192, 28672))
L2_BYTES = 126 << 20


def _peaks() -> dict:
    root = os.path.dirname(os.path.abspath(__file__))
    try:
        with open(os.path.join(root, "MEASURED_PEAKS.json")) as fh:
            m = json.load(fh)
        return {"int8_tops": 2.0 * m["bf16_tflops"], "hbm_gbs": m["hbm_gbs"], "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"int8_tops": 2.0 * 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


def _shard_points(tps):
    """(split, tp, n, k) per config-5 point: the unsplit GEMM at tp 1, and at
    tp > 1 one GPU's share of a column split (N / tp, K) and of a row split
    (N, K / tp; its int32 partial sums still need the all-reduce, not timed
    here)."""
    for (n, k) in SWEEP_NK:
        for tp in tps:
            if tp == 1:
                yield "none", 1, n, k
            else:
                yield "column", tp, n // tp, k
                yield "row", tp, n, k // tp


def sweep(out: str | None, tps=(1,), iters: int = 20, reps: int = 3) -> None:
    peaks = _peaks()
    lib = _lib.lib()
    rows = []
    for (split, tp, n, k) in _shard_points(tps):
        kp = K.kpad(k)
        for m in SWEEP_M:
            g = torch.Generator(device="cuda").manual_seed(m + n + k)
            per_copy = (m + n) * kp
            copies = max(1, min(16, -(-2 * L2_BYTES // per_copy)))
            a = [torch.randint(-127, 128, (m, kp), generator=g, device="cuda", dtype=torch.int8)
                 for _ in range(copies)]
            b = [torch.randint(-127, 128, (n, kp), generator=g, device="cuda", dtype=torch.int8)
                 for _ in range(copies)]
            xs = torch.rand(m, generator=g, device="cuda") * 1e-3 + 1e-3
            ws = torch.rand(n, generator=g, device="cuda") * 1e-3 + 1e-3
            y = torch.empty((m, n), device="cuda")
            skinny = m <= 128
            wsb = lib.reef_b200_gemm_skinny_workspace_bytes(m, k, n) if skinny else 0
            work = torch.empty(max(wsb, 16), dtype=torch.uint8, device="cuda")

            def call(i: int) -> None:
                c = i % copies
                st = torch.cuda.current_stream().cuda_stream
                if skinny:
                    _lib.call("reef_b200_gemm_w8a8_skinny", m, k, n, a[c].data_ptr(), xs.data_ptr(),
                              b[c].data_ptr(), ws.data_ptr(), None, work.data_ptr(), work.numel(),
                              y.data_ptr(), st)
                else:
                    _lib.call("reef_b200_gemm_w8a8", m, k, n, a[c].data_ptr(), xs.data_ptr(),
                              b[c].data_ptr(), ws.data_ptr(), None, y.data_ptr(), st)

            for i in range(3):
                call(i)
            torch.cuda.synchronize()
            # the timed calls replay from a CUDA graph, so the host's cost per
            # call (ctypes, tensor-map encoding) is off the clock, as in a
            # captured decode step
            graph = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream()
            with torch.cuda.stream(cap), torch.cuda.graph(graph, stream=cap):
                for i in range(iters):
                    call(i)
            graph.replay()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / (reps * iters)
            ops = 2.0 * m * n * k
            moved = m * k + n * k + 4.0 * m * n  # int8 A and B, fp32 y
            tops = ops / (ms * 1e-3) / 1e12
            gbs = moved / (ms * 1e-3) / 1e9
            tensor = m >= 1024
            r = {"m": m, "n": n, "k": k, "tp": tp, "split": split,
                 "path": "skinny split-K" if skinny else "tcgen05 persistent",
                 "ms": ms, "tops": tops, "gbs": gbs, "bound": "tensor" if tensor else "hbm",
                 "frac": tops / peaks["int8_tops"] if tensor else gbs / peaks["hbm_gbs"],
                 "peak_source": peaks["source"], "operand_copies": copies}
            rows.append(r)
            print(json.dumps(r), flush=True)
            del a, b, y, work, graph
            torch.cuda.empty_cache()
    if out:
        with open(out, "w") as fh:
            json.dump(rows, fh, indent=1)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["gemm", "flash", "qkv", "decode", "decode_step", "layer",
                                     "layer_timing", "sweep", "tp", "stream"])
    ap.add_argument("--sizes", default="35,69,138,276", help="stream: working sets in MB")
    ap.add_argument("--chunks", default="1,2,4", help="tp: chunk counts of the all-gather plan")
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=12288)
    ap.add_argument("--k", type=int, default=4096)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--heads", type=int, default=32)
    ap.add_argument("--kv-heads", type=int, default=32)
    ap.add_argument("--out", default=None)
    ap.add_argument("--tp", default="1", help="comma-separated TP degrees for the sweep")
    a = ap.parse_args()
    if a.case == "stream":
        stream([float(v) for v in a.sizes.split(",")])
        return
    if a.case == "tp":
        tp_forward(tuple(int(c) for c in a.chunks.split(",")), max(a.steps, 5))
        return
    if a.case == "sweep":
        sweep(a.out, tuple(int(t) for t in a.tp.split(",")))
    elif a.case == "gemm":
        gemm(a.m, a.n, a.k)
    elif a.case == "qkv":
        qkv(a.batch, a.seq, a.heads, a.kv_heads)
    elif a.case == "decode":
        decode(a.batch, a.heads, a.kv_heads, a.seq)
    elif a.case == "decode_step":
        decode_step(a.steps)
    elif a.case == "layer":
        layer(a.batch, a.steps)
    elif a.case == "layer_timing":
        layer_timing(a.batch, max(a.steps, 5))
    else:
        flash(a.batch, a.seq, a.heads, a.kv_heads)
    K.check_device_error()
    print("ok")


if __name__ == "__main__":
    main()
