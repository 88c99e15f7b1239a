#!/usr/bin/env python3
"""Benchmark: int8 TP decoder-layer TOPS and tokens/s on B200.

Workload: one Llama-7B-shape W8A8 decoder layer, prefill
of batch 8 x seq 2048 = 16384 tokens (hidden 4096, 32 heads x 128, SwiGLU
FFN 11008), synthetic seeded inputs and random-init weights.  At N GPUs the
layer runs Megatron tensor-parallel over N ranks (one process per GPU, launched
by torchrun): total work is fixed, so scaling is "strong".

A step = one forward of the layer over all 16384 tokens.  `value` is the
whole-job throughput in TOPS (algorithmic int ops: 2 per MAC of the four
projections, plus the causal q.k and p.v of attention) over the device-timed
steps (CUDA events, max over ranks), inputs resident in HBM (x is 256 MiB,
the weights 200 MiB: both larger than L2, so no flush is needed between
steps).  `e2e` is the same metric through the C ABI with host buffers: each
step copies x from pinned host memory and y back inside the timed region;
as in a serving loop, one step's copies overlap its neighbours' forwards
(a copy-in stream, the compute stream and a copy-out stream, two device
buffers of each, ordered by events).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

At one GPU the line also carries `decode_attention`: config 4's int8 decode
attention timed on its own against the measured HBM bandwidth.

--impl reference times reef's own engine (inference-engine/reference/cpp,
compiled in place into oracle/_ref) on the host cores, on a bounded sample of
the same workload; rank 0 prints its line, other ranks exit without work.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import ctypes as C
import datetime as dt
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = "llama7b-w8a8-prefill-layer"
BATCH, SEQ = 8, 2048
METRIC = "int8 TP decoder-layer TOPS (Llama-7B-shape W8A8 prefill layer, 8 x 2048 tokens)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="reef_b200", choices=["reef_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--tp-mode", default="allgather", choices=["allgather", "allreduce"],
                    help="tensor-parallel plan at N > 1: all-gather int8 activations "
                         "(column-sharded residual) or Megatron int32 all-reduce")
    return ap.parse_args()


def shape():
    from reef_b200.layer import LLAMA_7B
    return LLAMA_7B


def layer_ops(s, tokens: int, seq: int) -> dict:
    per = s.ops_per_token(seq)
    return dict(gemm=per["gemm"] * tokens, attention=per["attention"] * tokens,
                total=(per["gemm"] + per["attention"]) * tokens)


# ---- reef's engine on the host cores (CPU baseline / reference arm) ---------------

class RefSample:
    """reef's own W8A8 linear (operator/linear.hpp:106-134) and float head
    (attention.hpp:117-123), compiled in place (oracle/_ref), on a bounded
    sample of the layer.  Each host thread pushes ROWS tokens per linear()
    call, as a prefill does, through a slice (fraction `frac`) of each
    projection's output rows; the engine's QuantizedWeight for each slice is
    built once, outside the timed calls (reef's linear still transposes W
    inside every call, as it does in its own prefill).  Attention: the same
    ROWS queries, ending at a position spread over the sequence, through
    `frac` of the 32 heads."""

    ROWS = 128

    def __init__(self, s, threads: int, frac: float):
        import numpy as np

        from oracle import oracle as ro
        self.ro, self.np, self.s, self.threads, self.frac = ro, np, s, threads, frac
        self.lib = ro.ref()
        rng = np.random.default_rng(5)
        h, d = s.hidden, s.head_dim
        dims = [((s.heads_q + 2 * s.heads_kv) * d, h), (h, s.heads_q * d), (2 * s.ffn, h),
                (h, s.ffn)]
        i8 = C.POINTER(C.c_int8)
        f = C.POINTER(C.c_float)
        self.handles, self.shapes = [], []
        for n, k in dims:
            ns = max(1, int(round(n * frac)))
            w = rng.integers(-127, 128, (ns, k), dtype=np.int8)
            ws = np.full(ns, 1e-3, np.float32)
            hnd = self.lib.ref_weight_new(ns, k, w.ctypes.data_as(i8), ws.ctypes.data_as(f))
            if not hnd:
                raise RuntimeError("reef engine could not build a weight")
            self.handles.append(hnd)
            self.shapes.append((ns, k))
        self.heads = max(1, int(round(s.heads_q * frac)))
        self.kv = rng.standard_normal((2, SEQ, d)).astype(np.float32)
        self.x = [[rng.standard_normal((self.ROWS, k)).astype(np.float32) for _, k in self.shapes]
                  for _ in range(threads)]
        self.q = [rng.standard_normal((self.ROWS, d)).astype(np.float32) for _ in range(threads)]

    def close(self):
        for hnd in self.handles:
            self.lib.ref_weight_free(hnd)
        self.handles = []

    def _rows(self, i: int) -> float:
        np, s, L, R = self.np, self.s, self.lib, self.ROWS
        f = C.POINTER(C.c_float)
        ops = 0.0
        for hnd, (n, k), x in zip(self.handles, self.shapes, self.x[i]):
            y = np.empty((R, n), np.float32)
            rc = L.ref_linear_w8a8_weight(hnd, R, k, x.ctypes.data_as(f), y.ctypes.data_as(f))
            if rc != 0:
                raise RuntimeError(f"reef linear failed ({rc})")
            ops += 2.0 * R * n * k
        # queries at positions last - R + 1 .. last, causal over keys 0..last
        last = R - 1 + (i * (SEQ - R)) // max(1, self.threads - 1)
        kk = np.ascontiguousarray(self.kv[0, :last + 1])
        vv = np.ascontiguousarray(self.kv[1, :last + 1])
        o = np.empty((R, s.head_dim), np.float32)
        for _ in range(self.heads):
            L.ref_attend_head_f32(R, last + 1, s.head_dim, last - R + 1, 0,
                                  self.q[i].ctypes.data_as(f), kk.ctypes.data_as(f),
                                  vv.ctypes.data_as(f), o.ctypes.data_as(f))
            ops += 2.0 * 2 * s.head_dim * sum(last - R + 2 + j for j in range(R))
        return ops

    def run(self):
        t0 = time.perf_counter()
        with cf.ThreadPoolExecutor(self.threads) as ex:
            ops = sum(ex.map(self._rows, range(self.threads)))
        return ops, time.perf_counter() - t0

    def describe(self) -> str:
        cols = ", ".join(f"{n}x{k}" for n, k in self.shapes)
        return (f"reef engine (oracle/_ref, -O2 -ffp-contract=off), {self.threads} threads: each "
                f"pushes {self.ROWS} tokens per linear() call through slices of the 4 W8A8 "
                f"projections ({self.frac:.3g} of their output rows: {cols}; QuantizedWeight "
                f"built once, reef transposes W inside each call) and {self.heads} head(s) of "
                f"causal float attention for the same {self.ROWS} queries at a position spread "
                f"over 0..{SEQ - 1}")


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def calibrated_sample(s, threads: int, seconds: float):
    """A RefSample whose run() takes about `seconds` on these host cores:
    one small run measures the engine's rate, the slice is then scaled."""
    probe = RefSample(s, threads, 0.002)
    probe.run()
    _, t = probe.run()
    probe.close()
    frac = min(1.0, max(0.002, 0.002 * seconds / max(t, 1e-3)))
    return RefSample(s, threads, frac)


def cpu_baseline(s, threads: int, seconds: float = 10.0) -> dict:
    from oracle import oracle as ro
    if not ro.ref_available():
        return {"value": None, "unit": "TOPS", "cores": threads, "kind": "reference",
                "sample": "unavailable: oracle/_ref was not built (needs the reference checkout)"}
    rs = calibrated_sample(s, threads, seconds)
    ops, sec = rs.run()
    out = {"value": ops / sec / 1e12, "unit": "TOPS", "cores": threads, "kind": "reference",
           "seconds": sec, "tokens_per_s": ops / sec / layer_ops(s, 1, SEQ)["total"],
           "sample": rs.describe()}
    rs.close()
    return out


def run_reference(args) -> int:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    s = shape()
    threads = host_threads()
    from oracle import oracle as ro
    if not ro.ref_available():
        emit({"impl": "reference",
              "unavailable": "oracle/_ref not built: reef's engine headers were absent when "
                             "build() ran"})
        return 0
    # each timed step a bounded sample, so the whole run stays within minutes
    rs = calibrated_sample(s, threads, min(10.0, 150.0 / max(args.steps, 1)))
    for _ in range(max(args.warmup, 0)):
        rs.run()
    total_ops, total_s = 0.0, 0.0
    for _ in range(args.steps):
        ops, sec = rs.run()
        total_ops += ops
        total_s += sec
    v = total_ops / total_s / 1e12
    out = {
        "metric": METRIC, "value": v, "unit": "TOPS", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_s / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch": BATCH, "seq_len": SEQ, "tokens": BATCH * SEQ,
                   "hidden": s.hidden, "heads": s.heads_q, "ffn": s.ffn},
        # whole-layer tokens/s implied by the sampled rate (the sample's ops
        # are a fraction of the layer's ops per token)
        "tokens_per_s": v * 1e12 / (layer_ops(s, 1, SEQ)["total"]),
        "cpu_baseline": {"value": v, "unit": "TOPS", "cores": threads, "kind": "reference",
                         "sample": "per step: " + rs.describe()},
        "e2e": {"value": v, "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    rs.close()
    emit(out)
    return 0


# ---- clocks during the timed region ----------------------------------------------

class Clocks:
    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.lines = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self, t0: float, t1: float) -> dict:
        rows = []
        for (t, line) in self.lines:
            p = [x.strip() for x in line.split(",")]
            if len(p) < 10:
                continue
            try:
                rows.append(dict(t=t, sm=float(p[2]), smax=float(p[3]), power=float(p[4]),
                                 hw=p[6], hwt=p[7], swt=p[8], pcap=p[9]))
            except ValueError:
                continue
        inside = [r for r in rows if t0 <= r["t"] <= t1 + 0.05] or rows[-3:]
        if not inside:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        reasons = set()
        for r in inside:
            if r["hw"].lower() == "active":
                reasons.add("hw_slowdown")
            if r["hwt"].lower() == "active":
                reasons.add("hw_thermal_slowdown")
            if r["swt"].lower() == "active":
                reasons.add("sw_thermal_slowdown")
            if r["pcap"].lower() == "active":
                reasons.add("sw_power_cap")
        return {"sm_mhz": statistics.median(r["sm"] for r in inside),
                "sm_max_mhz": max(r["smax"] for r in inside), "reasons": sorted(reasons),
                "samples": len(inside), "power_w_max": max(r["power"] for r in inside)}


def peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            m = json.load(fh)
        return {"bf16_sustained": m["bf16_tflops_sustained"], "bf16": m["bf16_tflops"],
                "hbm": m["hbm_gbs"], "source": "measured"}
    except Exception:
        return {"bf16_sustained": 1400.0, "bf16": 1590.0, "hbm": 6650.0, "source": "fallback"}


# ---- the product ---------------------------------------------------------------

def decode_attention(dev, pk: dict) -> dict:
    """Config 4's decode attention (the Llama-70B TP=8 shard: 64 sequences, 8
    query heads on 1 KV head, 4096 cached int8 keys each), timed on its own:
    a CUDA graph of 12 calls over 4 rotating cache copies (277 MB, past L2, so
    every call reads its 69 MB shard from DRAM), replayed 20 times."""
    import torch
    from reef_b200 import _lib
    B, HQ, HKV, L, copies, calls, reps = 64, 8, 1, 4096, 4, 12, 20
    g = torch.Generator(device=dev).manual_seed(4)
    q8 = torch.randint(-127, 128, (B, HQ, 128), generator=g, device=dev, dtype=torch.int8)
    qs = torch.rand((B, HQ), generator=g, device=dev) * 0.02
    shp = (B, HKV, L)
    caches = []
    for _ in range(copies):
        caches.append((torch.randint(-127, 128, shp + (128,), generator=g, device=dev,
                                     dtype=torch.int8),
                       torch.rand(shp, generator=g, device=dev) * 0.02,
                       torch.randint(-127, 128, shp + (128,), generator=g, device=dev,
                                     dtype=torch.int8),
                       torch.rand(shp, generator=g, device=dev) * 0.02))
    out = torch.empty((B, HQ, 128), device=dev)
    n = _lib.lib().reef_b200_decode_attn_workspace_bytes(B, HQ, L)
    ws = torch.empty(n, dtype=torch.uint8, device=dev)

    def call(c: int) -> None:
        k8, ks, v8, vs = caches[c % copies]
        _lib.call("reef_b200_decode_attn_i8", B, HQ, HKV, 128, L, None, L, 1.0 / math.sqrt(128),
                  q8.data_ptr(), qs.data_ptr(), k8.data_ptr(), ks.data_ptr(), v8.data_ptr(),
                  vs.data_ptr(), ws.data_ptr(), n, out.data_ptr(),
                  torch.cuda.current_stream(dev).cuda_stream)

    for c in range(copies):
        call(c)
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    cap = torch.cuda.Stream(dev)
    with torch.cuda.stream(cap), torch.cuda.graph(graph, stream=cap):
        for i in range(calls):
            call(i)
    graph.replay()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / (reps * calls)
    nbytes = 2 * B * HKV * L * (128 + 4)  # int8 K and V rows + one fp32 scale each
    gbs = nbytes / (us * 1e-6) / 1e9
    return {"kernel": "decode_mma + decode_combine (config 4, TP=8 shard)", "us": us,
            "bytes": nbytes, "achieved_gbs": gbs, "peak_gbs": pk["hbm"],
            "frac": gbs / pk["hbm"], "peak_source": pk["source"],
            "timing": f"CUDA graph of {calls} calls over {copies} rotating cache copies, "
                      f"{reps} replays"}


def decode_step(dev, pk: dict, world: int, rank: int, comm) -> dict:
    """Config 4's whole decode layer (Llama-70B shape, 64 sequences, one new
    token each at position 4095 of a 4096-row int8 KV cache): at one GPU the
    TP=8 shard of one rank (8 q / 1 kv heads, FFN 3584, no collectives); at N
    GPUs the TP=N layer with its row-parallel all-reduces.  Each of `copies`
    layer copies has its own weights and caches (together past L2, so every
    step streams its weights and cache from DRAM, as successive layers of a
    model do); a CUDA graph of `calls` steps over the copies is replayed
    `reps` times.  HBM roofline: the shard's int8 weights + fp32 scales and
    the int8 K / V rows + fp32 scales the attention reads, per step."""
    import torch
    import torch.distributed as dist

    from reef_b200 import kernels as K
    from reef_b200.layer import LLAMA_70B, LlamaLayer
    s = LLAMA_70B
    B, Lmax, copies, calls, reps = 64, 4096, 4, 8, 20
    tp = world if world > 1 else 8
    layers, caches = [], []
    g = torch.Generator(device=dev).manual_seed(7)
    err = None
    try:  # every allocation and weight before any step with a collective
        for c in range(copies):
            if world > 1:
                L = LlamaLayer(s, B, 8, seed=11 + c, world=world, rank=rank, comm=comm,
                               device=dev)
            else:
                L = LlamaLayer(s, B, 8, seed=11 + c, world=8, rank=0, device=dev)
            cache = L.alloc_cache(Lmax)
            cache["k"].random_(-127, 128, generator=g)
            cache["v"].random_(-127, 128, generator=g)
            cache["ks"].uniform_(0.005, 0.015, generator=g)
            cache["vs"].uniform_(0.005, 0.015, generator=g)
            L._decode_tiles()
            layers.append(L)
            caches.append(cache)
        x = torch.randn((B, s.hidden), generator=g, device=dev)
        y = torch.empty_like(x)
        pos = torch.full((B,), Lmax - 1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
    except Exception as e:  # noqa: BLE001
        err = e
    if world > 1:  # every rank set up, or none runs a step
        ok = torch.tensor([0 if err is not None else 1], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if int(ok.item()) == 0:
            raise RuntimeError(f"decode set-up failed on some rank: {err}")
    elif err is not None:
        raise err
    for c in range(copies):  # workspaces allocated, tensor maps warmed
        layers[c].decode(x, pos, caches[c], out=y)
    torch.cuda.synchronize(dev)
    K.check_device_error()
    # One GPU: the steps replay from a CUDA graph (the host's launch cost off
    # the clock, as a serving loop would run them).  N > 1: the steps are
    # launched one by one on the stream, the library's NCCL all-reduces
    # among them, so the host's issue time is on the clock.
    graph = None
    if world == 1:
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(dev)
        with torch.cuda.stream(cap), torch.cuda.graph(graph, stream=cap):
            for i in range(calls):
                layers[i % copies].decode(x, pos, caches[i % copies], out=y)

    def run_once():
        if graph is not None:
            graph.replay()
        else:
            for i in range(calls):
                layers[i % copies].decode(x, pos, caches[i % copies], out=y)

    for _ in range(2):
        run_once()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        run_once()
    e1.record()
    torch.cuda.synchronize(dev)
    K.check_device_error()
    us = e0.elapsed_time(e1) * 1e3 / (reps * calls)
    if world > 1:
        t = torch.tensor([us], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
    del graph
    torch.cuda.synchronize(dev)
    L = layers[0]
    w_bytes = sum(getattr(L, n).numel() for n in ("w_qkv", "w_o", "w_gu", "w_down")) + \
        4 * sum(getattr(L, n).numel() for n in ("s_qkv", "s_o", "s_gu", "s_down"))
    kv_bytes = 2 * B * (s.heads_kv // tp) * Lmax * (128 + 4)
    nbytes = w_bytes + kv_bytes
    gbs = nbytes / (us * 1e-6) / 1e9
    ops = 2.0 * B * (w_bytes - 4 * sum(getattr(L, n).numel()
                                       for n in ("s_qkv", "s_o", "s_gu", "s_down"))) + \
        2.0 * 2 * B * (s.heads_q // tp) * 128 * Lmax
    return {"workload": "llama70b-w8a8-decode-layer (config 4)",
            "parallelism": (f"tp{world}" if world > 1 else "tp8 shard of rank 0, no collectives"),
            "us": us, "tokens_per_s": B / (us * 1e-6), "tops_per_gpu": ops / (us * 1e-6) / 1e12,
            "bytes_per_gpu": nbytes, "achieved_gbs": gbs, "peak_gbs": pk["hbm"],
            "frac": gbs / pk["hbm"], "peak_source": pk["source"],
            "timing": (f"CUDA graph of {calls} steps over {copies} layer copies (weights and "
                       f"caches past L2), {reps} replays" if world == 1 else
                       f"{calls} steps over {copies} layer copies (weights and caches past L2) "
                       f"launched one by one, {reps} times, max over ranks")}


def run_reef(args) -> int:
    import torch
    import torch.distributed as dist

    from reef_b200 import _lib, tp
    from reef_b200 import kernels as K
    from reef_b200.layer import TP_ALLGATHER, TP_ALLREDUCE, LlamaLayer

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=dt.timedelta(seconds=180), device_id=dev)
    s = shape()
    T = BATCH * SEQ
    comm = tp.Comm(rank, world, timeout_s=120.0) if world > 1 else None
    mode = TP_ALLGATHER if args.tp_mode == "allgather" else TP_ALLREDUCE
    L = LlamaLayer(s, BATCH, SEQ, seed=1, world=world, rank=rank, comm=comm, device=dev,
                   tp_mode=mode)
    g = torch.Generator(device=dev).manual_seed(1234)
    x = torch.randn((T, s.hidden), generator=g, device=dev)
    if world > 1 and mode == TP_ALLGATHER:  # this rank's hidden columns
        x = x[:, tp.col_slice(s.hidden, world, rank)].contiguous()
    y = torch.empty_like(x)
    lib = _lib.lib()
    launches = lib.reef_b200_llama_layer_kernel_launches(C.byref(L.desc))
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier()

    w_evs = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    warm = max(args.warmup, 3)
    for i in range(warm):
        if i == warm - 1:
            w_evs[0].record(stream)
        L.forward(x, y)
    w_evs[1].record(stream)
    torch.cuda.synchronize(dev)
    K.check_device_error()
    step_s = w_evs[0].elapsed_time(w_evs[1]) * 1e-3
    n_pre = max(1, int(1.0 / max(step_s, 1e-4)))
    if world > 1:  # every rank runs the same number of forwards (collectives)
        t_pre = torch.tensor([n_pre], device=dev)
        dist.all_reduce(t_pre, op=dist.ReduceOp.MAX)
        n_pre = int(t_pre.item())

    # The instrumented forwards' events (below), made before the timed region
    # so that nothing idles the GPU between the two: torch makes a CUDA event
    # at its first record.
    n_inst = max(3, min(200, n_pre // 2))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(12)] for _ in range(n_inst)]
    for row in evs:
        for e in row:
            e.record(stream)
    handles = [(C.c_void_p * 10)(*[e.cuda_event for e in row[1:11]]) for row in evs]

    # The timed region: K forwards through the public entry point.  A second
    # of the same forward runs just before it, so that the clock samples
    # (one per 50 ms) cover sustained load even when the region is short.
    K_steps = args.steps
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    clocks = Clocks(local)
    clocks.start()
    time.sleep(0.6)  # the sampler is up before the load starts
    barrier()
    torch.cuda.synchronize(dev)
    w0 = time.time()
    for _ in range(n_pre):
        L.forward(x, y)
    t_start.record(stream)
    for k in range(K_steps):
        L.forward(x, y)
    t_end.record(stream)
    torch.cuda.synchronize(dev)
    w1 = time.time()
    K.check_device_error()
    ms = t_start.elapsed_time(t_end) / K_steps

    # Per-kernel spans (QKV, flash, o-proj, gate/up, down) from the
    # instrumented forward, which runs its steps in sequence.  They run right
    # after the timed region, with no idle time between (an idle GPU leaves
    # the power cap and boosts its clock), for about half a second, with the
    # clock still sampled, so the spans are taken under the same load as the
    # timed forwards.  n_pre is the same on every rank, so is n_inst.
    wi0 = time.time()
    for k in range(n_inst):
        evs[k][0].record(stream)
        _lib.call("reef_b200_llama_layer_forward_events", C.byref(L.desc), x.data_ptr(),
                  y.data_ptr(), L.workspace.data_ptr(), L.workspace.numel(), handles[k],
                  stream.cuda_stream)
        evs[k][11].record(stream)
    torch.cuda.synchronize(dev)
    wi1 = time.time()
    barrier()
    time.sleep(0.25)
    clocks.stop()
    K.check_device_error()
    spans = [[row[1 + 2 * i].elapsed_time(row[2 + 2 * i]) for i in range(5)] for row in evs]
    gemm_ms = statistics.mean(sum(r[i] for i in (0, 2, 3, 4)) for r in spans)
    flash_ms = statistics.mean(r[1] for r in spans)
    per_gemm = [statistics.mean(r[i] for r in spans) for i in (0, 2, 3, 4)]
    instrumented = None
    try:  # where the instrumented forward's time goes; never fails the line
        names = ["qkv", "flash", "o_proj", "gate_up", "down"]
        mean = lambda f: statistics.mean(f(row) for row in evs)
        instrumented = {
            "forwards": n_inst,
            "forward_ms": mean(lambda r: r[0].elapsed_time(r[11])),
            "spans_ms": {nm: statistics.mean(sp[i] for sp in spans)
                         for i, nm in enumerate(names)},
            "before_qkv_ms": mean(lambda r: r[0].elapsed_time(r[1])),
            "between_ms": {f"{names[i]}->{names[i + 1]}":
                           mean(lambda r, i=i: r[2 + 2 * i].elapsed_time(r[3 + 2 * i]))
                           for i in range(4)},
            "after_down_ms": mean(lambda r: r[10].elapsed_time(r[11])),
            "clocks": clocks.summary(wi0, wi1),
            "note": "same kernels as the timed forward, an event pair around each GEMM and "
                    "flash; run right after the timed region under the same load",
        }
    except Exception as e:  # noqa: BLE001
        instrumented = {"error": str(e)[:200]}

    # end to end through the C ABI with host buffers: step i copies x in on
    # s_in, runs the forward on `stream` and reads y back on s_out; buffers
    # alternate, so step i's copy-in overlaps step i - 1's forward and its
    # copy-out overlaps step i + 1's forward (events order each reuse)
    xh = x.cpu().pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    xd = [torch.empty_like(x) for _ in range(2)]
    yd = [torch.empty_like(y) for _ in range(2)]
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()
    in_done = [ev(), ev()]
    fwd_done = [ev(), ev()]
    out_done = [ev(), ev()]

    def e2e_step(i):
        b = i % 2
        if i >= 2:
            s_in.wait_event(fwd_done[b])  # step i - 2's forward has read xd[b]
        with torch.cuda.stream(s_in):
            xd[b].copy_(xh, non_blocking=True)
        in_done[b].record(s_in)
        stream.wait_event(in_done[b])
        if i >= 2:
            stream.wait_event(out_done[b])  # step i - 2's y has left yd[b]
        L.forward(xd[b], yd[b])
        fwd_done[b].record(stream)
        s_out.wait_event(fwd_done[b])
        with torch.cuda.stream(s_out):
            yh.copy_(yd[b], non_blocking=True)
        out_done[b].record(s_out)

    e_steps = max(3, min(K_steps, 20))
    for i in range(2):
        e2e_step(i)
    torch.cuda.synchronize(dev)
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    s_in.wait_event(e0)
    for i in range(e_steps):
        e2e_step(i)
    stream.wait_event(out_done[(e_steps - 1) % 2])
    stream.wait_event(out_done[e_steps % 2])
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / e_steps
    barrier()

    # Parity at N > 1, outside every timed region: this rank runs the same
    # layer at TP=1 on its own GPU (same seed, same input) and compares its
    # output shard with it bit for bit; the line reports the AND over ranks.
    tp_ok = None
    if world > 1:
        L.forward(x, y)
        L1 = LlamaLayer(s, BATCH, SEQ, seed=1, device=dev)
        g1 = torch.Generator(device=dev).manual_seed(1234)
        xf = torch.randn((T, s.hidden), generator=g1, device=dev)
        y1 = L1.forward(xf)
        if mode == TP_ALLGATHER:
            y1 = y1[:, tp.col_slice(s.hidden, world, rank)].contiguous()
        torch.cuda.synchronize(dev)
        K.check_device_error()
        same = torch.tensor([int(torch.equal(y.view(torch.int32), y1.view(torch.int32)))],
                            device=dev)
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        tp_ok = bool(same.item())
        del L1, xf, y1
        torch.cuda.empty_cache()

    # max over ranks
    t = torch.tensor([ms, e2e_ms, gemm_ms, flash_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, e2e_ms, gemm_ms_max, flash_ms_max = t.tolist()

    ops = layer_ops(s, T, SEQ)
    value = ops["total"] / (ms * 1e-3) / 1e12
    pk = peaks()
    int8_peak = 2.0 * pk["bf16_sustained"]
    rank_gemm_ops = ops["gemm"] / world
    achieved = rank_gemm_ops / (gemm_ms * 1e-3) / 1e12
    traffic = None
    tf = os.path.join(ROOT, "profiles", "gemm_i8_llama7b_traffic.json")
    if os.path.exists(tf):
        try:
            with open(tf) as fh:
                traffic = json.load(fh).get("dram_bytes_per_launch")
        except Exception:
            traffic = None
    out = {
        "metric": METRIC, "value": value, "unit": "TOPS", "n_gpus": world, "steps": K_steps,
        "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch": BATCH, "seq_len": SEQ, "tokens": T,
                   "hidden": s.hidden, "heads": s.heads_q, "kv_heads": s.heads_kv,
                   "ffn": s.ffn, "parallelism": f"tp{world}",
                   "tp_plan": (args.tp_mode if world > 1 else "none"),
                   "l2": "inputs larger than L2 (x 256 MiB, weights 200 MiB): no flush"},
        "tokens_per_s": T / (ms * 1e-3),
        "ops_per_step": ops["total"],
        "roofline": {"bound": "tensor", "kernel": "gemm_i8 (tcgen05 kind::i8)",
                     "achieved": achieved, "peak": int8_peak, "unit": "TOPS",
                     "frac": achieved / int8_peak, "traffic": traffic,
                     "peak_source": (f"2 x bf16_tflops_sustained of {pk['source']} "
                                     "(B200 dense int8 rate = 2 x dense bf16)"),
                     "per_launch_ms": per_gemm,
                     "launch_ops": [2.0 * T * s.hidden * (s.heads_q + 2 * s.heads_kv) * 128 / world,
                                    2.0 * T * s.heads_q * 128 * s.hidden / world,
                                    2.0 * T * s.hidden * 2 * s.ffn / world,
                                    2.0 * T * s.ffn * s.hidden / world]},
        "attention": {"kernel": "flash_prefill_i8", "ms": flash_ms,
                      "achieved_tops": ops["attention"] / world / (flash_ms * 1e-3) / 1e12},
        "e2e": {"value": ops["total"] / (e2e_ms * 1e-3) / 1e12, "unit": "TOPS",
                "h2d_bytes_per_step": x.numel() * 4, "d2h_bytes_per_step": y.numel() * 4,
                "ms_per_step": e2e_ms},
        "gpu_launches": int(launches) * K_steps,
        "tp_bit_identical": tp_ok,
        "instrumented_forward": instrumented,
        "exchange": exchange_bytes(s, T, world, args.tp_mode, ms),
        "clocks": dict(clocks.summary(w0, w1),
                       window="the timed region and the 1 s of the same forward just before it"),
    }
    if rank == 0 and world == 1:
        try:  # after the measured line's own work; never lets it fail
            out["decode_attention"] = decode_attention(dev, pk)
        except Exception as e:  # noqa: BLE001
            out["decode_attention"] = {"error": str(e)[:200]}
    try:  # after the measured line's own work; every rank takes part at N > 1
        dstep = decode_step(dev, pk, world, rank, comm)
    except Exception as e:  # noqa: BLE001
        dstep = {"error": str(e)[:200]}
    out["decode_step"] = dstep
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = cpu_baseline(s, host_threads())
    if rank == 0:  # the line first: teardown cannot take it away
        emit(out)
    if comm is not None:
        torch.cuda.synchronize(dev)
        try:
            comm.close()
        except Exception as e:  # noqa: BLE001
            print(f"rank {rank}: communicator teardown: {e}", file=sys.stderr, flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def exchange_bytes(s, tokens: int, world: int, plan: str, ms: float) -> dict | None:
    """Bytes that cross NVLink into each rank per layer forward, and how long
    they take at the pool's measured 770 GB/s per direction (a lower bound
    on the exchange, set beside the step time).  All-gather plan: the int8
    activations of the four projections (3 x hidden + ffn bytes per token)
    from the N - 1 peers, plus the RMSNorm chunk sums and the row maxima.
    All-reduce plan: two int32 all-reduces of [tokens][hidden] (a ring moves
    2 (N - 1) / N of it in) and two fp32 MAX all-reduces of [tokens]."""
    if world <= 1:
        return None
    f = (world - 1) / world
    if plan == "allgather":
        s_words = 8 // world + 1
        b = f * tokens * (3 * s.hidden + s.ffn) + (world - 1) * tokens * (2 * 4 * s_words + 2 * 4)
    else:
        b = 2 * f * 2 * tokens * s.hidden * 4 + 2 * 2 * f * tokens * 4
    link_ms = b / 770e9 * 1e3
    return {"plan": plan, "bytes_in_per_rank": b, "link_ms_at_770_gbs": link_ms,
            "link_share_of_step": link_ms / ms}


_JSON_OUT = None


def emit(obj: dict) -> None:
    """Print the one JSON line on the real stdout."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(obj) + "\n")
    out.flush()


def main() -> int:
    global _JSON_OUT
    args = parse()
    # Libraries (NCCL, the CUDA runtime) may print to fd 1; keep stdout for the
    # one JSON line and send everything else to stderr.
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if args.impl == "reference":
        return run_reference(args)
    return run_reef(args)


if __name__ == "__main__":
    sys.exit(main())
