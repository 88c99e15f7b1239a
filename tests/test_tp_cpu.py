"""Tensor-parallel host logic on CPU ranks (gloo, world sizes 2, 4 and 8).

The GPU path shards with reef_b200.tp and runs the row-parallel algebra in
layer.cpp over NCCL.  Here the same shard functions and the same algebra run
on two gloo ranks with the oracle as the compute:

* row-parallel W8A8 linear: all-reduce MAX of per-token row maxima, quantise
  the K-slice with the full-row scale, int32 partial GEMM, all-reduce SUM,
  dequant epilogue + bias once  ==  TP=1 linear_w8a8, bit for bit;
* column-parallel q/k/v and gate/up row selections == the TP=1 columns;
* reef's GPT-Neo W8A8 block at TP=2 (config 2) == Block<float> at TP=1,
  bit for bit;
* the all-gather plan's algebra: each rank's RMSNorm chunk sums and
  max|x * gain| over its hidden columns, all-gathered, give TP=1's r and
  scale (the fixed 8-chunk tree; max|y| = max|x * gain| * r), so its int8
  columns are TP=1's; a column-sharded activation (SwiGLU's h, the attention
  output) quantised with the MAX-all-reduced row maxima is TP=1's; and a
  column-parallel GEMM on the all-gathered int8 rows gives TP=1's columns;
* a rank that fails before a collective surfaces as an error on its peer
  within the process-group timeout (no hang).
"""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as ro
from reef_b200 import tp
from tests import rms_ref
from tests.test_oracle import block_float_weights


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world=2, timeout_s=60):
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q, timeout_s))
             for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=timeout_s + 60) for _ in procs]
    for p in procs:
        p.join(timeout=30)
    return dict(results)


def _entry(fn, rank, world, port, q, timeout_s):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world,
                                timeout=datetime.timedelta(seconds=timeout_s))
        out = fn(rank, world)
        q.put((rank, ("ok", out)))
    except Exception:
        q.put((rank, ("error", traceback.format_exc())))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def quantize_with_max(x, row_max):
    """quantize_rows (quant.hpp:112-133) with a given row maximum."""
    rm = np.asarray(row_max, np.float32)
    scale = np.where(rm > 0, rm / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(x / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale


def rowpar_linear(x_loc, w_loc, ws, bias):
    rm = torch.from_numpy(np.abs(x_loc).max(axis=1).astype(np.float32))
    dist.all_reduce(rm, op=dist.ReduceOp.MAX)
    q, s = quantize_with_max(x_loc, rm.numpy())
    acc = torch.from_numpy(ro.gemm_i8(q, w_loc, threads=1))
    dist.all_reduce(acc, op=dist.ReduceOp.SUM)
    return ro.w8a8_epilogue(acc.numpy(), s, ws, bias)


def _rowpar_case(rank, world):
    M, K, N = 33, 512, 96
    x = ro.normal(1, (M, K))
    x[4] = 0.0
    w, ws = ro.quantize_rows(ro.normal(2, (N, K), 0, 0.02))
    b = ro.normal(3, (N,), 0, 0.02)
    cols = tp.col_slice(K, world, rank)
    y = rowpar_linear(np.ascontiguousarray(x[:, cols]), np.ascontiguousarray(w[:, cols]), ws, b)
    want = ro.linear_w8a8(x, w, ws, b, threads=1)
    return bool(np.array_equal(y.view(np.uint32), want.view(np.uint32)))


def _colpar_case(rank, world):
    hq, hkv, hd, hidden, ffn = 8, 4, 16, 64, 96
    x = ro.normal(5, (7, hidden))
    wqkv, sqkv = ro.quantize_rows(ro.normal(6, ((hq + 2 * hkv) * hd, hidden), 0, 0.02))
    rows = tp.qkv_rows(hq, hkv, hd, world, rank)
    full = ro.linear_w8a8(x, wqkv, sqkv, threads=1)
    mine = ro.linear_w8a8(x, np.ascontiguousarray(wqkv[rows]), sqkv[rows], threads=1)
    ok = np.array_equal(mine.view(np.uint32), full[:, rows].view(np.uint32))
    wgu, sgu = ro.quantize_rows(ro.normal(7, (2 * ffn, hidden), 0, 0.02))
    rows = tp.gate_up_rows(ffn, world, rank)
    full = ro.linear_w8a8(x, wgu, sgu, threads=1)
    mine = ro.linear_w8a8(x, np.ascontiguousarray(wgu[rows]), sgu[rows], threads=1)
    return bool(ok and np.array_equal(mine.view(np.uint32), full[:, rows].view(np.uint32)))


def _gptneo_tp_case(rank, world):
    """Config 2: the 256-d, 4-head, FFN-1024 block, TP=world, against TP=1."""
    seq, d, heads, ffn = 32, 256, 4, 1024
    fw = block_float_weights(d, ffn, seed=80)
    p = ro.quantize_block(fw)
    x = ro.normal(81, (seq, d))
    hd = d // heads
    h0, h1 = tp.shard_range(heads, world, rank)
    cols = slice(h0 * hd, h1 * hd)
    f0, f1 = tp.shard_range(ffn, world, rank)
    lin = lambda a, w, s, b=None: ro.linear_w8a8(a, np.ascontiguousarray(w), s, b, threads=1)
    h = ro.layernorm(x, p["ln1_g"], p["ln1_b"])
    q = lin(h, p["wq"][cols], p["sq"][cols])
    k = lin(h, p["wk"][cols], p["sk"][cols])
    v = lin(h, p["wv"][cols], p["sv"][cols])
    ctx = np.empty_like(q)
    for i in range(h1 - h0):
        sl = slice(i * hd, (i + 1) * hd)
        ctx[:, sl] = ro.attention_head_f32(np.ascontiguousarray(q[:, sl]),
                                           np.ascontiguousarray(k[:, sl]),
                                           np.ascontiguousarray(v[:, sl]), 0, 0)
    o = rowpar_linear(ctx, np.ascontiguousarray(p["wo"][:, cols]), p["so"], p["bo"])
    a = x + o
    h2 = ro.layernorm(a, p["ln2_g"], p["ln2_b"])
    f = lin(h2, p["wfc"][f0:f1], p["sfc"][f0:f1], p["bfc"][f0:f1])
    g = ro.gelu(f)
    y = a + rowpar_linear(g, np.ascontiguousarray(p["wproj"][:, f0:f1]), p["sproj"], p["bproj"])
    want = ro.gptneo_block_w8a8(x, p, heads, threads=1)
    return bool(np.array_equal(y.astype(np.float32).view(np.uint32), want.view(np.uint32)))


def _allgather_plan_case(rank, world):
    """The all-gather plan (layer.cpp llama_forward_ag*, llama.cu rms_stats /
    rms_apply) restated with numpy on this rank's columns."""
    rng = np.random.default_rng(41)
    eps = 1e-5
    ok = True
    for rows, width in ((6, 1024), (3, 4096), (2, 8192)):
        x = rng.normal(0, 1, (rows, width)).astype(np.float32)
        x[1] = 0.0  # a zero row: scale 1
        gain = rng.normal(1, 0.1, width).astype(np.float32)
        cols = tp.col_slice(width, world, rank)
        st = torch.from_numpy(rms_ref.rms_stats_local(x[:, cols], gain[cols], width))
        parts = [torch.empty_like(st) for _ in range(world)]
        dist.all_gather(parts, st)
        q, scale = rms_ref.rms_apply_local(x[:, cols], gain[cols],
                                           np.stack([t.numpy() for t in parts]), width, eps)
        q1, s1 = rms_ref.rmsnorm_quant_ref(x, gain, eps)
        ok &= bool(np.array_equal(q, q1[:, cols]))
        ok &= bool(np.array_equal(scale.view(np.uint32), s1.view(np.uint32)))
        # the all-gathered int8 rows [rank][rows][width/N] reassemble TP=1's
        got = [torch.empty_like(torch.from_numpy(q)) for _ in range(world)]
        dist.all_gather(got, torch.from_numpy(np.ascontiguousarray(q)))
        ok &= bool(np.array_equal(np.concatenate([t.numpy() for t in got], axis=1), q1))
    # a column-sharded activation quantised with the all-reduced row maxima,
    # then a column-parallel GEMM (this rank's output rows) on the gathered int8
    rows, width, n = 9, 704 * 8, 64
    h = rng.normal(0, 3, (rows, width)).astype(np.float32)
    h[4] = 0.0
    cols = tp.col_slice(width, world, rank)
    rm = torch.from_numpy(np.abs(h[:, cols]).max(axis=1).astype(np.float32))
    dist.all_reduce(rm, op=dist.ReduceOp.MAX)
    q, s = quantize_with_max(h[:, cols], rm.numpy())
    qf, sf = ro.quantize_rows(h)
    ok &= bool(np.array_equal(q, qf[:, cols]))
    ok &= bool(np.array_equal(s.view(np.uint32), sf.view(np.uint32)))
    got = [torch.empty_like(torch.from_numpy(q)) for _ in range(world)]
    dist.all_gather(got, torch.from_numpy(np.ascontiguousarray(q)))
    qa = np.concatenate([t.numpy() for t in got], axis=1)
    w, ws = ro.quantize_rows(ro.normal(42, (n * world, width), 0, 0.02))
    out = slice(rank * n, (rank + 1) * n)
    mine = ro.w8a8_epilogue(ro.gemm_i8(qa, np.ascontiguousarray(w[out]), threads=1), s, ws[out])
    full = ro.linear_w8a8(h, w, ws, threads=1)
    ok &= bool(np.array_equal(mine.view(np.uint32), full[:, out].view(np.uint32)))
    return ok


def _dead_peer_case(rank, world):
    if rank == 1:
        raise RuntimeError("rank 1 fails before the collective")
    t = torch.ones(4)
    try:
        dist.all_reduce(t)
    except Exception as e:  # the peer is gone: an error, not a hang
        return f"surfaced: {type(e).__name__}"
    return "no error"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_rowpar_linear_bit_identical_to_tp1(world):
    r = _run(_rowpar_case, world=world)
    assert len(r) == world and all(v == ("ok", True) for v in r.values()), r


@pytest.mark.parametrize("world", [2, 4])
def test_colpar_rows_are_the_tp1_columns(world):
    r = _run(_colpar_case, world=world)
    assert len(r) == world and all(v == ("ok", True) for v in r.values()), r


@pytest.mark.parametrize("world", [2, 4])
def test_gptneo_block_tp_bit_identical_to_tp1(world):
    r = _run(_gptneo_tp_case, world=world)
    assert len(r) == world and all(v == ("ok", True) for v in r.values()), r


@pytest.mark.parametrize("world", [2, 4, 8])
def test_allgather_plan_algebra_bit_identical_to_tp1(world):
    r = _run(_allgather_plan_case, world=world)
    assert len(r) == world and all(v == ("ok", True) for v in r.values()), r


def test_dead_peer_surfaces_as_error():
    r = _run(_dead_peer_case, timeout_s=8)
    assert r[1][0] == "error"
    assert r[0][0] == "error" or (r[0][0] == "ok" and r[0][1].startswith("surfaced")), r


def test_shard_functions():
    assert tp.shard_range(32, 8, 3) == (12, 16)
    with pytest.raises(ValueError):
        tp.shard_range(30, 8, 0)
    assert tp.qkv_rows(2, 2, 2, 2, 1) == [2, 3, 6, 7, 10, 11]
    assert tp.gate_up_rows(4, 2, 1) == [2, 3, 6, 7]
