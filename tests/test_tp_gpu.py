"""Tensor parallelism on two, four and eight B200s (NCCL and NVLink peer
stores): every rank's output is bit-identical to TP=1.

* reef_b200_linear_w8a8_rowpar (all-reduce MAX of row maxima, int32 partial
  GEMM, all-reduce SUM, dequant + bias) == reef_b200_linear_w8a8_bias;
* the Llama-shape layer at TP=N == the same layer at TP=1 (same seed), with
  the all-reduce plan and with the pipelined all-gather plan, on a small
  shape and at config 3's widths (hidden 4096, 32 x 128 heads, FFN 11008;
  batch 2 x 2048, so the all-gather plan pipelines two chunks);
* reef's GPT-Neo block at TP=N (config 2's shape) == the oracle, i.e.
  Block<float>::forward (its 4 heads split over 2 and 4 ranks).
Each world size is skipped when fewer GPUs are visible.
"""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

needs2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                            reason="needs two GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import ctypes as C

    import torch.distributed as dist

    from oracle import oracle as ro
    from reef_b200 import _lib, tp
    from reef_b200 import kernels as K
    from reef_b200 import layer as RL
    from tests.test_oracle import block_float_weights
    res = {}
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        comm = tp.Comm(rank, world, timeout_s=60)
        bits = lambda t: t.cpu().numpy().view(np.uint32)

        # row-parallel linear vs the unsplit linear
        M, Kd, N = 257, 1024, 768
        x = torch.from_numpy(ro.normal(1, (M, Kd))).to(dev)
        w, ws = ro.quantize_rows(ro.normal(2, (N, Kd), 0, 0.02))
        b = torch.from_numpy(ro.normal(3, (N,), 0, 0.02)).to(dev)
        wd, wsd = torch.from_numpy(w).to(dev), torch.from_numpy(ws).to(dev)
        cols = tp.col_slice(Kd, world, rank)
        xl = x[:, cols].contiguous()
        wl = wd[:, cols].contiguous()
        kl = xl.shape[1]
        xq = torch.empty((M, K.kpad(kl)), dtype=torch.int8, device=dev)
        xs = torch.empty(M, device=dev)
        rm = torch.empty(M, device=dev)
        acc = torch.empty((M, N), dtype=torch.int32, device=dev)
        y = torch.empty((M, N), device=dev)
        _lib.call("reef_b200_linear_w8a8_rowpar", comm.ptr, M, kl, N, xl.data_ptr(),
                  wl.data_ptr(), wsd.data_ptr(), b.data_ptr(), xq.data_ptr(), xs.data_ptr(),
                  rm.data_ptr(), acc.data_ptr(), y.data_ptr(),
                  torch.cuda.current_stream().cuda_stream)
        want = K.linear_w8a8(x, wd, wsd, b)
        res["rowpar"] = bool(np.array_equal(bits(y), bits(want)))

        # Llama-shape layers, TP=N shard vs TP=1 on this device, both plans;
        # the small shape has GQA (2 query heads per kv head) where the kv
        # heads split, and config 3's widths at two sequences of 2048
        kv_small = 4 if world <= 4 else 8
        cases = [("llama", RL.LlamaShape(hidden=1024, heads_q=8, heads_kv=kv_small, ffn=2816),
                  256, 9),
                 ("llama7b", RL.LLAMA_7B, 2048, 19)]
        for name, shape, seq, seed in cases:
            xin = torch.from_numpy(ro.normal(seed, (2 * seq, shape.hidden))).to(dev)
            L1 = RL.LlamaLayer(shape, 2, seq, seed=seed + 1, device=dev)
            y1 = L1.forward(xin)
            del L1
            L2 = RL.LlamaLayer(shape, 2, seq, seed=seed + 1, world=world, rank=rank, comm=comm,
                               device=dev)
            y2 = L2.forward(xin)
            res[name] = bool(np.array_equal(bits(y2), bits(y1)))
            del L2
            # the all-gather plan: x / y are this rank's hidden columns
            cols = tp.col_slice(shape.hidden, world, rank)
            L3 = RL.LlamaLayer(shape, 2, seq, seed=seed + 1, world=world, rank=rank, comm=comm,
                               device=dev, tp_mode=RL.TP_ALLGATHER)
            y3 = L3.forward(xin[:, cols].contiguous())
            res[name + "_allgather"] = bool(np.array_equal(bits(y3),
                                                           bits(y1[:, cols].contiguous())))
            del L3, y1, y2, y3, xin
            torch.cuda.synchronize(dev)
            torch.cuda.empty_cache()

        # GPT-Neo block (config 2 shape), TP=N vs the oracle (reef's Block<float>)
        if 4 % world == 0:
            fw = block_float_weights(256, 1024, seed=80)
            xb = ro.normal(81, (128, 256))
            blk = RL.GptNeoBlock(fw, 4, 128, world=world, rank=rank, comm=comm, device=dev)
            yb = blk.forward(torch.from_numpy(xb).to(dev))
            wantb = ro.gptneo_block_w8a8(xb, ro.quantize_block(fw), 4)
            res["gptneo"] = bool(np.array_equal(bits(yb), wantb.view(np.uint32)))
        torch.cuda.synchronize(dev)
        K.check_device_error()
        comm.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, ("ok", res)))
    except Exception:
        q.put((rank, ("error", traceback.format_exc())))


@needs2
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_bit_identical_to_tp1(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    want = {"rowpar": True, "llama": True, "llama_allgather": True, "llama7b": True,
            "llama7b_allgather": True}
    if 4 % world == 0:
        want["gptneo"] = True
    for r in range(world):
        status, res = out[r]
        assert status == "ok", res
        assert res == want, (r, res)
