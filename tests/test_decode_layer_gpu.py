"""The Llama-shape decode step against the prefill layer.

reef checks that decoding token by token gives the prefill's result
(test_gpt_neo.cpp:97-105).  Here each sequence is decoded one token at a time
into the int8 KV cache; the step's output for token t must match the prefill
layer's row t over the same inputs.  The q / k / v codes are identical in the
two paths (the same exact W8A8 GEMMs and quantiser); the attention kernels
differ (flash: f16 P on tensor cores; decode: fp32 P on CUDA cores), so the
outputs agree within the layer tolerance of test_layer_gpu.py.  Also runs
one step at config 4's TP=8 shard shape (hidden 8192, 8 q / 1 kv heads, FFN
3584, 64 sequences, 4096-row cache).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as ro
from reef_b200 import kernels as K
from reef_b200 import layer as RL

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_lib):
    yield
    K.check_device_error()


def test_decode_steps_match_prefill():
    shape = RL.LlamaShape(hidden=512, heads_q=4, heads_kv=2, ffn=1024)
    B, S = 2, 64
    L = RL.LlamaLayer(shape, B, S, seed=21)
    x = torch.from_numpy(ro.normal(22, (B * S, 512))).cuda()
    want = L.forward(x).view(B, S, 512)
    cache = L.alloc_cache(S)
    xs = x.view(B, S, 512)
    worst, mean = 0.0, []
    for t in range(S):
        pos = torch.full((B,), t, dtype=torch.int32, device="cuda")
        y = L.decode(xs[:, t].contiguous(), pos, cache)
        err = (y - want[:, t]).abs()
        worst = max(worst, float(err.max()))
        mean.append(float(err.mean()))
    assert worst < 5e-2, worst
    assert np.mean(mean) < 5e-3, np.mean(mean)


def test_decode_config4_tp8_shard_runs():
    # config 4 at TP=8, one rank's shard: hidden 8192, 64/8 = 8 q heads,
    # 8/8 = 1 kv head, FFN 28672/8 = 3584; 64 sequences, 4096-row cache
    shape = RL.LlamaShape(hidden=8192, heads_q=64, heads_kv=8, ffn=28672)
    L = RL.LlamaLayer(shape, 64, 8, seed=3, world=8, rank=0)
    cache = L.alloc_cache(4096)
    g = torch.Generator(device="cuda").manual_seed(5)
    cache["k"].random_(-127, 128, generator=g)
    cache["v"].random_(-127, 128, generator=g)
    cache["ks"].fill_(0.01)
    cache["vs"].fill_(0.01)
    x = torch.randn((64, 8192), generator=g, device="cuda")
    pos = torch.full((64,), 4095, dtype=torch.int32, device="cuda")
    y = L.decode(x, pos, cache)
    torch.cuda.synchronize()
    assert torch.isfinite(y).all()
    # the new token's k / v rows were written at row 4095
    assert cache["ks"][:, :, 4095].gt(0).all() and cache["vs"][:, :, 4095].ne(0.01).any()
