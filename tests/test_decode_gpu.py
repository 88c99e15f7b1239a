"""int8 decode attention (config 4) against reef's float head, within 1e-2.

Each sequence's new query sits at its last cached position, so it sees every
cached key: reef's attend_head(q, k, v) with query_start = len - 1 on the
dequantised inputs (the score scale folded into q).  Checked against the
oracle on every head of small cases (incl. ragged lengths, GQA groups 1..16,
lengths not multiple of the split chunk) and against torch fp64 at config
4's per-GPU shape at TP=8 (batch 64, 8 query heads over 1 KV head, 4096
cached keys).
"""
import math

import numpy as np
import pytest
import torch

from oracle import oracle as ro
from reef_b200 import _lib
from reef_b200 import kernels as K

pytestmark = pytest.mark.gpu
TOL = 1e-2


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_lib):
    yield
    K.check_device_error()


def qrows(x):
    """reef's quantiser per row of 128 (quant.hpp:51-81), on the device."""
    mx = x.abs().amax(dim=-1, keepdim=True)
    sc = torch.where(mx > 0, mx / 127.0, torch.ones_like(mx))
    return torch.clamp(torch.round(x / sc), -127, 127).to(torch.int8), sc.squeeze(-1)


def make(B, Hq, Hkv, L, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q8, qs = qrows(torch.randn((B, Hq, 128), generator=g, device="cuda") * 1.5)
    k8, ks = qrows(torch.randn((B, Hkv, L, 128), generator=g, device="cuda") * 1.5)
    v8, vs = qrows(torch.randn((B, Hkv, L, 128), generator=g, device="cuda"))
    return [t.contiguous() for t in (q8, qs, k8, ks, v8, vs)]


def run(B, Hq, Hkv, L, lens, sm, t):
    q8, qs, k8, ks, v8, vs = t
    ws = torch.empty(_lib.lib().reef_b200_decode_attn_workspace_bytes(B, Hq, L),
                     dtype=torch.uint8, device="cuda")
    out = torch.empty((B, Hq, 128), device="cuda")
    lens_t = None if lens is None else torch.tensor(lens, dtype=torch.int32, device="cuda")
    _lib.call("reef_b200_decode_attn_i8", B, Hq, Hkv, 128, L,
              None if lens_t is None else lens_t.data_ptr(), 0 if lens is not None else L, sm,
              q8.data_ptr(), qs.data_ptr(), k8.data_ptr(), ks.data_ptr(), v8.data_ptr(),
              vs.data_ptr(), ws.data_ptr(), ws.numel(), out.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("B,Hq,Hkv,L,lens", [(2, 4, 4, 300, None), (3, 8, 1, 1000, [1000, 257, 1]),
                                             (2, 16, 1, 520, [513, 256]),
                                             (1, 4, 2, 4096, None),
                                             # more (sequence, KV head) pairs than CTAs:
                                             # CTAs that end one sequence and start the next
                                             (300, 4, 2, 256, [1 + (37 * i) % 256 for i in range(300)]),
                                             (5, 32, 2, 1024, [1024, 129, 128, 700, 3])])
def test_decode_matches_reef_float_head(B, Hq, Hkv, L, lens):
    sm = 1.0 / math.sqrt(128)
    t = make(B, Hq, Hkv, L, seed=B + Hq + L)
    out = run(B, Hq, Hkv, L, lens, sm, t).cpu().numpy()
    q8, qs, k8, ks, v8, vs = (x.cpu().numpy() for x in t)
    worst = 0.0
    for b in range(B):
        n = L if lens is None else lens[b]
        for h in range(Hq):
            kh = h // (Hq // Hkv)
            q = (q8[b, h].astype(np.float32) * qs[b, h] * np.float32(sm))[None, :]
            k = k8[b, kh, :n].astype(np.float32) * ks[b, kh, :n, None]
            v = v8[b, kh, :n].astype(np.float32) * vs[b, kh, :n, None]
            want = ro.attention_head_f32(np.ascontiguousarray(q), np.ascontiguousarray(k),
                                         np.ascontiguousarray(v), n - 1, 0)
            worst = max(worst, float(np.abs(out[b, h] - want[0]).max()))
    assert worst < TOL, worst


def test_decode_config4_tp8_shard():
    B, Hq, Hkv, L = 64, 8, 1, 4096
    sm = 1.0 / math.sqrt(128)
    t = make(B, Hq, Hkv, L, seed=4)
    out = run(B, Hq, Hkv, L, None, sm, t)
    q8, qs, k8, ks, v8, vs = t
    q = q8.double() * qs.double()[..., None] * sm                     # [B, Hq, 128]
    k = (k8.double() * ks.double()[..., None])[:, 0]                   # [B, L, 128]
    v = (v8.double() * vs.double()[..., None])[:, 0]
    p = torch.softmax(torch.einsum("bhd,bld->bhl", q, k), dim=-1)
    want = torch.einsum("bhl,bld->bhd", p, v)
    assert float((out.double() - want).abs().max()) < TOL
