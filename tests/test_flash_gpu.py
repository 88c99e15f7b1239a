"""The int8 flash head against reef's float head (within 1e-2, max-abs).

reef's attend_head (attention.hpp:117-123) is unscaled and per head; the flash
kernel takes int8 q/k/v with per-(token, head) scales, a score scale and GQA.
The reference is attend_head on the dequantised inputs with the score scale
folded into q:  attend_head(q8*qs*sm_scale, k8*ks, v8*vs, causal).
* oracle (CPU restatement of attend_head) on small shapes, every head;
* torch fp64 at the config-3 shape (batch 8 x seq 2048, 32 heads x 128) on
  sampled (batch, head) pairs, and at config-4's GQA grouping (8 q per kv).
Also checks the RoPE / quantise packing kernel: v8 bit-exact with reef's
quantize_rows, vt exactly f16(v8 * v_scale) transposed, q8/k8 within one code
of a float64 RoPE then reef's quantiser.
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


def quant_heads(x, heads):
    """reef's quantiser (quant.hpp:51-81) per (token, head) of 128 values."""
    t = x.shape[0]
    xr = x.reshape(t, heads, 128).astype(np.float32)
    mx = np.abs(xr).max(axis=2)
    scale = np.where(mx > 0, mx / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q = np.clip(np.rint(xr / scale[:, :, None]), -127, 127).astype(np.int8)
    return q.reshape(t, heads * 128), scale


def flash(q8, qs, k8, ks, vt, B, S, Hq, Hkv, causal, sm):
    out = torch.empty((B * S, Hq * 128), dtype=torch.float32, device="cuda")
    _lib.call("reef_b200_flash_attn_i8", B, S, Hq, Hkv, 128, int(causal), sm,
              q8.data_ptr(), qs.data_ptr(), k8.data_ptr(), ks.data_ptr(), vt.data_ptr(),
              out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    return out


def quant_heads_dev(x, heads):
    """The same quantiser on the device (torch.round is half-to-even)."""
    t = x.shape[0]
    xr = x.reshape(t, heads, 128)
    mx = xr.abs().amax(dim=2)
    scale = torch.where(mx > 0, mx / 127.0, torch.ones_like(mx))
    q = torch.clamp(torch.round(xr / scale[:, :, None]), -127, 127).to(torch.int8)
    return q.reshape(t, heads * 128).contiguous(), scale.contiguous()


class Inputs:
    """Seeded int8 q/k/v with per-(token, head) scales, on the device; host
    copies of single heads on demand."""

    def __init__(self, B, S, Hq, Hkv, seed, qk_std=1.0):
        g = torch.Generator(device="cuda").manual_seed(seed)
        T = B * S
        rnd = lambda n, std: torch.randn((T, n), generator=g, device="cuda") * std
        self.q8, self.qsc = quant_heads_dev(rnd(Hq * 128, qk_std), Hq)
        self.k8, self.ksc = quant_heads_dev(rnd(Hkv * 128, qk_std), Hkv)
        self.v8, self.vsc = quant_heads_dev(rnd(Hkv * 128, 1.0), Hkv)
        bhs = lambda sc, H: sc.reshape(B, S, H).permute(0, 2, 1).contiguous()
        self.qs, self.ks, self.vs = bhs(self.qsc, Hq), bhs(self.ksc, Hkv), bhs(self.vsc, Hkv)
        vdeq = self.v8.reshape(T, Hkv, 128).float() * self.vsc[:, :, None]
        self.vt = vdeq.to(torch.float16).reshape(B, S, Hkv, 128).permute(0, 2, 3, 1).contiguous()
        self.B, self.S, self.Hq, self.Hkv = B, S, Hq, Hkv

    def head(self, b, h, sm):
        """Dequantised (q * sm, k, v) of one query head, float32 numpy."""
        S, g = self.S, self.Hq // self.Hkv
        rows = slice(b * S, (b + 1) * S)
        kh = h // g
        f = lambda x8, sc, hh: (x8[rows, hh * 128:(hh + 1) * 128].float() *
                                sc[rows, hh][:, None]).cpu().numpy()
        q = f(self.q8, self.qsc, h) * np.float32(sm)
        return q.astype(np.float32), f(self.k8, self.ksc, kh), f(self.v8, self.vsc, kh)


def make(B, S, Hq, Hkv, seed, qk_std=1.0):
    d = Inputs(B, S, Hq, Hkv, seed, qk_std)
    return d, dict(q8=d.q8, k8=d.k8, qs=d.qs, ks=d.ks, vt=d.vt)


def run(dev, B, S, Hq, Hkv, causal, sm):
    o = flash(dev["q8"], dev["qs"], dev["k8"], dev["ks"], dev["vt"], B, S, Hq, Hkv, causal, sm)
    torch.cuda.synchronize()
    return o.cpu().numpy()


def deq(d, b, h, Hq, Hkv, S, sm):
    return d.head(b, h, sm)


# one query tile (no second tile in the CTA), an odd tile count, ragged tails
# (136 = 128 + 8, 264 = 2*128 + 8), non-causal, and a wide score range
# (qk_std 3) that makes the lazy rescale of O fire
@pytest.mark.parametrize("B,S,Hq,Hkv,causal,qk_std", [
    (1, 128, 1, 1, True, 1.0), (2, 256, 4, 2, True, 1.0), (1, 384, 2, 2, False, 1.0),
    (1, 136, 2, 1, True, 1.0), (1, 264, 2, 2, True, 1.0), (1, 640, 2, 1, True, 1.0),
    (1, 264, 1, 1, False, 1.0), (1, 1024, 2, 1, True, 3.0)])
def test_flash_matches_reef_float_head(B, S, Hq, Hkv, causal, qk_std):
    sm = 1.0 / math.sqrt(128)
    d, dev = make(B, S, Hq, Hkv, seed=B * 100 + S + Hq, qk_std=qk_std)
    out = run(dev, B, S, Hq, Hkv, causal, sm)
    worst = 0.0
    for b in range(B):
        for h in range(Hq):
            q, k, v = deq(d, b, h, Hq, Hkv, S, sm)
            want = ro.attention_head_f32(q, k, v, 0, 0) if causal else \
                ro.attention_head_f32(q, k, v, S - 1, 0)  # rows at S-1.. see every key
            got = out[b * S:(b + 1) * S, h * 128:(h + 1) * 128]
            worst = max(worst, float(np.abs(got - want).max()))
    assert worst < TOL, worst


def test_flash_noncausal_all_rows():
    B, S, H = 1, 256, 2
    sm = 1.0 / math.sqrt(128)
    d, dev = make(B, S, H, H, seed=7)
    out = run(dev, B, S, H, H, False, sm)
    for h in range(H):
        q, k, v = deq(d, 0, h, H, H, S, sm)
        s = q.astype(np.float64) @ k.astype(np.float64).T
        p = np.exp(s - s.max(1, keepdims=True))
        want = (p / p.sum(1, keepdims=True)) @ v
        assert np.abs(out[:, h * 128:(h + 1) * 128] - want).max() < TOL


@pytest.mark.parametrize("B,S,Hq,Hkv", [(8, 2048, 32, 32), (2, 4096, 8, 1)])
def test_flash_config_shapes_sampled(B, S, Hq, Hkv):
    """Config 3 (prefill 8 x 2048, 32 heads) and config-4 GQA (8 q / kv)."""
    sm = 1.0 / math.sqrt(128)
    d, dev = make(B, S, Hq, Hkv, seed=S + Hq, qk_std=1.5)
    out = run(dev, B, S, Hq, Hkv, True, sm)
    for (b, h) in [(0, 0), (B - 1, Hq - 1), (B // 2, Hq // 3)]:
        q, k, v = (torch.from_numpy(a).cuda().double() for a in deq(d, b, h, Hq, Hkv, S, sm))
        s = q @ k.T
        s.masked_fill_(torch.ones(S, S, device="cuda").triu(1).bool(), float("-inf"))
        want = torch.softmax(s, 1) @ v
        got = torch.from_numpy(out[b * S:(b + 1) * S, h * 128:(h + 1) * 128]).cuda().double()
        assert float((got - want).abs().max()) < TOL


# (3, 40): the 64-token blocks of the V transpose straddle sequences
@pytest.mark.parametrize("B,S", [(2, 64), (3, 40)])
def test_rope_qkv_quant_packing(B, S):
    Hq, Hkv = 4, 2
    T = B * S
    W = (Hq + 2 * Hkv) * 128
    rng = np.random.default_rng(3)
    qkv = rng.normal(0, 1, (T, W)).astype(np.float32)
    qkv[5, (Hq + Hkv) * 128:(Hq + Hkv + 1) * 128] = 0  # an all-zero v head row
    q8 = torch.empty((T, Hq * 128), dtype=torch.int8, device="cuda")
    k8 = torch.empty((T, Hkv * 128), dtype=torch.int8, device="cuda")
    v8 = torch.empty((T, Hkv * 128), dtype=torch.int8, device="cuda")
    qs = torch.empty((B, Hq, S), device="cuda")
    ks = torch.empty((B, Hkv, S), device="cuda")
    vs = torch.empty((B, Hkv, S), device="cuda")
    vt = torch.empty((B, Hkv, 128, S), dtype=torch.float16, device="cuda")
    x = torch.from_numpy(qkv).cuda()
    _lib.call("reef_b200_rope_qkv_quant", B, S, Hq, Hkv, 10000.0, x.data_ptr(), q8.data_ptr(),
              k8.data_ptr(), v8.data_ptr(), qs.data_ptr(), ks.data_ptr(), vs.data_ptr(),
              vt.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    # v: reef's quantize_rows on each (token, head) row, bit for bit
    vrows = qkv[:, (Hq + Hkv) * 128:].reshape(T * Hkv, 128)
    wq, ws = ro.quantize_rows(np.ascontiguousarray(vrows))
    np.testing.assert_array_equal(v8.cpu().numpy().reshape(T * Hkv, 128), wq)
    np.testing.assert_array_equal(
        vs.cpu().numpy().transpose(0, 2, 1).reshape(T * Hkv).view(np.uint32), ws.view(np.uint32))
    vdeq = (v8.cpu().numpy().reshape(B, S, Hkv, 128).astype(np.float32) *
            vs.cpu().numpy().transpose(0, 2, 1)[:, :, :, None]).astype(np.float16)
    np.testing.assert_array_equal(vt.cpu().numpy().view(np.uint16),
                                  vdeq.transpose(0, 2, 3, 1).view(np.uint16))
    # q / k: float64 rotate-half RoPE, then reef's quantiser; within one code
    pos = np.tile(np.arange(S), B)[:, None].astype(np.float64)
    inv = 10000.0 ** (-np.arange(64) * 2 / 128.0)
    ang = pos * inv[None, :]
    for off, H, got in ((0, Hq, q8), (Hq * 128, Hkv, k8)):
        xh = qkv[:, off:off + H * 128].reshape(T, H, 128).astype(np.float64)
        lo, hi = xh[..., :64], xh[..., 64:]
        c, s = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
        rot = np.concatenate([lo * c - hi * s, hi * c + lo * s], axis=2).reshape(T, H * 128)
        want, _ = quant_heads(rot.astype(np.float32), H)
        diff = np.abs(got.cpu().numpy().astype(np.int32) - want.astype(np.int32))
        assert diff.max() <= 1


# QKV GEMM with RoPE + int8 packing in its epilogue == GEMM, then the packing
# kernel: one head per tile (1 + 2 heads), 40-token sequences (warps straddle
# two sequences), an all-zero token row, config 3's per-token width
@pytest.mark.parametrize("B,S,k,Hq,Hkv", [(2, 64, 256, 4, 2), (3, 40, 512, 2, 1),
                                          (1, 128, 4096, 32, 32), (2, 72, 128, 1, 1)])
def test_qkv_rope_gemm_matches_two_pass(B, S, k, Hq, Hkv):
    T, W = B * S, (Hq + 2 * Hkv) * 128
    g = torch.Generator(device="cuda").manual_seed(B * S + k + Hq)
    xq = torch.randint(-127, 128, (T, K.kpad(k)), generator=g, device="cuda", dtype=torch.int8)
    xq[5] = 0
    w = torch.randint(-127, 128, (W, K.kpad(k)), generator=g, device="cuda", dtype=torch.int8)
    xs = torch.rand((T,), generator=g, device="cuda") * 1e-3 + 1e-4
    ws = torch.rand((W,), generator=g, device="cuda") * 1e-3 + 1e-4
    st = torch.cuda.current_stream().cuda_stream

    def outputs():
        return dict(q8=torch.empty((T, Hq * 128), dtype=torch.int8, device="cuda"),
                    k8=torch.empty((T, Hkv * 128), dtype=torch.int8, device="cuda"),
                    v8=torch.empty((T, Hkv * 128), dtype=torch.int8, device="cuda"),
                    qs=torch.empty((B, Hq, S), device="cuda"),
                    ks=torch.empty((B, Hkv, S), device="cuda"),
                    vs=torch.empty((B, Hkv, S), device="cuda"),
                    vt=torch.empty((B, Hkv, 128, S), dtype=torch.float16, device="cuda"))

    y = K.gemm_w8a8(xq, xs, w, ws, in_features=k)
    ref = outputs()
    _lib.call("reef_b200_rope_qkv_quant", B, S, Hq, Hkv, 10000.0, y.data_ptr(),
              ref["q8"].data_ptr(), ref["k8"].data_ptr(), ref["v8"].data_ptr(),
              ref["qs"].data_ptr(), ref["ks"].data_ptr(), ref["vs"].data_ptr(),
              ref["vt"].data_ptr(), st)
    rope = torch.empty((S, 64, 2), device="cuda")
    for with_v in (True, False):
        got = outputs()
        _lib.call("reef_b200_linear_w8a8_qkv_rope", B, S, k, Hq, Hkv, 10000.0, xq.data_ptr(),
                  xs.data_ptr(), w.data_ptr(), ws.data_ptr(), got["q8"].data_ptr(),
                  got["k8"].data_ptr(), got["v8"].data_ptr() if with_v else None,
                  got["qs"].data_ptr(), got["ks"].data_ptr(),
                  got["vs"].data_ptr() if with_v else None, got["vt"].data_ptr(),
                  rope.data_ptr(), st)
        torch.cuda.synchronize()
        names = ["q8", "k8", "qs", "ks", "vt"] + (["v8", "vs"] if with_v else [])
        for name in names:
            a, b = got[name].cpu(), ref[name].cpu()
            if a.dtype in (torch.float32, torch.float16):
                a, b = a.view(torch.int32 if a.dtype == torch.float32 else torch.int16), \
                    b.view(torch.int32 if b.dtype == torch.float32 else torch.int16)
            assert torch.equal(a, b), (name, with_v)
