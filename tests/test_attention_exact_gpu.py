"""Parity of reef's two attention heads on the GPU (bit for bit).

* integer softmax / integer head against reef's golden vectors
  (gen_golden.cpp write_int8: 3 softmax cases incl. equal scores and a wide
  spread at shift 0; 7 heads incl. windows and query offsets);
* float head against reef's golden vectors (write_attention, 7 heads);
* both heads against the oracle on larger seeded shapes, and the multi-head
  launch (Attention::context) at the config-1 shape.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as ro
from reef_b200 import kernels as K
from tests import goldens

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    a = np.asarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_lib):
    yield
    K.check_device_error()


def test_softmax_int8_goldens():
    for c in goldens.cases("int8", "kInt8Softmax"):
        p = K.softmax_int8(dev(c["scores"].reshape(c["rows"], c["n"])), c["shift"],
                           K.exp_table_device(c["table"]))
        np.testing.assert_array_equal(host(p).ravel(), c["probs"])


def test_attention_int8_goldens():
    for c in goldens.cases("int8", "kInt8Attention"):
        d = c["head_dim"]
        y = K.attention_head_int8(dev(c["q"].reshape(-1, d)), dev(c["k"].reshape(-1, d)),
                                  dev(c["v"].reshape(-1, d)), c["query_start"], c["window"],
                                  c["score_shift"], K.exp_table_device(c["table"]),
                                  c["out_shift"])
        np.testing.assert_array_equal(host(y).ravel(), c["y"])


def test_attention_f32_goldens():
    for c in goldens.cases("attention", "kAttention"):
        d = c["head_dim"]
        y = K.attention_head_f32(dev(c["q"].reshape(-1, d)), dev(c["k"].reshape(-1, d)),
                                 dev(c["v"].reshape(-1, d)), c["query_start"], c["window"])
        np.testing.assert_array_equal(bits(host(y).ravel()), bits(c["y"]))


HEADS = [  # query_len, key_len, head_dim, query_start, window, score_shift
    (64, 64, 64, 0, 0, 10), (16, 300, 128, 284, 100, 9), (128, 128, 64, 0, 0, 8),
    (3, 5000, 64, 4997, 0, 11), (33, 1030, 128, 997, 256, 12), (1, 4096, 128, 4095, 0, 12),
]


@pytest.mark.parametrize("ql,kl,d,qs,win,sh", HEADS)
def test_attention_int8_matches_oracle(ql, kl, d, qs, win, sh):
    seed = ql + kl + d
    q = ro.int8_uniform(seed, (ql, d))
    k = ro.int8_uniform(seed + 1, (kl, d))
    v = ro.int8_uniform(seed + 2, (kl, d))
    want = ro.attention_head_int8(q, k, v, qs, win, sh, 8)
    got = K.attention_head_int8(dev(q), dev(k), dev(v), qs, win, sh,
                                K.exp_table_device(ro.exp_table()), 8)
    np.testing.assert_array_equal(host(got), want)


@pytest.mark.parametrize("ql,kl,d,qs,win,sh", HEADS)
def test_attention_f32_matches_oracle(ql, kl, d, qs, win, sh):
    seed = 3 * ql + kl + d
    q = ro.normal(seed, (ql, d), 0.0, 0.3)
    k = ro.normal(seed + 1, (kl, d), 0.0, 0.3)
    v = ro.normal(seed + 2, (kl, d))
    want = ro.attention_head_f32(q, k, v, qs, win)
    got = K.attention_head_f32(dev(q), dev(k), dev(v), qs, win)
    np.testing.assert_array_equal(bits(host(got)), bits(want))


def test_context_all_heads_config1_shape():
    """Attention::context at config 1: seq 128, 4 heads x 64, causal."""
    seq, dm, heads = 128, 256, 4
    hd = dm // heads
    q, k, v = (ro.normal(s, (seq, dm)) for s in (41, 42, 43))
    got = host(K.attention_heads_f32(dev(q), dev(k), dev(v), heads))
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        want = ro.attention_head_f32(q[:, sl].copy(), k[:, sl].copy(), v[:, sl].copy(), 0, 0)
        np.testing.assert_array_equal(bits(got[:, sl].copy()), bits(want))
