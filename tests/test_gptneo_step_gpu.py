"""reef's GPT-Neo W8A8 model generating on the GPU, pinned to reef's golden.

reef's kGptNeo golden (gen_golden.cpp:755-805) packs a small GPT-Neo (4
layers, global and local, window 8, 4 heads, vocab 96) at W8A8 and at float
precision, runs the engine's GPTNeo<float> on a 5-token prompt and greedily
generates 20 tokens, keeping the logits behind each; the Coral firmware is
held to it.  Here the blob is
loaded by reef_b200_blob_load_model and run by reef_b200_gptneo_step: every
logit must match bit for bit and every token, whether the prompt goes in at
once or a token at a time (the firmware's way).  The pieces are checked on
their own too: the embedding against reef's kEmbedding goldens, and a block
run in chunks over its KV cache against the same block run at once.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as ro
from reef_b200 import _lib
from reef_b200 import kernels as K
from reef_b200.layer import GptNeoModel
from tests import blob_fixture as BF
from tests import goldens

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_lib):
    yield
    K.check_device_error()


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def test_generation_matches_reef_golden():
    blob, prompt, tokens, logits = BF.golden_model("w8a8")
    m = GptNeoModel(blob, max_tokens=prompt.size + tokens.size)
    got_tokens, got_logits = m.generate(prompt, tokens.size)
    torch.cuda.synchronize()
    assert got_tokens.tolist() == tokens.tolist()
    np.testing.assert_array_equal(bits(got_logits.numpy()), bits(logits))


def test_float_generation_matches_reef_golden():
    """The float (kFloat32) model of the same golden: a float blob loads with
    its [in][out] weights and runs the exact float operators."""
    blob, prompt, tokens, logits = BF.golden_model("fp32")
    m = GptNeoModel(blob, max_tokens=prompt.size + tokens.size)
    got_tokens, got_logits = m.generate(prompt, tokens.size)
    torch.cuda.synchronize()
    assert got_tokens.tolist() == tokens.tolist()
    np.testing.assert_array_equal(bits(got_logits.numpy()), bits(logits))


def test_prompt_token_by_token_gives_same_bits():
    blob, prompt, tokens, logits = BF.golden_model("w8a8")
    m = GptNeoModel(blob, max_tokens=prompt.size + tokens.size)
    ids = torch.tensor(prompt.astype(np.int32), device="cuda")
    out = torch.empty((tokens.size, logits.shape[1]), device="cuda")
    nxt = torch.empty(tokens.size, dtype=torch.int32, device="cuda")
    for t in range(prompt.size - 1):  # no logits until the prompt's last token
        m.step(ids[t:t + 1])
    m.step(ids[prompt.size - 1:], out[0], nxt[0:1])
    for i in range(1, tokens.size):
        m.step(nxt[i - 1:i], out[i], nxt[i:i + 1])
    torch.cuda.synchronize()
    assert nxt.cpu().tolist() == tokens.astype(np.int64).tolist()
    np.testing.assert_array_equal(bits(out.cpu().numpy()), bits(logits))


def test_embedding_matches_reef_goldens():
    for c in goldens.cases("elementwise", "kEmbedding"):
        w = c["width"]
        wte = torch.from_numpy(c["wte"]).cuda()
        wpe = torch.from_numpy(c["wpe"]).cuda()
        ids = torch.tensor([c["id"]], dtype=torch.int32, device="cuda")
        y = torch.empty(w, device="cuda")
        _lib.call("reef_b200_embedding_f32", w, 1, ids.data_ptr(), c["position"],
                  wte.numel() // w, wpe.numel() // w, wte.data_ptr(), wpe.data_ptr(),
                  y.data_ptr(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(c["y"]))


def test_embedding_bad_token_is_reported():
    """An id past the vocabulary (the engine throws) is caught by the kernel's
    bounds check: the row is zeros and 0x202 is in the device error word."""
    wte = torch.ones((10, 37), device="cuda")
    wpe = torch.ones((8, 37), device="cuda")
    ids = torch.tensor([3, 10], dtype=torch.int32, device="cuda")
    y = torch.full((2, 37), 7.0, device="cuda")
    _lib.call("reef_b200_embedding_f32", 37, 2, ids.data_ptr(), 0, 10, 8, wte.data_ptr(),
              wpe.data_ptr(), y.data_ptr(), torch.cuda.current_stream().cuda_stream)
    code = C.c_int(-1)
    assert _lib.lib().reef_b200_device_error(C.byref(code)) == 0
    assert code.value == 0x202
    assert torch.equal(y[0].cpu(), torch.full((37,), 2.0))
    assert torch.equal(y[1].cpu(), torch.zeros(37))


@pytest.mark.parametrize("layer,split", [(0, (3, 5)), (1, (1, 1, 6, 2)), (1, (10,))])
def test_cached_block_equals_block_at_once(layer, split):
    """A blob layer run over its KV cache in chunks (prefill pieces, then
    single tokens) gives the bits of the same layer run on all positions at
    once, which the oracle pins (tests/test_blob_gpu.py)."""
    b = BF.data()
    h = BF.header(b)
    buf = C.create_string_buffer(b, len(b))
    info = _lib.BlobInfo()
    _lib.call("reef_b200_blob_read_info", buf, len(b), C.byref(info))
    arena = torch.zeros(_lib.lib().reef_b200_blob_layer_bytes(C.byref(info)), dtype=torch.uint8,
                        device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    desc = _lib.GptNeoBlockDesc()
    _lib.call("reef_b200_blob_load_layer", buf, len(b), layer, arena.data_ptr(), arena.numel(),
              C.byref(desc), st)
    total = sum(split)
    x = torch.from_numpy(ro.normal(70 + layer, (total, h["hidden"]))).cuda()
    p, local = BF.layer(b, layer)
    want = ro.gptneo_block_w8a8(x.cpu().numpy(), p, h["heads"],
                                window=h["window"] if local else 0, eps=h["eps"])
    kc = torch.zeros((total + 3, h["hidden"]), device="cuda")
    vc = torch.zeros_like(kc)
    y = torch.empty_like(x)
    pos = 0
    for n in split:
        desc.seq = n
        ws = torch.empty(_lib.lib().reef_b200_gptneo_block_workspace_bytes(C.byref(desc)),
                         dtype=torch.uint8, device="cuda")
        _lib.call("reef_b200_gptneo_block_forward_cached", C.byref(desc),
                  x[pos:pos + n].data_ptr(), y[pos:pos + n].data_ptr(), pos, kc.data_ptr(),
                  vc.data_ptr(), kc.shape[0], ws.data_ptr(), ws.numel(), st)
        pos += n
    torch.cuda.synchronize()
    np.testing.assert_array_equal(bits(y.cpu().numpy()), bits(want))


def test_step_rejects_positions_past_the_cache():
    blob, prompt, tokens, _ = BF.golden_model("w8a8")
    m = GptNeoModel(blob, max_tokens=6)
    ids = torch.tensor(prompt.astype(np.int32), device="cuda")
    m.step(ids)  # positions 0..4
    with pytest.raises(_lib.ReefError):
        m.step(torch.cat([ids[:1], ids[:1]]))  # 5..6 > 6 rows
