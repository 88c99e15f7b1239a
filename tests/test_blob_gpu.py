"""Layers of reef's packed model loaded onto the GPU and run, bit for bit.

Each layer of the fixture blob (written by reef's packer, W8A8) is loaded by
reef_b200_blob_load_layer into a device arena (its [in][out] int8 weights
repacked K-major) and run through reef_b200_gptneo_block_forward; the output
must equal the oracle's GPT-Neo block (reef's Block<float>::forward, pinned
to the engine) run on the same layer's arrays, read from the blob by numpy.
Layer 0 is global, layer 1 local (the blob's window).
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as ro
from reef_b200 import _lib
from reef_b200 import kernels as K
from tests import blob_fixture as BF

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_lib):
    yield
    K.check_device_error()


@pytest.mark.parametrize("index", [0, 1])
def test_loaded_layer_runs_bit_identical(index):
    b = BF.data()
    h = BF.header(b)
    buf = C.create_string_buffer(b, len(b))
    info = _lib.BlobInfo()
    _lib.call("reef_b200_blob_read_info", buf, len(b), C.byref(info))
    arena = torch.zeros(_lib.lib().reef_b200_blob_layer_bytes(C.byref(info)), dtype=torch.uint8,
                        device="cuda")
    desc = _lib.GptNeoBlockDesc()
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("reef_b200_blob_load_layer", buf, len(b), index, arena.data_ptr(), arena.numel(),
              C.byref(desc), st)
    p, local = BF.layer(b, index)
    window = h["window"] if local else 0
    assert (desc.hidden, desc.heads, desc.ffn, desc.window) == (h["hidden"], h["heads"],
                                                                h["inner"], window)
    seq = 24
    desc.seq = seq
    ws = torch.empty(_lib.lib().reef_b200_gptneo_block_workspace_bytes(C.byref(desc)),
                     dtype=torch.uint8, device="cuda")
    x = ro.normal(90 + index, (seq, h["hidden"]))
    xd = torch.from_numpy(x).cuda()
    y = torch.empty_like(xd)
    _lib.call("reef_b200_gptneo_block_forward", C.byref(desc), xd.data_ptr(), y.data_ptr(),
              ws.data_ptr(), ws.numel(), st)
    torch.cuda.synchronize()
    want = ro.gptneo_block_w8a8(x, p, h["heads"], window=window, eps=h["eps"])
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_float_blob_is_unsupported():
    b = bytearray(BF.data())
    b[8:12] = (0).to_bytes(4, "little")  # precision kFloat32
    buf = C.create_string_buffer(bytes(b), len(b))
    arena = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    desc = _lib.GptNeoBlockDesc()
    rc = _lib.lib().reef_b200_blob_load_layer(buf, len(b), 0, arena.data_ptr(), arena.numel(),
                                              C.byref(desc), None)
    assert rc == 4  # REEF_B200_ERR_UNSUPPORTED
