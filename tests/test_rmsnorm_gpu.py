"""The Llama RMSNorm + int8 kernel against the numpy float32 restatement of
its fixed summation order (tests/rms_ref.py), bit for bit.  The order is the
definition that makes the tensor-parallel shards (rms_stats / rms_apply)
reproduce TP=1 exactly: 8 chunks, 128 ordered partial sums per chunk, an xor
butterfly per 32 partials, then fixed trees.  No counterpart in reef (its
GPT-Neo block uses LayerNorm), so the restatement is the specification;
parity with a reference is unpinned.
"""
import numpy as np
import pytest
import torch

from reef_b200 import _lib

from tests.rms_ref import rmsnorm_quant_ref

pytestmark = pytest.mark.gpu
f32 = np.float32


# the config-3 hidden width, config-4's, a width whose chunks hold fewer
# float4 than the 128 partials, and an all-zero row
@pytest.mark.parametrize("rows,width", [(33, 4096), (9, 8192), (20, 1024), (5, 96)])
def test_rmsnorm_quant_exact(rows, width):
    rng = np.random.default_rng(rows + width)
    x = rng.normal(0, 1, (rows, width)).astype(f32)
    x[1] = 0
    gain = rng.normal(1, 0.1, width).astype(f32)
    xd, gd = torch.from_numpy(x).cuda(), torch.from_numpy(gain).cuda()
    q = torch.empty((rows, width), dtype=torch.int8, device="cuda")
    s = torch.empty(rows, device="cuda")
    _lib.call("reef_b200_rmsnorm_quant", rows, width, 1e-5, xd.data_ptr(), gd.data_ptr(),
              q.data_ptr(), s.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    wq, ws = rmsnorm_quant_ref(x, gain, 1e-5)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), ws.view(np.uint32))
    np.testing.assert_array_equal(q.cpu().numpy(), wq)
