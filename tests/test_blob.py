"""reef's packed model ("REEF" blob v1) read through the C ABI, on the CPU.

The fixture was written by reef's own packer (tests/golden/make_blob.py).
reef_b200_blob_read_info must return its header; malformed blobs (wrong
magic or version, truncated, an array running past the end or off its
16-byte alignment) must be refused.  Reading needs no GPU.
"""
import ctypes as C

import numpy as np

from reef_b200 import _lib
from tests import blob_fixture as BF


def read(b: bytes):
    info = _lib.BlobInfo()
    buf = C.create_string_buffer(b, len(b))
    rc = _lib.lib().reef_b200_blob_read_info(buf, len(b), C.byref(info))
    return rc, info


def test_header_of_reef_packed_blob():
    b = BF.data()
    cfg = BF.config()
    h = BF.header(b)
    rc, info = read(b)
    assert rc == 0
    assert h["magic"] == 0x46454552 and h["version"] == 1 and h["total_bytes"] == len(b)
    assert info.precision == 1  # W8A8
    assert (info.vocab, info.max_positions, info.hidden, info.layers, info.heads, info.inner,
            info.window) == (cfg["vocab"], cfg["positions"], cfg["hidden"], cfg["layers"],
                             cfg["heads"], cfg["inner"], cfg["window"])
    assert abs(info.eps - 1e-5) < 1e-12
    assert (info.wte, info.wpe, info.ln_f_weight, info.ln_f_bias) == (
        h["wte"], h["wpe"], h["ln_f_weight"], h["ln_f_bias"])
    need = _lib.lib().reef_b200_blob_layer_bytes(C.byref(info))
    d, f = cfg["hidden"], cfg["inner"]
    assert need >= 4 * d * d + 2 * d * f + 4 * (11 * d + 2 * f)


def test_malformed_blobs_are_refused():
    b = bytearray(BF.data())
    h = BF.header(bytes(b))
    bad = []
    x = bytearray(b)
    x[0] ^= 1  # magic
    bad.append(bytes(x))
    x = bytearray(b)
    x[4] = 2  # version
    bad.append(bytes(x))
    bad.append(bytes(b[: len(b) - 16]))  # shorter than total_bytes
    bad.append(bytes(b[:40]))  # shorter than the header
    x = bytearray(b)
    x[44:48] = (h["wte"] + 4).to_bytes(4, "little")  # wte off its 16-byte alignment
    bad.append(bytes(x))
    x = bytearray(b)
    x[48:52] = (len(b) - 16).to_bytes(4, "little")  # wpe runs past the end
    bad.append(bytes(x))
    x = bytearray(b)
    x[24:28] = (0).to_bytes(4, "little")  # no layers
    bad.append(bytes(x))
    for blob in bad:
        rc, _ = read(blob)
        assert rc == 1, rc  # REEF_B200_ERR_INVALID


def test_oracle_model_reproduces_reef_generation():
    """reef's kGptNeo golden (gen_golden.cpp:755-805): the W8A8 model generates
    20 tokens greedily from a 5-token prompt.  The oracle's blocks, final
    layernorm, tied lm_head and argmax over the whole sequence reproduce
    every logit bit for bit and every token -- the whole-model check the
    GPU decode loop is held to."""
    from oracle import oracle as ro
    blob, prompt, tokens, logits = BF.golden_model("w8a8")
    h = BF.header(blob)
    assert h["precision"] == 1 and h["total_bytes"] == len(blob)
    seq = np.concatenate([prompt, tokens[:-1]])
    got = BF.oracle_logits(blob, seq)[prompt.size - 1:]
    np.testing.assert_array_equal(got.view(np.uint32), logits.view(np.uint32))
    assert [ro.argmax_f32(r) for r in got] == list(tokens)


def test_model_loading_and_step_refuse_bad_arguments():
    """Argument checks that come before any device work (no GPU needed): the
    whole-model loader, the decode step, the cached block and the embedding
    refuse what the engine would throw on or what would run off a buffer."""
    L = _lib.lib()
    blob, prompt, _, _ = BF.golden_model("w8a8")
    rc, info = read(blob)
    assert rc == 0 and info.layers == 4
    need = L.reef_b200_blob_model_bytes(C.byref(info))
    assert need >= info.layers * L.reef_b200_blob_layer_bytes(C.byref(info))
    buf = C.create_string_buffer(blob, len(blob))
    model = _lib.GptNeoModelDesc()
    blocks = (_lib.GptNeoBlockDesc * info.layers)()
    fake = C.c_void_p(1 << 20)  # never dereferenced: each call fails its checks first
    # arena too small
    assert L.reef_b200_blob_load_model(buf, len(blob), fake, need - 256, C.byref(model), blocks,
                                       None, None) == 1
    # a W8A8 blob needs W8A8 blocks, a float blob float blocks
    assert L.reef_b200_blob_load_model(buf, len(blob), fake, need, C.byref(model), None, None,
                                       None) == 1
    fblob, _, _, _ = BF.golden_model("fp32")
    fbuf = C.create_string_buffer(fblob, len(fblob))
    rc, finfo = read(fblob)
    assert rc == 0 and finfo.precision == 0
    assert L.reef_b200_blob_model_bytes(C.byref(finfo)) > 0
    assert L.reef_b200_blob_load_model(fbuf, len(fblob), fake, 1 << 30, C.byref(model), blocks,
                                       None, None) == 1
    # the decode step: no model, no tokens, an empty model
    assert L.reef_b200_gptneo_step_workspace_bytes(None, 1) == 0
    assert L.reef_b200_gptneo_step(None, fake, 1, 0, fake, fake, 8, None, None, fake, 1 << 20,
                                   None) == 1
    empty = _lib.GptNeoModelDesc()
    assert L.reef_b200_gptneo_step_workspace_bytes(C.byref(empty), 1) == 0
    # the cached block: new rows past the cache
    blk = _lib.GptNeoBlockDesc()
    blk.seq = 4
    assert L.reef_b200_gptneo_block_forward_cached(C.byref(blk), fake, fake, 6, fake, fake, 8,
                                                   fake, 1 << 20, None) == 1
    # the embedding: positions past the table; nothing to do is fine
    assert L.reef_b200_embedding_f32(32, 4, fake, 30, 96, 32, fake, fake, fake, None) == 1
    assert L.reef_b200_embedding_f32(32, 0, fake, 30, 96, 32, fake, fake, fake, None) == 0


def test_oracle_float_model_reproduces_reef_generation():
    """The same kGptNeo golden at float precision: the oracle's exact float
    operators (linear with Coral's [in][out] weights, layernorm, the float
    head, gelu, residual adds, ln_f, lm_head) reproduce every logit and token."""
    from oracle import oracle as ro
    blob, prompt, tokens, logits = BF.golden_model("fp32")
    seq = np.concatenate([prompt, tokens[:-1]])
    got = BF.oracle_logits_f32(blob, seq)[prompt.size - 1:]
    np.testing.assert_array_equal(got.view(np.uint32), logits.view(np.uint32))
    assert [ro.argmax_f32(r) for r in got] == list(tokens)


def test_reader_survives_corrupted_blobs(tmp_path):
    """A blob is read from a file the caller may not control: corrupted ones
    must end in an error status, never a read outside the blob or a write
    outside the arena.  blob.cpp is compiled with AddressSanitizer over
    host-side copies (tests/host/blob_fuzz_test.cpp) and fed the layer
    fixture and both kGptNeo models (W8A8 and fp32): each must load intact,
    then 4000 seeded corruptions each (header and layer-table fields set to
    boundary and random values, truncations, flipped bytes) go through
    read_info and, where it accepts them, the layer and model loads."""
    import os

    from reef_b200 import build
    from tests.test_comm_host import HERE, _build_and_run
    paths = [BF.BLOB]
    for precision in ("w8a8", "fp32"):
        blob, _, _, _ = BF.golden_model(precision)
        p = tmp_path / f"kgptneo_{precision}.blob"
        p.write_bytes(blob)
        paths.append(str(p))
    passed = _build_and_run(tmp_path, "blob_fuzz_test", [
        os.path.join(build.CSRC, "blob.cpp"), os.path.join(HERE, "host", "blob_fuzz_test.cpp")],
        sanitize=True, args=tuple(paths))
    assert {line.split()[0] for line in passed} == set(paths)
