"""The C ABI loads and exports every symbol include/reef_b200.h declares.

CPU only: no call here reaches the GPU (only argument validation that returns
before any CUDA call, and pure helpers).
"""
import ctypes as C
import os

import pytest

from reef_b200 import _lib


@pytest.fixture(scope="module")
def L():
    return _lib.lib()


def test_exports_every_declared_symbol(L):
    declared = _lib.header_functions()
    assert declared, "header declares nothing"
    missing = [f for f in declared if not hasattr(L, f)]
    assert not missing, f"declared but not exported: {missing}"


def test_binding_covers_the_header():
    declared = set(_lib.header_functions())
    assert declared == set(_lib.SIGNATURES), (
        declared ^ set(_lib.SIGNATURES))


def _declared_arity() -> dict:
    """Parameter count of every function the header declares."""
    import re
    with open(_lib.HEADER) as fh:
        text = re.sub(r"/\*.*?\*/", "", fh.read(), flags=re.S)
    out = {}
    for m in re.finditer(r"\b(reef_b200_\w+)\s*\(([^;{]*?)\)\s*;", text):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_binding_arity_matches_the_header():
    arity = _declared_arity()
    assert set(arity) == set(_lib.SIGNATURES)
    wrong = {f: (arity[f], len(_lib.SIGNATURES[f][0])) for f in arity
             if arity[f] != len(_lib.SIGNATURES[f][0])}
    assert not wrong, f"header vs binding argument counts: {wrong}"


def test_pure_helpers(L):
    assert L.reef_b200_version() >= 200
    assert [L.reef_b200_kpad(n) for n in (1, 7, 16, 17, 4096, 11008)] == \
        [16, 16, 16, 32, 4096, 11008]
    assert L.reef_b200_status_string(0) == b"ok"
    assert b"invalid" in L.reef_b200_status_string(1)


def test_argument_validation_without_gpu(L):
    p = C.c_void_p(16)  # never dereferenced: validation fails or rows == 0 first
    # rows == 0 is a no-op, as the Coral loops are
    assert L.reef_b200_linear_w8a8(0, 8, 8, p, p, p, p, p, p, None) == 0
    assert L.reef_b200_linear_int8(0, 8, 8, p, p, 3, p, None) == 0
    # empty feature dims and null pointers are invalid (the engine rejects them)
    assert L.reef_b200_linear_w8a8(4, 0, 8, p, p, p, p, p, p, None) == 1
    assert L.reef_b200_linear_w8a8(4, 8, 0, p, p, p, p, p, p, None) == 1
    assert L.reef_b200_linear_w8a8(4, 8, 8, None, p, p, p, p, p, None) == 1
    assert L.reef_b200_gemm_w8a8(4, 8, 8, p, p, p, None, None, p, None) == 1
    # shifts above 31 are not a rounding_shift the engine defines
    assert L.reef_b200_linear_int8(4, 8, 8, p, p, 32, p, None) == 1
    assert L.reef_b200_quantize_rows(4, 0, p, p, p, None) == 1
    # the no-allocation linear refuses, before any CUDA call, the first shape
    # past its fixed scratch: 4093 rows of 4096 need 16,781,300 bytes of 16 MiB
    assert L.reef_b200_linear_w8a8_noalloc(4093, 4096, 8, p, p, p, None, p, None) == 7
    assert L.reef_b200_linear_w8a8_noalloc(256, 65536, 8, p, p, p, None, p, None) == 7


def test_decode_tiles_and_peer_wait_validation_without_gpu(L):
    p = C.c_void_p(16)
    # the decode layout: one 16 KiB block (128 rows x 128 bytes of K) per tile,
    # ragged edges rounded up to whole tiles
    assert L.reef_b200_weight_tiles_bytes(1280, 8192) == 10 * 64 * 16384
    assert L.reef_b200_weight_tiles_bytes(1, 1) == 16384
    assert L.reef_b200_weight_tiles_bytes(129, 130) == 2 * 2 * 16384
    assert L.reef_b200_weight_tiles_bytes(0, 8192) == 0
    assert L.reef_b200_weight_tiles_bytes(1280, 0) == 0
    # packing: no rows is a no-op; null pointers are invalid; the tiles'
    # base must be 1024-byte aligned, as the header requires
    assert L.reef_b200_pack_weight_tiles(0, 8192, p, p, None) == 0
    assert L.reef_b200_pack_weight_tiles(128, 128, None, C.c_void_p(1024), None) == 1
    assert L.reef_b200_pack_weight_tiles(128, 128, p, C.c_void_p(1024 + 16), None) == 2
    # the cross-rank wait's self-test: a counter and a limit of 1 us .. 2 s
    assert L.reef_b200_selftest_peer_wait_timeout(1000, None, 1, None) == 1
    assert L.reef_b200_selftest_peer_wait_timeout(0, p, 1, None) == 1
    assert L.reef_b200_selftest_peer_wait_timeout(2000001, p, 1, None) == 1


def test_layer_shapes_are_bounded_without_gpu(L):
    """The layer descriptions' workspace queries are arithmetic only: a
    config-3 layer and config 2's GPT-Neo block get a size; widths past the
    bounds, and a batch x seq whose product wraps around, get 0 (invalid)
    instead of a wrapped-around, too small workspace."""
    p = C.c_void_p(1 << 20)  # aligned, never dereferenced
    ptrs = {f: p for f in ("attn_norm", "w_qkv", "s_qkv", "w_o", "s_o", "mlp_norm", "w_gu",
                           "s_gu", "w_down", "s_down")}

    def llama(**over):
        kw = dict(batch=8, seq=2048, hidden=4096, heads_q=32, heads_kv=32, head_dim=128,
                  ffn=11008, rms_eps=1e-5, rope_base=1e4, **ptrs)
        kw.update(over)
        return L.reef_b200_llama_layer_workspace_bytes(C.byref(_lib.LlamaLayerDesc(**kw)))

    assert llama() > 0
    assert llama(hidden=1 << 21) == 0
    assert llama(ffn=1 << 23) == 0
    assert llama(heads_q=8192, heads_kv=8192) == 0
    assert llama(batch=1 << 62, seq=256) == 0  # 2^70 tokens wraps to 0 in 64 bits
    assert llama(batch=1 << 20, seq=1 << 11) == 0  # 2^31 tokens

    def neo(**over):
        kw = dict(seq=128, hidden=256, heads=4, head_dim=64, ffn=1024, window=0, eps=1e-5)
        kw.update({f: p for f in ("ln1_g", "ln1_b", "wq", "sq", "wk", "sk", "wv", "sv", "wo",
                                  "so", "bo", "ln2_g", "ln2_b", "wfc", "sfc", "bfc", "wproj",
                                  "sproj", "bproj")})
        kw.update(over)
        return L.reef_b200_gptneo_block_workspace_bytes(C.byref(_lib.GptNeoBlockDesc(**kw)))

    assert neo() > 0
    assert neo(hidden=1 << 21) == 0
    assert neo(head_dim=8192) == 0


def test_attention_validation_without_gpu(L):
    p = C.c_void_p(16)
    # a row that sees no key: query 9 at window 3 over 5 keys
    assert L.reef_b200_attention_head_int8(1, 5, 8, 9, 3, p, 8, p, p, 4, p, 8,
                                           None, None, p, 8, None) == 1
    assert L.reef_b200_attention_head_f32(1, 5, 8, 9, 3, p, 8, p, p, None, p, 8, None) == 1
    # no keys at all
    assert L.reef_b200_attention_head_f32(1, 0, 8, 0, 0, p, 8, p, p, None, p, 8, None) == 1
    # longer than the shared-memory score buffer
    assert L.reef_b200_attention_head_int8(1, 40000, 8, 0, 0, p, 8, p, p, 4, p, 8,
                                           None, None, p, 8, None) == 7
    # empty query is a no-op
    assert L.reef_b200_attention_head_f32(0, 5, 8, 0, 0, p, 8, p, p, None, p, 8, None) == 0


def test_header_is_c99_and_links_from_c(tmp_path):
    """The boundary is a C ABI: a strict C99 program (the language cgo, JNI
    and other FFI stubs bind through) includes the header, links the library
    and calls an entry point that needs no GPU."""
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("gcc not present")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    src = tmp_path / "c_abi.c"
    src.write_text('#include "reef_b200.h"\n'
                   "int main(void) { return reef_b200_version() >= 200 && "
                   "reef_b200_kpad(17) == 32 ? 0 : 1; }\n")
    exe = tmp_path / "c_abi"
    libdir = os.path.join(root, "reef_b200")
    cc = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                         "-I", os.path.join(root, "include"), str(src), "-L", libdir,
                         "-lreef_b200", f"-Wl,-rpath,{libdir}", "-o", str(exe)],
                        capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr[-2000:]
    assert subprocess.run([str(exe)]).returncode == 0
