"""The C++ binding a reef maintainer would add compiles against reef.

INTEGRATION.md's first C++ block is the drop-in `kernels_b200.cc`: reef's
own `reef_kernels` signatures (coral/include/reef_kernels/kernels.hpp) with
bodies that forward to this library's C ABI (include/reef_b200.h).  This
test extracts it and compiles it with g++ against both headers, so a change
to either side that breaks the binding fails here; the later snippets (weight
packing, blob loading, the decode loop) are compiled as function bodies
against the C ABI.  It needs the reef checkout (REEF_REFERENCE) and the CUDA
headers, and is skipped without them.
"""
import os
import re
import shutil
import subprocess

import pytest

from oracle.oracle import reference_root

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = reference_root() or ""
CORAL_INC = os.path.join(REF, "inference-engine", "coral", "include")
CUDA_INC = "/usr/local/cuda/include"


def test_integration_shim_compiles_against_reef_kernels(tmp_path):
    if not os.path.isfile(os.path.join(CORAL_INC, "reef_kernels", "kernels.hpp")):
        pytest.skip("reef checkout not present")
    if shutil.which("g++") is None or not os.path.isdir(CUDA_INC):
        pytest.skip("g++ or the CUDA headers not present")
    with open(os.path.join(ROOT, "INTEGRATION.md")) as fh:
        blocks = re.findall(r"```cpp\n(.*?)```", fh.read(), re.S)
    assert blocks and "namespace reef_kernels" in blocks[0]
    src = tmp_path / "kernels_b200.cc"
    src.write_text(blocks[0])
    p = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Werror",
                        "-I", os.path.join(ROOT, "include"), "-I", CORAL_INC, "-I", CUDA_INC,
                        str(src)], capture_output=True, text=True)
    assert p.returncode == 0, p.stderr[-3000:]


# the free names the later snippets use, as parameters of the function each
# one is compiled in (names a snippet declares itself are left out)
_PARAMS = ("size_t in, size_t out, const int8_t* wt_dev, reef_b200_stream_t stream, "
           "const void* blob, size_t blob_bytes, size_t seq, void* arena, "
           "const uint32_t* ids_dev, size_t prompt_len, float* k_cache, float* v_cache, "
           "size_t max_tokens, uint32_t* next_dev, void* ws, size_t ws_bytes, "
           "size_t new_tokens")


def test_integration_snippets_compile(tmp_path):
    if shutil.which("g++") is None or not os.path.isdir(CUDA_INC):
        pytest.skip("g++ or the CUDA headers not present")
    with open(os.path.join(ROOT, "INTEGRATION.md")) as fh:
        blocks = re.findall(r"```cpp\n(.*?)```", fh.read(), re.S)[1:]
    assert len(blocks) >= 3
    parts = ["#include \"reef_b200.h\"", "#include <cuda_runtime.h>", "#include <cstddef>",
             "#include <cstdint>", "#include <vector>", "void check(int);"]
    for i, body in enumerate(blocks):
        extra = "" if "reef_b200_blob_info info;" in body or "info" not in body else \
            ", const reef_b200_blob_info& info"
        parts.append(f"void snippet_{i}({_PARAMS}{extra}) {{\n{body}}}")
    src = tmp_path / "snippets.cc"
    src.write_text("\n".join(parts) + "\n")
    p = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-Wall", "-Werror",
                        "-I", os.path.join(ROOT, "include"), "-I", CUDA_INC, str(src)],
                       capture_output=True, text=True)
    assert p.returncode == 0, p.stderr[-3000:]
