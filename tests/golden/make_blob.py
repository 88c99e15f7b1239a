"""Write tests/golden/gptneo_w8a8.blob: a small GPT-Neo model packed by reef.

reef's own code makes it, compiled in place into oracle/_ref (needs the
reference checkout, so it runs here, never on a GPU box): random_gpt_neo
(weights.hpp:407), quantize_w8a8 (weights.hpp:460) and the firmware packer
pack_gpt_neo with Precision::kW8A8 (coral/host/pack_model.hpp:88-160).  The
blob is the "REEF" v1 layout of coral/include/reef_kernels/model_blob.hpp.
The shape is small (vocab 96, 48 positions, hidden 64, 2 layers -- one
global, one local -- 4 heads, inner 256, window 8) so the fixture stays
near 100 KB; the tests parse it independently and run its layers.

Usage:  python tests/golden/make_blob.py
"""
from __future__ import annotations

import ctypes as C
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as ro  # noqa: E402

CONFIG = dict(vocab=96, positions=48, hidden=64, layers=2, heads=4, inner=256, window=8, seed=2024)


def main() -> None:
    ro.build(reference=True)
    R = ro.ref()
    cap = 1 << 22
    buf = (C.c_uint8 * cap)()
    size = C.c_size_t(0)
    c = CONFIG
    rc = R.ref_pack_random_gpt_neo(c["vocab"], c["positions"], c["hidden"], c["layers"],
                                   c["heads"], c["inner"], c["window"], c["seed"], buf, cap,
                                   C.byref(size))
    if rc != 0 or size.value > cap:
        raise SystemExit(f"packer failed: rc {rc}, size {size.value}")
    with open(os.path.join(HERE, "gptneo_w8a8.blob"), "wb") as fh:
        fh.write(bytes(buf[:size.value]))
    with open(os.path.join(HERE, "gptneo_w8a8.json"), "w") as fh:
        json.dump(dict(c, bytes=size.value), fh, indent=1)
    print(f"gptneo_w8a8.blob: {size.value} bytes")


if __name__ == "__main__":
    main()
