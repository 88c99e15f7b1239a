"""The committed "REEF" blob fixture (tests/golden/gptneo_w8a8.blob, written
by reef's packer: tests/golden/make_blob.py), parsed here with numpy alone,
independently of the library's C++ reader: the header and layer records of
coral/include/reef_kernels/model_blob.hpp:18-66 and each layer's arrays in
the engine's [out][in] layout, keyed as the oracle's GPT-Neo block takes
them."""
from __future__ import annotations

import json
import os
import struct

import numpy as np

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
BLOB = os.path.join(HERE, "gptneo_w8a8.blob")

HEADER_FIELDS = ("magic", "version", "precision", "vocab", "max_positions", "hidden", "layers",
                 "heads", "inner", "window", "eps", "wte", "wpe", "ln_f_weight", "ln_f_bias",
                 "layer_table", "total_bytes")
LAYER_FIELDS = ("ln_1_weight", "ln_1_bias", "q_w", "q_s", "k_w", "k_s", "v_w", "v_s", "o_w",
                "o_s", "o_b", "ln_2_weight", "ln_2_bias", "fc_w", "fc_s", "fc_b", "proj_w",
                "proj_s", "proj_b", "is_local")


def data() -> bytes:
    with open(BLOB, "rb") as fh:
        return fh.read()


def config() -> dict:
    with open(os.path.join(HERE, "gptneo_w8a8.json")) as fh:
        return json.load(fh)


def header(b: bytes) -> dict:
    return dict(zip(HEADER_FIELDS, struct.unpack_from("<10If6I", b, 0)))


def layer(b: bytes, index: int):
    """(block weights for the oracle, is_local) of one layer."""
    h = header(b)
    r = dict(zip(LAYER_FIELDS, struct.unpack_from("<20I", b, h["layer_table"] + 80 * index)))
    d, f = h["hidden"], h["inner"]

    def floats(off, n):
        return np.frombuffer(b, np.float32, n, off).copy()

    def weight(off, n_in, n_out):  # stored [in][out] -> [out][in]
        return np.ascontiguousarray(np.frombuffer(b, np.int8, n_in * n_out, off)
                                    .reshape(n_in, n_out).T)

    p = {"ln1_g": floats(r["ln_1_weight"], d), "ln1_b": floats(r["ln_1_bias"], d),
         "wq": weight(r["q_w"], d, d), "sq": floats(r["q_s"], d),
         "wk": weight(r["k_w"], d, d), "sk": floats(r["k_s"], d),
         "wv": weight(r["v_w"], d, d), "sv": floats(r["v_s"], d),
         "wo": weight(r["o_w"], d, d), "so": floats(r["o_s"], d), "bo": floats(r["o_b"], d),
         "ln2_g": floats(r["ln_2_weight"], d), "ln2_b": floats(r["ln_2_bias"], d),
         "wfc": weight(r["fc_w"], d, f), "sfc": floats(r["fc_s"], f), "bfc": floats(r["fc_b"], f),
         "wproj": weight(r["proj_w"], f, d), "sproj": floats(r["proj_s"], d),
         "bproj": floats(r["proj_b"], d)}
    return p, bool(r["is_local"])
