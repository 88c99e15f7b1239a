"""reef's packed "REEF" v1 model blobs, parsed here with numpy alone,
independently of the library's C++ reader: the header and layer records of
coral/include/reef_kernels/model_blob.hpp:18-66, each layer's arrays in the
engine's [out][in] layout keyed as the oracle's GPT-Neo block takes them, and
the model-level arrays (wte, wpe, ln_f).

Two blobs are committed, both written by reef's own packer: the layer fixture
tests/golden/gptneo_w8a8.blob (tests/golden/make_blob.py) and the W8A8 model
of reef's kGptNeo golden (gen_golden.cpp:755-805, in tests/golden/gpt_neo.npz
with its prompt, generated tokens and the logits behind each token).  An
oracle forward of a whole model over a token sequence is here too."""
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


def golden_model(precision: str = "w8a8"):
    """(blob bytes, prompt, tokens, logits [tokens][vocab]) of reef's kGptNeo
    golden case for ``precision`` ("fp32" or "w8a8")."""
    from tests import goldens
    (c,) = [c for c in goldens.cases("gpt_neo", "kGptNeo")
            if header(c["blob"].astype("<u4").tobytes())["precision"] == (precision == "w8a8")]
    blob = c["blob"].astype("<u4").tobytes()
    assert c["prompt"].size == c["prompt_length"] and c["tokens"].size == c["new_tokens"]
    logits = c["logits"].reshape(c["new_tokens"], c["vocab_size"])
    return blob, c["prompt"].astype(np.uint32), c["tokens"].astype(np.uint32), logits


def model_arrays(b: bytes) -> dict:
    """wte [vocab][hidden], wpe [positions][hidden], ln_f gain and shift."""
    h = header(b)
    v, n, d = h["vocab"], h["max_positions"], h["hidden"]

    def floats(off, count):
        return np.frombuffer(b, np.float32, count, off).copy()

    return {"wte": floats(h["wte"], v * d).reshape(v, d),
            "wpe": floats(h["wpe"], n * d).reshape(n, d),
            "ln_f_g": floats(h["ln_f_weight"], d), "ln_f_b": floats(h["ln_f_bias"], d)}


def oracle_logits(b: bytes, tokens) -> np.ndarray:
    """The engine's GPTNeo forward over ``tokens`` at positions 0.. (W8A8
    blocks; model.hpp's embedding add, final layernorm and tied lm_head),
    restated with the oracle: logits [len(tokens)][vocab]."""
    from oracle import oracle as ro
    h = header(b)
    m = model_arrays(b)
    ids = np.asarray(tokens, np.int64)
    x = (m["wte"][ids] + m["wpe"][np.arange(ids.size)]).astype(np.float32)
    for i in range(h["layers"]):
        p, local = layer(b, i)
        x = ro.gptneo_block_w8a8(x, p, h["heads"], window=h["window"] if local else 0,
                                 eps=h["eps"])
    normed = ro.layernorm(x, m["ln_f_g"], m["ln_f_b"], h["eps"])
    out = np.empty((ids.size, h["vocab"]), np.float32)
    for t in range(ids.size):
        out[t], ok = ro.matvec_rows_f32(m["wte"], normed[t])
        assert ok
    return out


def layer_f32(b: bytes, index: int):
    """(float layer arrays, is_local) of a float (precision 0) blob: weights
    kept in the blob's [in][out] layout (Coral's linear_f32 takes them so)."""
    h = header(b)
    assert h["precision"] == 0
    r = dict(zip(LAYER_FIELDS, struct.unpack_from("<20I", b, h["layer_table"] + 80 * index)))
    d, f = h["hidden"], h["inner"]

    def floats(off, *shape):
        return np.frombuffer(b, np.float32, int(np.prod(shape)), off).reshape(shape).copy()

    p = {"ln1_g": floats(r["ln_1_weight"], d), "ln1_b": floats(r["ln_1_bias"], d),
         "wq": floats(r["q_w"], d, d), "wk": floats(r["k_w"], d, d), "wv": floats(r["v_w"], d, d),
         "wo": floats(r["o_w"], d, d), "bo": floats(r["o_b"], d),
         "ln2_g": floats(r["ln_2_weight"], d), "ln2_b": floats(r["ln_2_bias"], d),
         "wfc": floats(r["fc_w"], d, f), "bfc": floats(r["fc_b"], f),
         "wproj": floats(r["proj_w"], f, d), "bproj": floats(r["proj_b"], d)}
    return p, bool(r["is_local"])


def oracle_logits_f32(b: bytes, tokens) -> np.ndarray:
    """The engine's float GPTNeo forward over ``tokens`` (the firmware's
    kFloat32 step, gpt_neo.cc:123-188, on every position), restated with the
    oracle's exact float operators: logits [len(tokens)][vocab]."""
    from oracle import oracle as ro
    h = header(b)
    m = model_arrays(b)
    ids = np.asarray(tokens, np.int64)
    T, d, H = ids.size, h["hidden"], h["heads"]
    hd = d // H
    x = (m["wte"][ids] + m["wpe"][np.arange(T)]).astype(np.float32)
    for i in range(h["layers"]):
        p, local = layer_f32(b, i)
        win = h["window"] if local else 0
        n1 = ro.layernorm(x, p["ln1_g"], p["ln1_b"], h["eps"])
        q, k, v = (ro.linear_f32(n1, p[w]) for w in ("wq", "wk", "wv"))
        ctx = np.empty_like(q)
        for j in range(H):
            sl = slice(j * hd, (j + 1) * hd)
            ctx[:, sl] = ro.attention_head_f32(q[:, sl], k[:, sl], v[:, sl], 0, win)
        x = (x + ro.linear_f32(ctx, p["wo"], p["bo"])).astype(np.float32)
        n2 = ro.layernorm(x, p["ln2_g"], p["ln2_b"], h["eps"])
        f = ro.gelu(ro.linear_f32(n2, p["wfc"], p["bfc"]))
        x = (x + ro.linear_f32(f, p["wproj"], p["bproj"])).astype(np.float32)
    normed = ro.layernorm(x, m["ln_f_g"], m["ln_f_b"], h["eps"])
    out = np.empty((T, h["vocab"]), np.float32)
    for t in range(T):
        out[t], ok = ro.matvec_rows_f32(m["wte"], normed[t])
        assert ok
    return out


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
