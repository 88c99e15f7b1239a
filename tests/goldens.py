"""Loader for the committed golden fixtures (tests/golden/*.npz + *_cases.json).

The fixtures are reef's own golden vectors: tests/golden/make_golden.py
compiles the reference generator (inference-engine/coral/host/gen_golden.cpp)
and converts its headers.  Each case is returned as a dict with named fields,
the field names following the struct each table fills in
inference-engine/coral/tests/cases.hpp.
"""
from __future__ import annotations

import functools
import json
import os

import numpy as np

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

FIELDS = {
    "kW8a8": ("rows", "in", "out", "x", "qt", "qs", "y"),
    "kW8a8Bias": ("rows", "in", "out", "x", "qt", "qs", "bias", "y"),
    "kInt8Linear": ("rows", "in", "out", "shift", "x", "wt", "y"),
    "kInt8LinearBias": ("rows", "in", "out", "shift", "x", "wt", "bias", "y"),
    "kInt8Softmax": ("rows", "n", "shift", "table", "scores", "probs"),
    "kInt8Attention": ("query_len", "key_len", "head_dim", "query_start",
                       "window", "score_shift", "out_shift", "table", "q", "k",
                       "v", "y"),
    "kAttention": ("query_len", "key_len", "head_dim", "query_start",
                   "window", "q", "k", "v", "y"),
    "kExp": ("n", "x", "y"),
    "kTanh": ("n", "x", "y"),
    "kGelu": ("n", "x", "y"),
    "kLayerNorm": ("rows", "width", "eps", "x", "gain", "shift", "y"),
    "kMatvec": ("out", "in", "w", "x", "y"),
    "kArgmax": ("n", "x", "index"),
    "kAdd": ("n", "a", "b", "y"),
    "kLinear": ("rows", "in", "out", "x", "wt", "y"),
    "kLinearBias": ("rows", "in", "out", "x", "wt", "bias", "y"),
    "kInt8Gelu": ("n", "table", "x", "y"),
    "kInt8LayerNorm": ("rows", "width", "x", "gain", "shift", "y"),
    "kInt8Add": ("n", "a", "b", "y"),
    "kInt8Embedding": ("width", "id", "position", "wte", "wpe", "y"),
    "kEmbedding": ("width", "id", "position", "wte", "wpe", "y"),
    "kGptNeo": ("blob", "prompt_length", "prompt", "new_tokens", "tokens", "vocab_size",
                "logits"),
}


@functools.lru_cache(maxsize=None)
def _load(test: str):
    arrays = dict(np.load(os.path.join(HERE, f"{test}.npz")))
    with open(os.path.join(HERE, f"{test}_cases.json")) as fh:
        meta = json.load(fh)
    return arrays, meta


def cases(test: str, table: str):
    arrays, meta = _load(test)
    names = FIELDS[table]
    out = []
    for row in meta["tables"][table]["cases"]:
        assert len(row) == len(names), (table, row)
        case = {}
        for name, value in zip(names, row):
            case[name] = arrays[value] if isinstance(value, str) else value
        out.append(case)
    return out
