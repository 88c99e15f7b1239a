"""Regenerate the golden fixtures from reef's own golden generator.

reef pins every Coral kernel with ``inference-engine/coral/host/gen_golden.cpp``:
it draws seeded inputs, runs the host engine on them and writes C++ headers of
hex-float / integer literals (``golden/<test>.hpp``).  This script compiles that
generator directly from the reference checkout with g++ (its own flags:
C++17, ``-ffp-contract=off``; the reference's CMake is not run), runs it into a
temporary directory, parses the headers and stores every array and case table
as ``tests/golden/<test>.npz`` plus ``tests/golden/<test>_cases.json``.

Only the headers on the W8A8 / int8 / attention path and its lm_head are
kept: ``linear`` (matvec_rows_f32 included), ``int8``, ``attention``, ``math``
(exp_nonpositive), ``layernorm`` (used by the GPT-Neo block) and
``elementwise`` (argmax).  The committed fixtures are what the tests read; this
script needs the reference checkout and runs here, never on a GPU box.

Usage:  python tests/golden/make_golden.py [--reference <reef checkout>]
"""
from __future__ import annotations

import argparse
import json
import os
import re
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
KEEP = ("linear", "int8", "attention", "math", "layernorm", "elementwise", "gpt_neo")

_DTYPES = {
    "float": np.float32,
    "std::int8_t": np.int8,
    "std::uint8_t": np.uint8,
    "std::int32_t": np.int32,
    "std::uint16_t": np.uint16,
    "std::uint32_t": np.uint32,
}

_DECL = re.compile(
    r"(?:alignas\(16\) )?inline constexpr ([\w:]+) (\w+)\[\] = \{(.*?)\n\};",
    re.S)
_CONST = re.compile(r"inline constexpr std::size_t (\w+) = (\d+);")


def _literal(tok: str, dtype):
    tok = tok.strip()
    if dtype is np.float32:
        return float.fromhex(tok.rstrip("F"))
    return int(tok.rstrip("U"))


def parse_header(text: str):
    arrays, tables = {}, {}
    for ctype, name, body in _DECL.findall(text):
        if ctype in _DTYPES:
            dtype = _DTYPES[ctype]
            toks = [t for t in body.replace("\n", " ").split(",") if t.strip()]
            arrays[name] = np.array([_literal(t, dtype) for t in toks],
                                    dtype=dtype)
        else:
            rows = []
            for line in body.strip().splitlines():
                line = line.strip().rstrip(",")
                assert line.startswith("{") and line.endswith("}"), line
                fields = [f.strip() for f in line[1:-1].split(",")]
                rows.append([int(f) if re.fullmatch(r"-?\d+", f) else
                             (float.fromhex(f.rstrip("F")) if f.startswith(("0x", "-0x"))
                              else f) for f in fields])
            tables[name] = {"type": ctype, "cases": rows}
    consts = {k: int(v) for k, v in _CONST.findall(text)}
    return arrays, tables, consts


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="the reef checkout (default: $REEF_REFERENCE, else a checkout "
                         "named 'reference' beside this repository)")
    args = ap.parse_args()
    if args.reference is None:
        sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(
            os.path.abspath(__file__)))))
        from oracle.oracle import reference_root
        args.reference = reference_root()
    if args.reference is None:
        print("reef checkout not found: pass --reference or set REEF_REFERENCE",
              file=sys.stderr)
        return 1
    ie = os.path.join(args.reference, "inference-engine")
    src = os.path.join(ie, "coral", "host", "gen_golden.cpp")
    if not os.path.exists(src):
        print(f"gen_golden.cpp not found under {args.reference}", file=sys.stderr)
        return 1
    with tempfile.TemporaryDirectory() as tmp:
        exe = os.path.join(tmp, "gen_golden")
        subprocess.run(
            ["g++", "-std=c++17", "-O2", "-ffp-contract=off",
             "-I", os.path.join(ie, "reference", "cpp", "include"),
             "-I", os.path.join(ie, "coral", "include"),
             "-I", os.path.join(ie, "coral", "host"), src, "-o", exe],
            check=True)
        subprocess.run([exe, tmp], check=True)
        for test in KEEP:
            with open(os.path.join(tmp, "golden", f"{test}.hpp")) as fh:
                arrays, tables, consts = parse_header(fh.read())
            np.savez_compressed(os.path.join(HERE, f"{test}.npz"), **arrays)
            with open(os.path.join(HERE, f"{test}_cases.json"), "w") as fh:
                json.dump({"source": "inference-engine/coral/host/gen_golden.cpp",
                           "tables": tables, "constants": consts}, fh,
                          indent=1)
            print(f"{test}: {len(arrays)} arrays, "
                  f"{sum(len(t['cases']) for t in tables.values())} cases")
    return 0


if __name__ == "__main__":
    sys.exit(main())
