"""Extracts the literal golden vectors of the reference's CPU gtest suite.

    python tests/golden/extract_reference_goldens.py [REFERENCE_ROOT]

Reads tests/gpt2/test_{matmul,attention,layernorm,gelu,residual,
cross_entropy,encoder}.cpp of the reference as TEXT (nothing is compiled or
run) and writes tests/golden/reference_unit_vectors.json:

    {"<file>::<TEST name>": {"<C++ target expression>": [numbers...], ...}}

Numbers come from Eigen comma initialisers (`x << a, b, ...;`) and brace
initialisers (`Matf{{...},{...}}`, `VecBTC v{Matf{...}, Matf{...}}`), in
row-major order, which is the order Eigen fills them. The values are the
PyTorch outputs the reference's notebooks produced (tests/gpt2/*_note.ipynb in the reference tree).
"""
from __future__ import annotations

import json
import os
import re
import sys

FILES = ["test_matmul.cpp", "test_attention.cpp", "test_layernorm.cpp", "test_gelu.cpp", "test_residual.cpp",
         "test_cross_entropy.cpp", "test_encoder.cpp"]
NUM = re.compile(r"(?<![\w\]])-?\d+(?:\.\d*)?(?:[eE][-+]?\d+)?")


def strip_comments(s: str) -> str:
    s = re.sub(r"/\*.*?\*/", "", s, flags=re.S)
    return re.sub(r"//[^\n]*", "", s)


def test_bodies(src: str):
    for m in re.finditer(r"TEST_F\(\s*(\w+)\s*,\s*(\w+)\s*\)\s*\{", src):
        i, depth = m.end(), 1
        while depth:
            depth += {"{": 1, "}": -1}.get(src[i], 0)
            i += 1
        yield m.group(2), src[m.end():i - 1]


def numbers(text: str) -> list[float]:
    return [float(x) for x in NUM.findall(text)]


def parse_body(body: str) -> dict[str, list[float]]:
    out: dict[str, list[float]] = {}
    for stmt in body.split(";"):
        stmt = stmt.strip()
        m = re.match(r"EXPECT_NEAR\((.*),\s*([-\d\.eE+f]+)\s*,\s*([-\d\.eE+f]+)\s*\)$", stmt, flags=re.S)
        if m:
            # expected scalar and tolerance of EXPECT_NEAR(expr, expected, tol)
            out.setdefault("EXPECT_NEAR", []).append(
                [m.group(1).strip(), float(m.group(2).rstrip("f")), float(m.group(3).rstrip("f"))])
            continue
        if "<<" in stmt:
            # `a << 1, 2, b << 3, 4` (a typo in one reference test) is two fills.
            parts = re.split(r"([\w\.\[\]]+)\s*<<", stmt)
            # parts: [prefix, target1, values1, target2, values2, ...]
            for k in range(1, len(parts) - 1, 2):
                tgt = parts[k].strip()
                vals = parts[k + 1]
                vals = re.sub(r",\s*$", "", vals.strip())
                out[tgt] = numbers(vals)
        elif re.search(r"Matf\s*\{", stmt):
            m = re.match(r"(?:[\w:<>]+\s+)?([\w\.]+)\s*(?:=\s*)?(?:Matf\s*)?\{", stmt)
            if not m:
                continue
            name = m.group(1)
            out[name] = numbers(stmt[m.end() - 1:])
    return out


def main(root: str) -> None:
    res = {}
    for fn in FILES:
        path = os.path.join(root, "tests", "gpt2", fn)
        src = strip_comments(open(path).read())
        for name, body in test_bodies(src):
            res[f"{fn}::{name}"] = parse_body(body)
    here = os.path.dirname(os.path.abspath(__file__))
    with open(os.path.join(here, "reference_unit_vectors.json"), "w") as f:
        json.dump(res, f, indent=1)
    for k, v in res.items():
        print(k, {n: len(x) for n, x in v.items()})


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LLMK_REFERENCE_DIR")
    if not root:
        sys.exit("usage: extract_reference_goldens.py REFERENCE_ROOT (or set LLMK_REFERENCE_DIR)")
    main(root)
