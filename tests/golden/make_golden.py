"""Regenerates tests/golden/reference_kats.json from the reference's own tests.

Reads the TypeScript test sources of barhanc/wgpu-executorch as text (nothing
of the reference is executed) and extracts, per test case, the literal
expected-output arrays passed to ``expectTensorClose(out, [...], tol?)`` and
the literal ``toBeCloseTo`` expectations of the f16 mm test. The committed
JSON is what the tests read; this script only runs where the reference tree
is mounted:

    python tests/golden/make_golden.py /path/to/wgpu-executorch
"""
from __future__ import annotations

import json
import os
import re
import sys

FILES = {
    "mm": "tests/shaders/mm.test.ts",
    "convolution": "tests/shaders/convolution.test.ts",
    "conv_with_clamp": "tests/shaders/conv-with-clamp.test.ts",
    "program": "tests/api/program.test.ts",
}

IT_RE = re.compile(r"\bit\(\s*([`'\"])(.*?)\1\s*,", re.S)
EXPECT_RE = re.compile(r"expectTensorClose\(\s*out\s*,\s*\[(.*?)\]\s*(?:,\s*([0-9.e+-]+))?\s*\)",
                       re.S)
CLOSE_RE = re.compile(r"expect\(actual\[(\d+)\]\)\.toBeCloseTo\(([-0-9.e+]+)\s*,\s*(\d+)\)")


def extract(path: str):
    src = open(path).read()
    its = [(m.start(), m.group(2)) for m in IT_RE.finditer(src)]
    out = {}
    for i, (start, title) in enumerate(its):
        end = its[i + 1][0] if i + 1 < len(its) else len(src)
        body = src[start:end]
        line = src[:start].count("\n") + 1
        cases = []
        for m in EXPECT_RE.finditer(body):
            nums = [float(t) for t in re.findall(r"[-+]?\d+(?:\.\d+)?(?:e[-+]?\d+)?", m.group(1))]
            tol = float(m.group(2)) if m.group(2) else 1e-5
            cases.append({"expected": nums, "tolerance": tol})
        closes = [{"index": int(a), "value": float(b), "digits": int(c)}
                  for a, b, c in CLOSE_RE.findall(body)]
        if cases or closes:
            out[title] = {"line": line, "expectTensorClose": cases, "toBeCloseTo": closes}
    return out


def main(root: str) -> None:
    data = {"source": "barhanc/wgpu-executorch tests (literal expectations)", "files": {}}
    for key, rel in FILES.items():
        data["files"][key] = {"path": rel, "cases": extract(os.path.join(root, rel))}
    dst = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_kats.json")
    with open(dst, "w") as f:
        json.dump(data, f, indent=1)
    n = sum(len(v["cases"]) for v in data["files"].values())
    print(f"wrote {dst}: {n} test cases")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <reference checkout>")
    main(sys.argv[1])
