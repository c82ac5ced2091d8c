#!/usr/bin/env python3
"""Extracts the reference's Conv2D golden vectors into a JSON fixture.

The reference keeps its PyTorch-generated goldens as C++ arrays in
tests/data/traditional_reference.h (written by the reference's
tests/reference/gen_traditional_fixtures.py, seed 20261114, float32).  This
script reads that header as text and writes tests/golden/traditional_conv.json
with the Conv2D and DepthwiseConv2D arrays, so the test suite needs neither the
reference tree nor PyTorch to use them.

    python tests/golden/make_golden.py [/path/to/reference]
"""
import json
import re
import sys
from pathlib import Path

NAMES = {
    # name: shape, as declared in the header comments
    "kConvInput": [1, 2, 5, 5],
    "kConvWeight": [3, 2, 3, 3],
    "kConvBias": [3],
    "kConvExpected": [1, 3, 5, 5],
    "kDepthwiseInput": [1, 2, 3, 3],
    "kDepthwiseWeight": [2, 1, 2, 2],
    "kDepthwiseBias": [2],
    "kDepthwiseExpected": [1, 2, 2, 2],
}


def parse(header: str) -> dict:
    out = {}
    for name, shape in NAMES.items():
        m = re.search(r"%s\[(\d+)\]\s*=\s*\{(.*?)\};" % name, header, re.S)
        if m is None:
            raise SystemExit(f"{name} not found")
        vals = [float(v.strip().rstrip("f")) for v in m.group(2).split(",") if v.strip()]
        count = 1
        for d in shape:
            count *= d
        if len(vals) != int(m.group(1)) or len(vals) != count:
            raise SystemExit(f"{name}: size mismatch")
        out[name] = {"shape": shape, "values": vals}
    return out


def main() -> None:
    ref = Path(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
    src = ref / "tests/data/traditional_reference.h"
    data = parse(src.read_text())
    data["_source"] = "tests/data/traditional_reference.h (reference), read as text"
    dst = Path(__file__).resolve().parent / "traditional_conv.json"
    dst.write_text(json.dumps(data) + "\n")
    print(f"wrote {dst}")


if __name__ == "__main__":
    main()
