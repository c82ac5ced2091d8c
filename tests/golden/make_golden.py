#!/usr/bin/env python3
"""Extracts the reference's golden vectors into fixtures under tests/golden/.

The reference keeps its PyTorch / ONNX Runtime goldens as C++ arrays in
tests/data/*.h (written by the reference's
tests/reference/gen_traditional_fixtures.py).  This script reads those headers
as text and writes
  traditional_conv.json  the Conv2D and DepthwiseConv2D arrays
                         (traditional_reference.h, seed 20261114, float32)
  tiny_cnn.json          the tiny CNN's input and ONNX Runtime logits
                         (tiny_cnn_reference.h)
  tiny_cnn.onnx          the tiny CNN model those logits belong to (the
                         reference's tests/data/tiny_cnn.onnx, byte for byte)
so the test suite needs neither the reference tree nor PyTorch to use them.

    python tests/golden/make_golden.py [/path/to/reference]

The reference root defaults to $IE_REFERENCE_ROOT, else /root/reference.
"""
import json
import os
import re
import shutil
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


TINY_CNN = {
    "kTinyCnnInput": [1, 3, 8, 8],
    "kTinyCnnExpected": [1, 3],
}


def parse(header: str, names: dict = NAMES) -> dict:
    out = {}
    for name, shape in names.items():
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
    ref = Path(sys.argv[1] if len(sys.argv) > 1
               else os.environ.get("IE_REFERENCE_ROOT", "/root/reference"))
    here = Path(__file__).resolve().parent
    src = ref / "tests/data/traditional_reference.h"
    data = parse(src.read_text())
    data["_source"] = "tests/data/traditional_reference.h (reference), read as text"
    dst = here / "traditional_conv.json"
    dst.write_text(json.dumps(data) + "\n")
    print(f"wrote {dst}")
    tiny = parse((ref / "tests/data/tiny_cnn_reference.h").read_text(), TINY_CNN)
    tiny["_source"] = "tests/data/tiny_cnn_reference.h (reference), read as text"
    (here / "tiny_cnn.json").write_text(json.dumps(tiny) + "\n")
    shutil.copyfile(ref / "tests/data/tiny_cnn.onnx", here / "tiny_cnn.onnx")
    print(f"wrote {here / 'tiny_cnn.json'} and {here / 'tiny_cnn.onnx'}")


if __name__ == "__main__":
    main()
