"""Helpers for the C++ backend tests: the test driver binary and the
raw tensors it writes (name dtype dims... per manifest line)."""
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
DRIVER = ROOT / "computeengine_b200" / "_build" / "ie_cuda_backend_test"

# ie::DType enumerator order (src/core/base/types.h:10-22)
DTYPES = {0: np.float32, 3: np.int8, 5: np.uint8}


def driver() -> Path:
    if not DRIVER.exists():
        from computeengine_b200.build import build
        build()
    return DRIVER


def read_dump(outdir: Path) -> dict:
    out = {}
    for line in (outdir / "manifest.txt").read_text().splitlines():
        parts = line.split()
        name, dt, dims = parts[0], int(parts[1]), tuple(int(v) for v in parts[2:])
        out[name] = np.fromfile(outdir / f"{name}.bin", dtype=DTYPES[dt]).reshape(dims)
    return out
