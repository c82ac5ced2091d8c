import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def refconv():
    from oracle.oracle import RefConv
    if not RefConv.available():
        pytest.skip("reference Conv2DOp library (oracle/_ref) not built here")
    return RefConv()


@pytest.fixture(scope="session")
def golden():
    import json
    import numpy as np
    data = json.loads((ROOT / "tests" / "golden" / "traditional_conv.json").read_text())
    return {k: np.array(v["values"], np.float32).reshape(v["shape"])
            for k, v in data.items() if not k.startswith("_")}
