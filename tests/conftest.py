import os
import pathlib
import sys

import pytest

REPO = pathlib.Path(__file__).resolve().parent.parent
PKG = REPO / "eco-int8-opt_b200"
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = REPO / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) and the built library")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    has_gpu = False
    try:
        import torch

        has_gpu = torch.cuda.is_available()
    except Exception:
        pass
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    import json

    def load(name):
        return json.loads((GOLDEN / name).read_text())["data"]

    return load


os.environ.setdefault("OMP_NUM_THREADS", "4")
