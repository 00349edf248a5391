import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(autouse=True)
def _gather_mode():
    """PKV_GATHER=tma|cpasync runs every test with that decode gather (the
    library default otherwise), so the whole GPU suite can run on both."""
    mode = os.environ.get("PKV_GATHER")
    if not mode:
        yield
        return
    from persistentkv_attention_b200 import _native

    prev = _native.gather_mode()
    _native.set_gather_mode(mode)
    yield
    _native.set_gather_mode(prev)


@pytest.fixture(scope="session")
def smoke_kat():
    data = np.load(GOLDEN / "smoke_kat.npz", allow_pickle=True)
    return data


@pytest.fixture(scope="session")
def scheduler_golden():
    return json.loads((GOLDEN / "scheduler.json").read_text())


@pytest.fixture(scope="session")
def traces_golden():
    return json.loads((GOLDEN / "traces.json").read_text())


@pytest.fixture(scope="session")
def lib():
    from persistentkv_attention_b200 import _native

    return _native.load()


def gpu_available() -> bool:
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:  # pragma: no cover
        return False
