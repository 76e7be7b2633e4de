import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device")


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(ROOT / "tests" / "golden" / "golden.npz"))


@pytest.fixture(scope="session")
def port():
    from oracle import oracle as O
    O.build()
    return O.port()


@pytest.fixture(scope="session")
def lib():
    from tinymetalagent_b200 import runtime
    return runtime.load_library()


@pytest.fixture(scope="session")
def engine():
    import torch
    from tinymetalagent_b200 import AttnEngine
    torch.cuda.init()
    eng = AttnEngine(device=0)
    yield eng
    eng.close()
