import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a (B200) GPU; the parity tests proper")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return dict(np.load(ROOT / "tests" / "golden" / "golden.npz"))


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from stratametal_b200 import build
    build.build()
    dev = torch.device("cuda:0")
    # the C ABI requires an explicit, non-null stream (torch's default stream is the null stream)
    torch.cuda.set_stream(torch.cuda.Stream(dev))
    return dev
