import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def golden_cases():
    import numpy as np
    out = {}
    for f in sorted(GOLDEN.glob("*.npz")):
        z = dict(np.load(f))
        for name in ("q", "k", "v"):       # slim fixtures store bfloat16 bit patterns
            if name + "16" in z:
                z[name] = (z.pop(name + "16").astype(np.uint32) << 16).view(np.float32)
        out[f.stem] = z
    return out
