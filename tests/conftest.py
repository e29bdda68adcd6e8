import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def load_golden(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        out = {k: z[k] for k in z.files}
    for k in ("M", "N", "K", "group"):
        if k in out:
            out[k] = int(out[k])
    return out


def golden_names(prefix):
    return sorted(f[:-4] for f in os.listdir(GOLDEN)
                  if f.startswith(prefix) and f.endswith(".npz"))


@pytest.fixture(scope="session")
def oracle_mod():
    import oracle
    oracle.lib()
    return oracle
