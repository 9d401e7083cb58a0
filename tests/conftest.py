import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "aeo-quant_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    # GPU tests fail loudly when no GPU is present rather than skipping: the
    # driver selects them with -m gpu only on a GPU box.
    pass


@pytest.fixture(scope="session")
def quant_golden():
    import numpy as np
    return np.load(os.path.join(GOLDEN, "quant_golden.npz"))


@pytest.fixture(scope="session")
def moe_golden():
    import numpy as np
    return np.load(os.path.join(GOLDEN, "moe_golden.npz"))
