import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "neural-network_b200"), os.path.join(ROOT, "oracle"), os.path.dirname(__file__)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a); run with -m gpu")


@pytest.fixture(scope="session")
def oracle_built():
    import oracle

    oracle.build(ref=True)
    return oracle


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return dict(np.load(os.path.join(ROOT, "tests", "golden", "reference_cases.npz")))


@pytest.fixture(scope="session")
def gpu_lib():
    """The CUDA library, built in-tree; a GPU test fails loudly when it is missing."""
    sys.path.insert(0, os.path.join(ROOT, "neural-network_b200"))
    import build as nb_build  # neural-network_b200/build.py

    nb_build.build()
    import specdec_b200

    return specdec_b200.load_library()
