import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (runs on the B200 box)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle
    return Oracle()


@pytest.fixture(scope="session")
def reference():
    from oracle.oracle import REF_SO, Reference
    if not os.path.exists(REF_SO):
        pytest.skip("reference library oracle/_ref not built here")
    try:
        return Reference()
    except OSError as e:  # e.g. built for another host architecture
        pytest.skip(f"reference library not loadable: {e}")


@pytest.fixture(scope="session")
def manifest():
    with open(os.path.join(GOLDEN, "manifest.json")) as fh:
        return json.load(fh)


@pytest.fixture(scope="session")
def gpu():
    """The GPU library, with a device present; fails (not skips) if the library is missing."""
    import quiver_b200
    if quiver_b200.device_count() < 1:
        pytest.fail("no CUDA device visible to the GPU tests")
    return quiver_b200


def golden_flat_inputs(case):
    from quiver_b200.synthetic import clustered, gaussian, skewed_ints

    def gen(n, seed):
        if case["generator"] == "gaussian":
            return gaussian(n, case["dim"], seed)
        if case["generator"] == "clustered":
            return clustered(n, case["dim"], 20, seed)
        return skewed_ints(n, case["dim"], seed)

    base = gen(case["n"], case["seed"])
    q = gen(case["nq"], case["query_seed"])
    labels = np.arange(case["n"], dtype=np.uint64) * 3 + 7
    return base, q, labels


def golden_ivf_inputs(case):
    from quiver_b200.synthetic import clustered
    base = clustered(case["n"], case["dim"], case["clusters"], case["seed"])
    q = clustered(50, case["dim"], case["clusters"], case["query_seed"])
    return base, q
