"""Shared fixtures. GPU tests are marked ``gpu`` and call the CUDA library through its C ABI;
everything else runs on CPU (oracle vs golden fixtures, ABI surface, host logic, gloo ranks)."""

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and calls the CUDA library")


def _load_npz_cases(name):
    z = np.load(os.path.join(GOLDEN, name), allow_pickle=False)
    cases = {}
    for key in z.files:
        if "__" not in key:
            continue
        case, field = key.split("__", 1)
        cases.setdefault(case, {})[field] = z[key]
    return cases


@pytest.fixture(scope="session")
def golden_brute():
    return _load_npz_cases("brute_force.npz")


@pytest.fixture(scope="session")
def golden_kmeans():
    return _load_npz_cases("kmeans.npz")


@pytest.fixture(scope="session")
def golden_misc():
    return dict(np.load(os.path.join(GOLDEN, "misc.npz"), allow_pickle=False))


@pytest.fixture(scope="session")
def oracle():
    from oracle.cpu import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def ovvs():
    """The product binding; building the library first if needed (CPU-only build works)."""
    import ovvs_b200

    if not os.path.exists(ovvs_b200.library_path()):
        from ovvs_b200 import build

        build.build()
    return ovvs_b200


@pytest.fixture(scope="session")
def gpu(ovvs):
    """A Resources on cuda:0 for GPU tests; fails loudly (no skip) when the B200 is missing."""
    res = ovvs.Resources()
    assert res.gpu_available(), "GPU tests need an sm_100 device (B200)"
    yield res
    res.close()


@pytest.fixture(scope="session")
def golden_prims():
    return _load_npz_cases("prims.npz")


@pytest.fixture(scope="session")
def golden_ivf():
    return _load_npz_cases("ivf_flat.npz")
