"""Kernel watchdog on the GPU, without a GPU fault.

Every wait inside the library's kernels is bounded; a wait that runs out records a code in the
Resources' error word and the kernel returns. The self test runs a kernel whose wait nothing ever
satisfies (an mbarrier with no arrivals) with a short limit, and the test checks that the host
sees the error status and the code, and that the same Resources then runs a correct search.
"""
import time

import numpy as np
import pytest

from helpers import assert_search_equal

pytestmark = pytest.mark.gpu

SELF_TEST_CODE = 0x201


def test_watchdog_fires_and_context_survives(ovvs, oracle, gpu):
    res = ovvs.Resources()
    t0 = time.perf_counter()
    code = res.watchdog_self_test(50_000_000)  # 50 ms
    elapsed = time.perf_counter() - t0
    assert code == SELF_TEST_CODE
    assert elapsed < 5.0
    assert res.last_kernel_error() == 0  # the self test consumed its code

    rng = np.random.default_rng(7)
    data = rng.standard_normal((3000, 64), dtype=np.float32)
    queries = rng.standard_normal((50, 64), dtype=np.float32)
    ix = ovvs.BruteIndex.build(data, metric="l2", resources=res)
    nb, dist = ix.search(queries, 7)
    onb, odist = oracle.brute_search(data, queries, 7, "l2")
    assert_search_equal(nb, dist, onb, odist)
    assert res.last_kernel_error() == 0


def test_watchdog_limit_is_validated(ovvs, gpu):
    res = ovvs.Resources()
    with pytest.raises(ovvs.OvvsError):
        res.watchdog_self_test(10)  # below 1 ms
