"""Dynamic batcher (reference tests/test_neighbors.cpp:3697-3734): concurrent nq=1 searches
coalesce into one GPU search and return exactly the eager results."""

import threading

import numpy as np
import pytest

from oracle.cpu import make_data

pytestmark = pytest.mark.gpu


def test_batcher_matches_eager(ovvs, gpu):
    n, dim, nq, k = 30, 8, 4, 3
    data = make_data(n, dim, 490)
    q = make_data(nq, dim, 491)
    ix = ovvs.BruteIndex.build(data, resources=gpu)
    eager_nb, eager_ds = ix.search(q, k=k)
    b = ovvs.Batcher(ix, max_batch=4, max_wait_ms=250)
    out = [None] * nq
    go = threading.Barrier(nq)

    def work(i):
        go.wait()
        out[i] = b.search(q[i:i + 1], k=k)

    th = [threading.Thread(target=work, args=(i,)) for i in range(nq)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    assert b.last_batch_size() == nq
    got = np.vstack([o[0] for o in out])
    assert np.array_equal(got, eager_nb)
    b.close()
    ix.close()


def _batcher_index(ovvs, gpu):
    data = make_data(30, 8, 490)
    return ovvs.BruteIndex.build(data, resources=gpu)


def test_batcher_flushes_the_open_batch_when_k_changes(ovvs, gpu):
    """A member waiting with k=3 is searched as soon as a caller with k=5 arrives, long before its
    own max_wait_ms; the k=5 caller then forms its own batch."""
    import time

    ix = _batcher_index(ovvs, gpu)
    q = make_data(2, 8, 492)
    eager3 = ix.search(q[:1], k=3)
    eager5 = ix.search(q[1:2], k=5)
    b = ovvs.Batcher(ix, max_batch=8, max_wait_ms=1500)
    res, took = {}, {}

    def member():
        t0 = time.perf_counter()
        res["a"] = b.search(q[:1], k=3)
        took["a"] = time.perf_counter() - t0

    t = threading.Thread(target=member)
    t.start()
    time.sleep(0.15)
    res["b"] = b.search(q[1:2], k=5)
    t.join()
    assert took["a"] < 1.0, f"k change did not flush the waiting batch ({took['a']:.3f} s)"
    assert np.array_equal(res["a"][0], eager3[0]) and np.array_equal(res["a"][1], eager3[1])
    assert np.array_equal(res["b"][0], eager5[0]) and np.array_equal(res["b"][1], eager5[1])
    assert b.last_batch_size() == 1
    b.close()
    ix.close()


def test_batcher_flushes_after_max_wait(ovvs, gpu):
    """Below max_batch a batch is searched once a member has waited max_wait_ms; members arriving
    within the window share it; max_wait_ms = 0 searches at once."""
    import time

    ix = _batcher_index(ovvs, gpu)
    q = make_data(2, 8, 493)
    eager = ix.search(q, k=4)
    b = ovvs.Batcher(ix, max_batch=64, max_wait_ms=120)
    t0 = time.perf_counter()
    nb, ds = b.search(q[:1], k=4)
    assert time.perf_counter() - t0 >= 0.1
    assert b.last_batch_size() == 1
    assert np.array_equal(nb, eager[0][:1]) and np.array_equal(ds, eager[1][:1])
    out = [None, None]
    go = threading.Barrier(2)

    def work(i):
        go.wait()
        out[i] = b.search(q[i:i + 1], k=4)

    th = [threading.Thread(target=work, args=(i,)) for i in range(2)]
    for x in th:
        x.start()
    for x in th:
        x.join()
    assert b.last_batch_size() == 2
    assert np.array_equal(np.vstack([o[0] for o in out]), eager[0])
    b.close()
    b0 = ovvs.Batcher(ix, max_batch=64, max_wait_ms=0)
    t0 = time.perf_counter()
    nb, _ = b0.search(q[1:2], k=4)
    assert time.perf_counter() - t0 < 0.1 and b0.last_batch_size() == 1
    assert np.array_equal(nb, eager[0][1:2])
    b0.close()
    ix.close()


def test_batcher_destroy_fails_waiting_members(ovvs, gpu):
    """Destroying the batcher while a member waits in an open batch returns ERROR to that member
    (and destroy returns only after the member has left)."""
    import time

    ix = _batcher_index(ovvs, gpu)
    q = make_data(1, 8, 494)
    b = ovvs.Batcher(ix, max_batch=8, max_wait_ms=5000)
    err = {}

    def member():
        try:
            b.search(q, k=3)
        except ovvs.OvvsError as e:
            err["status"] = e.status

    t = threading.Thread(target=member)
    t.start()
    time.sleep(0.15)
    t0 = time.perf_counter()
    b.close()
    t.join()
    assert time.perf_counter() - t0 < 2.0
    assert err.get("status") == 1  # OVVS_STATUS_ERROR
    ix.close()
