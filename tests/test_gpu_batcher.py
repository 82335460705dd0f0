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
