"""Reference-facing code running unchanged on this library (the drop-in boundary).

* The reference's own C and C++ consumer programs (its tests/consumer.c and tests/consumer.cpp),
  compiled by oracle/Makefile against this repository's include/ovvs headers and linked to
  ovvs_b200/libovvs.so. The C program uses only brute-force entry points and must pass. The C++
  program walks every wrapper class: the brute-force (L2, allow list, Hamming), IVF-Flat, k-means
  and batcher parts are this library's; its first out-of-scope index (CAGRA) throws
  "unsupported", which ends the program there.
* The reference's Python binding (its python/ovvs package, installed into baseline/_ref) loaded
  with OVVS_LIBRARY pointing at this library: brute-force build + search (L2 and inner product,
  with an allow list), k-means fit + predict and the batcher, compared with the CPU oracle.
"""

import json
import os
import subprocess
import sys

import numpy as np
import pytest

from tests.helpers import assert_search_equal

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_BIN = os.path.join(ROOT, "oracle", "_ref")
REF_PY = os.path.join(ROOT, "baseline", "_ref")


def _run(exe):
    if not os.path.exists(exe):
        pytest.skip(f"{os.path.relpath(exe, ROOT)} not built (oracle/Makefile needs the reference)")
    # unbuffered stdout: a program that ends in abort() (an uncaught exception) keeps its output
    return subprocess.run(["stdbuf", "-o0", "-e0", exe], capture_output=True, text=True,
                          timeout=300)


def test_reference_c_consumer(ovvs, gpu):
    r = _run(os.path.join(REF_BIN, "consumer_c"))
    assert r.returncode == 0, r.stdout + r.stderr
    assert "consumer ok neighbors=" in r.stdout and "version=0.2.0" in r.stdout


def test_reference_cxx_consumer(ovvs, gpu):
    r = _run(os.path.join(REF_BIN, "consumer_cxx"))
    assert "cxx consumer ok neighbors=" in r.stdout, r.stdout + r.stderr
    # every in-scope part passed (a mismatch there returns 1 with a message) ...
    for bad in ("mismatch", "not in list", "out of range", "inertia"):
        assert bad not in r.stderr, r.stderr
    # ... and the first index outside this library's path stops it with "unsupported"
    assert r.returncode != 0 and "what():  unsupported" in r.stderr, r.stderr


_PY = r"""
import json, sys
import numpy as np
import ovvs
assert ovvs.__file__.startswith(sys.argv[1]), ovvs.__file__
rng = np.random.default_rng(31)
data = rng.standard_normal((5000, 24)).astype(np.float32)
q = rng.standard_normal((40, 24)).astype(np.float32)
res = ovvs.Resources()
out = {}
ix = ovvs.neighbors.brute_force.build(data, dim=24, resources=res)
nb, ds = ix.search(q, k=7)
out["l2"] = [np.asarray(nb).tolist(), np.asarray(ds, np.float32).view(np.uint32).tolist()]
ip = ovvs.neighbors.brute_force.build(data, dim=24, metric=2, resources=res)
nb, ds = ip.search(q, k=5, allow_list=list(range(0, 5000, 4)))
out["ip_allow"] = [np.asarray(nb).tolist(), np.asarray(ds, np.float32).view(np.uint32).tolist()]
km = ovvs.KMeans(data, nclusters=6, iters=5, resources=res)
labels, dist = km.predict(q)
out["km"] = [list(labels), np.asarray(dist, np.float32).view(np.uint32).tolist()]
b = ovvs.Batcher(ix, max_batch=4, max_wait_ms=0)
nb, ds = b.search(q[:1], k=7)
out["batch"] = np.asarray(nb).tolist()
print(json.dumps(out))
"""


def test_reference_python_binding(ovvs, gpu, oracle):
    if not os.path.isdir(os.path.join(REF_PY, "ovvs")):
        pytest.skip("the reference's Python binding is not installed in baseline/_ref")
    env = dict(os.environ, OVVS_LIBRARY=ovvs.library_path(), PYTHONPATH=REF_PY)
    r = subprocess.run([sys.executable, "-c", _PY, REF_PY], capture_output=True, text=True,
                       env=env, timeout=300, cwd=REF_PY)
    assert r.returncode == 0, r.stdout + r.stderr
    got = json.loads(r.stdout.strip().splitlines()[-1])
    rng = np.random.default_rng(31)
    data = rng.standard_normal((5000, 24)).astype(np.float32)
    q = rng.standard_normal((40, 24)).astype(np.float32)

    def f32(bits):
        return np.asarray(bits, np.uint32).view(np.float32)

    rnb, rds = oracle.brute_search(data, q, 7, "l2")
    assert_search_equal(got["l2"][0], f32(got["l2"][1]), rnb, rds, what="reference binding l2")
    bits = oracle.bitset_from_allow_list(5000, np.arange(0, 5000, 4))
    rnb, rds = oracle.brute_search(data, q, 5, "inner_product", bitset=bits)
    assert_search_equal(got["ip_allow"][0], f32(got["ip_allow"][1]), rnb, rds,
                        what="reference binding inner product + allow list")
    cent = oracle.kmeans_fit(data, 6, 5)
    rl, rd = oracle.kmeans_predict(cent, q)
    assert np.array_equal(got["km"][0], rl)
    assert np.array_equal(f32(got["km"][1]).view(np.uint32), rd.view(np.uint32))
    assert got["batch"][0] == list(oracle.brute_search(data, q[:1], 7, "l2")[0])
