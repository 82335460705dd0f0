"""The CPU oracle (oracle/ovvs_oracle.cpp) against the reference's own outputs.

tests/golden/*.npz were produced by the reference library compiled from its sources
(tests/golden/make_golden.py), so a bit-exact match here pins the restatement to the reference.
"""

import os

import numpy as np
import pytest

from tests.helpers import assert_search_equal, ivf_extend_lists, same_bits


def _brute_case(c, oracle):
    data32 = oracle.convert_to_f32(str(c["dtype"]), c["data"])
    bitset = c["bitset"] if c["bitset"].size else None
    fill = None
    if float(c["fill"][0]) != -1 or float(c["fill"][1]) != 0.0:
        fill = (int(c["fill"][0]), float(c["fill"][1]))
    return oracle.brute_search(data32, c["queries"], int(c["k"]), int(c["metric"]), bitset=bitset,
                               out_fill=fill)


def test_brute_force_cases_bit_exact(golden_brute, oracle):
    assert len(golden_brute) >= 39
    for name, c in golden_brute.items():
        nb, ds = _brute_case(c, oracle)
        assert_search_equal(nb, ds, c["neighbors"], c["distances"], what=name)


def test_kmeans_cases_bit_exact(golden_kmeans, oracle):
    for name, c in golden_kmeans.items():
        x = c["x"]
        cents = oracle.kmeans_fit(x, int(c["nclusters"]), max(4, int(c["iters"])))
        assert np.all(same_bits(cents, c["centroids"])), name
        assert int(c["reported_k"]) == int(c["nclusters"]), name
        if c["labels"].size:
            labels, dist = oracle.kmeans_predict(cents, x)
            assert np.array_equal(labels, c["labels"]), name
            assert np.all(same_bits(dist, c["distances"])), name


def test_topk_total_order(golden_misc, oracle):
    idx, val = oracle.topk(golden_misc["topk_scores"], 8)
    assert np.array_equal(idx, golden_misc["topk_idx"])
    assert np.all(same_bits(val, golden_misc["topk_val"]))


def test_bitset_from_allow_list(golden_misc, oracle):
    bs = oracle.bitset_from_allow_list(int(golden_misc["bitset_n"]), golden_misc["bitset_ids"])
    assert np.array_equal(bs, golden_misc["bitset"])


def test_kmeans_init_rows_follow_mt19937(oracle):
    # mixer.cpp:880-890: the first draw of std::mt19937(42) through uniform_int_distribution
    rows = oracle.kmeans_init_rows(1000, 16)
    assert rows.shape == (16,) and len(set(rows.tolist())) == 16
    assert np.all((rows >= 0) & (rows < 1000))
    assert np.array_equal(rows, oracle.kmeans_init_rows(1000, 16))


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(__file__), "..", "oracle", "_ref",
                                                    "libovvs_ref.so")),
                    reason="reference library not built in this checkout")
@pytest.mark.parametrize("metric", ["l2", "inner_product", "cosine", "l2_sqrt", "hamming", "lp"])
def test_reference_library_matches_oracle(oracle, metric):
    from oracle.cpu import Reference

    ref = Reference()
    rng = np.random.default_rng(7)
    X = rng.standard_normal((3000, 24)).astype(np.float32)
    Q = rng.standard_normal((20, 24)).astype(np.float32)
    a = oracle.brute_search(X, Q, 12, metric)
    b = ref.brute_search(X, Q, 12, metric)
    assert_search_equal(a[0], a[1], b[0], b[1], what=metric)


def _gemm_shape(c):
    m, k = c["a"].shape
    n = c["b"].shape[0] if int(c["trans_b"]) else c["b"].shape[1]
    return m, n, k


def test_primitive_cases_bit_exact(golden_prims, oracle):
    """resources.cpp:178-216 and graphs.cpp:3384-3396: the oracle's gemm / top-k / gather /
    pairwise / all-neighbors equal the reference's outputs bit for bit."""
    kinds = set()
    for name, c in golden_prims.items():
        kind = name.split("_", 1)[0]
        kinds.add(kind)
        if kind == "gemm":
            m, n, k = _gemm_shape(c)
            got = oracle.gemm(c["a"], c["b"], m, n, k, trans_b=bool(int(c["trans_b"])))
            assert np.all(same_bits(got, c["c"])), name
        elif kind == "topk":
            idx, val = oracle.topk(c["scores"], int(c["k"]), largest=bool(int(c["largest"])))
            assert np.array_equal(idx, c["idx"]), name
            assert np.all(same_bits(val, c["val"])), name
        elif kind == "gather":
            assert np.all(same_bits(oracle.gather_rows(c["src"], c["idx"]), c["out"])), name
        elif kind == "pw":
            got = oracle.pairwise(int(c["metric"]), c["x"], c["y"], float(c["arg"]))
            assert np.all(same_bits(got, c["out"])), name
        elif kind == "an":
            nb, ds = oracle.all_neighbors(c["data"], int(c["k"]), int(c["metric"]))
            assert_search_equal(nb, ds, c["neighbors"], c["distances"], what=name)
        else:
            raise AssertionError(name)
    assert kinds == {"gemm", "topk", "gather", "pw", "an"}


def test_ivf_flat_cases_bit_exact(golden_ivf, oracle):
    """IVF-Flat build (k-means lists) and search (indexes.cpp:281-358), extension included."""
    assert len(golden_ivf) >= 18
    for name, c in golden_ivf.items():
        x, extra = c["x"], c["extra"]
        cents, sizes, ids = oracle.ivf_flat_build(x, int(c["nlist"]))
        if extra.shape[0]:
            labels, _ = oracle.kmeans_predict(cents, extra)
            sizes, ids = ivf_extend_lists(cents, sizes, ids, x.shape[0], labels, cents.shape[0])
            x = np.concatenate([x, extra])
        assert np.all(same_bits(cents, c["centroids"])), name
        assert np.array_equal(sizes, c["sizes"]) and np.array_equal(ids, c["ids"]), name
        bits = c["bitset"] if c["bitset"].size else None
        nb, ds = oracle.ivf_flat_search(x, int(c["metric"]), cents, sizes, ids, c["queries"],
                                        int(c["k"]), int(c["nprobe"]), bits)
        assert_search_equal(nb, ds, c["neighbors"], c["distances"], what=name)


def test_ivf_flat_probing_every_list_is_brute_force(oracle):
    """With nprobe = nlist every row is a candidate, so the IVF-Flat search returns the brute-force
    distances (ids agree except between rows of equal distance: IVF breaks those ties by probe
    position, brute force by row id)."""
    rng = np.random.default_rng(12)
    x = rng.standard_normal((2000, 16)).astype(np.float32)
    q = rng.standard_normal((40, 16)).astype(np.float32)
    cents, sizes, ids = oracle.ivf_flat_build(x, 12)
    for metric in ("l2", "inner_product", "cosine"):
        nb, ds = oracle.ivf_flat_search(x, metric, cents, sizes, ids, q, 9, cents.shape[0])
        bnb, bds = oracle.brute_search(x, q, 9, metric)
        assert np.all(same_bits(ds.ravel(), bds)), metric
        assert np.mean(nb.ravel() == bnb) > 0.99, metric


def test_row_sharded_oracle_equals_serial(oracle):
    """Few queries over many rows take the oracle's row-sharded path (each thread a row shard,
    shard lists merged in the reference's total order): it must equal the serial search bit for
    bit, with NaN rows, duplicate rows across shard boundaries, bitsets and every metric."""
    rng = np.random.default_rng(0)
    x = rng.standard_normal((70_000, 24)).astype(np.float32)
    x[36_000] = x[5]
    x[200] = np.nan
    q = rng.standard_normal((5, 24)).astype(np.float32)
    q[1] = x[5]
    bits = np.packbits((rng.random(70_000) < 0.7).astype(np.uint8), bitorder="little")
    for metric in ("l2", "inner_product", "cosine", "hamming", "lp", "l2_sqrt"):
        for k in (1, 10, 100):
            for b in (None, bits):
                a = oracle.brute_search(x, q, k, metric, bitset=b, nthreads=1)
                c = oracle.brute_search(x, q, k, metric, bitset=b, nthreads=16)
                assert np.array_equal(a[0], c[0]), (metric, k)
                assert np.array_equal(a[1].view(np.uint32), c[1].view(np.uint32)), (metric, k)
