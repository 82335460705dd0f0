"""Host-side logic of bench.py that the round-end measurements rely on (no GPU needed)."""

import os

import numpy as np

import bench


def test_clock_summary_median_max_and_reasons():
    cs = bench.ClockSampler(0)
    cs.lines = [
        "1965, 1965, 0, Not Active, Not Active, Not Active, Not Active",
        "1700, 1965, 0, Not Active, Not Active, Not Active, Active",
        "1710, 1965, 0, Active, Not Active, Not Active, Active",
        "not a sample",
    ]
    s = cs.summary()
    assert s["samples"] == 3
    assert s["sm_mhz"] == 1710.0
    assert s["sm_max_mhz"] == 1965.0
    assert s["reasons"] == ["hw_slowdown", "sw_power_cap"]


def test_clock_summary_without_samples():
    s = bench.ClockSampler(0).summary()
    assert s["sm_mhz"] is None and s["samples"] == 0 and s["reasons"] == []


def test_search_launch_counts():
    # small k: query prep, fused kernel, merge + re-rank (+ cross-shard merge when sharded)
    assert bench._search_launches(10, 10_000_000, 1) == 3
    assert bench._search_launches(10, 1_250_000, 8) == 4
    # k = 100 (need 113 > 32): prep, bound pre-pass, k-th bound, append pass, select + re-rank
    assert bench._search_launches(100, 1_000_000, 1) == 5
    # no pre-pass at or below 4,096 rows
    assert bench._search_launches(100, 3_000, 1) == 3
    # k = 28 still fits the register lists (need 28 + 4 = 32)
    assert bench._search_launches(28, 1_000_000, 1) == 3


def test_metric_names():
    assert bench.metric_name(bench.CONFIGS["c3"]) == bench.METRIC_NAME
    assert "N=100M D=96 f16 inner_product k=100" in bench.metric_name(bench.CONFIGS["c5"])
    assert "N=100k" in bench.metric_name(bench.CONFIGS["c1"])


def test_traffic_figures_come_from_the_committed_profile():
    # both measured (read + write bytes of one launch), not scaled from a smaller case
    assert bench._traffic_from_profiles("c3s") == 793717504.0 + 22001408.0
    assert bench._traffic_from_profiles("c3") == 16770861824.0 + 50106624.0
    assert bench._traffic_from_profiles("no-such-config") is None


def test_ivf_file_lists_reads_the_reference_format(tmp_path):
    from oracle.cpu import write_ivf1

    rng = np.random.default_rng(3)
    x = rng.standard_normal((50, 6)).astype(np.float32)
    cents = rng.standard_normal((4, 6)).astype(np.float32)
    sizes = np.array([10, 0, 25, 15], np.int64)
    ids = rng.permutation(50).astype(np.int64)
    path = os.path.join(str(tmp_path), "ix.ivf")
    write_ivf1(path, x, cents, sizes, ids, 0)
    got_c, got_sizes = bench._ivf_file_lists(path)
    assert np.array_equal(got_c, cents)
    assert np.array_equal(got_sizes, sizes)


def test_reference_sample_sizes_are_bounded():
    threads, nq = bench._ivf_reference_sizes(bench.CONFIGS["ivf"], 12.0)
    assert threads >= 1 and threads <= nq <= bench.CONFIGS["ivf"]["nq"]
    rows = bench._reference_kmeans_rows(bench.CONFIGS["c4"], 12.0)
    assert bench.CONFIGS["c4"]["clusters"] <= rows <= bench.CONFIGS["c4"]["n"]


def _have_reference():
    from oracle.cpu import REFERENCE_SO

    return os.path.exists(REFERENCE_SO)


def test_reference_sample_merge_equals_unsharded_search(monkeypatch):
    """The bench's parity block merges the reference's per-shard answers; merged, they must be the
    reference's answer over all rows (here: the restatement's unsharded search), for L2 and for
    inner product (whose reported distances are negated scores), with duplicate rows across
    shard boundaries and k above a shard's row count."""
    import pytest

    if not _have_reference():
        pytest.skip("reference library not built")
    from oracle.cpu import Oracle

    monkeypatch.setattr(bench, "CHUNK", 700)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((2300, 16)).astype(np.float32)
    x[1500] = x[20]  # equal distances on both sides of a shard boundary
    x[699] = x[700]
    q = rng.standard_normal((9, 16)).astype(np.float32)
    q[3] = x[20]
    for metric, k in (("l2", 10), ("inner_product", 7), ("l2", 650)):
        cfg = dict(n=x.shape[0], k=k, metric=metric, dtype="f32")
        _, nb, ds = bench._reference_sample(cfg, x, q, 3, q.shape[0])
        rnb, rds = Oracle().brute_search(x, q, k, metric)
        ke = min(k, x.shape[0])
        assert np.array_equal(nb, rnb.reshape(-1, ke)), metric
        assert np.array_equal(ds.view(np.uint32), rds.reshape(-1, ke).view(np.uint32)), metric
        p = bench._parity(nb, ds, rnb.reshape(-1, ke), rds.reshape(-1, ke), 1e-4)
        assert p["ok"] and p["id_mismatch"] == 0 and p["max_rel_err"] == 0.0


def test_parity_flags_mismatches_beyond_ties():
    nb_ref = np.array([[1, 2, 3]], np.int64)
    ds_ref = np.array([[1.0, 2.0, 3.0]], np.float32)
    # a near-tie swap at the last rank is allowed
    p = bench._parity(np.array([[1, 2, 4]]), np.array([[1.0, 2.0, 3.0001]], np.float32),
                      nb_ref, ds_ref, 1e-4)
    assert p["ok"] and p["id_mismatch"] == 1 and p["id_mismatch_beyond_tie"] == 0
    # a different neighbour with a clearly different distance is not
    p = bench._parity(np.array([[1, 2, 4]]), np.array([[1.0, 2.0, 3.5]], np.float32),
                      nb_ref, ds_ref, 1e-4)
    assert not p["ok"] and p["id_mismatch_beyond_tie"] == 1
    # same ids with different distance bits fail
    p = bench._parity(nb_ref, np.array([[1.0, 2.0, 3.0000002]], np.float32), nb_ref, ds_ref, 1e-4)
    assert not p["ok"] and p["distance_bits_differ_where_ids_agree"] == 1


def test_primitive_configs():
    """The dense-primitive arms: seeded operands of the configured shapes, a named metric, and a
    reference sample sized to the requested seconds of the reference's single-threaded loop."""
    for name in ("pw", "gemm"):
        cfg = bench.CONFIGS[name]
        x, y = bench._prim_data(cfg)
        assert x.shape == (cfg["nx"], cfg["dim"]) and y.shape == (cfg["ny"], cfg["dim"])
        assert x.dtype == np.float32 and y.dtype == np.float32
        x2, _ = bench._prim_data(cfg)
        assert np.array_equal(x, x2)  # seeded
        assert cfg["op"] in bench._prim_metric(cfg)
        rows = bench._prim_reference_rows(cfg, 12.0)
        assert 1 <= rows <= cfg["nx"]
        # about 12 s at the reference's measured ~2.1 GFLOP/s
        assert abs(2.0 * rows * cfg["ny"] * cfg["dim"] / 2.1e9 - 12.0) < 1.0
        assert bench._prim_reference_rows(cfg, 1e9) == cfg["nx"]
