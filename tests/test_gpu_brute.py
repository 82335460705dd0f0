"""Brute-force kNN parity on the B200, through the C ABI.

Expected: neighbour ids identical to the reference, distances bit-identical (the merge kernel
re-evaluates each selected pair with the reference's own fp32 operation order). The only allowed
difference is a near-tie at the cut-off, where another row whose exact distance is within the
parity tolerance (fp32 1e-4, fp16 2e-3 relative) may be returned instead.
"""

import os

import numpy as np
import pytest

from tests.helpers import assert_search_close, assert_search_equal, same_bits

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "brute_force.npz")
_CASES = sorted({k.split("__")[0] for k in np.load(GOLDEN).files})
TOL = {"f32": 1e-4, "f16": 2e-3, "i8": 1e-4, "u8": 1e-4}


def _golden_fill(c):
    if float(c["fill"][0]) != -1 or float(c["fill"][1]) != 0.0:
        return int(c["fill"][0]), float(c["fill"][1])
    return None


@pytest.mark.parametrize("name", _CASES)
def test_golden_case(name, golden_brute, ovvs, gpu):
    c = golden_brute[name]
    k = int(c["k"])
    nq = c["queries"].shape[0]
    fill = _golden_fill(c) or (-1, 0.0)
    out = (np.full(nq * k, fill[0], np.int64), np.full(nq * k, fill[1], np.float32))
    ix = ovvs.BruteIndex.build(c["data"], metric=int(c["metric"]), dtype=str(c["dtype"]),
                               resources=gpu)
    bitset = c["bitset"] if c["bitset"].size else None
    nb, ds = ix.search(c["queries"], k=k, bitset=bitset, out=out)
    ix.close()
    assert_search_equal(nb, ds, c["neighbors"], c["distances"], what=name)
    assert gpu.last_device() == 3


def _dataset(rng, dtype, n, dim, kind):
    if kind == "uniform":
        x = rng.random((n, dim), dtype=np.float32)
    elif kind == "mixture":
        centres = rng.normal(0, 2, (64, dim)).astype(np.float32)
        x = centres[rng.integers(0, 64, n)] + rng.standard_normal((n, dim)).astype(np.float32)
    else:
        x = rng.standard_normal((n, dim)).astype(np.float32)
        x /= np.linalg.norm(x, axis=1, keepdims=True)
    if dtype == "f16":
        return x.astype(np.float16)
    if dtype == "i8":
        return np.clip(np.round(x * 40), -127, 127).astype(np.int8)
    if dtype == "u8":
        return np.clip(np.round((x + 1) * 100), 0, 255).astype(np.uint8)
    return x.astype(np.float32)


def _run_parity(ovvs, gpu, oracle, metric, dtype, n, dim, nq, k, kind="gauss", seed=0,
                bitset=None, fp16_queries=False):
    rng = np.random.default_rng(seed)
    data = _dataset(rng, dtype, n, dim, kind)
    q = _dataset(rng, "f32", nq, dim, kind).astype(np.float32)
    if dtype in ("i8", "u8"):
        q = np.round(q * 40).astype(np.float32)
    if fp16_queries:
        q = q.astype(np.float16).astype(np.float32)
    ix = ovvs.BruteIndex.build(data, metric=metric, dtype=dtype, resources=gpu)
    nb, ds = ix.search(q, k=k, bitset=bitset)
    ix.close()
    data32 = data.astype(np.float32)
    rnb, rds = oracle.brute_search(data32, q, k, metric, bitset=bitset)
    k_eff = min(k, n)
    nb, ds = nb.ravel()[: nq * k_eff], ds.ravel()[: nq * k_eff]
    rnb, rds = rnb[: nq * k_eff], rds[: nq * k_eff]

    def exact(qi, rid):
        v = oracle.pairwise(metric, q[qi:qi + 1], data32[rid:rid + 1])[0, 0]
        if bitset is not None and not (bitset[rid >> 3] >> (rid & 7)) & 1:
            v = np.float32(np.inf)
        return -v if metric == "inner_product" else v

    if metric == "lp":
        # The reference takes (sum |x-y|^p)^(1/p) with glibc powf, which is not correctly rounded
        # for the 1/2 power (1 ulp off sqrtf in ~0.06% of inputs); this library uses the
        # correctly rounded square root. Same ranking input, distances within 1 ulp.
        assert np.array_equal(nb, rnb), "lp ids"
        assert np.allclose(ds, rds, rtol=2.5e-7, atol=0), "lp distances beyond 1 ulp"
        return
    assert_search_close(nb, ds, rnb, rds, k_eff, exact, TOL[dtype],
                        what=f"{metric}/{dtype}/{n}x{dim}/q{nq}/k{k}", atol_floor=1.0)


@pytest.mark.parametrize("metric", ["l2", "inner_product", "cosine", "l2_sqrt", "hamming", "lp"])
@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_metrics_random(metric, dtype, ovvs, gpu, oracle):
    _run_parity(ovvs, gpu, oracle, metric, dtype, n=5000, dim=40, nq=150, k=10, seed=1)


@pytest.mark.parametrize("dtype", ["i8", "u8"])
@pytest.mark.parametrize("metric", ["l2", "inner_product", "cosine"])
def test_integer_dtypes(metric, dtype, ovvs, gpu, oracle):
    _run_parity(ovvs, gpu, oracle, metric, dtype, n=3000, dim=24, nq=70, k=8, seed=2)


@pytest.mark.parametrize("dim", [1, 2, 5, 16, 17, 31, 48, 64, 96, 100, 128, 160, 200])
def test_dims_and_chunking(dim, ovvs, gpu, oracle):
    _run_parity(ovvs, gpu, oracle, "l2", "f32", n=1700, dim=dim, nq=130, k=7, seed=dim)


@pytest.mark.parametrize("metric,dtype,dim", [
    ("l2", "f32", 320), ("l2", "f16", 384), ("inner_product", "f32", 512),
    ("cosine", "f32", 768), ("l2", "f32", 1000), ("inner_product", "f16", 1536),
    ("l2", "f16", 2048)])
def test_large_dims_streamed_queries(metric, dtype, dim, ovvs, gpu, oracle):
    """Dims whose 128-query tile does not fit shared memory with the ring run the fused kernel's
    streamed-query mode (query chunks travel with each database chunk)."""
    _run_parity(ovvs, gpu, oracle, metric, dtype, n=2500, dim=dim, nq=150, k=9, seed=dim)


def test_max_dim_4096(ovvs, gpu, oracle):
    _run_parity(ovvs, gpu, oracle, "l2", "f32", n=600, dim=4096, nq=40, k=5, seed=4096)


@pytest.mark.parametrize("n,nq,k", [(1, 1, 1), (3, 2, 5), (255, 129, 16), (256, 128, 28),
                                    (257, 127, 3), (513, 1, 1), (1000, 300, 20)])
def test_ragged_sizes(n, nq, k, ovvs, gpu, oracle):
    _run_parity(ovvs, gpu, oracle, "l2", "f32", n=n, dim=12, nq=nq, k=k, seed=n)


@pytest.mark.parametrize("k", [1, 2, 4, 8, 10, 11, 16, 28])
def test_list_sizes(k, ovvs, gpu, oracle):
    _run_parity(ovvs, gpu, oracle, "inner_product", "f16", n=20000, dim=64, nq=200, k=k, seed=k,
                kind="unit", fp16_queries=True)


def test_uniform_c1_shape_full(ovvs, gpu, oracle):
    """Config 1 at full size: L2 fp32, N=100k x 128 Uniform[0,1), Q=1000, k=10."""
    _run_parity(ovvs, gpu, oracle, "l2", "f32", n=100_000, dim=128, nq=1000, k=10, seed=0,
                kind="uniform")


def test_mixture_fp16_l2(ovvs, gpu, oracle):
    """Config-3 distribution (Gaussian mixture, fp16 rows, fp16-rounded queries), scaled down."""
    _run_parity(ovvs, gpu, oracle, "l2", "f16", n=300_000, dim=128, nq=256, k=10, seed=2,
                kind="mixture", fp16_queries=True)


@pytest.mark.parametrize("metric,dtype,k", [("l2", "f32", 1), ("inner_product", "f16", 32),
                                            ("cosine", "f32", 10), ("l2_sqrt", "f16", 7),
                                            ("hamming", "f32", 5)])
def test_small_batch_sampled_bound(metric, dtype, k, ovvs, gpu, oracle):
    """Small batches over a larger database: the work items of one query pair-tile all run at once
    (one wave), so every item fills its lists from nothing."""
    _run_parity(ovvs, gpu, oracle, metric, dtype, n=200_000, dim=48, nq=100, k=k, seed=77,
                kind="mixture")


def test_small_batch_sampled_bound_bitset(ovvs, gpu, oracle):
    """Small batch with few allowed rows (fewer than k in many work items: their lists hold
    filtered rows at +inf) and with more."""
    rng = np.random.default_rng(8)
    n = 200_000
    for frac in (0.001, 0.05):
        bs = ovvs.bitset_from_allow_list(n, np.nonzero(rng.random(n) < frac)[0])
        _run_parity(ovvs, gpu, oracle, "l2", "f32", n=n, dim=40, nq=60, k=32, seed=9, bitset=bs)


def test_bitset_filtering(ovvs, gpu, oracle):
    rng = np.random.default_rng(5)
    n = 9000
    for frac in (0.5, 0.01, 0.0005):
        ids = np.nonzero(rng.random(n) < frac)[0]
        bs = ovvs.bitset_from_allow_list(n, ids)
        _run_parity(ovvs, gpu, oracle, "l2", "f32", n=n, dim=32, nq=64, k=12, seed=6, bitset=bs)
        _run_parity(ovvs, gpu, oracle, "inner_product", "f32", n=n, dim=32, nq=64, k=12, seed=6,
                    bitset=bs)


@pytest.mark.parametrize("n", [9000, 40_000])
@pytest.mark.parametrize("metric", ["l2", "cosine", "l2_sqrt"])
@pytest.mark.parametrize("k", [1, 10])
def test_both_filters(n, metric, k, ovvs, gpu, oracle):
    """Databases of at most 64 tiles (16,384 rows) filter on every column's exact ranking value;
    larger ones on the tile group's conservative bound on the dot product. Both, with and
    without an allow list, against the oracle."""
    rng = np.random.default_rng(n + k)
    _run_parity(ovvs, gpu, oracle, metric, "f32", n=n, dim=32, nq=96, k=k, seed=n + k,
                kind="mixture")
    bs = ovvs.bitset_from_allow_list(n, np.nonzero(rng.random(n) < 0.02)[0])
    _run_parity(ovvs, gpu, oracle, metric, "f32", n=n, dim=32, nq=96, k=k, seed=n + k,
                kind="mixture", bitset=bs)


def test_duplicates_tie_by_lower_id(ovvs, gpu, oracle):
    rng = np.random.default_rng(9)
    base = rng.standard_normal((50, 16)).astype(np.float32)
    data = np.vstack([base[rng.integers(0, 50, 2000)], base])  # many exact duplicates
    q = base[:40] + 0.01
    ix = ovvs.BruteIndex.build(data, resources=gpu)
    nb, ds = ix.search(q, k=20)
    rnb, rds = oracle.brute_search(data, q, 20, "l2")
    assert_search_equal(nb, ds, rnb, rds, what="duplicates")


def test_k_larger_than_n_layout(ovvs, gpu, oracle):
    rng = np.random.default_rng(3)
    data = rng.standard_normal((7, 9)).astype(np.float32)
    q = rng.standard_normal((5, 9)).astype(np.float32)
    for metric in ("l2", "inner_product"):
        ix = ovvs.BruteIndex.build(data, metric=metric, resources=gpu)
        out = (np.full(5 * 12, 4, np.int64), np.full(5 * 12, 3.5, np.float32))
        nb, ds = ix.search(q, k=12, out=out)
        rnb, rds = oracle.brute_search(data, q, 12, metric, out_fill=(4, 3.5))
        assert_search_equal(nb, ds, rnb, rds, what=f"k>n {metric}")


def test_nan_and_inf_rows(ovvs, gpu, oracle):
    rng = np.random.default_rng(11)
    data = rng.standard_normal((600, 20)).astype(np.float32)
    data[17, 3] = np.nan
    data[300, :] = np.nan
    data[42, 0] = np.inf
    q = rng.standard_normal((9, 20)).astype(np.float32)
    for metric in ("l2", "inner_product", "cosine"):
        ix = ovvs.BruteIndex.build(data, metric=metric, resources=gpu)
        nb, ds = ix.search(q, k=600)
        rnb, rds = oracle.brute_search(data, q, 600, metric)
        assert np.array_equal(nb.ravel(), rnb), metric
        assert np.all(same_bits(ds.ravel(), rds)), metric


def test_device_pointer_search_matches_host(ovvs, gpu):
    import torch

    rng = np.random.default_rng(4)
    data = rng.standard_normal((10000, 64)).astype(np.float32)
    q = rng.standard_normal((300, 64)).astype(np.float32)
    ix = ovvs.BruteIndex.build(data, resources=gpu)
    nb, ds = ix.search(q, k=10)
    dq = torch.from_numpy(q).cuda()
    dn = torch.empty((300, 10), dtype=torch.int64, device="cuda")
    dd = torch.empty((300, 10), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ix.search_device(dq, 10, dn, dd)
    gpu.synchronize()
    assert np.array_equal(dn.cpu().numpy(), nb)
    assert np.array_equal(dd.cpu().numpy().view(np.uint32), ds.view(np.uint32))


def test_second_resources_same_index(ovvs, gpu, oracle):
    """ovvs.h: concurrent searches may share an immutable index with distinct Resources."""
    import threading

    rng = np.random.default_rng(12)
    data = rng.standard_normal((20000, 32)).astype(np.float32)
    qs = [rng.standard_normal((100, 32)).astype(np.float32) for _ in range(4)]
    ix = ovvs.BruteIndex.build(data, resources=gpu)
    results = [None] * 4

    def work(i):
        r = ovvs.Resources()
        idx = ovvs.BruteIndex(r, ix._h, ix.n, ix.dim, ix.metric)
        results[i] = idx.search(qs[i], k=5)
        idx._h = None  # borrowed handle
        r.close()

    th = [threading.Thread(target=work, args=(i,)) for i in range(4)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    for i in range(4):
        rnb, rds = oracle.brute_search(data, qs[i], 5, "l2")
        assert_search_equal(results[i][0], results[i][1], rnb, rds, what=f"thread {i}")


@pytest.mark.parametrize("k", [29, 32, 64, 100, 256, 1000])
def test_large_k(k, ovvs, gpu, oracle):
    """k + margin beyond the register lists: bound pre-pass + append buffers + exact select."""
    _run_parity(ovvs, gpu, oracle, "inner_product", "f32", n=40000, dim=48, nq=150, k=k, seed=k,
                kind="unit")


@pytest.mark.parametrize("metric", ["l2", "cosine"])
def test_large_k_l2_cosine_mixture(metric, ovvs, gpu, oracle):
    _run_parity(ovvs, gpu, oracle, metric, "f16", n=60000, dim=64, nq=130, k=100, seed=3,
                kind="mixture", fp16_queries=True)


def test_large_k_small_n_and_bitset(ovvs, gpu, oracle):
    rng = np.random.default_rng(8)
    n = 3000  # no pre-pass: every row is appended
    ids = np.nonzero(rng.random(n) < 0.3)[0]
    bs = ovvs.bitset_from_allow_list(n, ids)
    _run_parity(ovvs, gpu, oracle, "l2", "f32", n=n, dim=20, nq=40, k=200, seed=8, bitset=bs)
    few = ovvs.bitset_from_allow_list(n, ids[:50])  # fewer allowed rows than k
    _run_parity(ovvs, gpu, oracle, "inner_product", "f32", n=n, dim=20, nq=40, k=120, seed=9,
                bitset=few)


def test_large_k_overflow_retry(ovvs, gpu, oracle):
    """Thousands of exact duplicates at the cut-off overflow the append buffers; the bound is
    tightened (finally on keys) until every query fits, and ties still resolve by lower id."""
    rng = np.random.default_rng(10)
    base = rng.standard_normal((4, 24)).astype(np.float32)
    data = np.vstack([base[rng.integers(0, 4, 30000)],
                      rng.standard_normal((20000, 24)).astype(np.float32) * 3])
    q = base + 0.001
    ix = ovvs.BruteIndex.build(data, resources=gpu)
    nb, ds = ix.search(q, k=100)
    rnb, rds = oracle.brute_search(data, q, 100, "l2")
    assert_search_equal(nb, ds, rnb, rds, what="overflow retry")
    ix.close()


def test_phase_history_of_back_to_back_searches(ovvs, gpu):
    """Profiling keeps each search's phase times: three searches enqueued without a
    synchronisation in between give three rows, the last one the last search's phases (recorded
    by separate events at the same stream positions, so equal to within event resolution)."""
    import torch

    rng = np.random.default_rng(21)
    ix = ovvs.BruteIndex.build(rng.standard_normal((20000, 64)).astype(np.float32),
                               resources=gpu)
    dq = torch.from_numpy(rng.standard_normal((300, 64)).astype(np.float32)).cuda()
    dn = torch.empty((300, 10), dtype=torch.int64, device="cuda")
    dd = torch.empty((300, 10), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    gpu.set_profiling(True)
    for _ in range(3):
        ix.search_device(dq, 10, dn, dd)
    last = gpu.last_phase_ms()
    hist = gpu.phase_history()
    gpu.set_profiling(False)
    assert len(hist) == 3
    assert all(row[1] > 0.0 for row in hist)
    assert np.allclose(hist[-1], last, rtol=0.05, atol=0.02)
    assert gpu.phase_history() == []  # reading clears the record
    ix.close()
