"""The primitive entry points (ovvsGemm / GemmEx / Topk / KSelection / GatherRows /
PairwiseDistance, reference src/rt/resources.cpp:178-216) and ovvsAllNeighbors
(src/neighbors/graphs.cpp:3384-3396) on the B200, through the C ABI.

Expected: bit-identical to the reference's CPU path. GEMM, norms and direct distances sum their
products in k order with separately rounded multiply and add, exactly like the reference's naive
loops; top-k and gather move values without arithmetic. Two documented exceptions:
  * LP distances use the device powf, which may differ from the C library's powf by an ulp
    (checked to 2 ulp: rtol 2.5e-7);
  * all-neighbors runs through the brute-force search, whose only allowed difference is a near-tie
    at the cut-off (fp32 tolerance 1e-4 relative), as for ovvsBruteForceSearch.
"""

import os

import numpy as np
import pytest

from tests.helpers import assert_search_close, assert_search_equal, same_bits

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "prims.npz")
_CASES = sorted({k.split("__")[0] for k in np.load(GOLDEN).files})
LP_RTOL = 2.5e-7
METRICS = ["l2", "l2_sqrt", "inner_product", "cosine", "hamming", "lp"]


def _assert_lp_close(got, want, what):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert np.allclose(got, want, rtol=LP_RTOL, atol=0, equal_nan=True), what


@pytest.mark.parametrize("name", _CASES)
def test_golden_case(name, golden_prims, ovvs, gpu):
    c = golden_prims[name]
    kind = name.split("_", 1)[0]
    if kind == "gemm":
        m, k = c["a"].shape
        tb = int(c["trans_b"])
        n = c["b"].shape[0] if tb else c["b"].shape[1]
        got = gpu.gemm(c["a"], c["b"], m, n, k, trans_b=tb)
        assert np.all(same_bits(got, c["c"])), name
        assert gpu.last_compute_dtype() == 0
    elif kind == "topk":
        rows, cols = c["scores"].shape
        idx, val = gpu.topk(c["scores"], rows, cols, int(c["k"]), int(c["largest"]))
        assert np.array_equal(idx, c["idx"]), name
        assert np.all(same_bits(val, c["val"])), name
        idx2, val2 = gpu.k_selection(c["scores"], rows, cols, int(c["k"]), int(c["largest"]))
        assert np.array_equal(idx2, idx) and np.all(same_bits(val2, val))
    elif kind == "gather":
        src = c["src"]
        got = gpu.gather_rows(src, src.shape[0], src.shape[1], c["idx"])
        assert np.all(same_bits(got, c["out"])), name
    elif kind == "pw":
        got = gpu.pairwise_distance(c["x"], c["y"], int(c["metric"]), float(c["arg"]))
        if int(c["metric"]) == 5:
            _assert_lp_close(got, c["out"], name)
        else:
            assert np.all(same_bits(got, c["out"])), name
    elif kind == "an":
        nb, ds = gpu.all_neighbors(c["data"], int(c["k"]), int(c["metric"]))
        if int(c["metric"]) == 5:
            assert np.array_equal(nb, c["neighbors"]), name
            _assert_lp_close(ds, c["distances"], name)
        else:
            assert_search_equal(nb, ds, c["neighbors"], c["distances"], what=name)
    else:
        raise AssertionError(name)
    assert gpu.last_device() == 3


@pytest.mark.parametrize("trans_b", [0, 1])
@pytest.mark.parametrize("m,n,k", [(300, 257, 515), (1, 1, 1), (129, 64, 16), (64, 1000, 3)])
def test_gemm_random(m, n, k, trans_b, ovvs, gpu, oracle):
    rng = np.random.default_rng(m * 7 + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k) if trans_b else (k, n)).astype(np.float32)
    got = gpu.gemm(a, b, m, n, k, trans_b=trans_b)
    want = oracle.gemm(a, b, m, n, k, trans_b=bool(trans_b))
    assert np.all(same_bits(got, want))


def test_gemm_ex_compute_types(ovvs, gpu, oracle):
    """F16 rounds the operands to half (backend_gpu.cpp:523-548); other types compute in F32
    (mixer.cpp:85-90). The F16 result stays within the fp16 tolerance of the fp32 one."""
    rng = np.random.default_rng(3)
    m, n, k = 200, 150, 333
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    f16 = gpu.gemm(a, b, m, n, k, trans_b=1, compute_dtype=1)
    assert gpu.last_compute_dtype() == 1
    assert np.all(same_bits(f16, oracle.gemm(a, b, m, n, k, trans_b=True, round_f16=True)))
    f32 = oracle.gemm(a, b, m, n, k, trans_b=True)
    scale = np.abs(a) @ np.abs(b).T
    assert np.all(np.abs(f16 - f32) <= 2e-3 * scale)
    for dt in (2, 3, 4):
        got = gpu.gemm(a, b, m, n, k, trans_b=1, compute_dtype=dt)
        assert gpu.last_compute_dtype() == 0
        assert np.all(same_bits(got, f32))


def test_gemm_row_blocks(ovvs, gpu, oracle):
    """More output rows than one 1 GiB block: the host loop's blocks join seamlessly."""
    rng = np.random.default_rng(5)
    m, n, k = 70000, 2048, 8
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((n, k)).astype(np.float32)
    got = gpu.gemm(a, b, m, n, k, trans_b=1)
    rows = np.r_[0:50, 65000:m]
    want = oracle.gemm(a[rows], b, rows.size, n, k, trans_b=True)
    assert np.all(same_bits(got[rows], want))


@pytest.mark.parametrize("largest", [0, 1])
@pytest.mark.parametrize("rows,cols,k", [(1000, 5000, 100), (3, 7, 20), (64, 1, 1),
                                         (17, 33000, 700)])
def test_topk_random(rows, cols, k, largest, ovvs, gpu, oracle):
    rng = np.random.default_rng(rows + cols + k)
    s = rng.integers(-50, 50, (rows, cols)).astype(np.float32)  # many ties
    s[rng.random((rows, cols)) < 0.01] = np.nan
    s[rng.random((rows, cols)) < 0.01] = -0.0
    s[rng.random((rows, cols)) < 0.005] = np.inf
    s[rng.random((rows, cols)) < 0.005] = -np.inf
    idx, val = gpu.topk(s, rows, cols, k, largest)
    ridx, rval = oracle.topk(s, k, largest=bool(largest))
    assert np.array_equal(idx, ridx)
    assert np.all(same_bits(val, rval))


def test_topk_row_blocks(ovvs, gpu, oracle):
    """rows * cols past the per-block budget: several device blocks."""
    rng = np.random.default_rng(9)
    rows, cols, k = 12000, 5000, 8
    s = rng.standard_normal((rows, cols)).astype(np.float32)
    idx, val = gpu.topk(s, rows, cols, k, 0)
    sel = np.r_[0:20, 11980:rows]
    ridx, rval = oracle.topk(s[sel], k)
    assert np.array_equal(idx[sel], ridx)
    assert np.all(same_bits(val[sel], rval))
    assert np.all(np.diff(val, axis=1) >= 0)


def test_gather_random(ovvs, gpu, oracle):
    rng = np.random.default_rng(11)
    src = rng.standard_normal((100000, 96)).astype(np.float32)
    src[5, :] = np.nan
    idx = rng.integers(-10, 100010, 50000)
    idx[:3] = [5, -1, 100000]
    got = gpu.gather_rows(src, src.shape[0], src.shape[1], idx)
    assert np.all(same_bits(got, oracle.gather_rows(src, idx)))


@pytest.mark.parametrize("metric", METRICS + [7])
@pytest.mark.parametrize("nx,ny,dim", [(500, 700, 96), (1, 1, 1), (65, 130, 17)])
def test_pairwise_random(metric, nx, ny, dim, ovvs, gpu, oracle):
    rng = np.random.default_rng(nx + ny + dim)
    x = rng.standard_normal((nx, dim)).astype(np.float32)
    y = rng.standard_normal((ny, dim)).astype(np.float32)
    if nx > 1:
        x[0] = 0.0
    got = gpu.pairwise_distance(x, y, metric)
    want = oracle.pairwise(metric, x, y)
    if metric == "lp":
        _assert_lp_close(got, want, metric)
    else:
        assert np.all(same_bits(got, want)), metric


@pytest.mark.parametrize("p", [1.0, 3.0, 0.5, -1.0])
def test_pairwise_lp_orders(p, ovvs, gpu, oracle):
    rng = np.random.default_rng(13)
    x = rng.standard_normal((40, 33)).astype(np.float32)
    y = rng.standard_normal((50, 33)).astype(np.float32)
    got = gpu.pairwise_distance(x, y, "lp", p)
    want = oracle.pairwise("lp", x, y, p)
    assert np.allclose(got, want, rtol=4 * LP_RTOL, atol=0)


def _exact_self(oracle, data, metric):
    def exact(qi, rid):
        if qi == rid:
            v = np.float32(np.inf)
        else:
            v = oracle.pairwise(metric, data[qi:qi + 1], data[rid:rid + 1])[0, 0]
        return -v if metric == "inner_product" else v
    return exact


@pytest.mark.parametrize("metric", METRICS)
@pytest.mark.parametrize("n,dim,k", [(3000, 48, 10), (700, 130, 40), (300, 16, 299)])
def test_all_neighbors_random(metric, n, dim, k, ovvs, gpu, oracle):
    rng = np.random.default_rng(n + dim + k)
    data = rng.standard_normal((n, dim)).astype(np.float32)
    nb, ds = gpu.all_neighbors(data, k, metric)
    rnb, rds = oracle.all_neighbors(data, k, metric)
    ke = min(k, n - 1)
    assert nb.shape == (n, ke)
    if metric == "lp":
        assert np.array_equal(nb, rnb)
        _assert_lp_close(ds, rds, metric)
        return
    assert_search_close(nb, ds, rnb, rds, ke, _exact_self(oracle, data, metric), 1e-4,
                        what=f"all-neighbors {metric} {n}x{dim} k{k}", atol_floor=1.0)


def test_all_neighbors_large_k_and_duplicates(ovvs, gpu, oracle):
    """k beyond the register lists (the large-k search path) on data with exact duplicates,
    where ties resolve by lower row and a row's duplicates precede everything else."""
    rng = np.random.default_rng(17)
    base = rng.standard_normal((400, 24)).astype(np.float32)
    data = np.repeat(base, 3, axis=0)
    for metric in ("l2", "inner_product"):
        nb, ds = gpu.all_neighbors(data, 600, metric)
        rnb, rds = oracle.all_neighbors(data, 600, metric)
        assert_search_equal(nb, ds, rnb, rds, what=f"dup {metric}")


def test_all_neighbors_self_placement_with_nan_and_inf(ovvs, gpu, oracle):
    """The row itself scores +inf: it precedes NaN scores and follows equal +inf scores of lower
    rows (the reference's top-k order), so it can appear in the output."""
    rng = np.random.default_rng(19)
    data = rng.standard_normal((12, 4)).astype(np.float32)
    data[3] = np.nan
    data[7] = np.inf
    data[9] = np.inf
    for metric in ("l2", "inner_product", "l2_sqrt"):
        nb, ds = gpu.all_neighbors(data, 11, metric)
        rnb, rds = oracle.all_neighbors(data, 11, metric)
        assert_search_equal(nb, ds, rnb, rds, what=f"nan/inf {metric}")


def test_all_neighbors_mixture_l2(ovvs, gpu, oracle):
    rng = np.random.default_rng(23)
    centres = rng.normal(0, 2, (64, 64)).astype(np.float32)
    data = (centres[rng.integers(0, 64, 8000)]
            + rng.standard_normal((8000, 64)).astype(np.float32)).astype(np.float32)
    nb, ds = gpu.all_neighbors(data, 32, "l2")
    rnb, rds = oracle.all_neighbors(data, 32, "l2")
    assert_search_close(nb, ds, rnb, rds, 32, _exact_self(oracle, data, "l2"), 1e-4,
                        what="all-neighbors mixture", atol_floor=1.0)
