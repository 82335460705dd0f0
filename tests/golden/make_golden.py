"""Generates the golden fixtures in tests/golden/*.npz by running the REFERENCE library.

The reference (manan-ramnani/ovVS 0.2.0) is compiled from its own sources by oracle/Makefile into
oracle/_ref/libovvs_ref.so and driven through its public C ABI with policy FORCE_CPU. Each fixture
stores the inputs and the reference's outputs, so the tests need neither the reference checkout
nor its build on the GPU box.

Run from the repository root:  python tests/golden/make_golden.py
"""

from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle.cpu import Reference, make_data  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))
METRIC_IDS = {"l2": 0, "l2_sqrt": 1, "inner_product": 2, "cosine": 3, "hamming": 4, "lp": 5,
              "unknown7": 7}


def trunc_f16(x: np.ndarray) -> np.ndarray:
    """Truncating fp32->fp16 of the reference tests (internal.hpp:831-840 and
    tests/test_neighbors.cpp:3636-3646), vectorised."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.int64)
    sign = (b >> 16) & 0x8000
    exp = ((b >> 23) & 0xFF) - 127 + 15
    man = b & 0x7FFFFF
    out = np.where(exp <= 0, sign,
                   np.where(exp >= 31, sign | 0x7C00, sign | (np.clip(exp, 0, 31) << 10) | (man >> 13)))
    return out.astype(np.uint16)


def brute_cases(rng):
    """(name, data, dtype, queries, k, metric, bitset, out_fill)."""
    cases = []
    # --- the reference's own hot-path test scenarios (tests/test_neighbors.cpp) ---
    cases.append(("recall_one_l2", make_data(40, 8, 100), "f32", make_data(5, 8, 101), 4, "l2",
                  None, None))
    tri = np.array([[1, 0], [0, 1], [-1, 0]], np.float32)
    q10 = np.array([[1, 0]], np.float32)
    cases.append(("known_ip", tri, "f32", q10, 2, "inner_product", None, None))
    cases.append(("known_cosine", tri, "f32", q10, 2, "cosine", None, None))
    d16 = make_data(16, 4, 112)
    q16 = make_data(1, 4, 113)
    allow = np.zeros(2, np.uint8)
    for a in (2, 5, 9, 12):
        allow[a >> 3] |= 1 << (a & 7)
    cases.append(("allow_list_l2", d16, "f32", q16, 3, "l2", allow, None))
    cases.append(("allow_list_hamming", d16, "f32", q16, 3, "hamming", None, None))
    cases.append(("allow_list_lp", d16, "f32", q16, 3, "lp", None, None))
    d20 = make_data(20, 4, 110)
    even = np.zeros(3, np.uint8)
    for i in range(0, 20, 2):
        even[i >> 3] |= 1 << (i & 7)
    cases.append(("bitset_even", d20, "f32", make_data(1, 4, 111), 3, "l2", even, None))
    d480 = make_data(20, 8, 480)
    cases.append(("typed_f16_trunc", trunc_f16(d480), "f16", make_data(1, 8, 481), 4, "l2", None,
                  None))
    i8 = np.clip(np.round(d480 * 50.0), -127, 127).astype(np.int8)
    cases.append(("typed_i8", i8, "i8", make_data(1, 8, 481), 4, "l2", None, None))
    cons = (((np.arange(48) * 17) % 100) / np.float32(50.0) - np.float32(1.0)).astype(np.float32)
    cases.append(("consumer_c", cons.reshape(12, 4), "f32",
                  np.array([[0.1, -0.2, 0.3, 0.0]], np.float32), 3, "l2", None, None))

    # --- randomized coverage of every metric path ---
    X = rng.standard_normal((257, 40)).astype(np.float32)
    Q = rng.standard_normal((11, 40)).astype(np.float32)
    for m in METRIC_IDS:
        for k in (1, 10):
            cases.append((f"rand_{m}_k{k}", X, "f32", Q, k, m, None, None))
    U = rng.random((300, 64), dtype=np.float32)
    QU = rng.random((7, 64), dtype=np.float32)
    cases.append(("uniform_l2_k16", U, "f32", QU, 16, "l2", None, None))
    # typed datasets
    G = rng.standard_normal((300, 64)).astype(np.float32) * 3
    cases.append(("f16_rne_l2", G.astype(np.float16).view(np.uint16), "f16",
                  rng.standard_normal((9, 64)).astype(np.float32), 10, "l2", None, None))
    cases.append(("f16_rne_ip", G.astype(np.float16).view(np.uint16), "f16",
                  rng.standard_normal((9, 64)).astype(np.float32), 10, "inner_product", None,
                  None))
    B = rng.integers(0, 256, (200, 24), dtype=np.uint8)
    QB = rng.integers(0, 256, (5, 24)).astype(np.float32)
    cases.append(("u8_l2", B, "u8", QB, 8, "l2", None, None))
    cases.append(("f8e4m3_as_u8_l2", B, "f8e4m3", QB, 8, "l2", None, None))
    cases.append(("i8_cosine", B.view(np.int8), "i8", QB - 128, 8, "cosine", None, None))
    # k > n: output stride min(k, n), IP negates nq*k entries of caller memory
    S = rng.standard_normal((6, 5)).astype(np.float32)
    QS = rng.standard_normal((3, 5)).astype(np.float32)
    for m in ("l2", "inner_product"):
        cases.append((f"k_gt_n_{m}", S, "f32", QS, 9, m, None, (5, 7.0)))
    # fewer allowed rows than k: filtered rows come back as +inf (-inf for IP), by row id
    F = rng.standard_normal((40, 8)).astype(np.float32)
    QF = rng.standard_normal((4, 8)).astype(np.float32)
    few = np.zeros(5, np.uint8)
    for a in (3, 17, 30):
        few[a >> 3] |= 1 << (a & 7)
    for m in ("l2", "inner_product", "cosine"):
        cases.append((f"few_allowed_{m}", F, "f32", QF, 6, m, few, None))
    # exact duplicates (ties by lower id), zero rows, NaN and inf rows (NaN last)
    Dd = rng.standard_normal((64, 12)).astype(np.float32)
    Dd[10] = Dd[3]
    Dd[40] = Dd[3]
    Dd[20] = 0.0
    Dd[21] = 0.0
    Dd[50, 4] = np.nan
    Dd[51, 0] = np.inf
    Qd = np.vstack([Dd[3:4], rng.standard_normal((4, 12)).astype(np.float32)])
    for m in ("l2", "inner_product", "cosine", "l2_sqrt"):
        cases.append((f"ties_nan_{m}", Dd, "f32", Qd, 64, m, None, None))
    return cases


def kmeans_cases(rng):
    cases = []
    blobs = make_data(60, 4, 600)
    blobs[:30, 0] += 5.0  # tests/test_cluster.cpp:15-17
    cases.append(("two_blobs", blobs, 2, 15))
    centres = rng.normal(0, 3, (64, 32)).astype(np.float32)
    lab = rng.integers(0, 64, 3000)
    mix = (centres[lab] + rng.standard_normal((3000, 32)).astype(np.float32)).astype(np.float32)
    cases.append(("mixture_3000x32_k64", mix, 64, 10))
    cases.append(("k_gt_n", rng.standard_normal((20, 6)).astype(np.float32), 30, 3))
    cases.append(("iters0", mix[:500], 16, 0))
    return cases


def prims_cases(rng):
    """Inputs of the primitive entry points (resources.cpp:178-216) and ovvsAllNeighbors
    (graphs.cpp:3384-3396): odd shapes, the top-k edge values, out-of-range gather indices,
    every metric (and an unknown one), duplicate rows."""
    gemm = [
        ("gemm_small_nt", rng.standard_normal((5, 3)), rng.standard_normal((3, 7)), 0),
        ("gemm_small_t", rng.standard_normal((5, 3)), rng.standard_normal((7, 3)), 1),
        ("gemm_odd_t", make_data(33, 129, 11), make_data(65, 129, 12), 1),
        ("gemm_odd_nt", make_data(31, 70, 13), make_data(70, 17, 14), 0),
        ("gemm_k1", rng.standard_normal((4, 1)), rng.standard_normal((1, 6)), 0),
        ("gemm_cancel", np.array([[1e8, 1.0, -1e8]]), np.array([[1.0, 1.0, 1.0], [1.0, 0.5, 1.0]]), 1),
    ]
    edge = np.array([[np.nan, 0.0, -0.0, np.inf, -np.inf, 1.0, 1.0, np.nan],
                     [2.0, -1.0, 2.0, -1.0, np.nan, 0.0, -0.0, 3.0]], np.float32)
    ties = rng.integers(-5, 5, (50, 300)).astype(np.float32)
    topk = [("topk_edge_small", edge, 8, 0), ("topk_edge_large", edge, 8, 1),
            ("topk_k_gt_cols", edge, 10, 0), ("topk_ties_small", ties, 17, 0),
            ("topk_ties_large", ties, 17, 1), ("topk_k1", rng.standard_normal((7, 1000)), 1, 1)]
    gather = [("gather_mixed", rng.standard_normal((10, 5)), np.array([3, -1, 9, 10, 0, 3, 9]))]
    x = make_data(13, 19, 21)
    y = make_data(29, 19, 22)
    signs = rng.choice(np.array([-1.0, -0.0, 0.0, 1.0], np.float32), (29, 19))
    pairwise = [(f"pw_{m}", x, y, m, 2.0) for m in ("l2", "l2_sqrt", "inner_product", "cosine",
                                                   "hamming", "lp", "unknown7")]
    pairwise += [("pw_lp3", x, y, "lp", 3.0), ("pw_lp0", x, y, "lp", 0.0),
                 ("pw_lp1", x, y, "lp", 1.0), ("pw_hamming_zeros", signs[:11], signs, "hamming", 2.0),
                 ("pw_cos_zero_row", np.vstack([x[:3], np.zeros((1, 19))]), y, "cosine", 2.0)]
    base = make_data(200, 16, 31)
    dup = np.repeat(make_data(40, 8, 32), 3, axis=0)
    allnb = [(f"an_{m}", base, m, 7) for m in ("l2", "l2_sqrt", "inner_product", "cosine",
                                              "hamming", "lp")]
    allnb += [("an_dup_l2", dup, "l2", 5), ("an_dup_ip", dup, "inner_product", 4),
              ("an_k_gt_n", make_data(2, 4, 33), "l2", 3),
              ("an_ip_full", make_data(9, 4, 34), "inner_product", 8)]
    return gemm, topk, gather, pairwise, allnb


def write_prims(ref, rng):
    gemm, topk, gather, pairwise, allnb = prims_cases(rng)
    out = {}
    for name, a, b, tb in gemm:
        a = np.ascontiguousarray(a, np.float32)
        b = np.ascontiguousarray(b, np.float32)
        m, k = a.shape
        n = b.shape[0] if tb else b.shape[1]
        out[name + "__a"], out[name + "__b"], out[name + "__trans_b"] = a, b, np.array(tb)
        out[name + "__c"] = ref.gemm(a, b, m, n, k, trans_b=bool(tb))
    for name, sc, k, lg in topk:
        sc = np.ascontiguousarray(sc, np.float32)
        idx, val = ref.topk(sc, k, largest=bool(lg))
        out[name + "__scores"], out[name + "__k"], out[name + "__largest"] = sc, np.array(k), np.array(lg)
        out[name + "__idx"], out[name + "__val"] = idx, val
    for name, src, ix in gather:
        src = np.ascontiguousarray(src, np.float32)
        out[name + "__src"], out[name + "__idx"] = src, ix.astype(np.int64)
        out[name + "__out"] = ref.gather_rows(src, ix)
    for name, xx, yy, m, arg in pairwise:
        xx = np.ascontiguousarray(xx, np.float32)
        yy = np.ascontiguousarray(yy, np.float32)
        out[name + "__x"], out[name + "__y"] = xx, yy
        out[name + "__metric"], out[name + "__arg"] = np.array(METRIC_IDS[m]), np.array(arg, np.float32)
        out[name + "__out"] = ref.pairwise(METRIC_IDS[m], xx, yy, arg)
    for name, data, m, k in allnb:
        data = np.ascontiguousarray(data, np.float32)
        nb, ds = ref.all_neighbors(data, k, METRIC_IDS[m])
        out[name + "__data"], out[name + "__metric"], out[name + "__k"] = data, np.array(METRIC_IDS[m]), np.array(k)
        out[name + "__neighbors"], out[name + "__distances"] = nb, ds
    np.savez_compressed(os.path.join(OUT, "prims.npz"), **out)


def ivf_cases(rng):
    """(name, x, extra, nlist, metric, queries, k, nprobe, bitset) for ovvsIvfFlat*."""
    cases = []
    # the reference's own IVF-Flat scenarios (tests/test_neighbors.cpp)
    cases.append(("recall_l2", make_data(80, 8, 200), None, 8, "l2", make_data(6, 8, 201), 5, 8,
                  None))
    tri = np.array([[1, 0], [0, 1], [-1, 0], [0.5, 0.5]], np.float32)
    cases.append(("known_ip", tri, None, 1, "inner_product", np.array([[1, 0]], np.float32), 2, 1,
                  None))
    allx = make_data(45, 8, 450)
    cases.append(("serialize_extend", allx[:40], allx[40:], 8, "l2", make_data(4, 8, 451), 4, 8,
                  None))
    # every metric (unknown values score as squared L2), few probes
    x = rng.standard_normal((400, 12)).astype(np.float32)
    q = rng.standard_normal((20, 12)).astype(np.float32)
    for metric in ("l2", "l2_sqrt", "inner_product", "cosine", "hamming", "lp", "unknown7"):
        cases.append((f"metric_{metric}", x, None, 10, metric, q, 7, 3, None))
    # filtered rows score +inf and can still be returned
    x = rng.standard_normal((300, 16)).astype(np.float32)
    q = rng.standard_normal((15, 16)).astype(np.float32)
    bits = np.zeros((300 + 7) // 8, np.uint8)
    for i in range(0, 300, 3):
        bits[i >> 3] |= 1 << (i & 7)
    cases.append(("bitset_l2", x, None, 6, "l2", q, 9, 2, bits))
    few = np.zeros((300 + 7) // 8, np.uint8)
    for i in (4, 150, 299):
        few[i >> 3] |= 1 << (i & 7)
    cases.append(("bitset_ip_few", x, None, 6, "inner_product", q, 9, 6, few))
    # more neighbours than candidates: -1 / +inf padding
    x = rng.random((60, 4), dtype=np.float32)
    cases.append(("k_exceeds_candidates", x, None, 6, "l2", rng.random((5, 4), dtype=np.float32),
                  40, 1, None))
    # nprobe clamped to [1, nlist]
    cases.append(("nprobe_clamped", x, None, 5, "l2", rng.random((5, 4), dtype=np.float32), 6,
                  100, None))
    cases.append(("nprobe_zero", x, None, 5, "cosine", rng.random((5, 4), dtype=np.float32), 6, 0,
                  None))
    # nlist above n
    cases.append(("nlist_gt_n", rng.random((5, 3), dtype=np.float32), None, 16, "l2",
                  rng.random((4, 3), dtype=np.float32), 3, 2, None))
    # duplicate rows: equal scores, ties to the earlier position in the probe concatenation
    base = np.round(rng.standard_normal((40, 6)), 1).astype(np.float32)
    dup = np.concatenate([base, base[:20], base[5:15]])
    cases.append(("duplicates_ip", dup, None, 4, "inner_product",
                  np.round(rng.standard_normal((8, 6)), 1).astype(np.float32), 12, 4, None))
    cases.append(("duplicates_l2", dup, None, 4, "l2",
                  np.round(rng.standard_normal((8, 6)), 1).astype(np.float32), 12, 2, None))
    # k above the shared-memory list limit (the sort path)
    x = rng.standard_normal((700, 8)).astype(np.float32)
    cases.append(("large_k", x, None, 4, "l2", rng.standard_normal((6, 8)).astype(np.float32),
                  300, 3, None))
    return cases


def write_ivf(ref, rng):
    out = {}
    names = []
    for (name, x, extra, nlist, metric, q, k, nprobe, bits) in ivf_cases(rng):
        m = METRIC_IDS[metric]
        nb, ds, parts = ref.ivf_flat(x, nlist, m, q, k, nprobe, bitset=bits, extra=extra)
        p = f"{name}__"
        names.append(name)
        out[p + "x"] = np.ascontiguousarray(x, np.float32)
        out[p + "extra"] = (np.zeros((0, x.shape[1]), np.float32) if extra is None
                            else np.ascontiguousarray(extra, np.float32))
        out[p + "nlist"] = np.array(nlist)
        out[p + "metric"] = np.array(m)
        out[p + "queries"] = np.ascontiguousarray(q, np.float32)
        out[p + "k"] = np.array(k)
        out[p + "nprobe"] = np.array(nprobe)
        out[p + "bitset"] = np.zeros(0, np.uint8) if bits is None else bits
        out[p + "neighbors"] = nb
        out[p + "distances"] = ds
        out[p + "centroids"] = parts["centroids"]
        out[p + "sizes"] = parts["sizes"]
        out[p + "ids"] = parts["ids"]
    out["cases"] = np.array(names)
    np.savez_compressed(os.path.join(OUT, "ivf_flat.npz"), **out)


def main():
    ref = Reference()
    rng = np.random.default_rng(20261201)
    brute = {}
    for (name, data, dtype, q, k, metric, bitset, fill) in brute_cases(rng):
        nb, ds = ref.brute_search(data, q, k, metric=METRIC_IDS[metric] if metric in METRIC_IDS
                                  else metric, dtype=dtype, bitset=bitset, out_fill=fill)
        p = f"{name}__"
        brute[p + "data"] = np.ascontiguousarray(data)
        brute[p + "dtype"] = np.array(dtype)
        brute[p + "queries"] = np.ascontiguousarray(q, np.float32)
        brute[p + "k"] = np.array(k)
        brute[p + "metric"] = np.array(METRIC_IDS[metric])
        brute[p + "bitset"] = np.zeros(0, np.uint8) if bitset is None else bitset
        brute[p + "fill"] = np.array([-1, 0.0] if fill is None else list(fill), np.float64)
        brute[p + "neighbors"] = nb
        brute[p + "distances"] = ds
    np.savez_compressed(os.path.join(OUT, "brute_force.npz"), **brute)

    km = {}
    for (name, x, k, iters) in kmeans_cases(rng):
        cents, kk, labels, dist = ref.kmeans(x, k, iters, predict=k <= x.shape[0])
        p = f"{name}__"
        km[p + "x"] = x
        km[p + "nclusters"] = np.array(k)
        km[p + "iters"] = np.array(iters)
        km[p + "centroids"] = cents
        km[p + "reported_k"] = np.array(kk)
        km[p + "labels"] = labels
        km[p + "distances"] = dist
    np.savez_compressed(os.path.join(OUT, "kmeans.npz"), **km)

    # top-k total order (cpu_prims.cpp:24-32) on the reference's own edge values
    scores = np.array([[np.nan, 0.0, -0.0, np.inf, -np.inf, 1.0, 1.0, np.nan]], np.float32)
    idx, val = ref.topk(scores, 8, largest=False)
    bs = ref.bitset_from_allow_list(20, np.array([2, 5, 9, 12, -1, 25, 19], np.int64))
    np.savez_compressed(os.path.join(OUT, "misc.npz"), topk_scores=scores, topk_idx=idx,
                        topk_val=val, bitset_ids=np.array([2, 5, 9, 12, -1, 25, 19], np.int64),
                        bitset_n=np.array(20), bitset=bs,
                        version=np.array(ref.lib.ovvsGetVersion().decode()))
    write_prims(ref, np.random.default_rng(20261202))
    write_ivf(ref, np.random.default_rng(20261203))
    print("wrote", sorted(f for f in os.listdir(OUT) if f.endswith(".npz")))


if __name__ == "__main__":
    if sys.argv[1:] == ["ivf"]:  # only the IVF-Flat fixtures
        write_ivf(Reference(), np.random.default_rng(20261203))
    else:
        main()
