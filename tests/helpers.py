"""Comparison helpers shared by the parity tests."""

import numpy as np

DTYPE_NP = {"f32": np.float32, "f16": np.float16, "i8": np.int8, "u8": np.uint8,
            "f8e4m3": np.uint8, "f8e5m2": np.uint8, "f4e2m1": np.uint8}


def same_bits(a, b):
    """Bitwise float equality, with every NaN equal to every NaN."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    both_nan = np.isnan(a) & np.isnan(b)
    return (a.view(np.uint32) == b.view(np.uint32)) | both_nan


def assert_search_equal(nb, ds, nb_ref, ds_ref, what=""):
    """Exact parity: identical ids and bit-identical distances (NaN == NaN)."""
    nb = np.asarray(nb).ravel()
    nb_ref = np.asarray(nb_ref).ravel()
    bad_ids = np.nonzero(nb != nb_ref)[0]
    assert bad_ids.size == 0, f"{what}: ids differ at {bad_ids[:10]}: {nb[bad_ids[:10]]} vs {nb_ref[bad_ids[:10]]}"
    ok = same_bits(np.asarray(ds).ravel(), np.asarray(ds_ref).ravel())
    bad = np.nonzero(~ok)[0]
    assert bad.size == 0, (f"{what}: distances differ at {bad[:10]}: "
                           f"{np.asarray(ds).ravel()[bad[:10]]} vs {np.asarray(ds_ref).ravel()[bad[:10]]}")


def assert_search_close(nb, ds, nb_ref, ds_ref, k_eff, exact_dist, rtol, what="",
                        max_mismatch_frac=0.005, atol_floor=None):
    """Parity with near-tie allowance. nb/ds [nq, k_eff]. Where ids agree, distances must be
    bit-identical (both sides evaluate the same reference arithmetic). Where ids differ, the
    reported distance must equal the exact distance of the reported id, and stay within rtol of
    the reference distance at that rank (the neighbours are tied within tolerance)."""
    nb = np.asarray(nb).reshape(-1, k_eff)
    ds = np.asarray(ds).reshape(-1, k_eff)
    nb_ref = np.asarray(nb_ref).reshape(-1, k_eff)
    ds_ref = np.asarray(ds_ref).reshape(-1, k_eff)
    same = nb == nb_ref
    assert np.all(same_bits(ds[same], ds_ref[same])), f"{what}: distance bits differ where ids agree"
    rows, cols = np.nonzero(~same)
    frac = rows.size / max(1, nb.size)
    assert frac <= max_mismatch_frac, f"{what}: {rows.size} id mismatches ({frac:.4%})"
    for q, j in zip(rows, cols):
        d_ex = exact_dist(q, nb[q, j])
        assert same_bits(d_ex, ds[q, j]), f"{what}: reported distance is not exact at q={q}"
        ref = float(ds_ref[q, j])
        floor = atol_floor if atol_floor is not None else 0.0
        assert abs(float(ds[q, j]) - ref) <= rtol * max(abs(ref), floor) + 1e-30, (
            f"{what}: q={q} rank={j} {ds[q, j]} vs {ref} beyond near-tie tolerance")


def ivf_extend_lists(centroids, sizes, ids, n_old, labels, nlist):
    """The lists after ovvsIvfFlatExtend (indexes.cpp:447-455): each new row (id n_old + i) is
    appended to the list of its label, in row order. Returns (sizes, ids)."""
    off = np.concatenate([[0], np.cumsum(sizes)])
    new_sizes, new_ids = [], []
    for c in range(nlist):
        add = n_old + np.nonzero(labels == c)[0]
        new_ids.append(np.concatenate([ids[off[c]:off[c + 1]], add]).astype(np.int64))
        new_sizes.append(int(off[c + 1] - off[c]) + add.size)
    return np.array(new_sizes, np.int64), (np.concatenate(new_ids) if new_ids
                                            else np.zeros(0, np.int64))
