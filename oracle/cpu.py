"""ctypes bindings for the CPU checkers under oracle/_ref/.

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` and by bench.py's
CPU-baseline / reference arm. The product package (``ovvs_b200``) never imports this module.

Two checkers are exposed:

* :class:`Oracle` -- ``liboracle.so``, this repository's restatement of the reference's
  brute-force / k-means / IVF-Flat arithmetic (oracle/ovvs_oracle.cpp), bit-identical to the
  reference's FORCE_CPU path.

``read_ivf1`` / ``write_ivf1`` read and write index files in the reference's IVF-Flat format.
* :class:`Reference` -- ``libovvs_ref.so``, the reference library itself compiled from its own
  sources by oracle/Makefile (present when the reference checkout was available at build time).
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_float, c_int32, c_int64, c_uint8, c_uint16, c_void_p

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
ORACLE_SO = os.path.join(REF_DIR, "liboracle.so")
REFERENCE_SO = os.path.join(REF_DIR, "libovvs_ref.so")

METRICS = {
    "l2": 0,
    "l2_sqrt": 1,
    "inner_product": 2,
    "cosine": 3,
    "hamming": 4,
    "lp": 5,
}
DTYPES = {"f32": 0, "f16": 1, "i8": 2, "u8": 3, "f8e4m3": 4, "f8e5m2": 5, "f4e2m1": 6}
POLICY_FORCE_CPU = 6


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a, ctype):
    return a.ctypes.data_as(POINTER(ctype)) if a is not None else None


def build_checkers() -> None:
    """Compile oracle/_ref/*.so with oracle/Makefile (no-op when up to date)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", HERE, "-j8"], check=True)


class Oracle:
    """The C++ restatement (bit-identical to the reference's CPU arithmetic)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build_checkers()
        self.lib = ctypes.CDLL(path, mode=ctypes.RTLD_LOCAL)
        L = self.lib
        L.oracle_f16_to_f32.argtypes = [c_uint16]
        L.oracle_f16_to_f32.restype = c_float
        L.oracle_f32_to_f16_trunc.argtypes = [c_float]
        L.oracle_f32_to_f16_trunc.restype = c_uint16
        L.oracle_f32_to_f16_rne.argtypes = [c_float]
        L.oracle_f32_to_f16_rne.restype = c_uint16
        L.oracle_convert_to_f32.argtypes = [c_int32, c_void_p, c_int64, c_int64, POINTER(c_float)]
        L.oracle_pairwise.argtypes = [c_int32, POINTER(c_float), c_int64, POINTER(c_float), c_int64,
                                      c_int64, POINTER(c_float), c_float]
        L.oracle_topk.argtypes = [POINTER(c_float), c_int64, c_int64, c_int64, POINTER(c_int64),
                                  POINTER(c_float), c_int32]
        L.oracle_gemm.argtypes = [POINTER(c_float), POINTER(c_float), POINTER(c_float), c_int64,
                                  c_int64, c_int64, c_int32, c_int32]
        L.oracle_gather_rows.argtypes = [POINTER(c_float), c_int64, c_int64, POINTER(c_int64),
                                         c_int64, POINTER(c_float)]
        L.oracle_all_neighbors.argtypes = [POINTER(c_float), c_int64, c_int64, c_int32, c_int32,
                                           POINTER(c_int64), POINTER(c_float), c_int32]
        L.oracle_brute_search.argtypes = [POINTER(c_float), c_int64, c_int64, c_int32,
                                          POINTER(c_float), c_int64, c_int64, POINTER(c_uint8),
                                          POINTER(c_int64), POINTER(c_float), c_int32]
        L.oracle_kmeans_fit.argtypes = [POINTER(c_float), c_int64, c_int64, c_int32, c_int32,
                                        POINTER(c_float), c_int32]
        L.oracle_kmeans_fit.restype = c_int32
        L.oracle_kmeans_step.argtypes = [POINTER(c_float), c_int64, c_int64, c_int32,
                                         POINTER(c_float), POINTER(c_int64), POINTER(c_float),
                                         c_int32]
        L.oracle_kmeans_predict.argtypes = [POINTER(c_float), c_int32, c_int64, POINTER(c_float),
                                            c_int64, POINTER(c_int64), POINTER(c_float), c_int32]
        L.oracle_kmeans_init_rows.argtypes = [c_int64, c_int32, POINTER(c_int64)]
        L.oracle_kmeans_init_rows.restype = c_int32
        L.oracle_bitset_from_allow_list.argtypes = [c_int64, POINTER(c_int64), c_int64,
                                                    POINTER(c_uint8)]
        L.oracle_bitset_from_allow_list.restype = c_int32
        L.oracle_ivf_flat_build.argtypes = [POINTER(c_float), c_int64, c_int64, c_int32,
                                            POINTER(c_float), POINTER(c_int64), POINTER(c_int64),
                                            c_int32]
        L.oracle_ivf_flat_build.restype = c_int32
        L.oracle_ivf_flat_search.argtypes = [POINTER(c_float), c_int64, c_int64, c_int32,
                                             POINTER(c_float), c_int32, POINTER(c_int64),
                                             POINTER(c_int64), POINTER(c_float), c_int64, c_int64,
                                             c_int32, POINTER(c_uint8), POINTER(c_int64),
                                             POINTER(c_float), c_int32]
        self.nthreads = max(1, os.cpu_count() or 1)

    # -- conversions ---------------------------------------------------------------------
    def convert_to_f32(self, dtype: str, data: np.ndarray) -> np.ndarray:
        data = np.ascontiguousarray(data)
        n, dim = data.shape
        out = np.empty((n, dim), np.float32)
        self.lib.oracle_convert_to_f32(DTYPES[dtype], data.ctypes.data_as(c_void_p), n, dim,
                                       _ptr(out, c_float))
        return out

    def f16_trunc(self, x: np.ndarray) -> np.ndarray:
        """Truncating fp32->fp16 of the reference tests (internal.hpp:831-840), as uint16."""
        x = _f32(x)
        f = np.vectorize(lambda v: self.lib.oracle_f32_to_f16_trunc(float(v)), otypes=[np.uint16])
        return f(x).reshape(x.shape)

    # -- hot path ------------------------------------------------------------------------
    def pairwise(self, metric, x, y, metric_arg=2.0):
        x, y = _f32(x), _f32(y)
        out = np.empty((x.shape[0], y.shape[0]), np.float32)
        self.lib.oracle_pairwise(METRICS.get(metric, metric), _ptr(x, c_float), x.shape[0],
                                 _ptr(y, c_float), y.shape[0], x.shape[1], _ptr(out, c_float),
                                 metric_arg)
        return out

    def topk(self, scores, k, largest=False):
        scores = _f32(scores)
        rows, cols = scores.shape
        ke = min(k, cols)
        idx = np.empty((rows, ke), np.int64)
        val = np.empty((rows, ke), np.float32)
        self.lib.oracle_topk(_ptr(scores, c_float), rows, cols, k, _ptr(idx, c_int64),
                             _ptr(val, c_float), int(largest))
        return idx, val

    def gemm(self, a, b, m, n, k, trans_b=True, round_f16=False):
        a, b = _f32(a).reshape(-1), _f32(b).reshape(-1)
        c = np.empty((m, n), np.float32)
        self.lib.oracle_gemm(_ptr(a, c_float), _ptr(b, c_float), _ptr(c, c_float), m, n, k,
                             int(bool(trans_b)), int(bool(round_f16)))
        return c

    def gather_rows(self, src, indices):
        src = _f32(src)
        ix = np.ascontiguousarray(indices, np.int64)
        out = np.empty((ix.size, src.shape[1]), np.float32)
        self.lib.oracle_gather_rows(_ptr(src, c_float), src.shape[0], src.shape[1],
                                    _ptr(ix, c_int64), ix.size, _ptr(out, c_float))
        return out

    def all_neighbors(self, data, k, metric="l2"):
        data = _f32(data)
        n, dim = data.shape
        ke = min(k, n - 1)
        nb = np.empty((n, ke), np.int64)
        ds = np.empty((n, ke), np.float32)
        self.lib.oracle_all_neighbors(_ptr(data, c_float), n, dim, METRICS.get(metric, metric), k,
                                      _ptr(nb, c_int64), _ptr(ds, c_float), self.nthreads)
        return nb, ds

    def brute_search(self, data, queries, k, metric="l2", bitset=None, out_fill=None,
                     nthreads=None):
        """Returns (neighbors, distances) as flat buffers of nq*k entries (reference layout:
        the first nq*min(k,n) entries hold rows of stride min(k,n)). ``out_fill`` pre-fills the
        output buffers, mirroring caller-owned memory."""
        data, queries = _f32(data), _f32(queries)
        n, dim = data.shape
        nq = queries.shape[0]
        nb = np.full(nq * k, -1 if out_fill is None else out_fill[0], np.int64)
        ds = np.full(nq * k, 0.0 if out_fill is None else out_fill[1], np.float32)
        bs = None if bitset is None else np.ascontiguousarray(bitset, np.uint8)
        self.lib.oracle_brute_search(_ptr(data, c_float), n, dim, METRICS.get(metric, metric),
                                     _ptr(queries, c_float), nq, k, _ptr(bs, c_uint8),
                                     _ptr(nb, c_int64), _ptr(ds, c_float),
                                     nthreads or self.nthreads)
        return nb, ds

    def kmeans_fit(self, x, k, iters):
        x = _f32(x)
        n, dim = x.shape
        c = np.zeros((max(1, min(k, n)), dim), np.float32)
        keff = self.lib.oracle_kmeans_fit(_ptr(x, c_float), n, dim, k, iters, _ptr(c, c_float),
                                          self.nthreads)
        if keff < 0:
            raise ValueError("invalid k-means arguments")
        return c[:keff]

    def kmeans_step(self, x, centroids):
        x = _f32(x)
        c = np.array(centroids, np.float32, copy=True, order="C")
        n, dim = x.shape
        labels = np.empty(n, np.int64)
        dist = np.empty(n, np.float32)
        self.lib.oracle_kmeans_step(_ptr(x, c_float), n, dim, c.shape[0], _ptr(c, c_float),
                                    _ptr(labels, c_int64), _ptr(dist, c_float), self.nthreads)
        return c, labels, dist

    def kmeans_predict(self, centroids, x):
        centroids, x = _f32(centroids), _f32(x)
        n = x.shape[0]
        labels = np.empty(n, np.int64)
        dist = np.empty(n, np.float32)
        self.lib.oracle_kmeans_predict(_ptr(centroids, c_float), centroids.shape[0], x.shape[1],
                                       _ptr(x, c_float), n, _ptr(labels, c_int64),
                                       _ptr(dist, c_float), self.nthreads)
        return labels, dist

    def kmeans_init_rows(self, n, k):
        rows = np.empty(max(1, k), np.int64)
        keff = self.lib.oracle_kmeans_init_rows(n, k, _ptr(rows, c_int64))
        return rows[:keff]

    def ivf_flat_build(self, x, nlist):
        """(centroids [nlist_eff, dim], list sizes [nlist_eff], list ids concatenated [n])."""
        x = _f32(x)
        n, dim = x.shape
        ne = max(1, min(nlist, n))
        c = np.zeros((ne, dim), np.float32)
        sizes = np.zeros(ne, np.int64)
        ids = np.zeros(n, np.int64)
        keff = self.lib.oracle_ivf_flat_build(_ptr(x, c_float), n, dim, nlist, _ptr(c, c_float),
                                              _ptr(sizes, c_int64), _ptr(ids, c_int64),
                                              self.nthreads)
        if keff < 0:
            raise ValueError("invalid IVF-Flat arguments")
        return c[:keff], sizes[:keff], ids[: int(sizes[:keff].sum())]

    def ivf_flat_search(self, x, metric, centroids, sizes, ids, queries, k, nprobe, bitset=None):
        x, centroids, queries = _f32(x), _f32(centroids), _f32(queries)
        sizes = np.ascontiguousarray(sizes, np.int64)
        ids = np.ascontiguousarray(ids, np.int64)
        m = METRICS[metric] if isinstance(metric, str) else int(metric)
        nq = queries.shape[0]
        nb = np.empty(nq * k, np.int64)
        ds = np.empty(nq * k, np.float32)
        bs = None if bitset is None else np.ascontiguousarray(bitset, np.uint8)
        self.lib.oracle_ivf_flat_search(_ptr(x, c_float), x.shape[0], x.shape[1], m,
                                        _ptr(centroids, c_float), centroids.shape[0],
                                        _ptr(sizes, c_int64), _ptr(ids, c_int64),
                                        _ptr(queries, c_float), nq, k, nprobe,
                                        _ptr(bs, c_uint8) if bs is not None else None,
                                        _ptr(nb, c_int64), _ptr(ds, c_float), self.nthreads)
        return nb.reshape(nq, k), ds.reshape(nq, k)

    def bitset_from_allow_list(self, n, ids):
        ids = np.ascontiguousarray(ids, np.int64)
        bs = np.zeros((n + 7) // 8, np.uint8)
        st = self.lib.oracle_bitset_from_allow_list(n, _ptr(ids, c_int64), ids.size,
                                                    _ptr(bs, c_uint8))
        if st != 0:
            raise ValueError("invalid allow list")
        return bs


class Reference:
    """The reference libovvs compiled from its own sources (oracle/_ref/libovvs_ref.so), driven
    through its public C ABI with policy FORCE_CPU."""

    def __init__(self, path: str = REFERENCE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = ctypes.CDLL(path, mode=ctypes.RTLD_LOCAL)
        L = self.lib
        L.ovvsGetVersion.restype = ctypes.c_char_p
        L.ovvsResourcesCreate.argtypes = [POINTER(c_void_p)]
        L.ovvsResourcesDestroy.argtypes = [c_void_p]
        L.ovvsResourcesSetPolicy.argtypes = [c_void_p, c_int32]
        L.ovvsBruteForceBuildTyped.argtypes = [c_void_p, c_void_p, c_int64, c_int64, c_int32,
                                               c_int32, POINTER(c_void_p)]
        L.ovvsBruteForceSearch.argtypes = [c_void_p, c_void_p, POINTER(c_float), c_int64, c_int64,
                                           c_void_p, POINTER(c_int64), POINTER(c_float)]
        L.ovvsBruteForceDestroy.argtypes = [c_void_p]
        L.ovvsKMeansFit.argtypes = [c_void_p, POINTER(c_float), c_int64, c_int64, c_int32, c_int32,
                                    POINTER(c_void_p)]
        L.ovvsKMeansPredict.argtypes = [c_void_p, c_void_p, POINTER(c_float), c_int64,
                                        POINTER(c_int64), POINTER(c_float)]
        L.ovvsKMeansCentroids.argtypes = [c_void_p, POINTER(POINTER(c_float)), POINTER(c_int32),
                                          POINTER(c_int64)]
        L.ovvsKMeansDestroy.argtypes = [c_void_p]
        L.ovvsBitsetFromAllowList.argtypes = [c_int64, POINTER(c_int64), c_int64, POINTER(c_uint8)]
        L.ovvsTopk.argtypes = [c_void_p, POINTER(c_float), c_int64, c_int64, c_int64,
                               POINTER(c_int64), POINTER(c_float), c_int32]
        L.ovvsGemm.argtypes = [c_void_p, POINTER(c_float), POINTER(c_float), POINTER(c_float),
                               c_int64, c_int64, c_int64, c_int32]
        L.ovvsGatherRows.argtypes = [c_void_p, POINTER(c_float), c_int64, c_int64,
                                     POINTER(c_int64), c_int64, POINTER(c_float)]
        L.ovvsPairwiseDistance.argtypes = [c_void_p, c_int32, POINTER(c_float), c_int64,
                                           POINTER(c_float), c_int64, c_int64, POINTER(c_float),
                                           c_float]
        L.ovvsAllNeighbors.argtypes = [c_void_p, POINTER(c_float), c_int64, c_int64, c_int32,
                                       c_int32, POINTER(c_int64), POINTER(c_float)]

    def ivf_flat(self, x, nlist, metric, queries, k, nprobe, bitset=None, extra=None):
        """Builds an IVF-Flat index with the reference (FORCE_CPU), optionally extends it with
        `extra` rows, searches, and returns (neighbors [nq, k], distances [nq, k], the index as
        written by the reference's ovvsIvfFlatSerialize: dict of centroids / sizes / ids)."""
        import tempfile

        L = self.lib
        L.ovvsIvfFlatBuild.argtypes = [c_void_p, POINTER(c_float), c_int64, c_int64, c_int32,
                                       c_int32, POINTER(c_void_p)]
        L.ovvsIvfFlatSearch.argtypes = [c_void_p, c_void_p, POINTER(c_float), c_int64, c_int64,
                                        c_int32, c_void_p, POINTER(c_int64), POINTER(c_float)]
        L.ovvsIvfFlatSerialize.argtypes = [c_void_p, ctypes.c_char_p]
        L.ovvsIvfFlatExtend.argtypes = [c_void_p, c_void_p, POINTER(c_float), c_int64]
        L.ovvsIvfFlatDestroy.argtypes = [c_void_p]
        x, queries = _f32(x), _f32(queries)
        m = METRICS[metric] if isinstance(metric, str) else int(metric)
        res = self.resources()
        ix = c_void_p()
        assert L.ovvsIvfFlatBuild(res, _ptr(x, c_float), x.shape[0], x.shape[1], m, nlist,
                                  ctypes.byref(ix)) == 0
        if extra is not None:
            e = _f32(extra)
            assert L.ovvsIvfFlatExtend(res, ix, _ptr(e, c_float), e.shape[0]) == 0
        nq = queries.shape[0]
        nb = np.empty(nq * k, np.int64)
        ds = np.empty(nq * k, np.float32)
        bs = None if bitset is None else np.ascontiguousarray(bitset, np.uint8)
        assert L.ovvsIvfFlatSearch(res, ix, _ptr(queries, c_float), nq, k, nprobe,
                                   bs.ctypes.data if bs is not None else None,
                                   _ptr(nb, c_int64), _ptr(ds, c_float)) == 0
        with tempfile.TemporaryDirectory() as d:
            path = os.path.join(d, "ivf.bin")
            assert L.ovvsIvfFlatSerialize(ix, path.encode()) == 0
            parts = read_ivf1(path)
        L.ovvsIvfFlatDestroy(ix)
        L.ovvsResourcesDestroy(res)
        return nb.reshape(nq, k), ds.reshape(nq, k), parts

    def resources(self):
        r = c_void_p()
        assert self.lib.ovvsResourcesCreate(ctypes.byref(r)) == 0
        assert self.lib.ovvsResourcesSetPolicy(r, POLICY_FORCE_CPU) == 0
        return r

    def brute_search(self, data, queries, k, metric="l2", dtype="f32", bitset=None,
                     out_fill=None, res=None):
        data = np.ascontiguousarray(data)
        queries = _f32(queries)
        n, dim = data.shape
        nq = queries.shape[0]
        own = res is None
        res = res or self.resources()
        ix = c_void_p()
        st = self.lib.ovvsBruteForceBuildTyped(res, data.ctypes.data_as(c_void_p), n, dim,
                                               METRICS.get(metric, metric), DTYPES[dtype],
                                               ctypes.byref(ix))
        assert st == 0, st
        nb = np.full(nq * k, -1 if out_fill is None else out_fill[0], np.int64)
        ds = np.full(nq * k, 0.0 if out_fill is None else out_fill[1], np.float32)
        bs = None if bitset is None else np.ascontiguousarray(bitset, np.uint8)
        st = self.lib.ovvsBruteForceSearch(res, ix, _ptr(queries, c_float), nq, k,
                                           bs.ctypes.data_as(c_void_p) if bs is not None else None,
                                           _ptr(nb, c_int64), _ptr(ds, c_float))
        assert st == 0, st
        self.lib.ovvsBruteForceDestroy(ix)
        if own:
            self.lib.ovvsResourcesDestroy(res)
        return nb, ds

    def kmeans(self, x, nclusters, iters, predict_x=None, predict=True):
        """Fit, read the centroids and (when ``predict``) predict. Predict is undefined behaviour
        in the reference when nclusters > n (it reads past its centroid buffer), so callers pass
        predict=False there."""
        x = _f32(x)
        n, dim = x.shape
        res = self.resources()
        m = c_void_p()
        assert self.lib.ovvsKMeansFit(res, _ptr(x, c_float), n, dim, nclusters, iters,
                                      ctypes.byref(m)) == 0
        cp = POINTER(c_float)()
        kk = c_int32()
        dd = c_int64()
        assert self.lib.ovvsKMeansCentroids(m, ctypes.byref(cp), ctypes.byref(kk),
                                            ctypes.byref(dd)) == 0
        keff = max(1, min(nclusters, n))
        cents = np.ctypeslib.as_array(cp, shape=(keff * dim,)).reshape(keff, dim).copy()
        px = x if predict_x is None else _f32(predict_x)
        labels = np.empty(px.shape[0] if predict else 0, np.int64)
        dist = np.empty(px.shape[0] if predict else 0, np.float32)
        if predict:
            assert self.lib.ovvsKMeansPredict(res, m, _ptr(px, c_float), px.shape[0],
                                              _ptr(labels, c_int64), _ptr(dist, c_float)) == 0
        self.lib.ovvsKMeansDestroy(m)
        self.lib.ovvsResourcesDestroy(res)
        return cents, int(kk.value), labels, dist

    def bitset_from_allow_list(self, n, ids):
        ids = np.ascontiguousarray(ids, np.int64)
        bs = np.zeros((n + 7) // 8, np.uint8)
        st = self.lib.ovvsBitsetFromAllowList(n, _ptr(ids, c_int64), ids.size, _ptr(bs, c_uint8))
        assert st == 0
        return bs

    def topk(self, scores, k, largest=False):
        scores = _f32(scores)
        rows, cols = scores.shape
        ke = min(k, cols)
        res = self.resources()
        idx = np.empty((rows, ke), np.int64)
        val = np.empty((rows, ke), np.float32)
        assert self.lib.ovvsTopk(res, _ptr(scores, c_float), rows, cols, k, _ptr(idx, c_int64),
                                 _ptr(val, c_float), int(largest)) == 0
        self.lib.ovvsResourcesDestroy(res)
        return idx, val


    def gemm(self, a, b, m, n, k, trans_b=True):
        a, b = _f32(a).reshape(-1), _f32(b).reshape(-1)
        c = np.empty((m, n), np.float32)
        res = self.resources()
        assert self.lib.ovvsGemm(res, _ptr(a, c_float), _ptr(b, c_float), _ptr(c, c_float), m, n,
                                 k, int(bool(trans_b))) == 0
        self.lib.ovvsResourcesDestroy(res)
        return c

    def gather_rows(self, src, indices):
        src = _f32(src)
        ix = np.ascontiguousarray(indices, np.int64)
        out = np.empty((ix.size, src.shape[1]), np.float32)
        res = self.resources()
        assert self.lib.ovvsGatherRows(res, _ptr(src, c_float), src.shape[0], src.shape[1],
                                       _ptr(ix, c_int64), ix.size, _ptr(out, c_float)) == 0
        self.lib.ovvsResourcesDestroy(res)
        return out

    def pairwise(self, metric, x, y, metric_arg=2.0):
        x, y = _f32(x), _f32(y)
        out = np.empty((x.shape[0], y.shape[0]), np.float32)
        res = self.resources()
        assert self.lib.ovvsPairwiseDistance(res, METRICS.get(metric, metric), _ptr(x, c_float),
                                             x.shape[0], _ptr(y, c_float), y.shape[0], x.shape[1],
                                             _ptr(out, c_float), metric_arg) == 0
        self.lib.ovvsResourcesDestroy(res)
        return out

    def all_neighbors(self, data, k, metric="l2"):
        data = _f32(data)
        n, dim = data.shape
        ke = min(k, n - 1)
        nb = np.empty((n, ke), np.int64)
        ds = np.empty((n, ke), np.float32)
        res = self.resources()
        assert self.lib.ovvsAllNeighbors(res, _ptr(data, c_float), n, dim,
                                         METRICS.get(metric, metric), k, _ptr(nb, c_int64),
                                         _ptr(ds, c_float)) == 0
        self.lib.ovvsResourcesDestroy(res)
        return nb, ds


def make_data(n: int, dim: int, seed: int) -> np.ndarray:
    """The reference tests' deterministic LCG data (tests/test_harness.hpp:71-79): values on a
    0.001 grid in [-1, 1)."""
    out = np.empty(n * dim, np.float32)
    s = np.uint32(seed)
    vals = np.empty(n * dim, np.int64)
    with np.errstate(over="ignore"):
        for i in range(n * dim):
            s = np.uint32(s * np.uint32(1664525) + np.uint32(1013904223))
            vals[i] = int(s >> np.uint32(16))
    # C++: (static_cast<int>(s >> 16) % 2000) / 1000.f - 1.f
    out[:] = (vals % 2000).astype(np.float32) / np.float32(1000.0) - np.float32(1.0)
    return out.reshape(n, dim)


def read_ivf1(path):
    """Parses an index file in the reference's IVF1 format (indexes.cpp:368-394): magic, version,
    n, dim, nlist, metric, centroids, rows, then per list an int32 size and its int64 ids."""
    with open(path, "rb") as f:
        buf = f.read()
    n, dim = (int(v) for v in np.frombuffer(buf[8:24], np.int64))
    nlist, metric = (int(v) for v in np.frombuffer(buf[24:32], np.int32))
    at = 32
    cents = np.frombuffer(buf[at: at + 4 * nlist * dim], np.float32).reshape(nlist, dim).copy()
    at += 4 * nlist * dim
    x = np.frombuffer(buf[at: at + 4 * n * dim], np.float32).reshape(n, dim).copy()
    at += 4 * n * dim
    sizes, ids = [], []
    for _ in range(nlist):
        sz = max(0, int(np.frombuffer(buf[at: at + 4], np.int32)[0]))
        at += 4
        sizes.append(sz)
        ids.append(np.frombuffer(buf[at: at + 8 * sz], np.int64))
        at += 8 * sz
    return {"n": n, "dim": dim, "nlist": nlist, "metric": metric, "centroids": cents, "x": x,
            "sizes": np.array(sizes, np.int64),
            "ids": np.concatenate(ids) if ids else np.zeros(0, np.int64)}


def write_ivf1(path, x, centroids, sizes, ids, metric):
    """Writes an index in the reference's IVF1 format (the inverse of read_ivf1)."""
    x = np.ascontiguousarray(x, np.float32)
    centroids = np.ascontiguousarray(centroids, np.float32).reshape(-1, x.shape[1])
    with open(path, "wb") as f:
        f.write(np.array([0x31465649, 1], np.uint32).tobytes())
        f.write(np.array([x.shape[0], x.shape[1]], np.int64).tobytes())
        f.write(np.array([centroids.shape[0], metric], np.int32).tobytes())
        f.write(centroids.tobytes())
        f.write(x.tobytes())
        at = 0
        for sz in np.asarray(sizes, np.int64):
            f.write(np.array([sz], np.int32).tobytes())
            f.write(np.ascontiguousarray(ids[at: at + sz], np.int64).tobytes())
            at += int(sz)
