"""ovvs on B200: Python binding of libovvs.so (the ovvs C ABI, sm_100a kernels).

The API mirrors the reference binding's brute-force / k-means surface (python/ovvs/__init__.py:
``neighbors.brute_force.build``, ``BruteIndex.search``, ``KMeans``, ``Batcher``,
``bitset_from_allow_list``), with numpy arrays in and out, plus the B200 extensions of
include/ovvs/ovvs_cuda.h: device-pointer search (any object exposing ``data_ptr()``, e.g. a CUDA
torch tensor) and one-process-per-GPU sharding over NCCL.

The shared library is built in-tree by ``python -m ovvs_b200.build``; there is no CPU fallback
and importing fails loudly when the library is missing.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, byref, c_char_p, c_float, c_int32, c_int64, c_uint8, c_void_p

import numpy as np

__all__ = [
    "OvvsError", "Resources", "BruteIndex", "IvfFlatIndex", "KMeans", "Batcher", "neighbors",
    "bitset_from_allow_list", "version", "library_path", "nccl_unique_id",
    "METRIC", "DTYPE", "POLICY", "STATUS",
]

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "libovvs.so")

METRIC = {"l2": 0, "l2_sqrt": 1, "inner_product": 2, "cosine": 3, "hamming": 4, "lp": 5}
DTYPE = {"f32": 0, "f16": 1, "i8": 2, "u8": 3, "f8e4m3": 4, "f8e5m2": 5, "f4e2m1": 6}
POLICY = {"auto": 0, "npu_if_faster": 1, "gpu_if_faster": 2, "hetero": 3, "force_npu": 4,
          "force_gpu": 5, "force_cpu": 6}
STATUS = {0: "success", 1: "error", 2: "invalid argument", 3: "unsupported", 4: "out of memory",
          5: "compile fail", 6: "shape mismatch", 7: "device unavailable", 8: "io error"}
_NP_DTYPE = {np.dtype(np.float32): "f32", np.dtype(np.float16): "f16", np.dtype(np.int8): "i8",
             np.dtype(np.uint8): "u8"}


class OvvsError(RuntimeError):
    """A non-success ovvsStatus (python/ovvs/__init__.py:509-521)."""

    def __init__(self, operation: str, status: int):
        self.operation = operation
        self.status = int(status)
        super().__init__(f"{operation} failed: {STATUS.get(self.status, 'unknown')} ({status})")


def library_path() -> str:
    return os.environ.get("OVVS_B200_LIBRARY", LIBRARY)


def _bind(lib):
    P = POINTER
    sig = {
        "ovvsGetVersion": ([], c_char_p),
        "ovvsStatusString": ([c_int32], c_char_p),
        "ovvsResourcesCreate": ([P(c_void_p)], c_int32),
        "ovvsResourcesDestroy": ([c_void_p], c_int32),
        "ovvsResourcesSetPolicy": ([c_void_p, c_int32], c_int32),
        "ovvsResourcesGetPolicy": ([c_void_p, P(c_int32)], c_int32),
        "ovvsResourcesGpuAvailable": ([c_void_p, P(c_int32)], c_int32),
        "ovvsResourcesLastDevice": ([c_void_p, P(c_int32)], c_int32),
        "ovvsResourcesLastComputeDtype": ([c_void_p, P(c_int32)], c_int32),
        "ovvsResourcesSku": ([c_void_p, c_char_p, c_int32], c_int32),
        "ovvsBruteForceBuildTyped": ([c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32,
                                      P(c_void_p)], c_int32),
        "ovvsBruteForceSearch": ([c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                  c_void_p, c_void_p], c_int32),
        "ovvsBruteForceDestroy": ([c_void_p], c_int32),
        "ovvsBitsetFromAllowList": ([c_int64, c_void_p, c_int64, c_void_p], c_int32),
        "ovvsKMeansFit": ([c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32, P(c_void_p)],
                          c_int32),
        "ovvsKMeansPredict": ([c_void_p, c_void_p, c_void_p, c_int64, c_void_p, c_void_p],
                              c_int32),
        "ovvsKMeansCentroids": ([c_void_p, P(P(c_float)), P(c_int32), P(c_int64)], c_int32),
        "ovvsKMeansDestroy": ([c_void_p], c_int32),
        "ovvsBatcherCreate": ([c_void_p, c_void_p, c_int32, c_int32, P(c_void_p)], c_int32),
        "ovvsBatcherSearch": ([c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p],
                              c_int32),
        "ovvsBatcherLastBatchSize": ([c_void_p, P(c_int32)], c_int32),
        "ovvsBatcherDestroy": ([c_void_p], c_int32),
        "ovvsGemm": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                      c_int32], c_int32),
        "ovvsGemmEx": ([c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                        c_int32, c_int32], c_int32),
        "ovvsTopk": ([c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                      c_int32], c_int32),
        "ovvsKSelection": ([c_void_p, c_void_p, c_int64, c_int64, c_int64, c_void_p, c_void_p,
                            c_int32], c_int32),
        "ovvsGatherRows": ([c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_int64, c_void_p],
                           c_int32),
        "ovvsPairwiseDistance": ([c_void_p, c_int32, c_void_p, c_int64, c_void_p, c_int64,
                                  c_int64, c_void_p, c_float], c_int32),
        "ovvsAllNeighbors": ([c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32, c_void_p,
                              c_void_p], c_int32),
        "ovvsIvfFlatBuild": ([c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32,
                              P(c_void_p)], c_int32),
        "ovvsIvfFlatSearch": ([c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int32, c_void_p,
                               c_void_p, c_void_p], c_int32),
        "ovvsIvfFlatSerialize": ([c_void_p, c_char_p], c_int32),
        "ovvsIvfFlatDeserialize": ([c_void_p, c_char_p, P(c_void_p)], c_int32),
        "ovvsIvfFlatExtend": ([c_void_p, c_void_p, c_void_p, c_int64], c_int32),
        "ovvsIvfFlatDestroy": ([c_void_p], c_int32),
        # extensions (include/ovvs/ovvs_cuda.h)
        "ovvsIvfFlatSearchDevice": ([c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int32,
                                     c_void_p, c_void_p, c_void_p], c_int32),
        "ovvsResourcesStream": ([c_void_p, P(c_void_p)], c_int32),
        "ovvsResourcesSynchronize": ([c_void_p], c_int32),
        "ovvsResourcesDevice": ([c_void_p, P(c_int32)], c_int32),
        "ovvsBruteForceSearchDevice": ([c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                        c_void_p, c_void_p], c_int32),
        "ovvsBruteForceSearchDeviceNoAlloc": ([c_void_p, c_void_p, c_void_p, c_int64, c_int64,
                                               c_void_p, c_void_p, c_void_p, c_void_p], c_int32),
        "ovvsResourcesSetProfiling": ([c_void_p, c_int32], c_int32),
        "ovvsResourcesLastPhaseMs": ([c_void_p, P(c_float), c_int32], c_int32),
        "ovvsResourcesPhaseHistoryMs": ([c_void_p, P(c_float), c_int32, P(c_int32)], c_int32),
        "ovvsResourcesLastKernelError": ([c_void_p, P(c_int32)], c_int32),
        "ovvsResourcesPeerBounds": ([c_void_p, P(c_int32)], c_int32),
        "ovvsWatchdogSelfTest": ([c_void_p, c_int64, P(c_int32)], c_int32),
        "ovvsNcclUniqueIdSize": ([], c_int32),
        "ovvsNcclUniqueId": ([c_void_p, c_int32], c_int32),
        "ovvsResourcesCreateSharded": ([P(c_void_p), c_int32, c_int32, c_int32, c_void_p,
                                        c_int32], c_int32),
        "ovvsBruteForceBuildShard": ([c_void_p, c_void_p, c_int64, c_int64, c_int32, c_int32,
                                      c_int64, P(c_void_p)], c_int32),
        "ovvsKMeansFitShard": ([c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int32,
                                c_int32, P(c_void_p)], c_int32),
    }
    for name, (args, res) in sig.items():
        f = getattr(lib, name)
        f.argtypes = args
        f.restype = res
    return lib


_lib = None


def lib():
    """The loaded libovvs.so (raises if it has not been built: there is no fallback)."""
    global _lib
    if _lib is None:
        path = library_path()
        if not os.path.exists(path):
            raise ImportError(f"{path} is missing; build it with `python -m ovvs_b200.build`")
        _lib = _bind(ctypes.CDLL(path, mode=ctypes.RTLD_LOCAL))
    return _lib


def _check(status: int, what: str) -> None:
    if status != 0:
        raise OvvsError(what, status)


def version() -> str:
    return lib().ovvsGetVersion().decode()


def _ptr(a) -> c_void_p:
    return c_void_p(a.ctypes.data) if a is not None else c_void_p()


def _dev_ptr(t) -> c_void_p:
    if t is None:
        return c_void_p()
    if hasattr(t, "data_ptr"):
        return c_void_p(t.data_ptr())
    return c_void_p(int(t))


class Resources:
    """One CUDA device + stream (reference: ovvsResources_t). ``device`` defaults to
    OVVS_CUDA_DEVICE or 0."""

    def __init__(self, _handle=None):
        self._h = c_void_p()
        if _handle is not None:
            self._h = _handle
        else:
            _check(lib().ovvsResourcesCreate(byref(self._h)), "resources create")

    @classmethod
    def sharded(cls, device: int, rank: int, world: int, uid: bytes | None):
        """Rank ``rank`` of ``world`` ranks on CUDA device ``device`` (collective when world>1)."""
        h = c_void_p()
        buf = (c_uint8 * max(1, len(uid or b"")))(*(uid or b"\0"))
        _check(lib().ovvsResourcesCreateSharded(byref(h), device, rank, world,
                                                ctypes.cast(buf, c_void_p),
                                                len(uid or b"")), "sharded resources create")
        return cls(_handle=h)

    def close(self):
        if self._h:
            lib().ovvsResourcesDestroy(self._h)
            self._h = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def set_policy(self, policy) -> None:
        p = POLICY[policy] if isinstance(policy, str) else int(policy)
        _check(lib().ovvsResourcesSetPolicy(self._h, p), "set policy")

    def policy(self) -> int:
        v = c_int32()
        _check(lib().ovvsResourcesGetPolicy(self._h, byref(v)), "get policy")
        return v.value

    def gpu_available(self) -> bool:
        v = c_int32()
        _check(lib().ovvsResourcesGpuAvailable(self._h, byref(v)), "gpu available")
        return bool(v.value)

    def last_device(self) -> int:
        v = c_int32()
        _check(lib().ovvsResourcesLastDevice(self._h, byref(v)), "last device")
        return v.value

    def last_compute_dtype(self) -> int:
        v = c_int32()
        _check(lib().ovvsResourcesLastComputeDtype(self._h, byref(v)), "last compute dtype")
        return v.value

    def sku(self) -> str:
        buf = ctypes.create_string_buffer(256)
        _check(lib().ovvsResourcesSku(self._h, buf, 256), "sku")
        return buf.value.decode()

    def stream(self) -> int:
        s = c_void_p()
        _check(lib().ovvsResourcesStream(self._h, byref(s)), "stream")
        return s.value or 0

    def synchronize(self) -> None:
        _check(lib().ovvsResourcesSynchronize(self._h), "synchronize")

    def device(self) -> int:
        v = c_int32()
        _check(lib().ovvsResourcesDevice(self._h, byref(v)), "device")
        return v.value

    def set_profiling(self, enable: bool) -> None:
        _check(lib().ovvsResourcesSetProfiling(self._h, int(bool(enable))), "set profiling")

    def last_phase_ms(self):
        """[query prep, fused kernel, merge + re-rank, cross-shard merge] of the last search."""
        ms = (c_float * 4)()
        _check(lib().ovvsResourcesLastPhaseMs(self._h, ms, 4), "phase times")
        return list(ms)

    def phase_history(self, max_searches=64):
        """The four phase times of each of the last searches run with profiling on (oldest first,
        at most 64), read after they have all been enqueued back to back; clears the record."""
        ms = (c_float * (4 * max_searches))()
        n = c_int32()
        _check(lib().ovvsResourcesPhaseHistoryMs(self._h, ms, max_searches, byref(n)),
               "phase history")
        return [list(ms[4 * i: 4 * i + 4]) for i in range(n.value)]

    # Primitives (reference python/ovvs/__init__.py Resources.gemm / topk / gather_rows, which
    # return flat lists; these return numpy arrays of the same values, shaped [rows, cols]).
    def gemm(self, a, b, m, n, k, trans_b=1, compute_dtype=0) -> np.ndarray:
        """C[m, n] = A[m, k] @ (B[n, k].T if trans_b else B[k, n]) (ovvsGemm / ovvsGemmEx)."""
        a = np.ascontiguousarray(a, np.float32).reshape(-1)
        b = np.ascontiguousarray(b, np.float32).reshape(-1)
        if a.size < m * k or b.size < k * n:
            raise ValueError("gemm operands are smaller than m*k / k*n")
        c = np.empty((m, n), np.float32)
        if compute_dtype:
            st = lib().ovvsGemmEx(self._h, _ptr(a), _ptr(b), _ptr(c), m, n, k, int(trans_b),
                                  int(compute_dtype))
        else:
            st = lib().ovvsGemm(self._h, _ptr(a), _ptr(b), _ptr(c), m, n, k, int(trans_b))
        _check(st, "gemm")
        return c

    def topk(self, scores, rows, cols, k, largest=0):
        """(indices [rows, min(k, cols)], values) of each row's k smallest (largest) scores."""
        s = np.ascontiguousarray(scores, np.float32).reshape(-1)
        if s.size < rows * cols:
            raise ValueError("scores is smaller than rows*cols")
        ke = min(k, cols)
        idx = np.empty((rows, ke), np.int64)
        val = np.empty((rows, ke), np.float32)
        _check(lib().ovvsTopk(self._h, _ptr(s), rows, cols, k, _ptr(idx), _ptr(val),
                              int(largest)), "topk")
        return idx, val

    def k_selection(self, scores, rows, cols, k, largest=0):
        return self.topk(scores, rows, cols, k, largest)

    def gather_rows(self, src, src_rows, dim, indices) -> np.ndarray:
        """out[i] = src[indices[i]] (zeros for an index outside [0, src_rows))."""
        s = np.ascontiguousarray(src, np.float32).reshape(-1)
        if s.size < src_rows * dim:
            raise ValueError("src is smaller than src_rows*dim")
        ix = np.ascontiguousarray(indices, np.int64).reshape(-1)
        out = np.empty((ix.size, dim), np.float32)
        _check(lib().ovvsGatherRows(self._h, _ptr(s), src_rows, dim, _ptr(ix), ix.size,
                                    _ptr(out)), "gather rows")
        return out

    def pairwise_distance(self, x, y, metric="l2", metric_arg=2.0) -> np.ndarray:
        """[nx, ny] scores of ovvsPairwiseDistance."""
        x = np.ascontiguousarray(x, np.float32)
        y = np.ascontiguousarray(y, np.float32)
        if x.ndim != 2 or y.ndim != 2 or x.shape[1] != y.shape[1]:
            raise ValueError("x and y must be 2-D with the same dim")
        m = METRIC[metric] if isinstance(metric, str) else int(metric)
        out = np.empty((x.shape[0], y.shape[0]), np.float32)
        _check(lib().ovvsPairwiseDistance(self._h, m, _ptr(x), x.shape[0], _ptr(y), y.shape[0],
                                          x.shape[1], _ptr(out), float(metric_arg)),
               "pairwise distance")
        return out

    def all_neighbors(self, dataset, k, metric="l2"):
        """Exact kNN graph (ovvsAllNeighbors): (neighbors, distances), [n, min(k, n - 1)]."""
        a = np.ascontiguousarray(dataset, np.float32)
        if a.ndim != 2:
            raise ValueError("dataset must be 2-D [n, dim]")
        m = METRIC[metric] if isinstance(metric, str) else int(metric)
        ke = max(0, min(int(k), a.shape[0] - 1))
        nb = np.empty((a.shape[0], ke), np.int64)
        ds = np.empty((a.shape[0], ke), np.float32)
        _check(lib().ovvsAllNeighbors(self._h, _ptr(a), a.shape[0], a.shape[1], m, int(k),
                                      _ptr(nb), _ptr(ds)), "all neighbors")
        return nb, ds

    def last_kernel_error(self) -> int:
        """Watchdog code seen by the last synchronising call that failed (0 if none); clears it."""
        code = c_int32(0)
        _check(lib().ovvsResourcesLastKernelError(self._h, byref(code)), "last kernel error")
        return code.value

    def peer_bounds(self) -> bool:
        """Whether sharded searches share each query's bound with the other ranks (peer memory)."""
        v = c_int32(0)
        _check(lib().ovvsResourcesPeerBounds(self._h, byref(v)), "peer bounds")
        return bool(v.value)

    def watchdog_self_test(self, limit_ns: int = 50_000_000) -> int:
        """Runs a kernel whose bounded wait is never satisfied; returns the watchdog code (0x201)."""
        code = c_int32(0)
        _check(lib().ovvsWatchdogSelfTest(self._h, int(limit_ns), byref(code)), "watchdog self test")
        return code.value


def nccl_unique_id() -> bytes:
    n = lib().ovvsNcclUniqueIdSize()
    buf = (c_uint8 * n)()
    _check(lib().ovvsNcclUniqueId(ctypes.cast(buf, c_void_p), n), "nccl unique id")
    return bytes(buf)


def bitset_from_allow_list(n: int, ids) -> np.ndarray:
    """(n+7)//8 bytes, bit id (LSB first) set for each id in [0, n) (resources.cpp:218-229)."""
    ids = np.ascontiguousarray(np.asarray(list(ids) if not isinstance(ids, np.ndarray) else ids,
                                          dtype=np.int64))
    out = np.zeros(max(1, (int(n) + 7) // 8), np.uint8)
    _check(lib().ovvsBitsetFromAllowList(int(n), _ptr(ids) if ids.size else c_void_p(), ids.size,
                                         _ptr(out)), "bitset from allow list")
    return out


def _dataset(data, dtype):
    a = np.asarray(data)
    if a.ndim != 2:
        raise ValueError("dataset must be 2-D [n, dim]")
    if dtype is None:
        dtype = _NP_DTYPE.get(a.dtype, "f32")
        if a.dtype not in _NP_DTYPE:
            a = a.astype(np.float32)
    if dtype == "f16" and a.dtype == np.uint16:
        a = a.view(np.float16)
    want = {"f32": np.float32, "f16": np.float16, "i8": np.int8}.get(dtype, np.uint8)
    return np.ascontiguousarray(a, dtype=want if a.dtype != want else None), dtype


class BruteIndex:
    """Exact brute-force kNN index (ovvsBruteForce*). Results are [nq, k] arrays laid out as the
    reference writes them: rows of stride min(k, n) packed at the front of the buffer."""

    def __init__(self, res: Resources, handle: c_void_p, n: int, dim: int, metric: int,
                 own_res: bool = False):
        self._res, self._h, self.n, self.dim, self.metric = res, handle, n, dim, metric
        self._own = own_res

    @classmethod
    def build(cls, dataset, metric="l2", dtype=None, resources: Resources | None = None,
              row_offset: int | None = None):
        res = resources or Resources()
        a, dt = _dataset(dataset, dtype)
        m = METRIC[metric] if isinstance(metric, str) else int(metric)
        h = c_void_p()
        if row_offset is None:
            st = lib().ovvsBruteForceBuildTyped(res._h, _ptr(a), a.shape[0], a.shape[1], m,
                                                DTYPE[dt], byref(h))
        else:
            st = lib().ovvsBruteForceBuildShard(res._h, _ptr(a), a.shape[0], a.shape[1], m,
                                                DTYPE[dt], int(row_offset), byref(h))
        _check(st, "brute-force build")
        return cls(res, h, a.shape[0], a.shape[1], m, own_res=resources is None)

    def close(self):
        if self._h:
            lib().ovvsBruteForceDestroy(self._h)
            self._h = c_void_p()
        if self._own and self._res:
            self._res.close()
            self._res = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def search(self, queries, k=10, bitset=None, allow_list=None, out=None):
        q = np.ascontiguousarray(np.asarray(queries, dtype=np.float32).reshape(-1, self.dim))
        nq = q.shape[0]
        if allow_list is not None:
            bitset = bitset_from_allow_list(self.n, allow_list)
        bs = None if bitset is None else np.ascontiguousarray(bitset, dtype=np.uint8)
        if out is None:
            nb = np.full(nq * k, -1, np.int64)
            ds = np.zeros(nq * k, np.float32)
        else:
            nb, ds = out
        _check(lib().ovvsBruteForceSearch(self._res._h, self._h, _ptr(q), nq, k, _ptr(bs),
                                          _ptr(nb), _ptr(ds)), "brute-force search")
        return nb.reshape(nq, k), ds.reshape(nq, k)

    def search_device(self, queries, k, neighbors, distances, bitset=None):
        """Enqueue a search on device buffers (objects with data_ptr(), or raw pointers):
        queries [nq, dim] f32, neighbors [nq, min(k,n)] i64, distances [nq, min(k,n)] f32."""
        nq = int(queries.shape[0]) if hasattr(queries, "shape") else int(queries[1])
        qp = _dev_ptr(queries if hasattr(queries, "shape") else queries[0])
        _check(lib().ovvsBruteForceSearchDevice(self._res._h, self._h, qp, nq, k,
                                                _dev_ptr(bitset), _dev_ptr(neighbors),
                                                _dev_ptr(distances)), "device search")


    def search_device_no_alloc(self, queries, k, neighbors, distances, bitset=None, stream=0):
        """Like search_device, but the library allocates no device memory (intermediate buffers
        come from its fixed 32 MiB array); runs on `stream` and returns when the work is done."""
        nq = int(queries.shape[0])
        _check(lib().ovvsBruteForceSearchDeviceNoAlloc(self._res._h, self._h, _dev_ptr(queries),
                                                       nq, k, _dev_ptr(bitset),
                                                       _dev_ptr(neighbors), _dev_ptr(distances),
                                                       c_void_p(int(stream))),
               "device search without allocation")


class IvfFlatIndex:
    """IVF-Flat index (ovvsIvfFlat*): k-means lists (12 Lloyd iterations, squared-L2 coarse
    assignment) scanned exactly with the index metric. Results are [nq, k] arrays, -1 / +inf past
    a query's candidates (indexes.cpp:302-358)."""

    def __init__(self, res: Resources, handle: c_void_p, dim: int, own_res: bool = False):
        self._res, self._h, self.dim, self._own = res, handle, dim, own_res

    @classmethod
    def build(cls, dataset, nlist=16, metric="l2", resources: Resources | None = None):
        res = resources or Resources()
        a = np.ascontiguousarray(np.asarray(dataset, dtype=np.float32))
        m = METRIC[metric] if isinstance(metric, str) else int(metric)
        h = c_void_p()
        _check(lib().ovvsIvfFlatBuild(res._h, _ptr(a), a.shape[0], a.shape[1], m, int(nlist),
                                      byref(h)), "ivf-flat build")
        return cls(res, h, a.shape[1], own_res=resources is None)

    @classmethod
    def load(cls, path, dim=None, resources: Resources | None = None):
        """Reads an index file in the reference's IVF1 format (ovvsIvfFlatDeserialize)."""
        res = resources or Resources()
        h = c_void_p()
        _check(lib().ovvsIvfFlatDeserialize(res._h, os.fsencode(path), byref(h)),
               "ivf-flat deserialize")
        if dim is None:
            with open(path, "rb") as f:
                dim = int(np.frombuffer(f.read(24)[16:24], np.int64)[0])
        return cls(res, h, dim, own_res=resources is None)

    def save(self, path):
        _check(lib().ovvsIvfFlatSerialize(self._h, os.fsencode(path)), "ivf-flat serialize")

    def extend(self, rows):
        a = np.ascontiguousarray(np.asarray(rows, dtype=np.float32).reshape(-1, self.dim))
        _check(lib().ovvsIvfFlatExtend(self._res._h, self._h, _ptr(a), a.shape[0]),
               "ivf-flat extend")

    def search(self, queries, k=10, nprobe=1, bitset=None, allow_list=None, n=None):
        q = np.ascontiguousarray(np.asarray(queries, dtype=np.float32).reshape(-1, self.dim))
        nq = q.shape[0]
        if allow_list is not None:
            bitset = bitset_from_allow_list(int(n), allow_list)
        bs = None if bitset is None else np.ascontiguousarray(bitset, dtype=np.uint8)
        nb = np.full(nq * k, -1, np.int64)
        ds = np.zeros(nq * k, np.float32)
        _check(lib().ovvsIvfFlatSearch(self._res._h, self._h, _ptr(q), nq, k, int(nprobe),
                                       _ptr(bs), _ptr(nb), _ptr(ds)), "ivf-flat search")
        return nb.reshape(nq, k), ds.reshape(nq, k)

    def search_device(self, queries, k, nprobe, neighbors, distances, bitset=None):
        """Enqueue a search on device buffers: queries [nq, dim] f32, neighbors [nq, k] i64,
        distances [nq, k] f32 (objects with data_ptr(), e.g. CUDA torch tensors)."""
        nq = int(queries.shape[0])
        _check(lib().ovvsIvfFlatSearchDevice(self._res._h, self._h, _dev_ptr(queries), nq, k,
                                             int(nprobe), _dev_ptr(bitset), _dev_ptr(neighbors),
                                             _dev_ptr(distances)), "ivf-flat device search")

    def close(self):
        if self._h:
            lib().ovvsIvfFlatDestroy(self._h)
            self._h = c_void_p()
        if self._own and self._res:
            self._res.close()
            self._res = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class neighbors:  # noqa: N801  (mirrors the reference's namespace class)
    class brute_force:  # noqa: N801
        @staticmethod
        def build(dataset, dim=None, metric=0, resources=None, dtype=None):
            a = np.asarray(dataset)
            if a.ndim == 1 and dim:
                a = a.reshape(-1, dim)
            return BruteIndex.build(a, metric=metric, dtype=dtype, resources=resources)


class KMeans:
    """Lloyd k-means (ovvsKMeans*); ``iters`` below 4 runs 4, as the reference."""

    def __init__(self, dataset, nclusters=2, iters=12, dim=None, resources=None,
                 row_offset=None, n_total=None):
        self._res = resources or Resources()
        self._own = resources is None
        a = np.ascontiguousarray(np.asarray(dataset, dtype=np.float32))
        if a.ndim == 1 and dim:
            a = a.reshape(-1, dim)
        self.dim = a.shape[1]
        self._h = c_void_p()
        if row_offset is None:
            st = lib().ovvsKMeansFit(self._res._h, _ptr(a), a.shape[0], a.shape[1], nclusters,
                                     iters, byref(self._h))
        else:
            st = lib().ovvsKMeansFitShard(self._res._h, _ptr(a), a.shape[0], int(row_offset),
                                          int(n_total), a.shape[1], nclusters, iters,
                                          byref(self._h))
        _check(st, "kmeans fit")

    def centroids(self) -> np.ndarray:
        p = POINTER(c_float)()
        k = c_int32()
        d = c_int64()
        _check(lib().ovvsKMeansCentroids(self._h, byref(p), byref(k), byref(d)), "centroids")
        return np.ctypeslib.as_array(p, shape=(k.value * d.value,)).reshape(k.value, d.value).copy()

    def predict(self, x):
        a = np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1, self.dim))
        labels = np.empty(a.shape[0], np.int64)
        dist = np.empty(a.shape[0], np.float32)
        _check(lib().ovvsKMeansPredict(self._res._h, self._h, _ptr(a), a.shape[0], _ptr(labels),
                                       _ptr(dist)), "kmeans predict")
        return labels, dist

    def close(self):
        if self._h:
            lib().ovvsKMeansDestroy(self._h)
            self._h = c_void_p()
        if self._own and self._res:
            self._res.close()
            self._res = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Batcher:
    """Dynamic batcher over a BruteIndex (ovvsBatcher*)."""

    def __init__(self, brute_index: BruteIndex, max_batch=8, max_wait_ms=0):
        self._b = c_void_p()
        self.dim = brute_index.dim
        self._ix = brute_index
        _check(lib().ovvsBatcherCreate(brute_index._res._h, brute_index._h, max_batch,
                                       max_wait_ms, byref(self._b)), "batcher create")

    def search(self, queries, k=10):
        q = np.ascontiguousarray(np.asarray(queries, dtype=np.float32).reshape(-1, self.dim))
        nq = q.shape[0]
        nb = np.full(nq * k, -1, np.int64)
        ds = np.zeros(nq * k, np.float32)
        _check(lib().ovvsBatcherSearch(self._b, _ptr(q), nq, k, _ptr(nb), _ptr(ds)),
               "batcher search")
        return nb.reshape(nq, k), ds.reshape(nq, k)

    def last_batch_size(self) -> int:
        v = c_int32()
        _check(lib().ovvsBatcherLastBatchSize(self._b, byref(v)), "last batch size")
        return v.value

    def close(self):
        if self._b:
            lib().ovvsBatcherDestroy(self._b)
            self._b = c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
