"""The C ABI surface, host logic and error paths -- no GPU needed (no compute calls)."""

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
# The reference checkout: REF_DIR, else `reference` beside this repository (read only by the CPU
# tests that compare against it; they skip without it)
REF_DIR = os.environ.get("REF_DIR") or os.path.join(os.path.dirname(ROOT), "reference")

def _declared_symbols():
    names = set()
    for d, _, files in os.walk(os.path.join(ROOT, "include")):
        for f in files:
            if f.endswith(".h"):
                src = open(os.path.join(d, f)).read()
                names |= set(re.findall(r"OVVS_API\s+[^;(]*?\b(ovvs[A-Za-z0-9_]+)\s*\(", src))
    return names


def test_library_exports_every_declared_symbol(ovvs):
    lib = ctypes.CDLL(ovvs.library_path(), mode=ctypes.RTLD_LOCAL)
    names = _declared_symbols()
    assert len(names) >= 133
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_reference_abi_names_all_declared():
    """Every entry point of the reference ABI (124 names) is declared in include/ovvs/ovvs.h."""
    ref_h = os.path.join(REF_DIR, "include", "ovvs", "ovvs.h")
    if not os.path.exists(ref_h):
        pytest.skip("reference checkout not present")
    ref = set(re.findall(r"OVVS_API\s+[^;(]*?\b(ovvs[A-Za-z0-9_]+)\s*\(", open(ref_h).read()))
    assert len(ref) == 124
    assert ref <= _declared_symbols()


def test_version_and_status_strings(ovvs):
    L = ovvs.lib()
    assert ovvs.version() == "0.2.0"
    expect = ["success", "error", "invalid argument", "unsupported", "out of memory",
              "compile fail", "shape mismatch", "device unavailable", "io error"]
    for i, s in enumerate(expect):
        assert L.ovvsStatusString(i).decode() == s
    assert L.ovvsStatusString(99).decode() == "unknown"


def test_bitset_matches_reference(ovvs, golden_misc):
    bs = ovvs.bitset_from_allow_list(int(golden_misc["bitset_n"]), golden_misc["bitset_ids"])
    assert np.array_equal(bs, golden_misc["bitset"])
    L = ovvs.lib()
    assert L.ovvsBitsetFromAllowList(0, None, 0, ctypes.c_void_p(bs.ctypes.data)) == 2
    assert L.ovvsBitsetFromAllowList(8, None, -1, ctypes.c_void_p(bs.ctypes.data)) == 2
    assert L.ovvsBitsetFromAllowList(8, None, 0, None) == 2


def test_resources_without_gpu_report_unavailable(ovvs):
    import torch

    if torch.cuda.is_available():
        pytest.skip("host has a GPU")
    res = ovvs.Resources()
    assert not res.gpu_available()
    assert res.sku() == "no-cuda-device"
    assert res.last_device() == 1  # OVVS_DEVICE_CPU until something runs
    with pytest.raises(ovvs.OvvsError) as e:
        ovvs.BruteIndex.build(np.zeros((4, 2), np.float32), resources=res)
    assert e.value.status == 7  # DEVICE_UNAVAILABLE: no CPU fallback


def test_argument_validation_order(ovvs):
    """indexes.cpp:243/257-259 and cluster.cpp:48-49/61: null or non-positive -> INVALID_ARGUMENT,
    checked before any device work."""
    L = ovvs.lib()
    res = ovvs.Resources()
    h = ctypes.c_void_p()
    x = np.zeros((4, 2), np.float32)
    xp = ctypes.c_void_p(x.ctypes.data)
    assert L.ovvsBruteForceBuildTyped(None, xp, 4, 2, 0, 0, ctypes.byref(h)) == 2
    assert L.ovvsBruteForceBuildTyped(res._h, None, 4, 2, 0, 0, ctypes.byref(h)) == 2
    assert L.ovvsBruteForceBuildTyped(res._h, xp, 0, 2, 0, 0, ctypes.byref(h)) == 2
    assert L.ovvsBruteForceBuildTyped(res._h, xp, 4, 0, 0, 0, ctypes.byref(h)) == 2
    assert L.ovvsBruteForceBuildTyped(res._h, xp, 4, 2, 0, 0, None) == 2
    nb = np.zeros(4, np.int64)
    ds = np.zeros(4, np.float32)
    args = [res._h, ctypes.c_void_p(1), xp, 1, 1, None, ctypes.c_void_p(nb.ctypes.data),
            ctypes.c_void_p(ds.ctypes.data)]
    for i, bad in [(0, None), (1, None), (2, None), (3, 0), (4, 0), (6, None), (7, None)]:
        a = list(args)
        a[i] = bad
        assert L.ovvsBruteForceSearch(*a) == 2, i
    assert L.ovvsKMeansFit(res._h, xp, 4, 2, 0, 3, ctypes.byref(h)) == 2
    assert L.ovvsKMeansFit(res._h, xp, 4, 2, 2, 3, None) == 2
    assert L.ovvsKMeansPredict(res._h, None, xp, 4, ctypes.c_void_p(nb.ctypes.data), None) == 2


def test_primitive_argument_validation(ovvs):
    """resources.cpp:178-216 and graphs.cpp:3384: null pointers or non-positive sizes ->
    INVALID_ARGUMENT before any device work; with valid arguments and no GPU,
    DEVICE_UNAVAILABLE (no CPU fallback)."""
    import torch

    L = ovvs.lib()
    res = ovvs.Resources()
    x = np.ones((8, 4), np.float32)
    xp = ctypes.c_void_p(x.ctypes.data)
    ip = ctypes.c_void_p(np.zeros(64, np.int64).ctypes.data)
    i64 = ctypes.c_int64
    gemm = [res._h, xp, xp, xp, i64(2), i64(2), i64(2), 1]
    for i, bad in [(0, None), (1, None), (2, None), (3, None), (4, i64(0)), (5, i64(-1)),
                   (6, i64(0))]:
        a = list(gemm)
        a[i] = bad
        assert L.ovvsGemm(*a) == 2, i
        assert L.ovvsGemmEx(*a, 1) == 2, i
    topk = [res._h, xp, i64(2), i64(4), i64(2), ip, xp, 0]
    for i, bad in [(0, None), (1, None), (2, i64(0)), (3, i64(0)), (4, i64(0)), (5, None),
                   (6, None)]:
        a = list(topk)
        a[i] = bad
        assert L.ovvsTopk(*a) == 2, i
        assert L.ovvsKSelection(*a) == 2, i
    gather = [res._h, xp, i64(8), i64(4), ip, i64(2), xp]
    for i, bad in [(0, None), (1, None), (2, i64(0)), (3, i64(0)), (4, None), (5, i64(0)),
                   (6, None)]:
        a = list(gather)
        a[i] = bad
        assert L.ovvsGatherRows(*a) == 2, i
    pw = [res._h, 0, xp, i64(2), xp, i64(2), i64(4), xp, ctypes.c_float(2.0)]
    for i, bad in [(0, None), (2, None), (3, i64(0)), (4, None), (5, i64(0)), (6, i64(0)),
                   (7, None)]:
        a = list(pw)
        a[i] = bad
        assert L.ovvsPairwiseDistance(*a) == 2, i
    an = [res._h, xp, i64(8), i64(4), 0, 2, ip, xp]
    for i, bad in [(0, None), (1, None), (2, i64(1)), (5, 0), (6, None), (7, None)]:
        a = list(an)
        a[i] = bad
        assert L.ovvsAllNeighbors(*a) == 2, i
    if not torch.cuda.is_available():
        assert L.ovvsGemm(*gemm) == 7
        assert L.ovvsTopk(*topk) == 7
        assert L.ovvsGatherRows(*gather) == 7
        assert L.ovvsPairwiseDistance(*pw) == 7
        assert L.ovvsAllNeighbors(*an) == 7


def test_forced_cpu_or_npu_never_falls_back(ovvs):
    """FORCE_CPU / FORCE_NPU cannot be honoured by a GPU-only library: DEVICE_UNAVAILABLE
    (reference mixer.cpp:47-50: a forced device never falls back)."""
    res = ovvs.Resources()
    for pol in ("force_cpu", "force_npu"):
        res.set_policy(pol)
        assert res.policy() == ovvs.POLICY[pol]
        with pytest.raises(ovvs.OvvsError) as e:
            ovvs.BruteIndex.build(np.zeros((4, 2), np.float32), resources=res)
        assert e.value.status == 7


def test_out_of_scope_entry_points_are_unsupported(ovvs):
    L = ovvs.lib()
    res = ovvs.Resources()
    h = ctypes.c_void_p()
    x = np.zeros((8, 4), np.float32)
    xp = ctypes.c_void_p(x.ctypes.data)
    L.ovvsIvfPqBuild.restype = ctypes.c_int
    assert L.ovvsIvfPqBuild(res._h, xp, ctypes.c_int64(8), ctypes.c_int64(4), 0, 2, 2, 8,
                            ctypes.byref(h)) == 3
    # IVF-Flat is on the B200 path: without a GPU it reports the device as unavailable
    assert L.ovvsIvfFlatBuild(res._h, xp, 8, 4, 0, 2, ctypes.byref(h)) == 7
    assert L.ovvsCagraBuild(res._h, xp, ctypes.c_int64(8), ctypes.c_int64(4), 0, 4, 8, ctypes.byref(h)) == 3
    assert L.ovvsIvfFlatDestroy(None) == 0
    assert L.ovvsSyclEnabled() == 0
    assert L.ovvsGpuHasXmx() == -1
    uj = ctypes.c_int64(5)
    assert L.ovvsResourcesEnergyUj(None, ctypes.byref(uj)) == 3


def test_frozen_stats_structs(ovvs):
    """tests/consumer.c:66-80: stats queries succeed and stamp version + size."""
    L = ovvs.lib()
    res = ovvs.Resources()
    buf = (ctypes.c_uint8 * 256)()
    assert L.ovvsResourcesIvfPqSearchStatsV1(res._h, buf) == 0
    ver, size = np.frombuffer(bytes(buf[:8]), np.uint32)
    assert ver == 1 and size == 200
    assert L.ovvsResourcesCagraBuildStatsV1(res._h, buf) == 0
    ver, size = np.frombuffer(bytes(buf[:8]), np.uint32)
    assert ver == 1 and size == 256


def test_shave_helpers_match_reference_semantics(ovvs):
    L = ovvs.lib()
    scores = np.array([3.0, 1.0, 2.0, 1.0], np.float32)
    idx = np.zeros(3, np.int32)
    val = np.zeros(3, np.float32)
    L.ovvsShaveTopkSmallest(ctypes.c_void_p(scores.ctypes.data), 4, 3,
                            ctypes.c_void_p(idx.ctypes.data), ctypes.c_void_p(val.ctypes.data))
    assert idx.tolist() == [1, 3, 2] and val.tolist() == [1.0, 1.0, 2.0]
    t = np.arange(8, dtype=np.float32)
    code = np.array([1, 3], np.uint8)
    L.ovvsShavePqAdc.restype = ctypes.c_float
    assert L.ovvsShavePqAdc(ctypes.c_void_p(t.ctypes.data), ctypes.c_void_p(code.ctypes.data), 2, 4) == 1.0 + 7.0


def test_reference_python_binding_loads_this_library(ovvs, tmp_path):
    """Drop-in check: the reference's own ctypes binding (python/ovvs) imports against this
    libovvs.so -- every symbol it binds at import time resolves."""
    pkg = os.path.join(REF_DIR, "python")
    if not os.path.isdir(pkg):
        pytest.skip("reference checkout not present")
    import subprocess
    import sys

    env = dict(os.environ, OVVS_LIBRARY=ovvs.library_path(), PYTHONPATH=pkg)
    r = subprocess.run([sys.executable, "-c",
                        "import ovvs; print(ovvs.version()); "
                        "print(ovvs.bitset_from_allow_list(10, [1, 9])[1])"],
                       capture_output=True, text=True, env=env, cwd=str(tmp_path))
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == ["0.2.0", "2"]
