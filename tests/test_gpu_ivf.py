"""IVF-Flat on the B200 (ovvsIvfFlat* through the C ABI) against the reference and the oracle.

* Golden cases (outputs of the reference library, tests/golden/make_golden.py): the index built
  here must have the reference's centroids and lists, and the search results must be identical
  (ids and distance bits), extension and (de)serialisation included.
* The reference's own index files (IVF1 format) load here and search identically, which pins the
  search independently of the k-means build.
* Larger seeded cases: the search over this library's index equals the oracle's search over the
  same index parts (read back from the file this library writes), in both the shared-memory
  selection path (k <= 256) and the sort path (k > 256), with a bitset, over several query blocks.
"""

import os

import numpy as np
import pytest

from tests.helpers import assert_search_equal, same_bits

pytestmark = pytest.mark.gpu

LP = 5


def _assert_lp_close(nb, ds, c, name):
    """Lp scores go through powf, which the device evaluates within 2 ulp of glibc's: the ids must
    agree and the distances may differ in the last bits."""
    assert np.array_equal(nb, c["neighbors"]), name
    ref = c["distances"]
    fin = np.isfinite(ref)
    assert np.array_equal(np.isfinite(ds), fin), name
    ulp = np.abs(ds[fin].view(np.int32).astype(np.int64) - ref[fin].view(np.int32).astype(np.int64))
    assert ulp.max(initial=0) <= 2, f"{name}: {ulp.max()} ulp"


def _check(nb, ds, c, name):
    if int(c["metric"]) == LP:
        _assert_lp_close(nb, ds, c, name)
    else:
        assert_search_equal(nb, ds, c["neighbors"], c["distances"], what=name)


def test_golden_build_and_search(golden_ivf, ovvs, gpu, tmp_path):
    from oracle.cpu import read_ivf1

    for name, c in golden_ivf.items():
        ix = ovvs.IvfFlatIndex.build(c["x"], int(c["nlist"]), int(c["metric"]), resources=gpu)
        if c["extra"].shape[0]:
            ix.extend(c["extra"])
        path = str(tmp_path / f"{name}.ivf")
        ix.save(path)
        parts = read_ivf1(path)
        assert np.all(same_bits(parts["centroids"], c["centroids"])), f"{name}: centroids"
        assert np.array_equal(parts["sizes"], c["sizes"]), f"{name}: list sizes"
        assert np.array_equal(parts["ids"], c["ids"]), f"{name}: list ids"
        assert np.array_equal(parts["x"], np.concatenate([c["x"], c["extra"]])), name
        bits = c["bitset"] if c["bitset"].size else None
        nb, ds = ix.search(c["queries"], int(c["k"]), int(c["nprobe"]), bitset=bits)
        _check(nb, ds, c, name)
        ix.close()


def test_reference_index_files_load_and_search(golden_ivf, ovvs, gpu, tmp_path):
    from oracle.cpu import write_ivf1

    for name, c in golden_ivf.items():
        x = np.concatenate([c["x"], c["extra"]])
        path = str(tmp_path / f"{name}.ivf")
        write_ivf1(path, x, c["centroids"], c["sizes"], c["ids"], int(c["metric"]))
        ix = ovvs.IvfFlatIndex.load(path, resources=gpu)
        bits = c["bitset"] if c["bitset"].size else None
        nb, ds = ix.search(c["queries"], int(c["k"]), int(c["nprobe"]), bitset=bits)
        _check(nb, ds, c, name)
        # a round trip through this library's writer reproduces the file byte for byte
        again = str(tmp_path / f"{name}.again")
        ix.save(again)
        with open(path, "rb") as f1, open(again, "rb") as f2:
            assert f1.read() == f2.read(), name
        ix.close()


def _mixture(rng, n, dim, centres, std=2.0):
    c = rng.standard_normal((centres, dim)).astype(np.float32) * std
    return (c[rng.integers(0, centres, n)] + rng.standard_normal((n, dim))).astype(np.float32)


@pytest.mark.parametrize("metric,k,nprobe,with_bits", [
    ("l2", 10, 8, False),      # tensor-core scan
    ("l2", 10, 8, True),       # tensor-core scan with an allow list
    ("l2", 3, 2, 0.004),       # tensor-core scan, fewer allowed rows than k in most lists
    ("inner_product", 32, 4, True),
    ("cosine", 100, 6, False),
    ("l2", 300, 5, True),      # sort path
    ("hamming", 16, 3, False),
])
def test_seeded_search_vs_oracle(metric, k, nprobe, with_bits, ovvs, gpu, oracle, tmp_path):
    from oracle.cpu import read_ivf1

    rng = np.random.default_rng([k, nprobe, len(metric)])
    x = _mixture(rng, 20000, 48, 64)
    q = _mixture(rng, 700, 48, 64)
    ix = ovvs.IvfFlatIndex.build(x, 64, metric, resources=gpu)
    path = str(tmp_path / "ix.ivf")
    ix.save(path)
    parts = read_ivf1(path)
    assert parts["sizes"].sum() == x.shape[0]
    assert np.array_equal(np.sort(parts["ids"]), np.arange(x.shape[0]))
    bits = None
    if with_bits:
        frac = 0.3 if with_bits is True else with_bits
        bits = ovvs.bitset_from_allow_list(x.shape[0],
                                           np.nonzero(rng.random(x.shape[0]) < frac)[0])
    nb, ds = ix.search(q, k, nprobe, bitset=bits)
    rnb, rds = oracle.ivf_flat_search(x, metric, parts["centroids"], parts["sizes"], parts["ids"],
                                      q, k, nprobe, bits)
    assert_search_equal(nb, ds, rnb, rds, what=f"{metric} k={k}")
    ix.close()


def test_device_search_matches_host_search(ovvs, gpu):
    import torch

    rng = np.random.default_rng(5)
    x = _mixture(rng, 8000, 32, 40)
    q = _mixture(rng, 300, 32, 40)
    ix = ovvs.IvfFlatIndex.build(x, 40, "l2", resources=gpu)
    nb, ds = ix.search(q, 12, 5)
    dq = torch.from_numpy(q).cuda()
    dn = torch.full((300, 12), -5, dtype=torch.int64, device="cuda")
    dd = torch.zeros((300, 12), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    ix.search_device(dq, 12, 5, dn, dd)
    gpu.synchronize()
    assert np.array_equal(dn.cpu().numpy(), nb)
    assert np.all(same_bits(dd.cpu().numpy(), ds))
    ix.close()


def test_many_query_blocks(ovvs, gpu, oracle, tmp_path):
    """nlist = 16,384 limits a query block to 4,096 queries: 9,000 queries take three blocks."""
    from oracle.cpu import read_ivf1

    rng = np.random.default_rng(9)
    x = rng.standard_normal((40000, 8)).astype(np.float32)
    q = rng.standard_normal((9000, 8)).astype(np.float32)
    ix = ovvs.IvfFlatIndex.build(x, 16384, "l2", resources=gpu)
    path = str(tmp_path / "ix.ivf")
    ix.save(path)
    parts = read_ivf1(path)
    nb, ds = ix.search(q, 5, 3)
    rnb, rds = oracle.ivf_flat_search(x, "l2", parts["centroids"], parts["sizes"], parts["ids"],
                                      q, 5, 3)
    assert_search_equal(nb, ds, rnb, rds, what="blocks")
    ix.close()


def test_argument_handling(ovvs, gpu, tmp_path):
    rng = np.random.default_rng(1)
    x = rng.random((50, 4), dtype=np.float32)
    ix = ovvs.IvfFlatIndex.build(x, 4, "l2", resources=gpu)
    L = ovvs.lib()
    nb = np.zeros(4, np.int64)
    ds = np.zeros(4, np.float32)
    q = rng.random((1, 4), dtype=np.float32)
    # the reference writes nothing for nq = 0 or k = 0 and returns success
    assert L.ovvsIvfFlatSearch(gpu._h, ix._h, ovvs._ptr(q), 0, 4, 2, None, ovvs._ptr(nb),
                               ovvs._ptr(ds)) == 0
    assert L.ovvsIvfFlatSearch(gpu._h, ix._h, ovvs._ptr(q), 1, 0, 2, None, ovvs._ptr(nb),
                               ovvs._ptr(ds)) == 0
    assert L.ovvsIvfFlatSearch(gpu._h, ix._h, ovvs._ptr(q), -1, 4, 2, None, ovvs._ptr(nb),
                               ovvs._ptr(ds)) == 2
    assert L.ovvsIvfFlatSearch(gpu._h, ix._h, None, 1, 4, 2, None, ovvs._ptr(nb),
                               ovvs._ptr(ds)) == 2
    with pytest.raises(ovvs.OvvsError):
        ovvs.IvfFlatIndex.build(x, 0, "l2", resources=gpu)
    with pytest.raises(ovvs.OvvsError):
        ix.extend(np.zeros((0, 4), np.float32))
    bad = str(tmp_path / "bad.ivf")
    with open(bad, "wb") as f:
        f.write(b"NOPE" + bytes(40))
    with pytest.raises(ovvs.OvvsError) as e:
        ovvs.IvfFlatIndex.load(bad, dim=4, resources=gpu)
    assert e.value.status == 8  # OVVS_STATUS_IO
    with pytest.raises(ovvs.OvvsError):
        ovvs.IvfFlatIndex.load(os.path.join(str(tmp_path), "missing.ivf"), dim=4, resources=gpu)
    ix.close()


def test_device_search_unaligned_queries_and_odd_dim(ovvs, gpu, oracle, tmp_path):
    """Device queries that are not 16-byte aligned, and a dim that is not a multiple of 4, take
    the scan's scalar staging path; the results equal the oracle's."""
    import torch

    from oracle.cpu import read_ivf1

    rng = np.random.default_rng(31)
    for dim in (32, 30):
        x = _mixture(rng, 6000, dim, 20)
        q = _mixture(rng, 200, dim, 20)
        ix = ovvs.IvfFlatIndex.build(x, 20, "l2", resources=gpu)
        path = str(tmp_path / f"ix{dim}.ivf")
        ix.save(path)
        parts = read_ivf1(path)
        rnb, rds = oracle.ivf_flat_search(x, "l2", parts["centroids"], parts["sizes"],
                                          parts["ids"], q, 7, 4)
        buf = torch.zeros(200 * dim + 1, dtype=torch.float32, device="cuda")
        buf[1:].copy_(torch.from_numpy(q.ravel()))
        dq = buf[1:].view(200, dim)  # starts 4 bytes into the allocation
        assert dq.data_ptr() % 16 != 0
        dn = torch.empty((200, 7), dtype=torch.int64, device="cuda")
        dd = torch.empty((200, 7), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        ix.search_device(dq, 7, 4, dn, dd)
        gpu.synchronize()
        assert_search_equal(dn.cpu().numpy(), dd.cpu().numpy(), rnb, rds, what=f"dim {dim}")
        ix.close()
