"""Sharded search and k-means on 2 GPUs: one process per GPU, NCCL inside the library.

Rows are split with ovvs_b200.shard.row_range; each rank builds its shard with global ids
(offset + local id) and searches all queries; the library all-gathers the shards' exact top-k and
merges by (distance, global id), so every rank must return exactly the single-GPU result. The
sharded k-means sums per-shard partials in fp64 and all-reduces them, so its centroids match the
single-GPU fit to rounding on well-clustered data. Skipped on a box with one GPU."""
import multiprocessing as mp
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

N, DIM, NQ, K = 40_000, 64, 300, 10
KM_N, KM_K, KM_ITERS = 20_000, 32, 6


def _data():
    rng = np.random.default_rng(11)
    data = rng.standard_normal((N, DIM), dtype=np.float32)
    queries = rng.standard_normal((NQ, DIM), dtype=np.float32)
    # k-means data: well-separated mixture (centres ~ N(0, 9I), points = centre + N(0, I), as in
    # the k-means benchmark config) so that assignments do not hinge on last-bit rounding.
    centres = 3.0 * rng.standard_normal((KM_K, DIM), dtype=np.float32)
    km = (centres[rng.integers(0, KM_K, KM_N)]
          + rng.standard_normal((KM_N, DIM), dtype=np.float32)).astype(np.float32)
    return data, queries, km


def _worker(rank, world, uid, out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        import ovvs_b200 as ov
        from ovvs_b200.shard import row_range

        data, queries, km = _data()
        res = ov.Resources.sharded(rank, rank, world, uid)
        lo, hi = row_range(rank, world, N)
        ix = ov.BruteIndex.build(data[lo:hi], metric="l2", resources=res, row_offset=lo)
        nb, dist = ix.search(queries, K)
        klo, khi = row_range(rank, world, KM_N)
        model = ov.KMeans(km[klo:khi], nclusters=KM_K, iters=KM_ITERS, resources=res,
                          row_offset=klo, n_total=KM_N)
        out.put((rank, np.asarray(nb), np.asarray(dist), model.centroids(), None))
    except Exception as e:  # reported to the parent instead of hanging it
        out.put((rank, None, None, None, repr(e)))


def test_two_gpu_shards_match_one_gpu(ovvs, gpu):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    uid = ovvs.nccl_unique_id()
    procs = [ctx.Process(target=_worker, args=(r, 2, uid, out)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = {}
        for _ in range(2):
            rank, nb, dist, cent, err = out.get(timeout=300)
            assert err is None, f"rank {rank}: {err}"
            got[rank] = (nb, dist, cent)
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()

    data, queries, km = _data()
    ix = ovvs.BruteIndex.build(data, metric="l2", resources=gpu)
    nb1, dist1 = ix.search(queries, K)
    for rank in (0, 1):
        nb, dist, _ = got[rank]
        np.testing.assert_array_equal(nb, nb1)
        np.testing.assert_array_equal(dist.view(np.uint32), np.asarray(dist1).view(np.uint32))

    single = ovvs.KMeans(km, nclusters=KM_K, iters=KM_ITERS, resources=gpu).centroids()
    np.testing.assert_allclose(got[0][2], single, rtol=1e-4, atol=1e-5)
    np.testing.assert_array_equal(got[0][2], got[1][2])
