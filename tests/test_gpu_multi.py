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
        peer = res.peer_bounds()  # the ranks shared their query bounds through peer memory
        klo, khi = row_range(rank, world, KM_N)
        model = ov.KMeans(km[klo:khi], nclusters=KM_K, iters=KM_ITERS, resources=res,
                          row_offset=klo, n_total=KM_N)
        out.put((rank, np.asarray(nb), np.asarray(dist), model.centroids(), peer, None))
    except Exception as e:  # reported to the parent instead of hanging it
        out.put((rank, None, None, None, None, repr(e)))


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
            rank, nb, dist, cent, peer, err = out.get(timeout=300)
            assert err is None, f"rank {rank}: {err}"
            assert peer, f"rank {rank}: sharded search did not share bounds through peer memory"
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


def _group_worker(out):
    """A plain ovvsResourcesCreate over two GPUs (OVVS_CUDA_DEVICES): only ovvs.h entry points."""
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["OVVS_CUDA_DEVICES"] = "0,1"
    try:
        import ovvs_b200 as ov

        data, queries, km = _data()
        res = ov.Resources()
        ix = ov.BruteIndex.build(data, metric="l2", resources=res)
        nb, dist = ix.search(queries, K)
        peer = res.peer_bounds()
        ip = ov.BruteIndex.build(data, metric="inner_product", resources=res)
        bits = ov.bitset_from_allow_list(N, np.arange(0, N, 3))
        nb_ip, dist_ip = ip.search(queries, 25, bitset=bits)
        model = ov.KMeans(km, nclusters=KM_K, iters=KM_ITERS, resources=res)
        labels, _ = model.predict(km)
        out.put((np.asarray(nb), np.asarray(dist), np.asarray(nb_ip), np.asarray(dist_ip),
                 model.centroids(), np.asarray(labels), res.last_device(), peer, None))
        for o in (ix, ip, model, res):
            o.close()
    except Exception as e:
        out.put((None,) * 8 + (repr(e),))


def test_plain_abi_over_two_gpus(ovvs, gpu, oracle):
    """ovvsResourcesCreate with OVVS_CUDA_DEVICES=0,1: build and search shard the rows over both
    GPUs and return exactly the one-GPU results (which are the oracle's); the k-means fit sums
    both shards (fp64) and matches the one-GPU fit to rounding."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    p = ctx.Process(target=_group_worker, args=(out,))
    p.start()
    try:
        nb, dist, nb_ip, dist_ip, cent, labels, last, peer, err = out.get(timeout=300)
        assert err is None, err
        assert peer, "the two GPUs' shards did not share query bounds through peer memory"
        p.join(timeout=60)
        assert p.exitcode == 0
    finally:
        if p.is_alive():
            p.kill()
    assert last == 3  # OVVS_DEVICE_GPU
    data, queries, km = _data()
    ix = ovvs.BruteIndex.build(data, metric="l2", resources=gpu)
    nb1, dist1 = ix.search(queries, K)
    np.testing.assert_array_equal(nb, nb1)
    np.testing.assert_array_equal(dist.view(np.uint32), np.asarray(dist1).view(np.uint32))
    rnb, rds = oracle.brute_search(data, queries, K, "l2")
    np.testing.assert_array_equal(nb.ravel(), rnb)
    ip = ovvs.BruteIndex.build(data, metric="inner_product", resources=gpu)
    bits = ovvs.bitset_from_allow_list(N, np.arange(0, N, 3))
    nb1, dist1 = ip.search(queries, 25, bitset=bits)
    np.testing.assert_array_equal(nb_ip, nb1)
    np.testing.assert_array_equal(dist_ip.view(np.uint32), np.asarray(dist1).view(np.uint32))
    single = ovvs.KMeans(km, nclusters=KM_K, iters=KM_ITERS, resources=gpu).centroids()
    np.testing.assert_allclose(cent, single, rtol=1e-4, atol=1e-5)
    ref_labels, _ = oracle.kmeans_predict(cent, km)
    assert np.mean(labels == ref_labels) > 0.999


def _leaving_worker(rank, uid, out, go, log_path):
    """Rank 1 leaves after the first search (nothing in flight); rank 0 then searches again. Each
    step of rank 0 is logged (flushed) so that a stall shows where it happened."""
    import time

    def log(msg):
        with open(log_path, "a") as f:
            f.write(f"{time.time():.3f} rank {rank}: {msg}\n")
            f.flush()
            os.fsync(f.fileno())

    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["OVVS_NCCL_TIMEOUT_MS"] = "10000"
    # The surviving rank's next fused kernel would write its query bounds into the departed
    # rank's bound array (memory this process keeps mapped, so it stays allocated); this test
    # keeps to NCCL and plain device memory and leaves that case out.
    os.environ["OVVS_PEER_BOUNDS"] = "0"

    def leave(msg):
        out.put(msg)
        out.close()
        out.join_thread()  # the queue's feeder thread has written the message
        os._exit(0)

    try:
        import ovvs_b200 as ov
        from ovvs_b200.shard import row_range

        data, queries, _ = _data()
        res = ov.Resources.sharded(rank, rank, 2, uid)
        lo, hi = row_range(rank, 2, N)
        ix = ov.BruteIndex.build(data[lo:hi], metric="l2", resources=res, row_offset=lo)
        ix.search(queries, K)
        if rank == 1:
            leave((1, "left", None))  # leaves between steps: its search has completed
        go.wait(timeout=120)  # rank 1 has exited
        log("peer gone; searching")
        t0 = time.perf_counter()
        try:
            ix.search(queries, K)
            status = 0
        except ov.OvvsError as e:
            status = e.status
        took = time.perf_counter() - t0
        log(f"search returned status {status} after {took:.1f} s")
        try:
            ix.search(queries, K)  # the communicator is gone: fails at once
            again = 0
        except ov.OvvsError as e:
            again = e.status
        log(f"second search returned status {again}")
        leave((0, (status, took, again, time.perf_counter() - t0 - took), None))
    except Exception as e:
        out.put((rank, None, repr(e)))


def test_rank_leaving_between_steps_fails_closed(ovvs, gpu, tmp_path):
    """One of two ranks exits between searches; the other's next search ends with
    OVVS_STATUS_ERROR once the NCCL deadline (10 s here) passes, the communicator is aborted, and
    later searches fail immediately instead of hanging (fail closed, src/prim/mixer.cpp:47-50)."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    go = ctx.Event()
    uid = ovvs.nccl_unique_id()
    log_path = str(tmp_path / "ranks.log")
    procs = [ctx.Process(target=_leaving_worker, args=(r, uid, out, go, log_path))
             for r in range(2)]
    for p in procs:
        p.start()
    try:
        rank, msg, err = out.get(timeout=300)
        assert err is None and rank == 1 and msg == "left", (rank, msg, err)
        procs[1].join(timeout=60)
        go.set()
        try:
            rank, res, err = out.get(timeout=90)
        except Exception:
            log = open(log_path).read() if os.path.exists(log_path) else "(no log)"
            raise AssertionError("rank 0 did not report after its peer left:\n" + log)
        assert err is None, err
        status, took, again, took_again = res
        assert status == 1, f"search after a rank left returned {status}"  # OVVS_STATUS_ERROR
        assert took < 60, took
        assert again == 1 and took_again < 5, (again, took_again)
        procs[0].join(timeout=60)
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
