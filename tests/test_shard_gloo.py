"""Sharded search / k-means host logic with world_size 2 on CPU (gloo), no GPU.

Each rank computes its shard's exact top-k with the CPU oracle (global ids = shard offset +
local id), the ranks all-gather their lists, and the merge by (distance, global id) -- the order
the device cross-shard merge uses -- must equal the unsharded search. The k-means seeding split
(each rank contributes the seed rows it owns, the rest zeros, then a sum all-reduce) must equal
the whole-dataset seeding."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ovvs_b200.shard import row_range


def _order_key(v):
    """keys.cuh order_bits: ascending numbers, -0 == +0, NaN last."""
    v = np.float32(v)
    if np.isnan(v):
        return 0xFFFFFFFF
    u = int(np.float32(0.0).view(np.uint32)) if v == 0 else int(v.view(np.uint32))
    return (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)


def merge_shards(ranks, gids, k_eff, negate):
    """Host restatement of the device shard merge (select.cu shard_merge_kernel)."""
    out_n, out_d = [], []
    for q in range(ranks[0].shape[0]):
        cand = []
        for r in range(len(ranks)):
            for j in range(k_eff):
                g = int(gids[r][q, j])
                cand.append((_order_key(ranks[r][q, j]), g, float(ranks[r][q, j])))
        cand.sort(key=lambda c: (c[0], c[1]))
        out_n.append([c[1] for c in cand[:k_eff]])
        out_d.append([(-c[2] if negate else c[2]) for c in cand[:k_eff]])
    return np.array(out_n, np.int64), np.array(out_d, np.float32)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.cpu import Oracle

        oracle = Oracle()
        rng = np.random.default_rng(21)
        n, dim, nq, k = 1001, 16, 37, 9
        data = rng.standard_normal((n, dim)).astype(np.float32)
        data[500] = data[10]  # an exact duplicate across the shard boundary
        data[777, 3] = np.nan
        q = rng.standard_normal((nq, dim)).astype(np.float32)
        lo, hi = row_range(rank, world, n)
        for metric in ("l2", "inner_product", "cosine"):
            nb, ds = oracle.brute_search(data[lo:hi], q, k, metric)
            k_eff = min(k, hi - lo)
            nb = nb[: nq * k_eff].reshape(nq, k_eff) + lo
            ds = ds[: nq * k_eff].reshape(nq, k_eff)
            rank_vals = -ds if metric == "inner_product" else ds
            t_r = torch.from_numpy(np.ascontiguousarray(rank_vals))
            t_g = torch.from_numpy(np.ascontiguousarray(nb))
            all_r = [torch.empty_like(t_r) for _ in range(world)]
            all_g = [torch.empty_like(t_g) for _ in range(world)]
            dist.all_gather(all_r, t_r)
            dist.all_gather(all_g, t_g)
            mn, md = merge_shards([a.numpy() for a in all_r], [a.numpy() for a in all_g],
                                  min(k, n), metric == "inner_product")
            rn, rd = oracle.brute_search(data, q, k, metric)
            assert np.array_equal(mn.ravel(), rn), metric
            assert np.array_equal(md.ravel().view(np.uint32), rd.view(np.uint32)) or \
                np.all((md.ravel() == rd) | (np.isnan(md.ravel()) & np.isnan(rd))), metric
        # k-means seeding split over shards
        kc = 12
        rows = oracle.kmeans_init_rows(n, kc)
        init = np.zeros((kc, dim), np.float32)
        for c, g in enumerate(rows):
            if lo <= g < hi:
                init[c] = data[g]
        t = torch.from_numpy(init)
        dist.all_reduce(t)
        assert np.array_equal(t.numpy(), data[rows])
        results[rank] = True
    finally:
        dist.destroy_process_group()


def test_sharded_merge_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        results = m.dict()
        mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world,
                           join=True, start_method="spawn")
        assert dict(results) == {0: True, 1: True}


@pytest.mark.parametrize("n,world", [(10_000_000, 8), (7, 3), (1, 1), (100, 8)])
def test_row_range_partition(n, world):
    spans = [row_range(r, world, n) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = [b - a for a, b in spans]
    assert max(sizes) - min(sizes) <= 1
