"""Parity at the benchmark configurations' full sizes, through the C ABI.

The whole query set is searched on the GPU, so the work decomposition of the measured runs
(super-chunks, items per pair of CTAs, the per-query bound shared across waves, the large-k
append and overflow path) is the one checked; a sample of queries spread over every query tile is
compared with the CPU oracle (the reference's arithmetic, row-sharded over the host cores). Data
comes from bench.py's own generator, so these are the benchmark's inputs.

Expected: ids identical to the oracle's and distances bit-identical, except at near-ties of the
k-th distance within the parity tolerance (fp16 2e-3, fp32 1e-4 relative).
"""

import numpy as np
import pytest

import bench
from tests.helpers import assert_search_close

pytestmark = pytest.mark.gpu


def _config_data(name):
    import torch

    cfg = bench.CONFIGS[name]
    dev = torch.device("cuda", 0)
    data = bench._gen_rows(cfg, 0, cfg["n"], dev, torch).cpu().numpy()
    q = bench._queries(cfg, dev, torch).cpu().numpy()
    torch.cuda.empty_cache()
    return cfg, data, q


def _check(cfg, data, q, sample, ovvs, gpu, oracle, rtol):
    k, metric = cfg["k"], cfg["metric"]
    dtype = cfg["dtype"]
    ix = ovvs.BruteIndex.build(data, metric=metric, dtype=dtype, resources=gpu)
    nb, ds = ix.search(q, k=k)
    ix.close()
    nb, ds = nb[sample], ds[sample]
    data32 = data.astype(np.float32)
    qs = np.ascontiguousarray(q[sample])
    rnb, rds = oracle.brute_search(data32, qs, k, metric)

    def exact(qi, rid):
        v = oracle.pairwise(metric, qs[qi:qi + 1], data32[rid:rid + 1])[0, 0]
        return -v if metric == "inner_product" else v

    assert_search_close(nb, ds, rnb, rds, k, exact, rtol,
                        what=f"{cfg['desc']} ({len(sample)} sampled queries)")


def test_config3_full_size(ovvs, gpu, oracle):
    """Config 3: L2, 10M x 128 fp16 Gaussian mixture, Q = 10k (all searched), k = 10."""
    cfg, data, q = _config_data("c3")
    data = data.view(np.float16)
    sample = np.linspace(0, cfg["nq"] - 1, 32).astype(np.int64)
    _check(cfg, data, q, sample, ovvs, gpu, oracle, 2e-3)


def test_config2_full_size(ovvs, gpu, oracle):
    """Config 2: inner product, 1M x 96 fp32 unit rows, Q = 10k (all searched), k = 100 (the
    large-k path: bound pre-pass, append pass, select + exact re-rank)."""
    cfg, data, q = _config_data("c2")
    sample = np.linspace(0, cfg["nq"] - 1, 200).astype(np.int64)
    _check(cfg, data, q, sample, ovvs, gpu, oracle, 1e-4)
