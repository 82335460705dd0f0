#!/usr/bin/env python
"""Benchmark of the ovvs brute-force kNN path on B200.

Workload (default; the headline metric "kNN queries/sec @ N=10M D=128 fp16 k=10"): config 3 --
L2 kNN over N=10,000,000 x 128 fp16 rows drawn from a Gaussian mixture of 1,024 centres
(centres ~ N(0, 4I), rows = centre + N(0, I)), Q=10,000 queries from the same mixture rounded to
fp16, k=10, seed 2. Data is synthetic and generated on the GPU with torch's seeded CUDA RNG in
1M-row chunks (chunk c uses seed 1000*seed + c), so every GPU count sees the same rows.

One step = one search of all Q queries. `value` times K device-pointer searches
(ovvsBruteForceSearchDevice, inputs resident in HBM) with CUDA events on the library's stream;
`e2e` times K host-buffer searches through the C ABI (ovvsBruteForceSearch: pageable host
queries in, host results out, copies inside the timed region). N>1 GPUs (torchrun): rows are
sharded, every rank searches all queries, per-shard candidates meet in an NCCL all-gather;
times are the max over ranks.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config c3]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CONFIGS = {
    "c1": dict(metric="l2", dtype="f32", n=100_000, dim=128, nq=1_000, k=10, dist="uniform",
               seed=0, desc="L2 fp32, N=100k x 128 Uniform[0,1), Q=1000, k=10"),
    "c2": dict(metric="inner_product", dtype="f32", n=1_000_000, dim=96, nq=10_000, k=100,
               dist="unit", seed=1, desc="IP fp32, N=1M x 96 unit-norm N(0,1), Q=10k, k=100"),
    "c3": dict(metric="l2", dtype="f16", n=10_000_000, dim=128, nq=10_000, k=10, dist="mixture",
               centres=1024, centre_std=2.0, seed=2,
               desc="L2 fp16, N=10M x 128 Gaussian mixture (1024 centres, var 4), Q=10k, k=10"),
    # profiling case: config 3's distribution and queries with 2M rows (512 MB, > L2)
    "c3s": dict(metric="l2", dtype="f16", n=2_000_000, dim=128, nq=10_000, k=10, dist="mixture",
                centres=1024, centre_std=2.0, seed=2,
                desc="L2 fp16, N=2M x 128 Gaussian mixture (1024 centres), Q=10k, k=10"),
    # one rank's share of config 3 on 8 GPUs (1.25M rows), searched by one GPU: the per-rank kernel
    "c3r": dict(metric="l2", dtype="f16", n=1_250_000, dim=128, nq=10_000, k=10, dist="mixture",
                centres=1024, centre_std=2.0, seed=2,
                desc="L2 fp16, N=1.25M x 128 Gaussian mixture (1024 centres), Q=10k, k=10 "
                     "(one rank's rows of config 3 on 8 GPUs)"),
    # small query batch over config 3's database: one pair tile of 256 queries, HBM-bound
    "c3b": dict(metric="l2", dtype="f16", n=10_000_000, dim=128, nq=256, k=10, dist="mixture",
                centres=1024, centre_std=2.0, seed=2, bound="hbm",
                desc="L2 fp16, N=10M x 128 Gaussian mixture (1024 centres), Q=256, k=10 "
                     "(small batch: HBM-bound)"),
    # profiling case of c3b: 2M rows (512 MB, > L2)
    "c3sb": dict(metric="l2", dtype="f16", n=2_000_000, dim=128, nq=256, k=10, dist="mixture",
                 centres=1024, centre_std=2.0, seed=2, bound="hbm",
                 desc="L2 fp16, N=2M x 128 Gaussian mixture (1024 centres), Q=256, k=10 "
                      "(small batch: HBM-bound)"),
    "c5": dict(metric="inner_product", dtype="f16", n=100_000_000, dim=96, nq=100_000, k=100,
               dist="unit", seed=4, desc="IP fp16, N=100M x 96 unit-norm, Q=100k, k=100"),
    # profiling case: config 4's distribution with 500k rows (256 MB, > L2)
    "c4s": dict(kind="kmeans", metric="l2", dtype="f32", n=500_000, dim=128, clusters=4096,
                iters=10, dist="mixture", centres=4096, centre_std=3.0, seed=3,
                desc="k-means fp32, N=500k x 128 Gaussian mixture (4096 centres), C=4096, "
                     "10 iterations"),
    # IVF-Flat (ovvsIvfFlatSearch), the next caller of the k-means path: one step = one search
    # of all queries over a built index
    "ivf": dict(kind="ivf", metric="l2", dtype="f32", n=1_000_000, dim=128, nq=10_000, k=10,
                nlist=1024, nprobe=32, dist="mixture", centres=1024, centre_std=2.0, seed=5,
                desc="IVF-Flat L2 fp32, N=1M x 128 Gaussian mixture (1024 centres, var 4), "
                     "nlist=1024, nprobe=32, Q=10k, k=10"),
    # the dense primitives (ovvsPairwiseDistance / ovvsGemm, host buffers in and out): one step =
    # one call over a [nx x dim] x [ny x dim] problem whose output block fits one launch
    "pw": dict(kind="prim", op="pairwise", metric="l2", nx=4096, ny=65536, dim=128,
               dist="mixture", centres=1024, centre_std=2.0, seed=6,
               desc="ovvsPairwiseDistance L2 fp32, 4096 x 65536 pairs, D=128"),
    "gemm": dict(kind="prim", op="gemm", nx=4096, ny=65536, dim=128, dist="mixture",
                 centres=1024, centre_std=2.0, seed=7,
                 desc="ovvsGemm fp32, C[4096 x 65536] = A[4096 x 128] B[65536 x 128]^T"),
    # k-means (ovvsKMeansFit): one step = one full fit of `iters` Lloyd iterations
    "c4": dict(kind="kmeans", metric="l2", dtype="f32", n=5_000_000, dim=128, clusters=4096,
               iters=10, dist="mixture", centres=4096, centre_std=3.0, seed=3,
               desc="k-means fp32, N=5M x 128 Gaussian mixture (4096 centres, var 9), "
                    "C=4096, 10 iterations"),
}
KMEANS_METRIC = "k-means Lloyd iterations/sec @ N=5M D=128 C=4096 fp32; % of roofline"
IVF_METRIC = "IVF-Flat queries/sec @ N=1M D=128 fp32 L2 nlist=1024 nprobe=32 k=10"
METRIC_NAME = "kNN queries/sec @ N=10M D=128 fp16 k=10 at 1/2/4/8 B200; % of roofline"


def metric_name(cfg):
    """The headline metric for config 3; the same quantity named with its own shape for the other
    kNN configs (their lines are measurements of those configs, not of the headline)."""
    if cfg is CONFIGS["c3"]:
        return METRIC_NAME
    n = cfg["n"]
    ns = f"{n // 1_000_000}M" if n % 1_000_000 == 0 else f"{n // 1000}k"
    return (f"kNN queries/sec @ N={ns} D={cfg['dim']} {cfg['dtype']} {cfg['metric']} "
            f"k={cfg['k']}; % of roofline")
CHUNK = 1_000_000


# ---------------------------------------------------------------------------------------------
# data
# ---------------------------------------------------------------------------------------------
def _gen_rows(cfg, start, stop, device, torch, queries=False):
    """Rows [start, stop) of the dataset (or of the query set), as torch tensors on `device`."""
    dim = cfg["dim"]
    out = []
    base_seed = cfg["seed"] * 1000 + (500 if queries else 0)
    centres = None
    if cfg["dist"] == "mixture":
        g = torch.Generator(device=device).manual_seed(cfg["seed"] * 1000 + 999)
        centres = torch.randn(cfg["centres"], dim, generator=g, device=device) * cfg["centre_std"]
    for c in range(start // CHUNK, (stop + CHUNK - 1) // CHUNK):
        lo, hi = max(start, c * CHUNK), min(stop, (c + 1) * CHUNK)
        g = torch.Generator(device=device).manual_seed(base_seed + c)
        rows = CHUNK
        if cfg["dist"] == "uniform":
            x = torch.rand(rows, dim, generator=g, device=device)
        elif cfg["dist"] == "unit":
            x = torch.randn(rows, dim, generator=g, device=device)
            x = x / x.norm(dim=1, keepdim=True)
        else:
            lab = torch.randint(0, cfg["centres"], (rows,), generator=g, device=device)
            x = centres[lab] + torch.randn(rows, dim, generator=g, device=device)
        out.append(x[lo - c * CHUNK: hi - c * CHUNK])
    x = torch.cat(out) if len(out) > 1 else out[0]
    if cfg["dtype"] == "f16":
        x = x.half()
    return x.contiguous()


def _queries(cfg, device, torch):
    q = _gen_rows(cfg, 0, cfg["nq"], device, torch, queries=True)
    return q.float().contiguous()  # fp16-rounded values for fp16 configs, passed as fp32


# ---------------------------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------------------------
class ClockSampler:
    """SM clock and clock-event reasons sampled DURING the timed region (read-only queries).

    NVML is polled from a thread every ~2 ms, so even a timed region of a few milliseconds (a
    sharded search on 8 GPUs) gets samples; the first sample is taken before __enter__ returns.
    Without NVML it falls back to `nvidia-smi -lms 100` (and waits for its first line)."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvmlClocksEventReason*)
    REASON_BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
                   "hw_thermal_slowdown": 0x40}

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None
        self.lines = []
        self.nvml = None
        self._stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        import torch

        pynvml.nvmlInit()
        try:
            p = torch.cuda.get_device_properties(self.dev)
            bus = f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.dev)

    def _poll(self):
        nv, h = self.nvml
        try:
            mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        except Exception:
            mx = 0
        while True:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                fl = ["Active" if bits & self.REASON_BITS[n] else "Not Active"
                      for n in ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                                "sw_power_cap")]
                self.lines.append(", ".join([str(sm), str(mx), "0"] + fl))
            except Exception:
                pass
            if self._stop.wait(0.002):
                break

    def __enter__(self):
        try:
            self.nvml = self._nvml_handle()
        except Exception:
            self.nvml = None
        if self.nvml is not None:
            self.t = threading.Thread(target=self._poll, daemon=True)
            self.t.start()
            t0 = time.perf_counter()
            while not self.lines and time.perf_counter() - t0 < 2.0:
                time.sleep(0.001)
            return self
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.dev)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.perf_counter()
            while not self.lines and time.perf_counter() - t0 < 5.0:
                time.sleep(0.01)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.nvml is not None:
            self._stop.set()
            self.t.join(timeout=5)
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = max(mx, float(parts[1]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[3:7]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def _search_launches(k_eff, n_local, world):
    """This library's kernels per brute-force search: query prep, the fused kernel and the merge +
    re-rank; for k beyond the register lists (k + margin > 32) query prep, the bound pre-pass
    (more than 4,096 rows), its k-th bound, the append pass and the select + re-rank; plus the
    cross-shard merge on more than one GPU (the NCCL all-gathers are library code)."""
    need = k_eff + max(2, (k_eff + 7) // 8)
    per = 3 if need <= 32 else (5 if n_local > 4096 else 3)
    return per + (1 if world > 1 else 0)


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return p, "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, \
            "fallback"


def _traffic_from_profiles(config_name):
    """DRAM bytes per fused-kernel launch from the committed ncu summary, scaled to the config."""
    path = os.path.join(ROOT, "profiles", "knn_fused_traffic.txt")
    try:
        for line in open(path):
            if line.startswith(f"{config_name} "):
                return float(line.split()[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------------------------
# the reference CPU path (oracle/_ref/libovvs_ref.so, the reference built from its sources)
# ---------------------------------------------------------------------------------------------
def _order_key(v):
    """uint32 image of float32 scores in the reference's top-k order (cpu_prims.cpp:24-32):
    numbers ascending, -0 equal to +0, NaN after every number."""
    v = np.asarray(v, np.float32)
    u = v.view(np.uint32).copy()
    u[v == 0] = 0
    key = np.where(u & 0x80000000, ~u, u | 0x80000000).astype(np.uint32)
    key[np.isnan(v)] = 0xFFFFFFFF
    return key


def _merge_shard_topk(parts, k_eff, inner_product):
    """Merges per-shard top-k lists [(nb [nq, ks] global ids, ds [nq, ks])] into the top k_eff of
    their union, ordered like the reference's cpu_topk: score (for inner product the score is the
    negated distance it reports), then lower global id. Exact: every score depends only on its
    (query, row) pair and the order is strict."""
    nb = np.concatenate([p[0] for p in parts], axis=1)
    ds = np.concatenate([p[1] for p in parts], axis=1)
    score = -ds if inner_product else ds
    key = _order_key(score)
    out_nb = np.empty((nb.shape[0], k_eff), np.int64)
    out_ds = np.empty((nb.shape[0], k_eff), np.float32)
    for q in range(nb.shape[0]):
        o = np.lexsort((nb[q], key[q]))[:k_eff]
        out_nb[q] = nb[q, o]
        out_ds[q] = ds[q, o]
    return out_nb, out_ds


def _parity(nb, ds, nb_ref, ds_ref, rtol):
    """Parity of this library's results with the reference's on the same queries: ids equal, and
    where they differ the two distances at that rank within `rtol` (a near-tie at the cut-off);
    distances bit-identical where ids agree."""
    nb, ds = np.asarray(nb), np.asarray(ds, np.float32)
    same = nb == nb_ref
    both_nan = np.isnan(ds) & np.isnan(ds_ref)
    bits = (ds.view(np.uint32) == ds_ref.view(np.uint32)) | both_nan
    with np.errstate(invalid="ignore", divide="ignore"):
        rel = np.abs(ds.astype(np.float64) - ds_ref) / np.maximum(np.abs(ds_ref.astype(np.float64)),
                                                                   1e-30)
    rel[both_nan | (ds == ds_ref)] = 0.0
    ties = ~same & (rel <= rtol)
    out = {"queries": int(nb.shape[0]), "positions": int(nb.size),
           "id_mismatch": int((~same).sum()), "id_mismatch_beyond_tie": int((~same & ~ties).sum()),
           "distance_bits_differ_where_ids_agree": int((same & ~bits).sum()),
           "max_rel_err": float(rel.max()) if rel.size else 0.0, "rtol": rtol}
    out["ok"] = out["id_mismatch_beyond_tie"] == 0 and out["distance_bits_differ_where_ids_agree"] == 0
    return out


def _reference_sample(cfg, data_host, q_host, threads, n_queries):
    """Times the reference's FORCE_CPU ovvsBruteForceSearch on `n_queries` queries against all
    rows: row shards of 1M, `threads` host threads per shard (one Resources each, sharing the
    shard's immutable index as the reference allows). Returns (seconds, neighbours, distances):
    the shards' top-k lists merged into the reference's answer over all rows (the merge is not
    timed)."""
    import ctypes

    from oracle.cpu import DTYPES, METRICS, Reference

    ref = Reference()
    L = ref.lib
    qs = np.ascontiguousarray(q_host[:n_queries], np.float32)
    k = cfg["k"]
    per = [np.array_split(np.arange(n_queries), threads)[t] for t in range(threads)]
    res = [ref.resources() for _ in range(threads)]
    total = 0.0
    parts = []
    for s0 in range(0, cfg["n"], CHUNK):
        shard = np.ascontiguousarray(data_host[s0: s0 + CHUNK])
        ks = min(k, shard.shape[0])
        part_nb = np.empty((n_queries, ks), np.int64)
        part_ds = np.empty((n_queries, ks), np.float32)
        ix = ctypes.c_void_p()
        assert L.ovvsBruteForceBuildTyped(res[0], shard.ctypes.data_as(ctypes.c_void_p),
                                          shard.shape[0], shard.shape[1], METRICS[cfg["metric"]],
                                          DTYPES[cfg["dtype"]], ctypes.byref(ix)) == 0

        def work(t):
            idx = per[t]
            if idx.size == 0:
                return
            qq = np.ascontiguousarray(qs[idx])
            nb = np.empty(idx.size * k, np.int64)
            ds = np.empty(idx.size * k, np.float32)
            st = L.ovvsBruteForceSearch(res[t], ix, qq.ctypes.data_as(ctypes.POINTER(ctypes.c_float)),
                                        idx.size, k, None,
                                        nb.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)),
                                        ds.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
            assert st == 0
            part_nb[idx] = nb[: idx.size * ks].reshape(idx.size, ks) + s0
            part_ds[idx] = ds[: idx.size * ks].reshape(idx.size, ks)

        th = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
        t0 = time.perf_counter()
        for x in th:
            x.start()
        for x in th:
            x.join()
        total += time.perf_counter() - t0
        L.ovvsBruteForceDestroy(ix)
        parts.append((part_nb, part_ds))
    for r in res:
        L.ovvsResourcesDestroy(r)
    nb, ds = _merge_shard_topk(parts, min(k, cfg["n"]), cfg["metric"] == "inner_product")
    return total, nb, ds


def _reference_sizes(cfg, seconds):
    threads = max(1, min(os.cpu_count() or 1, 64))
    rate = 1.0e9  # reference naive fp32 GEMM, MAC/s per thread (measured ~1.06e9 on C1)
    nq = int(seconds * rate * threads / (cfg["n"] * cfg["dim"]))
    nq = max(threads, min(cfg["nq"], nq // threads * threads))
    return threads, nq


def _reference_kmeans_sample(cfg, data_host, rows, out=None):
    """Times the reference's FORCE_CPU ovvsKMeansFit (its minimum of 4 iterations) on the first
    `rows` rows with the config's cluster count. Returns (seconds, iterations); the fitted
    centroids go to out["centroids"] when `out` is given (the fit is timed, the copy is not)."""
    from oracle.cpu import Reference

    ref = Reference()
    x = np.ascontiguousarray(data_host[:rows], np.float32)
    t0 = time.perf_counter()
    cents = ref.kmeans(x, cfg["clusters"], 4, predict=False)[0]
    secs = time.perf_counter() - t0
    if out is not None:
        out["centroids"] = cents
    return secs, 4


def _reference_kmeans_rows(cfg, seconds):
    rate = 2.1e9  # reference naive fp32 GEMM, FLOP/s on one thread (measured on C1)
    rows = int(seconds * rate / (4 * 2.0 * cfg["clusters"] * cfg["dim"]))
    return max(cfg["clusters"], min(cfg["n"], rows))


def _reference_kmeans_line(args, cfg, secs, rows, iters):
    # iterations/s of the full config, extrapolated linearly by rows (cost ~ N * C * D)
    value = iters * len(secs) / sum(secs) * rows / cfg["n"]
    sample = (f"{iters}-iteration fits of {rows} of {cfg['n']} rows x C={cfg['clusters']}, "
              "FORCE_CPU (the reference fit is single-threaded), iterations/s scaled by "
              f"{rows}/{cfg['n']} rows")
    return value, sample


def run_reference_arm(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if cfg.get("kind") == "kmeans":
        import torch

        dev = "cuda" if torch.cuda.is_available() else "cpu"
        rows = _reference_kmeans_rows(cfg, args.ref_seconds)
        data_host = _gen_rows(cfg, 0, rows, dev, torch).cpu().numpy()
        for _ in range(max(1, args.warmup // 3)):
            _reference_kmeans_sample(cfg, data_host, min(rows, 2 * cfg["clusters"]))
        runs = [_reference_kmeans_sample(cfg, data_host, rows) for _ in range(args.steps)]
        secs = [r[0] for r in runs]
        value, sample = _reference_kmeans_line(args, cfg, secs, rows, runs[0][1])
        line = {
            "metric": KMEANS_METRIC, "value": value, "unit": "iterations/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * sum(secs) / len(secs), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": {"workload": f"{args.config}: {cfg['desc']}",
                                            "sample": sample},
            "cpu_baseline": {"value": value, "unit": "iterations/s", "cores": 1,
                             "kind": "reference", "sample": sample},
            "e2e": {"value": value, "unit": "iterations/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0
    import torch

    dev = "cuda" if torch.cuda.is_available() else "cpu"
    data = _gen_rows(cfg, 0, cfg["n"], dev, torch)
    data_host = data.cpu().numpy()
    if cfg["dtype"] == "f16":
        data_host = data_host.view(np.float16)
    q_host = _queries(cfg, dev, torch).cpu().numpy()
    del data
    threads, nq = _reference_sizes(cfg, args.ref_seconds)
    for _ in range(args.warmup):
        _reference_sample(cfg, data_host, q_host, threads, threads)
    secs = [_reference_sample(cfg, data_host, q_host, threads, nq)[0] for _ in range(args.steps)]
    t = sum(secs)
    value = nq * args.steps / t
    line = {
        "metric": metric_name(cfg), "value": value, "unit": "queries/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * t / args.steps,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": f"{args.config}: {cfg['desc']}",
                   "sample": f"{nq} of {cfg['nq']} queries x all {cfg['n']} rows per step"},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": threads,
                         "kind": "reference",
                         "sample": f"{nq} queries x {cfg['n']} rows (1M-row shards, {threads} "
                                   "threads with one Resources each, FORCE_CPU)"},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------
def run_ours(args, cfg):
    import torch
    import torch.distributed as dist

    import ovvs_b200 as ov
    from ovvs_b200.shard import row_range

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        uid = [ov.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        res = ov.Resources.sharded(local, rank, world, uid[0])
    else:
        res = ov.Resources.sharded(local, 0, 1, None)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    n, dim, nq, k = cfg["n"], cfg["dim"], cfg["nq"], cfg["k"]
    lo, hi = row_range(rank, world, n)
    shard = _gen_rows(cfg, lo, hi, dev, torch)
    shard_host = shard.cpu().numpy()
    if cfg["dtype"] == "f16":
        shard_host = shard_host.view(np.float16)
    del shard
    t0 = time.perf_counter()
    ix = ov.BruteIndex.build(shard_host, metric=cfg["metric"], dtype=cfg["dtype"], resources=res,
                             row_offset=lo if world > 1 else None)
    build_s = time.perf_counter() - t0
    dq = _queries(cfg, dev, torch)
    q_host = dq.cpu().numpy()
    k_eff = min(k, n)
    dn = torch.empty((nq, k_eff), dtype=torch.int64, device=dev)
    dd = torch.empty((nq, k_eff), dtype=torch.float32, device=dev)
    stream = torch.cuda.ExternalStream(res.stream(), device=dev)
    torch.cuda.synchronize()

    # warm-up (also grows the workspaces)
    for _ in range(args.warmup):
        ix.search_device(dq, k, dn, dd)
    res.synchronize()

    # ---- device-resident timing, phase events per launch --------------------------------
    # The K searches are enqueued back to back (no host synchronisation between them, so a rank
    # whose host is late does not hold up the others' all-gather); each search's phase events are
    # kept by the library and read after the timed region.
    res.set_profiling(True)
    barrier()
    with ClockSampler(local) as clocks:
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            ix.search_device(dq, k, dn, dd)
        ev1.record(stream)
        ev1.synchronize()
        res.synchronize()
        barrier()
    phases = res.phase_history(min(args.steps, 64))
    res.set_profiling(False)
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    ms_step = ms / args.steps
    value = nq / (ms_step / 1e3)
    # every rank's mean phases (prep, fused kernel, merge, cross-shard exchange): the exchange phase
    # of a rank includes its wait for the slowest rank
    rank_phases = [[round(statistics.mean(p[i] for p in phases), 4) for i in range(4)]]
    if world > 1:
        rank_phases = [None] * world
        dist.all_gather_object(rank_phases, [round(statistics.mean(p[i] for p in phases), 4)
                                             for i in range(4)])

    # ---- end to end through the C ABI with host buffers --------------------------------
    nb_h = np.empty(nq * k, np.int64)
    ds_h = np.empty(nq * k, np.float32)
    for _ in range(max(1, args.warmup)):
        ix.search(q_host, k=k, out=(nb_h, ds_h))
    barrier()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        ix.search(q_host, k=k, out=(nb_h, ds_h))
    e1.record(stream)
    e1.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    # results must agree between the two paths
    assert np.array_equal(nb_h[: nq * k_eff].reshape(nq, k_eff), dn.cpu().numpy())

    fused_ms = statistics.mean(p[1] for p in phases)
    peaks, peak_kind = _peaks()
    flops = 2.0 * nq * (hi - lo) * dim
    traffic = _traffic_from_profiles(args.config)
    if traffic is not None:  # the profiled figure is for the whole config; a rank streams its shard
        traffic *= (hi - lo) / n
    if cfg.get("bound") == "hbm":
        # small batch: the database stream bounds the kernel. Algorithmic bytes per launch: the
        # rows (fp16 operand: 2 bytes per element, 4 for fp32 data split hi + lo), one 4-byte aux
        # per row, the queries and the k results.
        row_bytes = dim * (2 if cfg["dtype"] == "f16" else 4) + 4
        hbm_bytes = (hi - lo) * row_bytes + 4.0 * nq * dim + 12.0 * nq * k
        roof = {"bound": "hbm", "achieved": hbm_bytes / (fused_ms / 1e3) / 1e9,
                "peak": float(peaks["hbm_gbs"]), "unit": "GB/s", "traffic": traffic,
                "kernel": "knn_fused_kernel", "bytes_per_launch": hbm_bytes,
                "peak_source": f"{peak_kind} HBM copy bandwidth"}
    else:
        # One fused launch per search (~25 ms on config 3), timed in a region well under a second:
        # the burst figure is the kernel's ceiling (the sustained one is for seconds-long steps).
        roof = {"bound": "tensor", "achieved": flops / (fused_ms / 1e3) / 1e12,
                "peak": float(peaks.get("bf16_tflops", peaks.get("bf16_tflops_sustained"))),
                "unit": "TFLOP/s", "traffic": traffic, "kernel": "knn_fused_kernel",
                "flops_per_launch": flops,
                "peak_source": f"{peak_kind} bf16 dense burst (fp16 MMA rate)"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    clk = clocks.summary()

    line = None
    if rank == 0:
        line = {
            "metric": metric_name(cfg), "value": value, "unit": "queries/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16" if cfg["dtype"] == "f16" else "f32", "data": "synthetic",
            "config": {
                "workload": f"{args.config}: {cfg['desc']}", "n": n, "dim": dim, "nq": nq, "k": k,
                "metric": cfg["metric"], "rows_per_gpu": hi - lo,
                "parallelism": f"rows sharded over {world} GPU(s), NCCL all-gather merge"
                if world > 1 else "1 GPU",
                **({"peer_bounds": res.peer_bounds()} if world > 1 else {}),
                "l2": "inputs larger than L2 (database >> 126 MB), no flush needed",
                "build_s": round(build_s, 3),
                "phase_ms_mean": [round(statistics.mean(p[i] for p in phases), 4)
                                  for i in range(4)],
                **({"phase_ms_ranks": rank_phases} if world > 1 else {}),
            },
            "e2e": {"value": nq / (e2e_ms / 1e3), "unit": "queries/s",
                    "h2d_bytes_per_step": nq * dim * 4, "d2h_bytes_per_step": nq * k_eff * 12},
            "gpu_launches": args.steps * _search_launches(k_eff, n // world, world),
            "roofline": roof,
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                       "reasons": clk["reasons"]},
        }
    ix.close()
    if world > 1:
        dist.barrier()
    res.close()
    if world > 1:
        dist.destroy_process_group()

    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads, nq_s = _reference_sizes(cfg, args.ref_seconds)
        data_host = shard_host
        secs, nb_ref, ds_ref = _reference_sample(cfg, data_host, q_host, threads, nq_s)
        line["cpu_baseline"] = {
            "value": nq_s / secs, "unit": "queries/s", "cores": threads, "kind": "reference",
            "sample": f"{nq_s} queries x all {n} rows: the reference library built from its "
                      f"sources (oracle/_ref), FORCE_CPU, 1M-row shards, {threads} threads"}
        # The same sampled queries' results from the timed runs above, against the reference's.
        parity = _parity(nb_h[: nq_s * k_eff].reshape(nq_s, k_eff),
                         ds_h[: nq_s * k_eff].reshape(nq_s, k_eff), nb_ref, ds_ref,
                         2e-3 if cfg["dtype"] == "f16" else 1e-4)
        parity["against"] = "the reference library (oracle/_ref), FORCE_CPU, same queries"
        line["parity"] = parity
    if rank == 0:
        print(json.dumps(line), flush=True)
        if "parity" in line and not line["parity"]["ok"]:
            print("parity FAILED against the reference", file=sys.stderr)
            return 1
    return 0


def run_kmeans(args, cfg):
    """k-means arm: each step is one ovvsKMeansFit (ovvsKMeansFitShard on N > 1 GPUs: rows
    sharded, centroids replicated, fp64 sums all-reduced per iteration). `value` = Lloyd
    iterations per second over the fit's device phase of iterations (CUDA events on the
    library's stream, max over ranks); `e2e` = the same from the fit's wall time, which includes
    the upload of the host dataset (pageable memory) and the centroid download."""
    import torch
    import torch.distributed as dist

    import ovvs_b200 as ov
    from ovvs_b200.shard import row_range

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
        uid = [ov.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        res = ov.Resources.sharded(local, rank, world, uid[0])
    else:
        res = ov.Resources.sharded(local, 0, 1, None)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    n, dim, C, iters = cfg["n"], cfg["dim"], cfg["clusters"], cfg["iters"]
    lo, hi = row_range(rank, world, n)
    shard = _gen_rows(cfg, lo, hi, dev, torch)
    shard_host = np.ascontiguousarray(shard.cpu().numpy(), np.float32)
    del shard
    torch.cuda.synchronize()

    def fit():
        if world > 1:
            return ov.KMeans(shard_host, nclusters=C, iters=iters, resources=res, row_offset=lo,
                             n_total=n)
        return ov.KMeans(shard_host, nclusters=C, iters=iters, resources=res)

    res.set_profiling(True)
    for _ in range(args.warmup):
        fit().close()
    barrier()
    walls, iter_ms, up_ms = [], [], []
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            m = fit()
            walls.append(time.perf_counter() - t0)
            ph = res.last_phase_ms()
            iter_ms.append(ph[1])
            up_ms.append(ph[0])
            m.close()
        barrier()
    res.set_profiling(False)
    dev_s = max_over_ranks(sum(iter_ms) / 1e3)
    wall_s = max_over_ranks(sum(walls))
    total_iters = iters * args.steps
    peaks, peak_kind = _peaks()
    peak = float(peaks.get("bf16_tflops_sustained", peaks.get("bf16_tflops")))
    flops_local = 2.0 * (hi - lo) * C * dim * total_iters
    achieved = flops_local / max_over_ranks(sum(iter_ms) / 1e3) / 1e12
    clk = clocks.summary()
    line = None
    if rank == 0:
        line = {
            "metric": KMEANS_METRIC, "value": total_iters / dev_s, "unit": "iterations/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * dev_s / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.config}: {cfg['desc']}", "n": n, "dim": dim,
                       "clusters": C, "iters": iters, "rows_per_gpu": hi - lo,
                       "parallelism": ("1 GPU" if world == 1 else
                                       f"rows sharded over {world} GPU(s), fp64 sums "
                                       "all-reduced per iteration (NCCL)"),
                       "l2": "inputs larger than L2 (dataset >> 126 MB), no flush needed",
                       "upload_ms_mean": sum(up_ms) / len(up_ms),
                       "fit_wall_s_mean": wall_s / args.steps},
            "e2e": {"value": total_iters / wall_s, "unit": "iterations/s",
                    "h2d_bytes_per_step": int(shard_host.nbytes),
                    "d2h_bytes_per_step": int(C * dim * 4)},
            # per iteration, ours: centroid index build (row stats, scatter, tile and group
            # bounds), query prep, fused kernel, merge + re-rank, label keys, centroid update
            # per Lloyd iteration: the centroid index rebuild (row stats, scatter, tile bounds),
            # the bound, query multipliers, fused kernel, merge, label keys, centroid update; per
            # fit the final index rebuild (CUB sorts and scans are library code)
            "gpu_launches": 9 * total_iters + 3 * args.steps,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak,
                         "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                         "kernel": "knn_fused_kernel (assignment) + update",
                         "flops_per_launch": 2.0 * (hi - lo) * C * dim,
                         "note": "algorithmic 2*N*C*D per iteration; fp32 rows and points run "
                                 "as three fp16 MMA passes (hi*hi + lo*hi + hi*lo)",
                         "peak_source": f"{peak_kind} bf16 dense sustained (fp16 MMA rate)"},
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                       "reasons": clk["reasons"]},
        }
    if world > 1:
        dist.barrier()
    res.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows = _reference_kmeans_rows(cfg, args.ref_seconds)
        ref_out = {}
        secs, it = _reference_kmeans_sample(cfg, shard_host, rows, ref_out)
        value, sample = _reference_kmeans_line(args, cfg, [secs], rows, it)
        line["cpu_baseline"] = {"value": value, "unit": "iterations/s", "cores": 1,
                                "kind": "reference", "sample": sample}
        # The same fit on this library (same rows, clusters and iterations; both seed with the
        # reference's mt19937(42) row sample): centroids must be bit-identical.
        res = ov.Resources.sharded(local, 0, 1, None)
        m = ov.KMeans(np.ascontiguousarray(shard_host[:rows]), nclusters=C, iters=it,
                      resources=res)
        ours = m.centroids()
        m.close()
        res.close()
        ref_c = ref_out["centroids"]
        same = (ours.shape == ref_c.shape and
                np.array_equal(ours.view(np.uint32), ref_c.view(np.uint32)))
        rel = float(np.max(np.abs(ours.astype(np.float64) - ref_c) /
                           np.maximum(np.abs(ref_c.astype(np.float64)), 1e-30))) \
            if ours.shape == ref_c.shape else float("inf")
        line["parity"] = {"rows": rows, "clusters": C, "iters": it,
                          "centroids_bit_identical": bool(same), "max_rel_err": rel,
                          "ok": bool(same),
                          "against": "the reference library (oracle/_ref), FORCE_CPU, same rows"}
    if rank == 0:
        print(json.dumps(line), flush=True)
        if "parity" in line and not line["parity"]["ok"]:
            print("parity FAILED against the reference", file=sys.stderr)
            return 1
    return 0


def _ivf_reference_search(path, q_host, cfg, threads, nq_s):
    """Times the reference's FORCE_CPU ovvsIvfFlatSearch over the index file `path` (the
    reference's own format, read by its own ovvsIvfFlatDeserialize) on the first nq_s queries,
    split over `threads` host threads, one Resources each (concurrent searches of one index are
    allowed). Returns seconds."""
    import ctypes

    from oracle.cpu import Reference

    ref = Reference()
    L = ref.lib
    L.ovvsIvfFlatDeserialize.argtypes = [ctypes.c_void_p, ctypes.c_char_p,
                                         ctypes.POINTER(ctypes.c_void_p)]
    L.ovvsIvfFlatSearch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                    ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    L.ovvsIvfFlatDestroy.argtypes = [ctypes.c_void_p]
    res = [ref.resources() for _ in range(threads)]
    ix = ctypes.c_void_p()
    assert L.ovvsIvfFlatDeserialize(res[0], path.encode(), ctypes.byref(ix)) == 0
    k = cfg["k"]
    parts = np.array_split(np.arange(nq_s), threads)

    def work(t):
        idx = parts[t]
        if idx.size == 0:
            return
        qq = np.ascontiguousarray(q_host[idx], np.float32)
        nb = np.empty(idx.size * k, np.int64)
        ds = np.empty(idx.size * k, np.float32)
        assert L.ovvsIvfFlatSearch(res[t], ix, qq.ctypes.data, idx.size, k, cfg["nprobe"], None,
                                   nb.ctypes.data, ds.ctypes.data) == 0

    th = [threading.Thread(target=work, args=(t,)) for t in range(threads)]
    t0 = time.perf_counter()
    for x in th:
        x.start()
    for x in th:
        x.join()
    secs = time.perf_counter() - t0
    L.ovvsIvfFlatDestroy(ix)
    for r in res:
        L.ovvsResourcesDestroy(r)
    return secs


def _ivf_file_lists(path):
    """Centroids and list sizes from an IVF1 file (header: magic, version, n, dim, nlist,
    metric; centroids; rows; per list an int32 size and its int64 ids)."""
    with open(path, "rb") as f:
        head = f.read(32)
        n, dim = (int(v) for v in np.frombuffer(head[8:24], np.int64))
        nlist = int(np.frombuffer(head[24:28], np.int32)[0])
        cents = np.frombuffer(f.read(4 * nlist * dim), np.float32).reshape(nlist, dim)
        f.seek(4 * n * dim, os.SEEK_CUR)
        sizes = np.empty(nlist, np.int64)
        for c in range(nlist):
            sizes[c] = max(0, int(np.frombuffer(f.read(4), np.int32)[0]))
            f.seek(8 * int(sizes[c]), os.SEEK_CUR)
    return cents, sizes


def _ivf_reference_sizes(cfg, seconds):
    threads = max(1, min(os.cpu_count() or 1, 64))
    per_query = cfg["dim"] * (cfg["nlist"] + cfg["n"] * cfg["nprobe"] / cfg["nlist"])
    nq = int(seconds * 1.0e9 * threads / per_query)
    return threads, max(threads, min(cfg["nq"], nq // threads * threads))


def _ivf_setup(cfg, dev, torch, ov, res):
    """Data, queries and the built index (timed) for the IVF config."""
    data = _gen_rows(cfg, 0, cfg["n"], dev, torch)
    data_host = data.cpu().numpy()
    del data
    t0 = time.perf_counter()
    ix = ov.IvfFlatIndex.build(data_host, cfg["nlist"], cfg["metric"], resources=res)
    build_s = time.perf_counter() - t0
    dq = _queries(cfg, dev, torch)
    return ix, build_s, dq, dq.cpu().numpy()


def run_ivf(args, cfg):
    """IVF-Flat arm (one GPU; with --gpus N each rank is an independent replica searching the
    same queries, no collective). `value` = device-resident searches (ovvsIvfFlatSearchDevice),
    `e2e` = host-buffer searches through ovvsIvfFlatSearch. Roofline: the list scan kernel, whose
    exact sequential fp32 sums run on the CUDA cores (two dependent instructions per MAC), against
    the FP32 issue rate of the SMs at the sampled clock."""
    import tempfile

    import torch
    import torch.distributed as dist

    import ovvs_b200 as ov

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    res = ov.Resources.sharded(local, 0, 1, None)
    nq, k, dim = cfg["nq"], cfg["k"], cfg["dim"]
    ix, build_s, dq, q_host = _ivf_setup(cfg, dev, torch, ov, res)
    dn = torch.empty((nq, k), dtype=torch.int64, device=dev)
    dd = torch.empty((nq, k), dtype=torch.float32, device=dev)
    stream = torch.cuda.ExternalStream(res.stream(), device=dev)
    for _ in range(args.warmup):
        ix.search_device(dq, k, cfg["nprobe"], dn, dd)
    res.synchronize()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    res.set_profiling(True)
    phases = []
    barrier()
    with ClockSampler(local) as clocks:
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for _ in range(args.steps):
            ix.search_device(dq, k, cfg["nprobe"], dn, dd)
            phases.append(res.last_phase_ms())
        ev1.record(stream)
        ev1.synchronize()
        barrier()
    res.set_profiling(False)
    ms_step = max_over_ranks(ev0.elapsed_time(ev1)) / args.steps
    nb_h, ds_h = ix.search(q_host, k, cfg["nprobe"])
    barrier()
    e0 = time.perf_counter()
    for _ in range(args.steps):
        nb_h, ds_h = ix.search(q_host, k, cfg["nprobe"])
    e2e_ms = max_over_ranks((time.perf_counter() - e0) * 1e3 / args.steps)
    assert np.array_equal(nb_h, dn.cpu().numpy())
    scan_ms = statistics.mean(p[1] for p in phases)
    clk = clocks.summary()
    # candidates actually scored: the probed lists' sizes per query
    path = os.path.join(tempfile.mkdtemp(), "ivf.bin")
    ix.save(path)
    cents, sizes = _ivf_file_lists(path)
    cn = (cents ** 2).sum(1)
    qs = q_host[:2000]
    d = (qs ** 2).sum(1)[:, None] + cn[None, :] - 2 * qs @ cents.T
    probes = np.argsort(d, axis=1, kind="stable")[:, :cfg["nprobe"]]
    cand_mean = float(sizes[probes].sum(1).mean())
    macs = nq * cand_mean * dim
    sm_mhz = clk["sm_mhz"] or 1965.0
    # L2 without a bitset and k <= 10 scans on the tensor cores (the fused kernel over (list,
    # 256 probing pairs) items); the other cases on the CUDA cores, whose peak is the FP32 lanes
    # per SM x SMs x clock (one separately rounded multiply and one add per MAC)
    tensor = cfg["metric"] in ("l2", "l2_sqrt") and k <= 10
    fp32_gops = 128 * torch.cuda.get_device_properties(dev).multi_processor_count * sm_mhz / 1e3
    achieved = 2 * macs / (scan_ms / 1e3) / 1e12
    peaks, _ = _peaks()
    peak = float(peaks.get("bf16_tflops", 1590.0)) if tensor else fp32_gops / 1e3
    ix.close()
    res.close()
    line = None
    if rank == 0:
        line = {
            "metric": IVF_METRIC, "value": world * nq / (ms_step / 1e3), "unit": "queries/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": f"{args.config}: {cfg['desc']}", "n": cfg["n"], "dim": dim,
                       "nq": nq, "k": k, "nlist": cfg["nlist"], "nprobe": cfg["nprobe"],
                       "parallelism": "1 GPU" if world == 1 else
                       f"{world} independent replicas (the IVF path is not sharded)",
                       "l2": "inputs larger than L2 (rows 512 MB >> 126 MB), no flush needed",
                       "build_s": round(build_s, 3), "candidates_per_query": round(cand_mean, 1),
                       "phase_ms_mean": [round(statistics.mean(p[i] for p in phases), 4)
                                         for i in range(4)]},
            "e2e": {"value": world * nq / (e2e_ms / 1e3), "unit": "queries/s",
                    "h2d_bytes_per_step": nq * dim * 4, "d2h_bytes_per_step": nq * k * 12},
            # row norms, coarse GEMM + L2 epilogue + probe selection, probe offsets, pair
            # grouping, item counts, list scan, merge/emit; the tensor-core scan adds slot counts,
            # slot fill, query prep, slot gather and the re-score and replaces the scan by the
            # fused kernel (the CUB scans are library code)
            "gpu_launches": (14 if tensor else 9) * args.steps,
            "roofline": ({"bound": "tensor", "achieved": achieved, "peak": peak,
                          "unit": "TFLOP/s", "frac": achieved / peak, "traffic": None,
                          "kernel": "knn_fused_kernel (list items) + exact re-score",
                          "flops_per_launch": 2 * macs,
                          "note": "algorithmic 2*D*(rows of the probed lists) per query; fp32 "
                                  "rows and queries run as three fp16 MMA passes; phase [1] = "
                                  "slot layout, fused kernel and re-score; peak = measured "
                                  "bf16 dense burst"}
                         if tensor else
                         {"bound": "fp32", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                          "frac": achieved / peak, "traffic": None, "kernel": "list_scan_kernel",
                          "flops_per_launch": 2 * macs,
                          "note": "exact sequential fp32 scores (separate multiply and add) on "
                                  "the CUDA cores; peak = 128 FP32 lanes x SMs x median SM clock, "
                                  "one instruction per flop"}),
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                       "reasons": clk["reasons"]},
        }
        if world == 1 and not args.no_cpu_baseline:
            threads, nq_s = _ivf_reference_sizes(cfg, args.ref_seconds)
            secs = _ivf_reference_search(path, q_host, cfg, threads, nq_s)
            line["cpu_baseline"] = {
                "value": nq_s / secs, "unit": "queries/s", "cores": threads, "kind": "reference",
                "sample": f"{nq_s} of {nq} queries through the reference library built from its "
                          f"sources (oracle/_ref), FORCE_CPU, {threads} threads, over this "
                          "index written in the reference's IVF1 file format"}
    os.remove(path)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_ivf_reference(args, cfg):
    """--impl reference for the IVF config: the reference's own ovvsIvfFlatDeserialize +
    ovvsIvfFlatSearch (FORCE_CPU, all host threads) over an index file in its format. Building
    the reference's index on the host (12 Lloyd iterations over 1M x 1024 x 128) would take
    about half an hour, so the index is built on the GPU by this library and written in the
    reference's file format; only the reference's search is timed."""
    import tempfile

    import torch

    import ovvs_b200 as ov

    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    res = ov.Resources.sharded(dev.index, 0, 1, None)
    ix, _, _, q_host = _ivf_setup(cfg, dev, torch, ov, res)
    path = os.path.join(tempfile.mkdtemp(), "ivf.bin")
    ix.save(path)
    ix.close()
    res.close()
    threads, nq_s = _ivf_reference_sizes(cfg, args.ref_seconds)
    for _ in range(args.warmup):
        _ivf_reference_search(path, q_host, cfg, threads, threads)
    secs = [_ivf_reference_search(path, q_host, cfg, threads, nq_s) for _ in range(args.steps)]
    os.remove(path)
    value = nq_s * args.steps / sum(secs)
    sample = (f"{nq_s} of {cfg['nq']} queries per step, FORCE_CPU, {threads} threads with one "
              "Resources each, over an index in the reference's IVF1 file format")
    print(json.dumps({
        "metric": IVF_METRIC, "value": value, "unit": "queries/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(secs) / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": f"{args.config}: {cfg['desc']}", "sample": sample},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": threads,
                         "kind": "reference", "sample": sample},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)
    return 0


def _prim_data(cfg):
    """Host operands of a primitive config (seeded mixture rows, fp32)."""
    rng = np.random.default_rng(cfg["seed"])
    centres = rng.normal(0, cfg["centre_std"], (cfg["centres"], cfg["dim"])).astype(np.float32)

    def rows(n):
        return (centres[rng.integers(0, cfg["centres"], n)]
                + rng.standard_normal((n, cfg["dim"]), dtype=np.float32)).astype(np.float32)

    return rows(cfg["nx"]), rows(cfg["ny"])


def _prim_metric(cfg):
    return (f"{cfg['op']} outputs/sec @ {cfg['nx']} x {cfg['ny']} x D={cfg['dim']} fp32"
            + (f" {cfg['metric']}" if cfg["op"] == "pairwise" else ""))


def _prim_call(obj, cfg, x, y):
    """One call of the config's primitive through the C ABI: `obj` is this library's Resources or
    the reference library's wrapper (oracle.cpu.Reference)."""
    if cfg["op"] == "gemm":
        return obj.gemm(x, y, x.shape[0], y.shape[0], x.shape[1], 1)
    if hasattr(obj, "pairwise_distance"):  # this library
        return obj.pairwise_distance(x, y, cfg["metric"])
    return obj.pairwise(cfg["metric"], x, y)  # the reference


def _prim_reference_rows(cfg, seconds):
    rate = 2.1e9  # reference naive fp32 GEMM, FLOP/s on one thread (measured on C1)
    return max(1, min(cfg["nx"], int(seconds * rate / (2.0 * cfg["ny"] * cfg["dim"]))))


def run_prim(args, cfg):
    """Dense primitive arm (one GPU; with --gpus N each rank is an independent replica). `value` =
    outputs per second of the kernels alone (phase [1] of the call, CUDA events on the library's
    stream: row norms, the sequential fp32 GEMM and the metric epilogue for the whole output,
    which fits one block); `e2e` = the same calls with the host copies (operands in, the nx x ny
    output back), CUDA events around each call. The kernels keep the reference's sequential fp32
    operation order (bit-identical results), so they run on the CUDA cores: the roofline is the
    FP32 issue rate (one instruction per flop: separately rounded multiply and add)."""
    import torch
    import torch.distributed as dist

    import ovvs_b200 as ov

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    res = ov.Resources.sharded(local, 0, 1, None)
    x, y = _prim_data(cfg)
    nx, ny, dim = cfg["nx"], cfg["ny"], cfg["dim"]
    out = None
    for _ in range(args.warmup):
        out = _prim_call(res, cfg, x, y)
    stream = torch.cuda.ExternalStream(res.stream(), device=dev)
    res.set_profiling(True)
    kern, e2e = [], []
    if world > 1:
        dist.barrier()
    with ClockSampler(local) as clocks:
        for _ in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            out = _prim_call(res, cfg, x, y)
            e1.record(stream)
            e1.synchronize()
            kern.append(res.last_phase_ms()[1])
            e2e.append(e0.elapsed_time(e1))
    res.set_profiling(False)
    clk = clocks.summary()

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    kern_ms = max_over_ranks(statistics.mean(kern))
    e2e_ms = max_over_ranks(statistics.mean(e2e))
    flops = 2.0 * nx * ny * dim
    sm_mhz = clk["sm_mhz"] or 1965.0
    peak = 128 * torch.cuda.get_device_properties(dev).multi_processor_count * sm_mhz / 1e6
    achieved = flops / (kern_ms / 1e3) / 1e12
    line = None
    if rank == 0:
        line = {
            "metric": _prim_metric(cfg), "value": world * nx * ny / (kern_ms / 1e3),
            "unit": "outputs/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": kern_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": f"{args.config}: {cfg['desc']}", "nx": nx, "ny": ny,
                       "dim": dim, "parallelism": "1 GPU" if world == 1 else
                       f"{world} independent replicas (the primitives are not sharded)",
                       "l2": "output 1 GiB >> 126 MB L2, no flush needed",
                       "e2e_ms_per_step": e2e_ms},
            "e2e": {"value": world * nx * ny / (e2e_ms / 1e3), "unit": "outputs/s",
                    "h2d_bytes_per_step": (nx + ny) * dim * 4, "d2h_bytes_per_step": nx * ny * 4},
            "gpu_launches": (4 if cfg["op"] == "pairwise" else 1) * args.steps,
            "roofline": {"bound": "fp32", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None,
                         "kernel": "gemm_seq_kernel" + (" + norms + pairwise_expand"
                                                        if cfg["op"] == "pairwise" else ""),
                         "flops_per_launch": flops,
                         "note": "sequential fp32 sums in the reference's order on the CUDA "
                                 "cores; peak = 128 FP32 lanes x SMs x median SM clock, one "
                                 "instruction per flop"},
            "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"],
                       "reasons": clk["reasons"]},
        }
        if world == 1 and not args.no_cpu_baseline:
            from oracle.cpu import Reference

            ref = Reference()
            rows = _prim_reference_rows(cfg, args.ref_seconds)
            xs = np.ascontiguousarray(x[:rows])
            t0 = time.perf_counter()
            ref_out = np.asarray(_prim_call(ref, cfg, xs, y), np.float32).reshape(rows, ny)
            secs = time.perf_counter() - t0
            line["cpu_baseline"] = {
                "value": rows * ny / secs, "unit": "outputs/s", "cores": 1, "kind": "reference",
                "sample": f"{rows} of {nx} rows x all {ny} through the reference library built "
                          "from its sources (oracle/_ref), FORCE_CPU (its naive loop is "
                          "single-threaded)"}
            got = np.asarray(out, np.float32).reshape(nx, ny)[:rows]
            same = got.view(np.uint32) == ref_out.view(np.uint32)
            line["parity"] = {"rows": rows, "outputs": int(same.size),
                              "bit_identical": int(same.sum()), "ok": bool(same.all()),
                              "against": "the reference library (oracle/_ref), FORCE_CPU"}
    res.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)
        if "parity" in line and not line["parity"]["ok"]:
            return 1
    return 0


def run_prim_reference(args, cfg):
    """--impl reference for a primitive config: the reference's own ovvsPairwiseDistance /
    ovvsGemm (FORCE_CPU, single-threaded naive loop) on a row sample of the same operands, in
    outputs per second."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    from oracle.cpu import Reference

    ref = Reference()
    x, y = _prim_data(cfg)
    rows = _prim_reference_rows(cfg, args.ref_seconds / max(1, args.steps))
    xs = np.ascontiguousarray(x[:rows])
    _prim_call(ref, cfg, xs[:max(1, rows // 8)], y)
    secs = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        _prim_call(ref, cfg, xs, y)
        secs.append(time.perf_counter() - t0)
    value = rows * cfg["ny"] / statistics.mean(secs)
    sample = (f"{rows} of {cfg['nx']} rows x all {cfg['ny']} per step, FORCE_CPU, 1 thread "
              "(the reference's naive loop)")
    line = {"metric": _prim_metric(cfg), "value": value, "unit": "outputs/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * statistics.mean(secs), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": {"workload": f"{args.config}: {cfg['desc']}",
                                            "sample": sample},
            "cpu_baseline": {"value": value, "unit": "outputs/s", "cores": 1,
                             "kind": "reference", "sample": sample},
            "e2e": {"value": value, "unit": "outputs/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c3")
    ap.add_argument("--ref-seconds", type=float, default=12.0,
                    help="target seconds of reference CPU work per sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        print("note: warm-up raised to 3", file=sys.stderr)
        args.warmup = 3
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        if cfg.get("kind") == "ivf":
            return run_ivf_reference(args, cfg)
        if cfg.get("kind") == "prim":
            return run_prim_reference(args, cfg)
        return run_reference_arm(args, cfg)
    if cfg.get("kind") == "kmeans":
        return run_kmeans(args, cfg)
    if cfg.get("kind") == "ivf":
        return run_ivf(args, cfg)
    if cfg.get("kind") == "prim":
        return run_prim(args, cfg)
    return run_ours(args, cfg)


if __name__ == "__main__":
    sys.exit(main())
