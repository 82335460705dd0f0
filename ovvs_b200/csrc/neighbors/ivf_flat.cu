// IVF-Flat build / search / extend / (de)serialisation (see ivf_flat.hpp).
#include "ivf_flat.hpp"

#include <cub/device/device_scan.cuh>
#include <cub/device/device_segmented_sort.cuh>

#include <algorithm>
#include <cstdio>
#include <cstring>

#include "../cluster/kmeans.hpp"
#include "../prim/dense.cuh"
#include "../prim/ivf_scan.cuh"
#include "../prim/prep.cuh"

namespace ovvs {
namespace ivf {
namespace {

constexpr int kDTypeF32 = 0;
constexpr uint32_t kIvf1Magic = 0x31465649u;  // 'IVF1' (indexes.cpp:366)
constexpr int kKMeansIters = 12;              // indexes.cpp:289

size_t bytes_of(int64_t count, size_t elem) {
  return static_cast<size_t>(count > 0 ? count : 1) * elem;
}

bool tc_metric(int metric) {
  return metric == OVVS_METRIC_L2_EXPANDED || metric == OVVS_METRIC_L2_SQRT_EXPANDED;
}

// The tensor-core scan's operand: every list padded to whole 256-row tiles, in list order.
ovvsStatus assemble_tc(rt::Resources& r, IvfFlatIndex& ix) {
  ix.tc_ready = false;
  const int64_t rows = ix.list_off.back();
  if (!tc_metric(ix.metric) || rows <= 0 || ix.nlist <= 0) return OVVS_STATUS_SUCCESS;
  cudaStream_t s = r.stream;
  std::vector<int64_t> lpos(static_cast<size_t>(ix.nlist) + 1, 0);
  std::vector<int2> tiles(static_cast<size_t>(ix.nlist));
  for (int c = 0; c < ix.nlist; ++c) {
    const int64_t size = ix.list_off[c + 1] - ix.list_off[c];
    lpos[c + 1] = lpos[c] + (size + 255) / 256 * 256;
    tiles[c] = make_int2(static_cast<int>(lpos[c] / 256), static_cast<int>(lpos[c + 1] / 256));
  }
  const int64_t n_tc = lpos.back();
  std::vector<int64_t> pos_row(static_cast<size_t>(n_tc), -1);
  for (int c = 0; c < ix.nlist; ++c)
    for (int64_t i = 0; i < ix.list_off[c + 1] - ix.list_off[c]; ++i)
      pos_row[static_cast<size_t>(lpos[c] + i)] = ix.list_off[c] + i;
  OVVS_TRY_CUDA(ix.d_pos_row.reserve(bytes_of(n_tc, sizeof(int64_t))));
  OVVS_TRY_CUDA(ix.d_list_tiles.reserve(bytes_of(ix.nlist, sizeof(int2))));
  OVVS_TRY_CUDA(cudaMemcpyAsync(ix.d_pos_row.get(), pos_row.data(), n_tc * sizeof(int64_t),
                                cudaMemcpyHostToDevice, s));
  OVVS_TRY_CUDA(cudaMemcpyAsync(ix.d_list_tiles.get(), tiles.data(), ix.nlist * sizeof(int2),
                                cudaMemcpyHostToDevice, s));
  rt::DeviceBuffer padded, pnorm;
  OVVS_TRY_CUDA(padded.reserve(bytes_of(n_tc * ix.dim, sizeof(float))));
  OVVS_TRY_CUDA(pnorm.reserve(bytes_of(n_tc, sizeof(float))));
  OVVS_TRY_CUDA(prim::launch_ivf_gather_rows(ix.d_rows.as<float>(), rows, static_cast<int>(ix.dim),
                                             ix.d_pos_row.as<int64_t>(), n_tc,
                                             padded.as<float>(), pnorm.as<float>(), s));
  const ovvsStatus st = nb::build_in_order(r, ix.tc, padded.as<float>(), n_tc, ix.dim, ix.metric,
                                           ix.d_pos_row.as<int64_t>());
  if (st == OVVS_STATUS_UNSUPPORTED) return OVVS_STATUS_SUCCESS;  // the CUDA-core scan serves
  OVVS_TRY(st);
  ix.tc_ready = true;
  return r.finish();
}

// Device copies of the host list layout, the list-ordered rows gathered from d_x and the
// tensor-core scan's operand.
ovvsStatus assemble(rt::Resources& r, IvfFlatIndex& ix) {
  cudaStream_t s = r.stream;
  const int64_t rows = ix.list_off.back();
  OVVS_TRY_CUDA(ix.d_loff.reserve(bytes_of(ix.nlist + 1, sizeof(int64_t))));
  OVVS_TRY_CUDA(cudaMemcpyAsync(ix.d_loff.get(), ix.list_off.data(),
                                (ix.nlist + 1) * sizeof(int64_t), cudaMemcpyHostToDevice, s));
  OVVS_TRY_CUDA(ix.d_ids.reserve(bytes_of(rows, sizeof(int64_t))));
  OVVS_TRY_CUDA(ix.d_rows.reserve(bytes_of(rows * ix.dim, sizeof(float))));
  OVVS_TRY_CUDA(ix.d_rnorm.reserve(bytes_of(rows, sizeof(float))));
  if (rows > 0) {
    OVVS_TRY_CUDA(cudaMemcpyAsync(ix.d_ids.get(), ix.list_ids.data(), rows * sizeof(int64_t),
                                  cudaMemcpyHostToDevice, s));
    OVVS_TRY_CUDA(prim::launch_ivf_gather_rows(ix.d_x.as<float>(), ix.n, static_cast<int>(ix.dim),
                                               ix.d_ids.as<int64_t>(), rows, ix.d_rows.as<float>(),
                                               ix.d_rnorm.as<float>(), s));
  }
  OVVS_TRY(r.finish());
  // The tensor-core operand is an accelerator: without room for it the CUDA-core scan serves.
  const ovvsStatus st = assemble_tc(r, ix);
  if (st == OVVS_STATUS_OOM) {
    (void)cudaGetLastError();
    ix.tc_ready = false;
    for (rt::DeviceBuffer* b : {&ix.tc.rows16, &ix.tc.exact32, &ix.tc.aux, &ix.tc.tile_aux,
                                &ix.tc.norm_sorted, &ix.tc.row_id, &ix.tc.inv_perm})
      b->release();
    ix.d_pos_row.release();
    ix.d_list_tiles.release();
    return r.finish();
  }
  return st;
}

// Device centroids, their norms (nrm2sq, sequential) and the assignment index.
ovvsStatus set_centroids(rt::Resources& r, IvfFlatIndex& ix) {
  cudaStream_t s = r.stream;
  const int64_t cnt = static_cast<int64_t>(ix.nlist) * ix.dim;
  OVVS_TRY_CUDA(ix.d_cent.reserve(bytes_of(cnt, sizeof(float))));
  OVVS_TRY_CUDA(ix.d_cnorm.reserve(bytes_of(ix.nlist, sizeof(float))));
  if (ix.nlist <= 0) return OVVS_STATUS_SUCCESS;
  OVVS_TRY_CUDA(cudaMemcpyAsync(ix.d_cent.get(), ix.centroids.data(), cnt * sizeof(float),
                                cudaMemcpyHostToDevice, s));
  OVVS_TRY_CUDA(prim::launch_row_norms_seq(ix.d_cent.as<float>(), ix.nlist, ix.dim,
                                           ix.d_cnorm.as<float>(), s));
  OVVS_TRY(nb::build_from_device(r, ix.cindex, ix.d_cent.get(), kDTypeF32, ix.nlist, ix.dim,
                                 OVVS_METRIC_L2_EXPANDED, 0));
  return r.finish();
}

// Nearest centroid (squared L2, ties to the lower id) of `n` device rows: the reference's
// prim_pairwise(L2) + prim_topk(k = 1) (indexes.cpp:290-293, 447-451).
ovvsStatus assign(rt::Resources& r, IvfFlatIndex& ix, const float* d_rows, int64_t n,
                  std::vector<int64_t>& labels) {
  rt::DeviceBuffer lab, dist;
  OVVS_TRY_CUDA(lab.reserve(bytes_of(n, sizeof(int64_t))));
  OVVS_TRY_CUDA(dist.reserve(bytes_of(n, sizeof(float))));
  int64_t ke = 0;
  OVVS_TRY(nb::search_device(r, ix.cindex, d_rows, n, 1, nullptr, lab.as<int64_t>(),
                             dist.as<float>(), &ke));
  labels.resize(static_cast<size_t>(n));
  OVVS_TRY_CUDA(cudaMemcpyAsync(labels.data(), lab.get(), n * sizeof(int64_t),
                                cudaMemcpyDeviceToHost, r.stream));
  return r.finish();
}

// The list scan of one query block on the tensor cores (ivf_flat.hpp: L2 metrics, k <= 10): slots for the block's (query, probe) pairs grouped by list, one fused-kernel item per
// (list, 256 slots) over the list's tiles with the exact-value filter, then every pair's
// candidates re-scored exactly into p.cand (select-mode lists of k for launch_ivf_emit).
ovvsStatus scan_tc(rt::Resources& r, const IvfFlatIndex& ix, prim::IvfScanParams& p, int64_t k,
                   const int* lcnt, const int* loff, const int* pairs, void* tmp,
                   size_t tmp_bytes) {
  cudaStream_t s = r.stream;
  const int nlist = ix.nlist;
  const nb::BruteIndex& tc = ix.tc;
  const int kl = nb::list_size_for(k);
  const int2* tiles = ix.d_list_tiles.as<int2>();
  const int64_t npairs = p.nq * p.nprobe;
  // 1. slots and items per list, and their totals on the host
  int* cnt = nullptr;
  OVVS_TRY(r.scratch(rt::kWsIvfTcCounts, static_cast<size_t>(4) * (nlist + 1), &cnt));
  int* slot_cnt = cnt;
  int* item_cnt = cnt + (nlist + 1);
  int* slot_off = cnt + 2 * (nlist + 1);
  int* item_off = cnt + 3 * (nlist + 1);
  OVVS_TRY_CUDA(prim::launch_ivf_tc_counts(lcnt, tiles, nlist, slot_cnt, item_cnt, s));
  size_t tb = tmp_bytes;
  OVVS_TRY_CUDA(cub::DeviceScan::ExclusiveSum(tmp, tb, slot_cnt, slot_off, nlist + 1, s));
  tb = tmp_bytes;
  OVVS_TRY_CUDA(cub::DeviceScan::ExclusiveSum(tmp, tb, item_cnt, item_off, nlist + 1, s));
  int totals[2] = {0, 0};
  OVVS_TRY_CUDA(cudaMemcpyAsync(&totals[0], slot_off + nlist, sizeof(int), cudaMemcpyDeviceToHost, s));
  OVVS_TRY_CUDA(cudaMemcpyAsync(&totals[1], item_off + nlist, sizeof(int), cudaMemcpyDeviceToHost, s));
  OVVS_TRY_CUDA(cudaStreamSynchronize(s));
  const int64_t slots = totals[0];
  const int items = totals[1];
  // 2. slot <-> pair maps and the item table
  int *slot_pair = nullptr, *pair_slot = nullptr;
  int4* item_tab = nullptr;
  OVVS_TRY(r.scratch(rt::kWsIvfTcSlotPair, static_cast<size_t>(std::max<int64_t>(slots, 1)),
                     &slot_pair));
  OVVS_TRY(r.scratch(rt::kWsIvfTcPairSlot, static_cast<size_t>(npairs), &pair_slot));
  OVVS_TRY(r.scratch(rt::kWsIvfTcItems, static_cast<size_t>(std::max(items, 1)), &item_tab));
  OVVS_TRY_CUDA(cudaMemsetAsync(pair_slot, 0xFF, npairs * sizeof(int), s));
  OVVS_TRY_CUDA(prim::launch_ivf_tc_fill(lcnt, loff, pairs, slot_off, item_off, tiles, nlist,
                                         slot_pair, pair_slot, item_tab, s));
  uint64_t* cand = nullptr;
  OVVS_TRY(r.scratch(rt::kWsIvfTcCand,
                     static_cast<size_t>(std::max<int64_t>(slots, 1)) * 2 * kl, &cand));
  if (items > 0) {
    // 3. the fused kernel's query operand per slot
    const int64_t q_pad = prim::pad_queries(p.nq);
    const int halves = 2 * tc.dp;
    __half *qa = nullptr, *sa = nullptr;
    float *qmul = nullptr, *smul = nullptr, *qxn = nullptr;
    int* flag = nullptr;
    uint64_t* bound = nullptr;
    OVVS_TRY(r.scratch(rt::kWsIvfTcQueryA, static_cast<size_t>(q_pad) * halves, &qa));
    OVVS_TRY(r.scratch(rt::kWsIvfTcSlotA, static_cast<size_t>(slots) * halves, &sa));
    OVVS_TRY(r.scratch(rt::kWsIvfTcQueryMul, static_cast<size_t>(q_pad), &qmul));
    OVVS_TRY(r.scratch(rt::kWsIvfTcSlotMul, static_cast<size_t>(slots), &smul));
    OVVS_TRY(r.scratch(rt::kWsIvfTcQueryNorm, static_cast<size_t>(q_pad), &qxn));
    OVVS_TRY(r.scratch(rt::kWsIvfTcFlag, 4, &flag));
    OVVS_TRY(r.scratch(rt::kWsIvfTcBound, static_cast<size_t>(slots), &bound));
    OVVS_TRY_CUDA(cudaMemsetAsync(flag, 0, sizeof(int), s));
    prim::launch_query_prep(p.queries, p.nq, q_pad, p.dim, tc.dp, tc.metric, tc.e_db, qa, qmul,
                            qxn, flag, s);
    OVVS_TRY_CUDA(cudaGetLastError());
    OVVS_TRY_CUDA(prim::launch_ivf_tc_gather(qa, qmul, slot_pair, p.nprobe, slots, halves, sa,
                                             smul, s));
    // 4. one item per (list, 256 slots) over the list's tiles
    nb::SearchCtx c;
    c.q_pad = slots;
    c.num_qtiles = static_cast<int>(slots / prim::kTileQ);
    c.a16 = sa;
    c.q_mul = smul;
    c.xn = qxn;
    c.flag = flag;
    OVVS_TRY(nb::encode_query_maps(c, tc.dp));
    c.maps.b64 = tc.b64;
    c.maps.b32 = tc.b32;
    c.maps.b16 = tc.b16;
    prim::FusedParams fp;
    OVVS_TRY(nb::base_params(r, tc, c, slots, &fp));
    fp.item_tab = item_tab;
    fp.slot_pair = slot_pair;
    fp.num_items = items;
    fp.num_sc = 1;
    fp.tiles_per_item = 1;
    fp.exact_filter = 1;
    OVVS_TRY_CUDA(cudaMemsetAsync(bound, 0xFF, static_cast<size_t>(slots) * sizeof(uint64_t), s));
    fp.q_bound = bound;
    fp.k_pub = static_cast<int>(k);
    fp.out = cand;
    if (p.bitset) {  // allow bits by padded position; the re-score also gives filtered rows +inf
      uint32_t* allow = nullptr;
      OVVS_TRY(r.scratch(rt::kWsIvfTcAllow, static_cast<size_t>(tc.n_pad / 32), &allow));
      OVVS_TRY_CUDA(prim::launch_ivf_tc_allow(p.bitset, p.bitset_bits, ix.d_pos_row.as<int64_t>(),
                                              ix.d_ids.as<int64_t>(), tc.n_pad, allow, s));
      fp.allow = allow;
    }
    OVVS_TRY_CUDA(prim::launch_knn_fused(c.maps, fp, kl,
                                         prim::fused_grid(items, nb::pair_sms(r, fp)), s));
  }
  // 5. exact re-score of every pair's candidates
  p.k_sel = static_cast<int>(k);
  OVVS_TRY_CUDA(prim::launch_ivf_tc_refine(p, cand, kl, pair_slot, ix.d_pos_row.as<int64_t>(), s));
  return OVVS_STATUS_SUCCESS;
}

}  // namespace

ovvsStatus build(rt::Resources& r, IvfFlatIndex& ix, const float* x, int64_t n, int64_t dim,
                 int metric, int32_t nlist) {
  // kmeans_fit_impl rejects n > INT32_MAX (mixer.cpp:869) and the candidate positions of a query
  // are 32-bit here.
  if (n > INT32_MAX) return OVVS_STATUS_SHAPE_MISMATCH;
  ix.device = r.device;
  ix.n = n;
  ix.dim = dim;
  ix.metric = metric;
  ix.nlist = static_cast<int32_t>(std::min<int64_t>(nlist, n));
  {
    km::KMeansModel m;
    OVVS_TRY(km::fit(r, x, n, 0, n, dim, ix.nlist, kKMeansIters, m));
    ix.centroids.assign(m.host.begin(), m.host.begin() + static_cast<size_t>(ix.nlist) * dim);
  }
  OVVS_TRY(set_centroids(r, ix));
  OVVS_TRY_CUDA(ix.d_x.reserve(bytes_of(n * dim, sizeof(float))));
  OVVS_TRY(rt::upload(r, ix.d_x.get(), x, n * dim * sizeof(float)));
  std::vector<int64_t> labels;
  OVVS_TRY(assign(r, ix, ix.d_x.as<float>(), n, labels));
  // build_ivf_lists (indexes.cpp:50-57): list c = rows labelled c, ascending.
  ix.list_off.assign(static_cast<size_t>(ix.nlist) + 1, 0);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t c = labels[static_cast<size_t>(i)];
    if (c >= 0 && c < ix.nlist) ++ix.list_off[static_cast<size_t>(c) + 1];
  }
  for (int32_t c = 0; c < ix.nlist; ++c) ix.list_off[c + 1] += ix.list_off[c];
  ix.list_ids.assign(static_cast<size_t>(ix.list_off.back()), 0);
  std::vector<int64_t> fill(ix.list_off.begin(), ix.list_off.end() - 1);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t c = labels[static_cast<size_t>(i)];
    if (c >= 0 && c < ix.nlist) ix.list_ids[static_cast<size_t>(fill[c]++)] = i;
  }
  return assemble(r, ix);
}

ovvsStatus extend(rt::Resources& r, IvfFlatIndex& ix, const float* extra, int64_t nextra) {
  if (ix.n + nextra > INT32_MAX) return OVVS_STATUS_SHAPE_MISMATCH;
  cudaStream_t s = r.stream;
  // the dataset grows by the new rows (indexes.cpp:442-443)
  rt::DeviceBuffer grown;
  OVVS_TRY_CUDA(grown.reserve(bytes_of((ix.n + nextra) * ix.dim, sizeof(float))));
  if (ix.n > 0)
    OVVS_TRY_CUDA(cudaMemcpyAsync(grown.get(), ix.d_x.get(), ix.n * ix.dim * sizeof(float),
                                  cudaMemcpyDeviceToDevice, s));
  float* dst = grown.as<float>() + ix.n * ix.dim;
  OVVS_TRY(rt::upload(r, dst, extra, nextra * ix.dim * sizeof(float)));
  std::vector<int64_t> labels(static_cast<size_t>(nextra), -1);
  if (ix.nlist > 0) OVVS_TRY(assign(r, ix, dst, nextra, labels));
  OVVS_TRY(r.finish());
  ix.d_x.swap(grown);
  // new rows are appended to their lists in row order (indexes.cpp:452-455)
  std::vector<int64_t> add(static_cast<size_t>(ix.nlist) + 1, 0);
  for (int64_t i = 0; i < nextra; ++i) {
    const int64_t c = labels[static_cast<size_t>(i)];
    if (c >= 0 && c < ix.nlist) ++add[static_cast<size_t>(c)];
  }
  std::vector<int64_t> off(static_cast<size_t>(ix.nlist) + 1, 0), ids;
  for (int32_t c = 0; c < ix.nlist; ++c)
    off[c + 1] = off[c] + (ix.list_off[c + 1] - ix.list_off[c]) + add[static_cast<size_t>(c)];
  ids.assign(static_cast<size_t>(off.back()), 0);
  std::vector<int64_t> fill(off.begin(), off.end() - 1);
  for (int32_t c = 0; c < ix.nlist; ++c)
    for (int64_t g = ix.list_off[c]; g < ix.list_off[c + 1]; ++g)
      ids[static_cast<size_t>(fill[c]++)] = ix.list_ids[static_cast<size_t>(g)];
  for (int64_t i = 0; i < nextra; ++i) {
    const int64_t c = labels[static_cast<size_t>(i)];
    if (c >= 0 && c < ix.nlist) ids[static_cast<size_t>(fill[c]++)] = ix.n + i;
  }
  ix.list_off.swap(off);
  ix.list_ids.swap(ids);
  ix.n += nextra;
  return assemble(r, ix);
}

ovvsStatus search_device(rt::Resources& r, const IvfFlatIndex& ix, const float* d_queries,
                         int64_t nq, int64_t k, int32_t nprobe_in, const uint8_t* d_bitset,
                         int64_t* d_neighbors, float* d_distances) {
  cudaStream_t s = r.stream;
  if (nq <= 0 || k <= 0) return OVVS_STATUS_SUCCESS;
  const int dim = static_cast<int>(ix.dim);
  const int nlist = ix.nlist;
  const float inf = __builtin_huge_valf();
  if (nlist <= 0) {  // no centroid: every probe is skipped (indexes.cpp:317-325)
    std::vector<int64_t> nb(static_cast<size_t>(nq * k), -1);
    std::vector<float> ds(static_cast<size_t>(nq * k), inf);
    OVVS_TRY_CUDA(cudaMemcpyAsync(d_neighbors, nb.data(), nq * k * sizeof(int64_t),
                                  cudaMemcpyHostToDevice, s));
    OVVS_TRY_CUDA(cudaMemcpyAsync(d_distances, ds.data(), nq * k * sizeof(float),
                                  cudaMemcpyHostToDevice, s));
    return r.finish();
  }
  const int nprobe = std::max(1, std::min(nprobe_in, nlist));  // indexes.cpp:307
  const bool sort_mode = k > prim::kIvfMaxSelect;
  // Largest candidate count of a query: its nprobe largest lists.
  std::vector<int64_t> sizes(static_cast<size_t>(nlist));
  for (int c = 0; c < nlist; ++c) sizes[c] = ix.list_off[c + 1] - ix.list_off[c];
  std::partial_sort(sizes.begin(), sizes.begin() + nprobe, sizes.end(), std::greater<int64_t>());
  int64_t max_total = 0;
  for (int pp = 0; pp < nprobe; ++pp) max_total += sizes[pp];
  max_total = std::max<int64_t>(max_total, 1);
  // Query blocks bound the scratch: coarse scores, per-pair lists / candidate keys.
  int64_t qb = nq;
  qb = std::min<int64_t>(qb, std::max<int64_t>(1, (int64_t(1) << 26) / nlist));
  qb = std::min<int64_t>(qb, std::max<int64_t>(1, (int64_t(1) << 30) / nprobe));
  if (sort_mode)
    qb = std::min<int64_t>(qb, std::max<int64_t>(1, (int64_t(1) << 28) / max_total));
  else
    qb = std::min<int64_t>(qb, std::max<int64_t>(1, (int64_t(1) << 27) / (int64_t(nprobe) * k)));
  const bool coarse_sort = nprobe > prim::kIvfMaxSelect;
  // the tensor-core scan: L2 metrics, k within its 12-entry lists
  const bool use_tc = ix.tc_ready && k <= 10 && !sort_mode;

  float *qn = nullptr, *sc = nullptr, *pval = nullptr;
  int64_t* probe = nullptr;
  uint32_t* cum = nullptr;
  int *lcnt = nullptr, *loff = nullptr, *cursor = nullptr, *pairs = nullptr, *icnt = nullptr,
      *ioff = nullptr;
  OVVS_TRY(r.scratch(rt::kWsIvfQueryNorm, static_cast<size_t>(nq), &qn));
  OVVS_TRY(r.scratch(rt::kWsIvfScores, static_cast<size_t>(qb) * nlist, &sc));
  OVVS_TRY(r.scratch(rt::kWsIvfProbe, static_cast<size_t>(qb) * nprobe, &probe));
  OVVS_TRY(r.scratch(rt::kWsIvfCum, static_cast<size_t>(qb) * (nprobe + 1), &cum));
  OVVS_TRY(r.scratch(rt::kWsIvfListCount, static_cast<size_t>(nlist) + 1, &lcnt));
  OVVS_TRY(r.scratch(rt::kWsIvfListOff, static_cast<size_t>(nlist) + 1, &loff));
  OVVS_TRY(r.scratch(rt::kWsIvfCursor, static_cast<size_t>(nlist), &cursor));
  OVVS_TRY(r.scratch(rt::kWsIvfPairs, static_cast<size_t>(qb) * nprobe, &pairs));
  OVVS_TRY(r.scratch(rt::kWsIvfItemCount, static_cast<size_t>(nlist) + 1, &icnt));
  OVVS_TRY(r.scratch(rt::kWsIvfItemOff, static_cast<size_t>(nlist) + 1, &ioff));
  uint64_t *ckeys = nullptr, *ckeys2 = nullptr;
  int64_t* seg = nullptr;
  int *seg_b = nullptr, *seg_e = nullptr;
  size_t cand_count = sort_mode ? static_cast<size_t>(qb) * max_total
                                : static_cast<size_t>(qb) * nprobe * k;
  if (coarse_sort) cand_count = std::max(cand_count, static_cast<size_t>(qb) * nlist);
  OVVS_TRY(r.scratch(rt::kWsIvfCand, cand_count, &ckeys));
  if (sort_mode || coarse_sort) {
    OVVS_TRY(r.scratch(rt::kWsIvfCand2, cand_count, &ckeys2));
    OVVS_TRY(r.scratch(rt::kWsIvfSeg, static_cast<size_t>(std::max<int64_t>(qb, nlist)) + 1, &seg));
    OVVS_TRY(r.scratch(rt::kWsIvfSegBegin, static_cast<size_t>(qb) + 1, &seg_b));
    OVVS_TRY(r.scratch(rt::kWsIvfSegEnd, static_cast<size_t>(qb) + 1, &seg_e));
  }
  if (coarse_sort) OVVS_TRY(r.scratch(rt::kWsIvfProbeVal, static_cast<size_t>(qb) * nprobe, &pval));
  // CUB temporary storage (the largest of the scans and sorts below)
  size_t tmp_bytes = 0, b = 0;
  OVVS_TRY_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, b, lcnt, loff, nlist + 1, s));
  tmp_bytes = std::max(tmp_bytes, b);
  if (sort_mode) {
    b = 0;
    OVVS_TRY_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, b, seg, seg, qb + 1, s));
    tmp_bytes = std::max(tmp_bytes, b);
    b = 0;
    OVVS_TRY_CUDA(cub::DeviceSegmentedSort::SortKeys(nullptr, b, ckeys, ckeys2,
                                                     static_cast<int>(cand_count),
                                                     static_cast<int>(qb), seg_b, seg_e, s));
    tmp_bytes = std::max(tmp_bytes, b);
  }
  if (coarse_sort) tmp_bytes = std::max(tmp_bytes, prim::topk_tmp_bytes(qb, nlist));
  void* tmp = nullptr;
  OVVS_TRY(r.scratch(rt::kWsIvfTmp, tmp_bytes, reinterpret_cast<uint8_t**>(&tmp)));

  const bool marks = qb >= nq;  // phases are recorded for single-block searches
  r.mark(0);
  OVVS_TRY_CUDA(prim::launch_row_norms_seq(d_queries, nq, dim, qn, s));
  for (int64_t q0 = 0; q0 < nq; q0 += qb) {
    const int64_t nb = std::min(qb, nq - q0);
    const float* qblk = d_queries + q0 * dim;
    // coarse: squared L2 against the centroids (indexes.cpp:310-312), nprobe smallest
    OVVS_TRY_CUDA(prim::launch_gemm_seq(qblk, ix.d_cent.as<float>(), sc, nb, nlist, dim, true,
                                        prim::kRoundNone, s));
    OVVS_TRY_CUDA(prim::launch_pairwise_expand(sc, qn + q0, ix.d_cnorm.as<float>(), nb, nlist,
                                               OVVS_METRIC_L2_EXPANDED, s));
    if (!coarse_sort) {
      OVVS_TRY_CUDA(prim::launch_ivf_coarse_select(sc, nb, nlist, nprobe, probe, s));
    } else {
      OVVS_TRY_CUDA(prim::launch_topk(sc, nb, nlist, nprobe, false, ckeys, ckeys2,
                                      reinterpret_cast<int*>(seg), tmp, tmp_bytes, probe, pval, s));
    }
    // group the (query, probe) pairs by list and lay out the work items
    OVVS_TRY_CUDA(cudaMemsetAsync(lcnt, 0, (nlist + 1) * sizeof(int), s));
    OVVS_TRY_CUDA(cudaMemsetAsync(cursor, 0, nlist * sizeof(int), s));
    OVVS_TRY_CUDA(prim::launch_ivf_probe_offsets(probe, nb, nprobe, ix.d_loff.as<int64_t>(), nlist,
                                                 cum, lcnt, s));
    size_t tb = tmp_bytes;
    OVVS_TRY_CUDA(cub::DeviceScan::ExclusiveSum(tmp, tb, lcnt, loff, nlist + 1, s));
    OVVS_TRY_CUDA(prim::launch_ivf_group_pairs(probe, nb, nprobe, nlist, loff, cursor, pairs, s));
    OVVS_TRY_CUDA(prim::launch_ivf_item_counts(lcnt, nlist, icnt, s));
    tb = tmp_bytes;
    OVVS_TRY_CUDA(cub::DeviceScan::ExclusiveSum(tmp, tb, icnt, ioff, nlist + 1, s));

    prim::IvfScanParams p{};
    p.queries = qblk;
    p.q_norm = qn + q0;
    p.rows = ix.d_rows.as<float>();
    p.row_norm = ix.d_rnorm.as<float>();
    p.row_ids = ix.d_ids.as<int64_t>();
    p.list_off = ix.d_loff.as<int64_t>();
    p.bitset = d_bitset;
    p.bitset_bits = ix.n;
    p.list_q_off = loff;
    p.pair_of = pairs;
    p.item_off = ioff;
    p.cum = cum;
    p.probe = probe;
    p.nq = nb;
    p.nprobe = nprobe;
    p.nlist = nlist;
    p.dim = dim;
    p.metric = ix.metric;
    const int64_t grid = prim::ivf_max_items(nb, nprobe, nlist);
    if (marks) r.mark(1);  // phase 1 = the list scan (and, for k > 256, the segment sort)
    int64_t* out_n = d_neighbors + q0 * k;
    float* out_d = d_distances + q0 * k;
    if (use_tc) {
      p.cand = ckeys;
      OVVS_TRY(scan_tc(r, ix, p, k, lcnt, loff, pairs, tmp, tmp_bytes));
      if (marks) r.mark(2);
      OVVS_TRY_CUDA(prim::launch_ivf_emit(p, nullptr, k, out_n, out_d, s));
    } else if (!sort_mode) {
      p.k_sel = static_cast<int>(k);
      p.cand = ckeys;
      OVVS_TRY_CUDA(prim::launch_ivf_scan_select(p, grid, s));
      if (marks) r.mark(2);
      OVVS_TRY_CUDA(prim::launch_ivf_emit(p, nullptr, k, out_n, out_d, s));
    } else {
      OVVS_TRY_CUDA(prim::launch_ivf_totals(cum, nb, nprobe, seg, s));
      tb = tmp_bytes;
      OVVS_TRY_CUDA(cub::DeviceScan::ExclusiveSum(tmp, tb, seg, seg, nb + 1, s));
      OVVS_TRY_CUDA(prim::launch_ivf_seg_bounds(seg, cum, nb, nprobe, seg_b, seg_e, s));
      p.seg_base = seg;
      p.keys = ckeys;
      OVVS_TRY_CUDA(prim::launch_ivf_scan_sort(p, grid, s));
      tb = tmp_bytes;
      OVVS_TRY_CUDA(cub::DeviceSegmentedSort::SortKeys(tmp, tb, ckeys, ckeys2,
                                                       static_cast<int>(cand_count),
                                                       static_cast<int>(nb), seg_b, seg_e, s));
      if (marks) r.mark(2);
      OVVS_TRY_CUDA(prim::launch_ivf_emit(p, ckeys2, k, out_n, out_d, s));
    }
  }
  if (!marks) {
    r.mark(1);
    r.mark(2);
  }
  r.mark(3);
  r.mark(4);
  return OVVS_STATUS_SUCCESS;
}

// ---- the 'IVF1' file format (indexes.cpp:368-434) ------------------------------------------

ovvsStatus serialize(const IvfFlatIndex& ix, const char* path) {
  std::vector<float> x(static_cast<size_t>(ix.n * ix.dim));
  if (!x.empty()) {
    OVVS_TRY_CUDA(cudaSetDevice(ix.device));
    OVVS_TRY_CUDA(cudaMemcpy(x.data(), ix.d_x.get(), x.size() * sizeof(float),
                             cudaMemcpyDeviceToHost));
  }
  FILE* f = std::fopen(path, "wb");
  if (!f) return OVVS_STATUS_IO;
  bool ok = true;
  auto put = [&](const void* p, size_t bytes) {
    if (bytes && std::fwrite(p, 1, bytes, f) != bytes) ok = false;
  };
  const int32_t ver = 1, metric = ix.metric;
  put(&kIvf1Magic, 4);
  put(&ver, 4);
  put(&ix.n, 8);
  put(&ix.dim, 8);
  put(&ix.nlist, 4);
  put(&metric, 4);
  put(ix.centroids.data(), ix.centroids.size() * sizeof(float));
  put(x.data(), x.size() * sizeof(float));
  for (int32_t c = 0; c < ix.nlist; ++c) {
    const int32_t sz = static_cast<int32_t>(ix.list_off[c + 1] - ix.list_off[c]);
    put(&sz, 4);
    put(ix.list_ids.data() + ix.list_off[c], static_cast<size_t>(sz) * sizeof(int64_t));
  }
  if (std::fclose(f) != 0) ok = false;
  return ok ? OVVS_STATUS_SUCCESS : OVVS_STATUS_IO;
}

ovvsStatus deserialize(rt::Resources& r, const char* path, IvfFlatIndex& ix) {
  FILE* f = std::fopen(path, "rb");
  if (!f) return OVVS_STATUS_IO;
  struct Closer {
    FILE* f;
    ~Closer() { std::fclose(f); }
  } closer{f};
  auto get = [&](void* p, size_t bytes) { return bytes == 0 || std::fread(p, 1, bytes, f) == bytes; };
  uint32_t magic = 0;
  int32_t ver = 0, metric = 0, nlist = 0;
  int64_t n = 0, dim = 0;
  if (!get(&magic, 4) || magic != kIvf1Magic) return OVVS_STATUS_IO;
  if (!get(&ver, 4) || !get(&n, 8) || !get(&dim, 8) || !get(&nlist, 4) || !get(&metric, 4))
    return OVVS_STATUS_IO;
  // sizes the reference would accept without crashing
  if (n < 0 || dim < 0 || nlist < 0 || n > INT32_MAX || (n > 0 && dim > (int64_t(1) << 40) / n) ||
      (nlist > 0 && dim > (int64_t(1) << 40) / nlist))
    return OVVS_STATUS_IO;
  ix.device = r.device;
  ix.n = n;
  ix.dim = dim;
  ix.metric = metric;
  ix.nlist = nlist;
  ix.centroids.resize(static_cast<size_t>(nlist) * dim);
  std::vector<float> x(static_cast<size_t>(n * dim));
  if (!get(ix.centroids.data(), ix.centroids.size() * sizeof(float)) ||
      !get(x.data(), x.size() * sizeof(float)))
    return OVVS_STATUS_IO;
  ix.list_off.assign(static_cast<size_t>(nlist) + 1, 0);
  ix.list_ids.clear();
  for (int32_t c = 0; c < nlist; ++c) {
    int32_t sz = 0;
    if (!get(&sz, 4)) return OVVS_STATUS_IO;
    sz = std::max(sz, 0);
    const size_t at = ix.list_ids.size();
    ix.list_ids.resize(at + static_cast<size_t>(sz));
    if (!get(ix.list_ids.data() + at, static_cast<size_t>(sz) * sizeof(int64_t)))
      return OVVS_STATUS_IO;
    ix.list_off[c + 1] = static_cast<int64_t>(ix.list_ids.size());
  }
  if (static_cast<int64_t>(ix.list_ids.size()) > INT32_MAX) return OVVS_STATUS_SHAPE_MISMATCH;
  OVVS_TRY_CUDA(ix.d_x.reserve(bytes_of(n * dim, sizeof(float))));
  if (!x.empty())
    OVVS_TRY_CUDA(cudaMemcpyAsync(ix.d_x.get(), x.data(), x.size() * sizeof(float),
                                  cudaMemcpyHostToDevice, r.stream));
  if (dim > 0) OVVS_TRY(set_centroids(r, ix));
  return assemble(r, ix);
}

}  // namespace ivf
}  // namespace ovvs
