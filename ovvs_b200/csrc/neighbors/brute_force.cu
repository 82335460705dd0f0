// Brute-force index build and search orchestration (see brute_force.hpp).
#include "brute_force.hpp"

#include <cub/device/device_radix_sort.cuh>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <vector>

#include "../prim/prep.cuh"
#include "../prim/select.cuh"

namespace ovvs {
namespace nb {
namespace {

using prim::kTileN;
using prim::kTileQ;

constexpr int kDTypeF32 = 0, kDTypeF16 = 1, kDTypeI8 = 2;
constexpr int kItemOverheadTiles = 4;  // query-tile load + pipeline refill + list warm-up

size_t elem_size(int dtype) {
  if (dtype == kDTypeF32) return 4;
  if (dtype == kDTypeF16) return 2;
  return 1;  // I8, U8 and the byte-read F8/F4 types
}

// Splits dp (multiple of 16) into K chunks of 64 (SWIZZLE_128B), then 32 / 16 for the tail.
// Splits a padded dim into K chunks of 64 fp16 columns plus 32- and 16-wide tails. Returns false
// (writing nothing past `cap`) when more than `cap` chunks would be needed.
bool plan_chunks(int dp, int cap, int* nchunk, int* cx, int* cw) {
  if (dp / 64 + 2 > cap) return false;
  int n = 0, x = 0;
  while (dp - x >= 64) {
    cx[n] = x;
    cw[n++] = 64;
    x += 64;
  }
  if (dp - x >= 32) {
    cx[n] = x;
    cw[n++] = 32;
    x += 32;
  }
  if (dp - x >= 16) {
    cx[n] = x;
    cw[n++] = 16;
    x += 16;
  }
  *nchunk = n;
  return true;
}

}  // namespace

// Databases of at most this many 256-row tiles (k-means centroids, coarse quantisers) are
// filtered on every column's exact ranking value (FusedParams::exact_filter).
constexpr int kExactFilterTiles = 64;

int list_size_for(int64_t k_eff) {
  const int64_t need = k_eff + std::max<int64_t>(2, (k_eff + 7) / 8);
  for (int kl : {4, 8, 12, 16, 32})
    if (need <= kl) return kl;
  return 0;
}

// Number of super-chunks per query pair-tile: balances the per-pair work of the statically
// strided item schedule (CTA pair c runs items c, c + pairs, ...) against the per-item
// overhead.
int choose_num_sc(int num_qtiles, int num_dbtiles, int num_sms, int64_t cand_per_sc_bytes,
                  int* tiles_per_item) {
  int best_sc = 1, best_L = num_dbtiles;
  double best = std::numeric_limits<double>::infinity();
  const int max_sc = std::min(num_dbtiles, 512);
  for (int sc = 1; sc <= max_sc; ++sc) {
    const int L = (num_dbtiles + sc - 1) / sc;
    const int sc_eff = (num_dbtiles + L - 1) / L;
    if (sc_eff != sc) continue;
    if (static_cast<double>(cand_per_sc_bytes) * sc > 1.5e9) break;
    const int64_t items = static_cast<int64_t>(num_qtiles / 2) * sc;
    const int64_t grid = std::min<int64_t>(items, num_sms / 2);
    const int64_t waves = (items + grid - 1) / grid;
    const double cost = static_cast<double>(waves) * (L + kItemOverheadTiles);
    if (cost < best * 0.999) {
      best = cost;
      best_sc = sc;
      best_L = L;
    }
  }
  *tiles_per_item = best_L;
  return best_sc;
}

ovvsStatus build_from_device(rt::Resources& r, BruteIndex& ix, const void* d_data, int dtype,
                             int64_t n, int64_t dim, int metric_raw, int64_t row_offset) {
  if (n >= static_cast<int64_t>(keys::kEmptyId) || dim > 4096) return OVVS_STATUS_SHAPE_MISMATCH;
  ix.device = r.device;
  ix.sharded = false;
  ix.n = n;
  ix.n_total = n;
  ix.row_offset = row_offset;
  ix.dim = dim;
  ix.metric_raw = metric_raw;
  ix.metric = prim::normalize_metric(metric_raw);
  ix.dtype = dtype;
  ix.dp = static_cast<int>((dim + 15) / 16 * 16);
  if (!plan_chunks(ix.dp, prim::kMaxChunks, &ix.nchunk, ix.chunk_x, ix.chunk_w))
    return OVVS_STATUS_UNSUPPORTED;
  const bool hamming = ix.metric == prim::kMetricHamming;
  ix.b_parts = (dtype == kDTypeF32 && !hamming) ? 2 : 1;
  ix.n_pad = (n + kTileN - 1) / kTileN * kTileN;
  ix.num_tiles = static_cast<int>(ix.n_pad / kTileN);
  cudaStream_t s = r.stream;

  rt::DeviceBuffer norm, key, ids, perm, keys_out, absmax, cub_tmp;
  OVVS_TRY_CUDA(norm.reserve(n * sizeof(float)));
  OVVS_TRY_CUDA(key.reserve(n * sizeof(float)));
  OVVS_TRY_CUDA(ids.reserve(n * sizeof(uint32_t)));
  OVVS_TRY_CUDA(perm.reserve(n * sizeof(uint32_t)));
  OVVS_TRY_CUDA(keys_out.reserve(n * sizeof(float)));
  OVVS_TRY_CUDA(absmax.reserve(sizeof(unsigned int)));
  OVVS_TRY_CUDA(cudaMemsetAsync(absmax.get(), 0, sizeof(unsigned int), s));
  prim::launch_row_stats(d_data, dtype, n, static_cast<int>(dim), ix.metric, norm.as<float>(),
                         key.as<float>(), absmax.as<unsigned int>(), s);
  OVVS_TRY_CUDA(cudaGetLastError());

  ix.e_db = 0;
  if (ix.b_parts == 2) {
    unsigned int bits = 0;
    OVVS_TRY_CUDA(cudaMemcpyAsync(&bits, absmax.get(), sizeof(bits), cudaMemcpyDeviceToHost, s));
    OVVS_TRY_CUDA(cudaStreamSynchronize(s));
    float mx;
    std::memcpy(&mx, &bits, sizeof(mx));
    if (mx > 0.f) ix.e_db = std::min(14 - std::ilogb(mx), 127);
  }

  // Stable sort of row ids by their ranking aux (radix sort keeps equal keys in id order, so
  // identical rows stay in ascending id order).
  {
    std::vector<uint32_t> iota(static_cast<size_t>(n));
    for (int64_t i = 0; i < n; ++i) iota[static_cast<size_t>(i)] = static_cast<uint32_t>(i);
    OVVS_TRY_CUDA(cudaMemcpyAsync(ids.get(), iota.data(), n * sizeof(uint32_t),
                                  cudaMemcpyHostToDevice, s));
    size_t tmp_bytes = 0;
    OVVS_TRY_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp_bytes, key.as<float>(),
                                                  keys_out.as<float>(), ids.as<uint32_t>(),
                                                  perm.as<uint32_t>(), static_cast<int>(n), 0, 32,
                                                  s));
    OVVS_TRY_CUDA(cub_tmp.reserve(tmp_bytes + 16));
    OVVS_TRY_CUDA(cub::DeviceRadixSort::SortPairs(cub_tmp.get(), tmp_bytes, key.as<float>(),
                                                  keys_out.as<float>(), ids.as<uint32_t>(),
                                                  perm.as<uint32_t>(), static_cast<int>(n), 0, 32,
                                                  s));
    OVVS_TRY_CUDA(cudaStreamSynchronize(s));  // iota must outlive the copy
  }

  const int stride = ix.b_parts * ix.dp;
  OVVS_TRY_CUDA(ix.rows16.reserve(static_cast<size_t>(ix.n_pad) * stride * 2));
  const bool keep_exact32 = dtype == kDTypeF32 && !hamming;
  if (keep_exact32) OVVS_TRY_CUDA(ix.exact32.reserve(static_cast<size_t>(ix.n_pad) * dim * 4));
  OVVS_TRY_CUDA(ix.aux.reserve(ix.n_pad * sizeof(float)));
  OVVS_TRY_CUDA(ix.norm_sorted.reserve(ix.n_pad * sizeof(float)));
  OVVS_TRY_CUDA(ix.row_id.reserve(ix.n_pad * sizeof(uint32_t)));
  OVVS_TRY_CUDA(ix.inv_perm.reserve(n * sizeof(uint32_t)));
  OVVS_TRY_CUDA(ix.tile_aux.reserve((ix.num_tiles + prim::group_count(ix.num_tiles)) * sizeof(float2)));
  prim::launch_scatter_rows(d_data, dtype, n, ix.n_pad, static_cast<int>(dim), ix.dp, ix.b_parts,
                            ix.metric, ix.e_db, perm.as<uint32_t>(), norm.as<float>(),
                            key.as<float>(), ix.rows16.as<__half>(),
                            keep_exact32 ? ix.exact32.as<float>() : nullptr, ix.aux.as<float>(),
                            ix.norm_sorted.as<float>(), ix.row_id.as<uint32_t>(),
                            ix.inv_perm.as<uint32_t>(), s);
  OVVS_TRY_CUDA(cudaGetLastError());
  prim::launch_tile_bounds(ix.aux.as<float>(), n, ix.num_tiles, ix.tile_aux.as<float2>(), s);
  OVVS_TRY_CUDA(cudaGetLastError());
  if (!keep_exact32) ix.exact32.release();

  const uint64_t cols = static_cast<uint64_t>(stride);
  if (!rt::encode_f16_2d(&ix.b64, ix.rows16.get(), cols, ix.n_pad, 64, prim::kHalfN) ||
      !rt::encode_f16_2d(&ix.b32, ix.rows16.get(), cols, ix.n_pad, 32, prim::kHalfN) ||
      !rt::encode_f16_2d(&ix.b16, ix.rows16.get(), cols, ix.n_pad, 16, prim::kHalfN)) {
    return OVVS_STATUS_ERROR;
  }
  OVVS_TRY_CUDA(cudaStreamSynchronize(s));
  return OVVS_STATUS_SUCCESS;
}

namespace {

__global__ void mask_padding_aux_kernel(float* __restrict__ aux, const int64_t* __restrict__ real,
                                        int64_t n) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n && real[i] < 0) aux[i] = __int_as_float(0x7f800000);
}

}  // namespace

ovvsStatus build_in_order(rt::Resources& r, BruteIndex& ix, const float* d_rows, int64_t n,
                          int64_t dim, int metric_raw, const int64_t* d_real) {
  if (n >= static_cast<int64_t>(keys::kEmptyId) || dim > 4096) return OVVS_STATUS_SHAPE_MISMATCH;
  ix.device = r.device;
  ix.sharded = false;
  ix.n = n;
  ix.n_total = n;
  ix.row_offset = 0;
  ix.dim = dim;
  ix.metric_raw = metric_raw;
  ix.metric = prim::normalize_metric(metric_raw);
  ix.dtype = kDTypeF32;
  ix.dp = static_cast<int>((dim + 15) / 16 * 16);
  if (!plan_chunks(ix.dp, prim::kMaxChunks, &ix.nchunk, ix.chunk_x, ix.chunk_w))
    return OVVS_STATUS_UNSUPPORTED;
  if (prim::rank_kind_of(ix.metric) != prim::kRankAffine) return OVVS_STATUS_UNSUPPORTED;
  ix.b_parts = 2;
  ix.n_pad = (n + kTileN - 1) / kTileN * kTileN;
  ix.num_tiles = static_cast<int>(ix.n_pad / kTileN);
  cudaStream_t s = r.stream;
  rt::DeviceBuffer norm, key, perm, absmax;
  OVVS_TRY_CUDA(norm.reserve(n * sizeof(float)));
  OVVS_TRY_CUDA(key.reserve(n * sizeof(float)));
  OVVS_TRY_CUDA(perm.reserve(n * sizeof(uint32_t)));
  OVVS_TRY_CUDA(absmax.reserve(sizeof(unsigned int)));
  OVVS_TRY_CUDA(cudaMemsetAsync(absmax.get(), 0, sizeof(unsigned int), s));
  prim::launch_row_stats(d_rows, kDTypeF32, n, static_cast<int>(dim), ix.metric, norm.as<float>(),
                         key.as<float>(), absmax.as<unsigned int>(), s);
  OVVS_TRY_CUDA(cudaGetLastError());
  std::vector<uint32_t> iota(static_cast<size_t>(n));
  for (int64_t i = 0; i < n; ++i) iota[static_cast<size_t>(i)] = static_cast<uint32_t>(i);
  OVVS_TRY_CUDA(cudaMemcpyAsync(perm.get(), iota.data(), n * sizeof(uint32_t),
                                cudaMemcpyHostToDevice, s));
  unsigned int bits = 0;
  OVVS_TRY_CUDA(cudaMemcpyAsync(&bits, absmax.get(), sizeof(bits), cudaMemcpyDeviceToHost, s));
  OVVS_TRY_CUDA(cudaStreamSynchronize(s));  // iota and bits
  float mx;
  std::memcpy(&mx, &bits, sizeof(mx));
  ix.e_db = mx > 0.f ? std::min(14 - std::ilogb(mx), 127) : 0;
  const int stride = ix.b_parts * ix.dp;
  OVVS_TRY_CUDA(ix.rows16.reserve(static_cast<size_t>(ix.n_pad) * stride * 2));
  ix.exact32.release();
  OVVS_TRY_CUDA(ix.aux.reserve(ix.n_pad * sizeof(float)));
  OVVS_TRY_CUDA(ix.norm_sorted.reserve(ix.n_pad * sizeof(float)));
  OVVS_TRY_CUDA(ix.row_id.reserve(ix.n_pad * sizeof(uint32_t)));
  OVVS_TRY_CUDA(ix.inv_perm.reserve(n * sizeof(uint32_t)));
  OVVS_TRY_CUDA(ix.tile_aux.reserve((ix.num_tiles + prim::group_count(ix.num_tiles)) * sizeof(float2)));
  prim::launch_scatter_rows(d_rows, kDTypeF32, n, ix.n_pad, static_cast<int>(dim), ix.dp,
                            ix.b_parts, ix.metric, ix.e_db, perm.as<uint32_t>(), norm.as<float>(),
                            key.as<float>(), ix.rows16.as<__half>(), nullptr, ix.aux.as<float>(),
                            ix.norm_sorted.as<float>(), ix.row_id.as<uint32_t>(),
                            ix.inv_perm.as<uint32_t>(), s);
  OVVS_TRY_CUDA(cudaGetLastError());
  if (d_real && n > 0) {
    mask_padding_aux_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
        ix.aux.as<float>(), d_real, n);
    OVVS_TRY_CUDA(cudaGetLastError());
  }
  prim::launch_tile_bounds(ix.aux.as<float>(), n, ix.num_tiles, ix.tile_aux.as<float2>(), s);
  OVVS_TRY_CUDA(cudaGetLastError());
  const uint64_t cols = static_cast<uint64_t>(stride);
  if (!rt::encode_f16_2d(&ix.b64, ix.rows16.get(), cols, ix.n_pad, 64, prim::kHalfN) ||
      !rt::encode_f16_2d(&ix.b32, ix.rows16.get(), cols, ix.n_pad, 32, prim::kHalfN) ||
      !rt::encode_f16_2d(&ix.b16, ix.rows16.get(), cols, ix.n_pad, 16, prim::kHalfN)) {
    return OVVS_STATUS_ERROR;
  }
  OVVS_TRY_CUDA(cudaStreamSynchronize(s));
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus build_from_host(rt::Resources& r, BruteIndex& ix, const void* data, int dtype,
                           int64_t n, int64_t dim, int metric_raw, int64_t row_offset,
                           bool sharded) {
  const size_t bytes = static_cast<size_t>(n) * dim * elem_size(dtype);
  rt::DeviceBuffer raw;
  OVVS_TRY_CUDA(raw.reserve(bytes));
  OVVS_TRY(rt::upload(r, raw.get(), data, bytes));
  ovvsStatus st = build_from_device(r, ix, raw.get(), dtype, n, dim, metric_raw, row_offset);
  if (st != OVVS_STATUS_SUCCESS) return st;
  ix.sharded = sharded && r.world > 1;
  if (ix.sharded) {
    int64_t total = n;
    OVVS_TRY(rt::allreduce_i64_sum(r, &total));
    ix.n_total = total;
  }
  return r.finish();
}

// Fused-kernel parameters common to every launch of one search.
ovvsStatus base_params(rt::Resources& r, const BruteIndex& ix, const SearchCtx& c, int64_t nq,
                       prim::FusedParams* out) {
  prim::FusedParams& p = *out;
  p = prim::FusedParams{};
  p.dp = ix.dp;
  p.nchunk = ix.nchunk;
  for (int i = 0; i < ix.nchunk; ++i) {
    p.chunk_x[i] = ix.chunk_x[i];
    p.chunk_w[i] = ix.chunk_w[i];
  }
  p.b_parts = ix.b_parts;
  p.nunits = ix.b_parts * ix.nchunk;
  if (!prim::plan_fused_smem(p, r.max_smem_optin)) return OVVS_STATUS_UNSUPPORTED;
  p.query_split = ix.metric != prim::kMetricHamming;
  p.q_lo_flag = c.flag;
  p.num_qtiles = c.num_qtiles;
  p.num_dbtiles = ix.num_tiles;
  p.n_rows = ix.n;
  p.row_aux = ix.aux.as<float>();
  p.group_aux = ix.tile_aux.as<float2>() + ix.num_tiles;
  p.row_id = ix.row_id.as<uint32_t>();
  p.q_mul = c.q_mul;
  p.allow = c.allow;
  p.rank_kind = prim::rank_kind_of(ix.metric);
  p.nq = nq;
  p.err = r.d_err;
  return OVVS_STATUS_SUCCESS;
}

prim::MergeParams merge_params(const BruteIndex& ix, const SearchCtx& c, const float* d_queries,
                               int64_t nq, int64_t k_eff) {
  prim::MergeParams m{};
  m.nq = nq;
  m.dim = static_cast<int>(ix.dim);
  m.queries = d_queries;
  m.xn = c.xn;
  m.metric = ix.metric;
  m.exact32 = ix.exact32.get() ? ix.exact32.as<float>() : nullptr;
  m.rows16 = ix.rows16.as<__half>();
  m.rows16_stride = ix.b_parts * ix.dp;
  m.norm_sorted = ix.norm_sorted.as<float>();
  m.inv_perm = ix.inv_perm.as<uint32_t>();
  m.allow = c.allow;
  m.row_offset = ix.row_offset;
  m.k_eff = static_cast<int>(k_eff);
  m.negate_output = ix.metric == prim::kMetricInnerProduct;
  return m;
}

int pair_sms(const rt::Resources& r, const prim::FusedParams& p) {
  return 2 * std::min(r.num_sms / 2, prim::fused_max_pairs(p.smem_bytes));
}

ovvsStatus encode_query_maps(SearchCtx& c, int dp) {
  const uint64_t a_cols = static_cast<uint64_t>(2 * dp);
  if (!rt::encode_f16_2d(&c.maps.a64, c.a16, a_cols, c.q_pad, 64, kTileQ) ||
      !rt::encode_f16_2d(&c.maps.a32, c.a16, a_cols, c.q_pad, 32, kTileQ) ||
      !rt::encode_f16_2d(&c.maps.a16, c.a16, a_cols, c.q_pad, 16, kTileQ)) {
    return OVVS_STATUS_ERROR;
  }
  return OVVS_STATUS_SUCCESS;
}

namespace {

int launch_grid(const prim::FusedParams& p, int num_sms) {
  return prim::fused_grid(p.num_items, num_sms);
}

// Sharded list-mode searches: *own = this rank's bound array in the peer window and
// p.peer_bound = the other ranks' arrays, so the fused kernel shares each query's bound across
// ranks. The window is created (and grown) here, collectively: every rank of a sharded search
// reaches this point with the same q_pad. *own stays null when the window is unavailable (every
// rank then agrees) or switched off with OVVS_PEER_BOUNDS=0 (which must then be set on every
// rank); the search then keeps its bound on its own rank.
ovvsStatus peer_bound_arrays(rt::Resources& r, int64_t q_pad, uint64_t** own,
                             prim::FusedParams& p) {
  *own = nullptr;
  if (r.peer_bounds == 0) {
    const char* e = std::getenv("OVVS_PEER_BOUNDS");
    if ((e && std::strcmp(e, "0") == 0) || r.world < 2 || r.world - 1 > prim::kMaxPeers)
      r.peer_bounds = -1;
  }
  if (r.peer_bounds < 0) return OVVS_STATUS_SUCCESS;
  const size_t need = static_cast<size_t>(q_pad) * sizeof(uint64_t);
  if (!r.bound_win.ready() || r.bound_win.bytes() < need) {
    // this rank's kernels stop using the old window before it is unmapped
    if (r.bound_win.ready()) OVVS_TRY(r.finish());
    const uint64_t tag =
        r.comm_tag ^ (0x9E3779B97F4A7C15ull * static_cast<uint64_t>(++r.window_seq));
    // descriptor exchange bounded by 10 s (or the NCCL deadline if shorter): where the ranks
    // cannot reach one another's sockets, the search goes on with local bounds after it
    const ovvsStatus st = r.bound_win.create(r, std::max(need, size_t(1) << 20), tag,
                                             std::min<int64_t>(r.nccl_timeout_ms, 10000));
    if (st == OVVS_STATUS_UNSUPPORTED) {
      r.peer_bounds = -1;
      return OVVS_STATUS_SUCCESS;
    }
    OVVS_TRY(st);
    r.peer_bounds = 1;
  }
  *own = static_cast<uint64_t*>(r.bound_win.ptr(r.rank));
  p.n_peers = 0;
  for (int g = 0; g < r.world; ++g)
    if (g != r.rank) p.peer_bound[p.n_peers++] = static_cast<uint64_t*>(r.bound_win.ptr(g));
  return OVVS_STATUS_SUCCESS;
}

// Large k (k plus re-rank margin above the register lists): bound pre-pass on a sample of the
// tiles, append pass with that bound, then per-query sort + exact re-rank; repeated with a
// tighter bound for queries whose buffer overflowed.
ovvsStatus search_large(rt::Resources& r, const BruteIndex& ix, const SearchCtx& c,
                        const float* d_queries, int64_t nq, int64_t k_eff, prim::MergeParams m) {
  cudaStream_t s = r.stream;
  const int margin = static_cast<int>(std::max<int64_t>(2, (k_eff + 7) / 8));
  const int64_t need = k_eff + margin;
  const bool prepass = ix.n > 4096;
  int cap = 32;
  const int64_t want = prepass ? 32 * need : std::max<int64_t>(ix.n, need);
  while (cap < want && cap < prim::kSelectMaxCap) cap <<= 1;
  if (need > cap) return OVVS_STATUS_UNSUPPORTED;  // k beyond ~7k rows per query

  uint64_t* tau = nullptr;
  uint32_t* count = nullptr;
  uint64_t* buf = nullptr;
  int* overflow = nullptr;
  OVVS_TRY(r.scratch(rt::kWsBound, static_cast<size_t>(c.q_pad), &tau));
  OVVS_TRY(r.scratch(rt::kWsAppCount, static_cast<size_t>(c.q_pad), &count));
  OVVS_TRY(r.scratch(rt::kWsAppBuf, static_cast<size_t>(c.q_pad) * cap, &buf));
  OVVS_TRY(r.scratch(rt::kWsOverflow, 1, &overflow));
  OVVS_TRY_CUDA(cudaMemsetAsync(tau, 0xFF, static_cast<size_t>(c.q_pad) * sizeof(uint64_t), s));

  if (prepass) {
    // Lists of kPreKL over every stride-th tile; the need-th smallest key of their union bounds
    // the need-th best key of the whole database (the union holds real rows). Short lists keep
    // the pre-pass cheap (each insertion walks the list): enough of them are used for the union
    // to hold twice `need` keys, which still contains the sample's best `need`; longer lists only
    // when 256 lists of 8 (or 16) cannot hold that many.
    const int kPreKL = need <= 1024 ? 8 : (need <= 2048 ? 16 : 32);
    const int stride = ix.num_tiles >= 64 ? 8 : 1;
    const int sampled = (ix.num_tiles + stride - 1) / stride;
    prim::FusedParams p;
    OVVS_TRY(base_params(r, ix, c, nq, &p));
    p.tile_stride = stride;
    p.num_dbtiles = sampled;
    const int64_t cand_per_sc =
        c.q_pad * kPreKL * prim::kListsPerItem * static_cast<int64_t>(sizeof(uint64_t));
    int num_sc = choose_num_sc(c.num_qtiles, sampled, pair_sms(r, p), cand_per_sc, &p.tiles_per_item);
    const int per_sc = kPreKL * prim::kListsPerItem;
    const int min_sc = static_cast<int>(
        std::min<int64_t>(sampled, (2 * need + per_sc - 1) / per_sc));
    if (num_sc < min_sc) {
      p.tiles_per_item = (sampled + min_sc - 1) / min_sc;
      num_sc = (sampled + p.tiles_per_item - 1) / p.tiles_per_item;
    }
    const int lists = num_sc * prim::kListsPerItem;
    if (lists <= 256 && static_cast<int64_t>(lists) * kPreKL >= need) {
      p.num_sc = num_sc;
      p.num_items = prim::fused_items(c.num_qtiles, num_sc);
      p.k_pub = 0;  // short lists cannot bound rank `need`
      uint64_t* cand = nullptr;
      uint64_t* shared_bound = nullptr;
      OVVS_TRY(r.scratch(rt::kWsCand, static_cast<size_t>(c.q_pad) * lists * kPreKL, &cand));
      OVVS_TRY(r.scratch(rt::kWsAppBound, static_cast<size_t>(c.q_pad), &shared_bound));
      OVVS_TRY_CUDA(cudaMemsetAsync(shared_bound, 0xFF, static_cast<size_t>(c.q_pad) * 8, s));
      p.q_bound = shared_bound;
      p.out = cand;
      OVVS_TRY_CUDA(prim::launch_knn_fused(c.maps, p, kPreKL, launch_grid(p, pair_sms(r, p)), s));
      OVVS_TRY_CUDA(prim::launch_kth_bound(cand, lists, nq, static_cast<int>(need), kPreKL, tau, s));
    }
  }

  prim::FusedParams p;
  OVVS_TRY(base_params(r, ix, c, nq, &p));
  p.q_tau_key = tau;
  p.app_count = count;
  p.app_buf = buf;
  p.app_cap = cap;
  // The append pass runs in two stages when the bound came from a sample: after the first half
  // of the tiles each query's bound is tightened to the need-th best key it has appended (about
  // the 2 x need-th best row instead of the sample's 8 x need-th), so the second half appends
  // few rows and its epilogue rarely leaves the filter.
  const bool two_stage = prepass && ix.num_tiles >= 64;
  const int half = two_stage ? (ix.num_tiles + 1) / 2 : ix.num_tiles;
  auto stage = [&](int base, int tiles) {
    prim::FusedParams q = p;
    q.tile_base = base;
    q.num_dbtiles = tiles;
    q.num_sc = choose_num_sc(c.num_qtiles, tiles, pair_sms(r, q), 0, &q.tiles_per_item);
    q.num_items = prim::fused_items(c.num_qtiles, q.num_sc);
    return prim::launch_knn_fused(c.maps, q, 0, launch_grid(q, pair_sms(r, q)), s);
  };
  prim::SelectParams sp{};
  sp.m = m;
  sp.count = count;
  sp.buf = buf;
  sp.cap = cap;
  sp.margin = margin;
  sp.tau_key = tau;
  sp.overflow = overflow;
  constexpr int kMaxRounds = 16;
  for (int round = 0; round < kMaxRounds; ++round) {
    p.app_exact = round >= 2;  // persistent overflow: strict key bound (ties cannot pile up)
    OVVS_TRY_CUDA(cudaMemsetAsync(count, 0, static_cast<size_t>(c.q_pad) * sizeof(uint32_t), s));
    OVVS_TRY_CUDA(cudaMemsetAsync(overflow, 0, sizeof(int), s));
    OVVS_TRY_CUDA(stage(0, half));
    if (two_stage) {
      OVVS_TRY_CUDA(prim::launch_tighten_tau(buf, count, cap, nq, static_cast<int>(need), tau, s));
      OVVS_TRY_CUDA(stage(half, ix.num_tiles - half));
    }
    OVVS_TRY_CUDA(prim::launch_select_rerank(sp, s));
    int host_overflow = 0;
    OVVS_TRY_CUDA(cudaMemcpyAsync(&host_overflow, overflow, sizeof(int), cudaMemcpyDeviceToHost, s));
    OVVS_TRY_CUDA(cudaStreamSynchronize(s));
    if (!host_overflow) return OVVS_STATUS_SUCCESS;
  }
  return OVVS_STATUS_ERROR;
}

}  // namespace

ovvsStatus prepare_queries(rt::Resources& r, const BruteIndex& ix, const float* d_queries,
                           int64_t nq, PreparedQueries& pq) {
  cudaStream_t s = r.stream;
  pq.nq = nq;
  pq.q_pad = prim::pad_queries(nq);
  pq.dp = ix.dp;
  pq.metric = ix.metric;
  OVVS_TRY_CUDA(pq.a16.reserve(static_cast<size_t>(pq.q_pad) * 2 * ix.dp * sizeof(__half)));
  OVVS_TRY_CUDA(pq.xn.reserve(static_cast<size_t>(pq.q_pad) * sizeof(float)));
  OVVS_TRY_CUDA(pq.e_q.reserve(static_cast<size_t>(pq.q_pad) * sizeof(int16_t)));
  OVVS_TRY_CUDA(pq.flag.reserve(sizeof(int)));
  float* q_mul = nullptr;
  OVVS_TRY(r.scratch(rt::kWsQueryMul, pq.q_pad, &q_mul));
  OVVS_TRY_CUDA(cudaMemsetAsync(pq.flag.get(), 0, sizeof(int), s));
  prim::launch_query_prep(d_queries, nq, pq.q_pad, static_cast<int>(ix.dim), ix.dp, ix.metric,
                          ix.e_db, pq.a16.as<__half>(), q_mul, pq.xn.as<float>(),
                          pq.flag.as<int>(), s, pq.e_q.as<int16_t>());
  OVVS_TRY_CUDA(cudaGetLastError());
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus search_from_host(rt::Resources& r, const BruteIndex& ix, const float* queries,
                            int64_t nq, int64_t k, const uint8_t* bitset, int64_t* neighbors,
                            float* distances, int64_t* k_eff_out) {
  const int64_t k_eff = std::min<int64_t>(k, ix.n_total);
  float* dq = nullptr;
  OVVS_TRY(r.scratch(rt::kWsQueries, static_cast<size_t>(nq) * ix.dim, &dq));
  OVVS_TRY_CUDA(cudaMemcpyAsync(dq, queries, static_cast<size_t>(nq) * ix.dim * sizeof(float),
                                cudaMemcpyHostToDevice, r.stream));
  uint8_t* db = nullptr;
  if (bitset) {
    const int64_t bytes = (ix.row_offset + ix.n + 7) / 8;
    OVVS_TRY(r.scratch(rt::kWsBitset, static_cast<size_t>(bytes), &db));
    OVVS_TRY_CUDA(cudaMemcpyAsync(db, bitset, static_cast<size_t>(bytes), cudaMemcpyHostToDevice,
                                  r.stream));
  }
  int64_t* dn = nullptr;
  float* dd = nullptr;
  OVVS_TRY(r.scratch(rt::kWsNeighbors, static_cast<size_t>(nq) * k_eff, &dn));
  OVVS_TRY(r.scratch(rt::kWsDistances, static_cast<size_t>(nq) * k_eff, &dd));
  int64_t ke = 0;
  OVVS_TRY(search_device(r, ix, dq, nq, k, db, dn, dd, &ke));
  // A copy into pageable host memory returns only once the stream's earlier work is done, so with
  // the exchange of a sharded search in the stream it would wait without a bound on the peers:
  // the bounded wait comes first.
  if (ix.sharded) OVVS_TRY(r.finish());
  if (neighbors) {
    OVVS_TRY_CUDA(cudaMemcpyAsync(neighbors, dn, static_cast<size_t>(nq) * ke * sizeof(int64_t),
                                  cudaMemcpyDeviceToHost, r.stream));
    OVVS_TRY_CUDA(cudaMemcpyAsync(distances, dd, static_cast<size_t>(nq) * ke * sizeof(float),
                                  cudaMemcpyDeviceToHost, r.stream));
  }
  *k_eff_out = ke;
  return r.finish();
}

ovvsStatus search_device(rt::Resources& r, const BruteIndex& ix, const float* d_queries, int64_t nq,
                         int64_t k, const uint8_t* d_bitset, int64_t* d_neighbors,
                         float* d_distances, int64_t* k_eff_out, const uint64_t* d_init_bound,
                         const PreparedQueries* prepared, bool labels_only) {
  cudaStream_t s = r.stream;
  const int64_t k_eff = std::min<int64_t>(k, ix.n_total);
  *k_eff_out = k_eff;
  if (!ix.shards.empty()) return OVVS_STATUS_UNSUPPORTED;  // a group's index: its shards search
  if (ix.device != r.device) return OVVS_STATUS_INVALID_ARGUMENT;
  // Sharded after a communicator failure: fail before touching the stream or the workspaces.
  if (ix.sharded) OVVS_TRY(r.comm_ready());
  const int kl = list_size_for(k_eff);
  const int dim = static_cast<int>(ix.dim);

  SearchCtx c;
  c.q_pad = prim::pad_queries(nq);
  c.num_qtiles = static_cast<int>(c.q_pad / kTileQ);
  r.mark(0);
  OVVS_TRY(r.scratch(rt::kWsQueryMul, c.q_pad, &c.q_mul));
  const bool reuse = prepared && prepared->nq == nq && prepared->q_pad == c.q_pad &&
                     prepared->dp == ix.dp && prepared->metric == ix.metric;
  if (reuse) {
    c.a16 = prepared->a16.as<__half>();
    c.xn = prepared->xn.as<float>();
    c.flag = prepared->flag.as<int>();
    prim::launch_query_mul(prepared->e_q.as<int16_t>(), nq, c.q_pad, ix.metric, ix.e_db,
                           c.q_mul, s);
  } else {
    OVVS_TRY(r.scratch(rt::kWsQueryA, static_cast<size_t>(c.q_pad) * 2 * ix.dp, &c.a16));
    OVVS_TRY(r.scratch(rt::kWsQueryNorm, c.q_pad, &c.xn));
    OVVS_TRY(r.scratch(rt::kWsFlags, 4, &c.flag));
    OVVS_TRY_CUDA(cudaMemsetAsync(c.flag, 0, sizeof(int), s));
    prim::launch_query_prep(d_queries, nq, c.q_pad, dim, ix.dp, ix.metric, ix.e_db, c.a16,
                            c.q_mul, c.xn, c.flag, s);
  }
  OVVS_TRY_CUDA(cudaGetLastError());
  if (d_bitset) {
    OVVS_TRY(r.scratch(rt::kWsAllow, ix.n_pad / 32, &c.allow));
    prim::launch_allow_bits(d_bitset, ix.row_offset, ix.row_id.as<uint32_t>(), ix.n, ix.n_pad,
                            c.allow, s);
    OVVS_TRY_CUDA(cudaGetLastError());
  }
  OVVS_TRY(encode_query_maps(c, ix.dp));
  c.maps.b64 = ix.b64;
  c.maps.b32 = ix.b32;
  c.maps.b16 = ix.b16;

  prim::MergeParams m = merge_params(ix, c, d_queries, nq, k_eff);
  m.labels_only = labels_only && r.world <= 1 ? 1 : 0;
  float *srank = nullptr, *grank = nullptr;
  int64_t *sgid = nullptr, *ggid = nullptr;
  const size_t cnt = static_cast<size_t>(nq) * k_eff;
  if (ix.sharded) {
    OVVS_TRY(r.scratch(rt::kWsShardRank, cnt, &srank));
    OVVS_TRY(r.scratch(rt::kWsShardGid, cnt, &sgid));
    OVVS_TRY(r.scratch(rt::kWsGatherRank, cnt * r.world, &grank));
    OVVS_TRY(r.scratch(rt::kWsGatherGid, cnt * r.world, &ggid));
    m.shard_rank = srank;
    m.shard_gid = sgid;
  } else {
    m.neighbors = d_neighbors;
    m.distances = d_distances;
  }

  if (kl == 0) {
    r.mark(1);
    OVVS_TRY(search_large(r, ix, c, d_queries, nq, k_eff, m));
    r.mark(2);
    r.mark(3);
  } else {
    prim::FusedParams p;
    OVVS_TRY(base_params(r, ix, c, nq, &p));
    const int64_t cand_per_sc =
        c.q_pad * kl * prim::kListsPerItem * static_cast<int64_t>(sizeof(uint64_t));
    p.num_sc = choose_num_sc(c.num_qtiles, ix.num_tiles, pair_sms(r, p), cand_per_sc,
                             &p.tiles_per_item);
    p.num_items = prim::fused_items(c.num_qtiles, p.num_sc);
    uint64_t* cand = nullptr;
    OVVS_TRY(r.scratch(rt::kWsCand,
                       static_cast<size_t>(c.q_pad) * p.num_sc * prim::kListsPerItem * kl, &cand));
    p.out = cand;
    uint64_t* bound = nullptr;
    if (ix.sharded && p.rank_kind != prim::kRankColumnScaled)
      OVVS_TRY(peer_bound_arrays(r, c.q_pad, &bound, p));
    if (!bound) OVVS_TRY(r.scratch(rt::kWsBound, static_cast<size_t>(c.q_pad), &bound));
    OVVS_TRY_CUDA(cudaMemsetAsync(bound, 0xFF, static_cast<size_t>(c.q_pad) * sizeof(uint64_t), s));
    if (d_init_bound)
      OVVS_TRY_CUDA(cudaMemcpyAsync(bound, d_init_bound, static_cast<size_t>(nq) * sizeof(uint64_t),
                                    cudaMemcpyDeviceToDevice, s));
    p.q_bound = bound;
    p.k_pub = static_cast<int>(k_eff);
    p.exact_filter = ix.num_tiles <= kExactFilterTiles ? 1 : 0;
    r.mark(1);
    OVVS_TRY_CUDA(prim::launch_knn_fused(c.maps, p, kl, launch_grid(p, pair_sms(r, p)), s));
    r.mark(2);
    m.cand = cand;
    m.num_sc = p.num_sc * prim::kListsPerItem;  // lists per query
    m.kl = kl;
    OVVS_TRY_CUDA(prim::launch_merge_rerank(m, s));
    r.mark(3);
  }
  if (!ix.sharded) {
    r.mark(4);
    return OVVS_STATUS_SUCCESS;
  }
  // Sharded: exact per-shard top-k, all-gather over NVLink, then an exact (rank, id) merge. The
  // communicator is non-blocking: the group's enqueue is settled (bounded) before the merge kernel
  // that reads the gathered lists is launched behind it.
  const rt::NcclApi* nc = rt::nccl();
  OVVS_TRY(r.comm_ready());
  OVVS_TRY(rt::status_of(nc->GroupStart()));
  OVVS_TRY(r.collective(nc->AllGather(srank, grank, cnt, ncclFloat32, r.comm, s)));
  OVVS_TRY(r.collective(nc->AllGather(sgid, ggid, cnt, ncclInt64, r.comm, s)));
  OVVS_TRY(r.collective(nc->GroupEnd()));
  OVVS_TRY_CUDA(prim::launch_shard_merge(grank, ggid, r.world, nq, static_cast<int>(k_eff),
                                         m.negate_output, d_neighbors, d_distances, s));
  r.mark(4);
  return OVVS_STATUS_SUCCESS;
}

}  // namespace nb
}  // namespace ovvs
