/* CPU restatement of the reference's brute-force kNN / k-means arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see ovvs_oracle.h): used by tests/ and by bench.py's CPU-baseline
 * leg as the checker, never by the product library. Compiled with -ffp-contract=off so that
 * every multiply and add rounds separately, like the reference's scalar loops on x86-64.
 *
 * Citations are file:line in the reference repository (manan-ramnani/ovVS 0.2.0). */

#include "ovvs_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <limits>
#include <numeric>
#include <random>
#include <thread>
#include <vector>

namespace {

constexpr int32_t kL2 = 0, kL2Sqrt = 1, kIP = 2, kCos = 3, kHamming = 4, kLp = 5;

/* internal.hpp:215-225: sequential dot product and squared norm. */
float dot_seq(const float* a, const float* b, int64_t d) {
  float s = 0.f;
  for (int64_t i = 0; i < d; ++i) s += a[i] * b[i];
  return s;
}
float nrm2sq_seq(const float* a, int64_t d) {
  float s = 0.f;
  for (int64_t i = 0; i < d; ++i) s += a[i] * a[i];
  return s;
}
/* internal.hpp:57-64. */
float l2sq_seq(const float* a, const float* b, int64_t d) {
  float s = 0.f;
  for (int64_t i = 0; i < d; ++i) {
    const float t = a[i] - b[i];
    s += t * t;
  }
  return s;
}

/* internal.hpp:240-272 distance_one: the non-expanded metrics. */
float distance_direct(int32_t metric, const float* x, const float* y, int64_t d, float arg) {
  switch (metric) {
    case kL2:
      return l2sq_seq(x, y, d);
    case kL2Sqrt:
      return std::sqrt(l2sq_seq(x, y, d));
    case kIP:
      return -dot_seq(x, y, d);
    case kCos: {
      const float nx = std::sqrt(std::max(nrm2sq_seq(x, d), 1e-12f));
      const float ny = std::sqrt(std::max(nrm2sq_seq(y, d), 1e-12f));
      return 1.f - dot_seq(x, y, d) / (nx * ny);
    }
    case kHamming: {
      int s = 0;
      for (int64_t i = 0; i < d; ++i) {
        const uint32_t ax = static_cast<uint32_t>(x[i] >= 0.f);
        const uint32_t ay = static_cast<uint32_t>(y[i] >= 0.f);
        s += static_cast<int>(ax ^ ay);
      }
      return static_cast<float>(s);
    }
    case kLp: {
      const float p = arg > 0.f ? arg : 2.f;
      float s = 0.f;
      for (int64_t i = 0; i < d; ++i) s += std::pow(std::fabs(x[i] - y[i]), p);
      return std::pow(s, 1.f / p);
    }
    default:
      return l2sq_seq(x, y, d);
  }
}

bool expanded(int32_t metric) { return metric == kL2 || metric == kIP || metric == kCos; }

/* cpu_prims.cpp:24-32 topk_before: numbers before NaN, direction, then lower ordinal. */
inline bool before(float a, int64_t ia, float b, int64_t ib, bool largest) {
  if (a < b) return !largest;
  if (a > b) return largest;
  const bool an = std::isnan(a), bn = std::isnan(b);
  if (an != bn) return !an;
  return ia < ib;
}

/* cpu_prims.cpp:61-106. The heap (k <= 64) and partial_sort (k > 64) branches both produce the
   first k elements of the total order, so one selection routine covers both. */
void topk_rows(const float* scores, int64_t rows, int64_t cols, int64_t k, int64_t* indices,
               float* values, bool largest) {
  if (rows <= 0 || cols <= 0 || k <= 0) return;
  k = std::min(k, cols);
  std::vector<int64_t> idx(static_cast<size_t>(cols));
  for (int64_t r = 0; r < rows; ++r) {
    const float* row = scores + r * cols;
    std::iota(idx.begin(), idx.end(), 0);
    std::partial_sort(idx.begin(), idx.begin() + k, idx.end(),
                      [&](int64_t i, int64_t j) { return before(row[i], i, row[j], j, largest); });
    for (int64_t t = 0; t < k; ++t) {
      indices[r * k + t] = idx[static_cast<size_t>(t)];
      values[r * k + t] = row[idx[static_cast<size_t>(t)]];
    }
  }
}

/* mixer.cpp:174-221 for a block of queries against all rows; ynorm precomputed. */
void pairwise_block(int32_t metric, const float* x, int64_t nx, const float* y, int64_t ny,
                    int64_t dim, const float* ynorm, float* out, float arg) {
  if (!expanded(metric)) {
    for (int64_t i = 0; i < nx; ++i)
      for (int64_t j = 0; j < ny; ++j)
        out[i * ny + j] = distance_direct(metric, x + i * dim, y + j * dim, dim, arg);
    return;
  }
  for (int64_t i = 0; i < nx; ++i) {
    const float* xi = x + i * dim;
    const float xn = nrm2sq_seq(xi, dim);
    for (int64_t j = 0; j < ny; ++j) {
      /* cpu_prims.cpp:48-58 naive GEMM (trans_b): sequential fp32 accumulation. */
      const float ip = dot_seq(xi, y + j * dim, dim);
      float v;
      if (metric == kIP) {
        v = -ip;
      } else if (metric == kCos) {
        const float nxv = std::sqrt(std::max(xn, 1e-12f));
        const float nyv = std::sqrt(std::max(ynorm[j], 1e-12f));
        v = 1.f - ip / (nxv * nyv);
      } else {
        v = xn + ynorm[j] - 2.f * ip;
      }
      out[i * ny + j] = v;
    }
  }
}

template <class F>
void parallel_for(int64_t n, int32_t nthreads, F&& fn) {
  if (nthreads <= 1 || n <= 1) {
    fn(int64_t{0}, n);
    return;
  }
  const int64_t t = std::min<int64_t>(nthreads, n);
  std::vector<std::thread> th;
  for (int64_t i = 0; i < t; ++i) {
    const int64_t b = n * i / t, e = n * (i + 1) / t;
    th.emplace_back([&fn, b, e] { fn(b, e); });
  }
  for (auto& x : th) x.join();
}

}  // namespace

extern "C" {

float oracle_f16_to_f32(uint16_t h) {
  /* internal.hpp:804-829 */
  const uint32_t sign = (static_cast<uint32_t>(h & 0x8000u) << 16);
  const uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int32_t e = 127 - 15 + 1;
      while ((man & 0x400u) == 0) {
        man <<= 1;
        --e;
      }
      man &= 0x3ffu;
      bits = sign | (static_cast<uint32_t>(e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | (man << 13);
  } else {
    bits = sign | ((exp + (127 - 15)) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, sizeof(f));
  return f;
}

uint16_t oracle_f32_to_f16_trunc(float f) {
  /* internal.hpp:831-840: exponent clamp, mantissa truncated, subnormals flushed to signed 0. */
  uint32_t bits = 0;
  std::memcpy(&bits, &f, sizeof(bits));
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const int32_t exp = static_cast<int32_t>((bits >> 23) & 0xffu) - 127 + 15;
  const uint32_t man = bits & 0x7fffffu;
  if (exp <= 0) return static_cast<uint16_t>(sign);
  if (exp >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
  return static_cast<uint16_t>(sign | (static_cast<uint32_t>(exp) << 10) | (man >> 13));
}

uint16_t oracle_f32_to_f16_rne(float value) {
  /* internal.hpp:83-106 */
  uint32_t f;
  std::memcpy(&f, &value, sizeof(f));
  const uint16_t sign = static_cast<uint16_t>((f >> 16) & 0x8000u);
  const uint32_t a = f & 0x7FFFFFFFu;
  if (a > 0x7F800000u) return static_cast<uint16_t>(sign | 0x7E00u);
  if (a >= 0x47800000u) return static_cast<uint16_t>(sign | 0x7C00u);
  if (a >= 0x38800000u) {
    const uint32_t mant = a & 0x7FFFFFu;
    const uint32_t e = (a >> 23) - 112u;
    uint32_t half = (e << 10) | (mant >> 13);
    const uint32_t rest = mant & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (half & 1u))) ++half;
    return static_cast<uint16_t>(sign | half);
  }
  if (a <= 0x33000000u) return sign;
  const uint32_t mant = (a & 0x7FFFFFu) | 0x800000u;
  const uint32_t shift = 126u - (a >> 23);
  uint32_t half = mant >> shift;
  const uint32_t rest = mant & ((1u << shift) - 1u);
  const uint32_t halfway = 1u << (shift - 1u);
  if (rest > halfway || (rest == halfway && (half & 1u))) ++half;
  return static_cast<uint16_t>(sign | half);
}

void oracle_convert_to_f32(int32_t dtype, const void* src, int64_t n, int64_t dim, float* out) {
  const int64_t cells = n * dim;
  if (dtype == 0) {
    std::memcpy(out, src, static_cast<size_t>(cells) * sizeof(float));
  } else if (dtype == 1) {
    const auto* h = static_cast<const uint16_t*>(src);
    for (int64_t i = 0; i < cells; ++i) out[i] = oracle_f16_to_f32(h[i]);
  } else if (dtype == 2) {
    const auto* p = static_cast<const int8_t*>(src);
    for (int64_t i = 0; i < cells; ++i) out[i] = static_cast<float>(p[i]);
  } else {
    const auto* p = static_cast<const uint8_t*>(src);
    for (int64_t i = 0; i < cells; ++i) out[i] = static_cast<float>(p[i]);
  }
}

void oracle_pairwise(int32_t metric, const float* x, int64_t nx, const float* y, int64_t ny,
                     int64_t dim, float* out, float metric_arg) {
  std::vector<float> ynorm(static_cast<size_t>(ny));
  for (int64_t j = 0; j < ny; ++j) ynorm[static_cast<size_t>(j)] = nrm2sq_seq(y + j * dim, dim);
  pairwise_block(metric, x, nx, y, ny, dim, ynorm.data(), out, metric_arg);
}

void oracle_topk(const float* scores, int64_t rows, int64_t cols, int64_t k, int64_t* indices,
                 float* values, int32_t largest) {
  topk_rows(scores, rows, cols, k, indices, values, largest != 0);
}

namespace {

/* Few queries against many rows: each thread takes a contiguous row shard, selects every query's
   top min(k, shard rows) there with the reference's arithmetic and total order (cpu_prims.cpp:
   24-32), and the shard lists are merged by the same order on (value, global id). Every score
   depends only on its (query, row) pair and the order is strict, so the result equals the
   unsharded brute_search_impl (mixer.cpp:843-864) bit for bit. */
void brute_search_row_sharded(const float* data, int64_t n, int64_t dim, int32_t metric,
                              const float* queries, int64_t nq, int64_t k, const uint8_t* bitset,
                              int64_t* neighbors, float* distances, int32_t nthreads) {
  const int64_t shards = std::max<int64_t>(1, std::min<int64_t>(nthreads, n / 16384));
  const int64_t k_eff = std::min(k, n);
  const float inf = std::numeric_limits<float>::infinity();
  std::vector<std::vector<int64_t>> sid(static_cast<size_t>(shards));
  std::vector<std::vector<float>> sval(static_cast<size_t>(shards));
  std::vector<int64_t> lo(static_cast<size_t>(shards) + 1);
  for (int64_t t = 0; t <= shards; ++t) lo[static_cast<size_t>(t)] = n * t / shards;
  parallel_for(shards, static_cast<int32_t>(shards), [&](int64_t t0, int64_t t1) {
    for (int64_t t = t0; t < t1; ++t) {
      const int64_t b = lo[static_cast<size_t>(t)], rows = lo[static_cast<size_t>(t) + 1] - b;
      const int64_t ks = std::min(k, rows);
      std::vector<float> ynorm(static_cast<size_t>(rows));
      for (int64_t j = 0; j < rows; ++j)
        ynorm[static_cast<size_t>(j)] = nrm2sq_seq(data + (b + j) * dim, dim);
      auto& ids = sid[static_cast<size_t>(t)];
      auto& vals = sval[static_cast<size_t>(t)];
      ids.resize(static_cast<size_t>(nq * ks));
      vals.resize(static_cast<size_t>(nq * ks));
      const int64_t block = 16;
      std::vector<float> scores(static_cast<size_t>(block * rows));
      for (int64_t q0 = 0; q0 < nq; q0 += block) {
        const int64_t m = std::min(block, nq - q0);
        pairwise_block(metric, queries + q0 * dim, m, data + b * dim, rows, dim, ynorm.data(),
                       scores.data(), 2.f);
        if (bitset) {
          for (int64_t i = 0; i < m; ++i)
            for (int64_t j = 0; j < rows; ++j) {
              const int64_t g = b + j;
              if (!((bitset[g >> 3] >> (g & 7)) & 1u)) scores[static_cast<size_t>(i * rows + j)] = inf;
            }
        }
        topk_rows(scores.data(), m, rows, k, ids.data() + q0 * ks, vals.data() + q0 * ks, false);
      }
      for (auto& v : ids) v += b;
    }
  });
  parallel_for(nq, nthreads, [&](int64_t q0, int64_t q1) {
    std::vector<std::pair<float, int64_t>> all;
    for (int64_t q = q0; q < q1; ++q) {
      all.clear();
      for (int64_t t = 0; t < shards; ++t) {
        const int64_t rows = lo[static_cast<size_t>(t) + 1] - lo[static_cast<size_t>(t)];
        const int64_t ks = std::min(k, rows);
        for (int64_t i = 0; i < ks; ++i)
          all.emplace_back(sval[static_cast<size_t>(t)][static_cast<size_t>(q * ks + i)],
                           sid[static_cast<size_t>(t)][static_cast<size_t>(q * ks + i)]);
      }
      std::partial_sort(all.begin(), all.begin() + k_eff, all.end(),
                        [](const std::pair<float, int64_t>& x, const std::pair<float, int64_t>& y) {
                          return before(x.first, x.second, y.first, y.second, false);
                        });
      for (int64_t i = 0; i < k_eff; ++i) {
        neighbors[q * k_eff + i] = all[static_cast<size_t>(i)].second;
        distances[q * k_eff + i] = all[static_cast<size_t>(i)].first;
      }
    }
  });
}

}  // namespace

void oracle_brute_search(const float* data, int64_t n, int64_t dim, int32_t metric,
                         const float* queries, int64_t nq, int64_t k, const uint8_t* bitset,
                         int64_t* neighbors, float* distances, int32_t nthreads) {
  if (nthreads > 1 && nq < 4 * static_cast<int64_t>(nthreads) && n >= 2 * 16384) {
    brute_search_row_sharded(data, n, dim, metric, queries, nq, k, bitset, neighbors, distances,
                             nthreads);
    /* mixer.cpp:860-862: negation covers nq*k entries (k as requested, not min(k, n)). */
    if (metric == kIP)
      for (int64_t i = 0; i < nq * k; ++i) distances[i] = -distances[i];
    return;
  }
  std::vector<float> ynorm(static_cast<size_t>(n));
  for (int64_t j = 0; j < n; ++j) ynorm[static_cast<size_t>(j)] = nrm2sq_seq(data + j * dim, dim);
  const int64_t k_eff = std::min(k, n);
  const float inf = std::numeric_limits<float>::infinity();
  parallel_for(nq, nthreads, [&](int64_t q0, int64_t q1) {
    const int64_t block = 16;
    std::vector<float> scores(static_cast<size_t>(block * n));
    for (int64_t b = q0; b < q1; b += block) {
      const int64_t m = std::min(block, q1 - b);
      /* metric_arg 2.f: mixer.cpp:847 */
      pairwise_block(metric, queries + b * dim, m, data, n, dim, ynorm.data(), scores.data(), 2.f);
      if (bitset) {
        /* mixer.cpp:849-857 + internal.hpp:274-277 (LSB-first) */
        for (int64_t i = 0; i < m; ++i)
          for (int64_t j = 0; j < n; ++j)
            if (!((bitset[j >> 3] >> (j & 7)) & 1u)) scores[static_cast<size_t>(i * n + j)] = inf;
      }
      topk_rows(scores.data(), m, n, k, neighbors + b * k_eff, distances + b * k_eff, false);
    }
  });
  /* mixer.cpp:860-862: negation covers nq*k entries (k as requested, not min(k, n)). */
  if (metric == kIP)
    for (int64_t i = 0; i < nq * k; ++i) distances[i] = -distances[i];
}

void oracle_gemm(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                 int32_t trans_b, int32_t round_f16) {
  /* cpu_prims.cpp:48-58 naive loop; round_f16 rounds each operand to half (RNE) first. */
  auto op = [round_f16](float v) {
    return round_f16 ? oracle_f16_to_f32(oracle_f32_to_f16_rne(v)) : v;
  };
  for (int64_t i = 0; i < m; ++i) {
    for (int64_t j = 0; j < n; ++j) {
      float s = 0.f;
      for (int64_t t = 0; t < k; ++t)
        s += op(a[i * k + t]) * op(trans_b ? b[j * k + t] : b[t * n + j]);
      c[i * n + j] = s;
    }
  }
}

void oracle_gather_rows(const float* src, int64_t src_rows, int64_t dim, const int64_t* idx,
                        int64_t nidx, float* out) {
  /* cpu_prims.cpp:108-118 */
  for (int64_t i = 0; i < nidx; ++i) {
    const int64_t r = idx[i];
    for (int64_t d = 0; d < dim; ++d)
      out[i * dim + d] = (r >= 0 && r < src_rows) ? src[r * dim + d] : 0.f;
  }
}

void oracle_all_neighbors(const float* data, int64_t n, int64_t dim, int32_t metric, int32_t k,
                          int64_t* neighbors, float* distances, int32_t nthreads) {
  /* graphs.cpp:3384-3396: pairwise (metric_arg 2), diagonal +inf, k = min(k, n - 1) smallest. */
  std::vector<float> ynorm(static_cast<size_t>(n));
  for (int64_t j = 0; j < n; ++j) ynorm[static_cast<size_t>(j)] = nrm2sq_seq(data + j * dim, dim);
  const int64_t ke = std::min<int64_t>(k, n - 1);
  const float inf = std::numeric_limits<float>::infinity();
  parallel_for(n, nthreads, [&](int64_t q0, int64_t q1) {
    std::vector<float> scores(static_cast<size_t>(n));
    for (int64_t i = q0; i < q1; ++i) {
      pairwise_block(metric, data + i * dim, 1, data, n, dim, ynorm.data(), scores.data(), 2.f);
      scores[static_cast<size_t>(i)] = inf;
      topk_rows(scores.data(), 1, n, ke, neighbors + i * ke, distances + i * ke, false);
    }
  });
  if (metric == kIP)
    for (int64_t i = 0; i < n * ke; ++i) distances[i] = -distances[i];
}

int32_t oracle_kmeans_init_rows(int64_t n, int32_t k, int64_t* rows) {
  /* mixer.cpp:879-890: std::mt19937(42), uniform_int_distribution<int64_t>(0, n-1), up to 8
     redraws when the row was already used. */
  if (n <= 0 || k <= 0) return -1;
  k = std::max(1, std::min(k, static_cast<int32_t>(std::min<int64_t>(n, INT32_MAX))));
  std::mt19937 rng(42u);
  std::uniform_int_distribution<int64_t> pick(0, n - 1);
  std::vector<int64_t> used;
  for (int32_t c = 0; c < k; ++c) {
    int64_t i = pick(rng);
    for (int t = 0; t < 8 && std::find(used.begin(), used.end(), i) != used.end(); ++t)
      i = pick(rng);
    used.push_back(i);
    rows[c] = i;
  }
  return k;
}

void oracle_kmeans_predict(const float* centroids, int32_t k, int64_t dim, const float* x,
                           int64_t n, int64_t* labels, float* distances, int32_t nthreads) {
  /* cluster.cpp:59-69: prim_pairwise(L2_EXPANDED) then prim_topk(k=1). */
  std::vector<float> cnorm(static_cast<size_t>(k));
  for (int32_t c = 0; c < k; ++c) cnorm[static_cast<size_t>(c)] = nrm2sq_seq(centroids + c * dim, dim);
  parallel_for(n, nthreads, [&](int64_t b, int64_t e) {
    std::vector<float> row(static_cast<size_t>(k));
    for (int64_t i = b; i < e; ++i) {
      pairwise_block(kL2, x + i * dim, 1, centroids, k, dim, cnorm.data(), row.data(), 2.f);
      int64_t li;
      float lv;
      topk_rows(row.data(), 1, k, 1, &li, &lv, false);
      labels[i] = li;
      if (distances) distances[i] = lv;
    }
  });
}

void oracle_kmeans_step(const float* x, int64_t n, int64_t dim, int32_t k, float* centroids,
                        int64_t* labels_out, float* dist_out, int32_t nthreads) {
  std::vector<int64_t> labels(static_cast<size_t>(n));
  std::vector<float> dist(static_cast<size_t>(n));
  oracle_kmeans_predict(centroids, k, dim, x, n, labels.data(), dist.data(), nthreads);
  /* mixer.cpp:902-918: serial fp32 sums in row order; centroid = sum * (1/cnt); empty clusters
     keep the previous centroid. */
  std::vector<float> sum(static_cast<size_t>(k) * static_cast<size_t>(dim), 0.f);
  std::vector<int32_t> cnt(static_cast<size_t>(k), 0);
  for (int64_t i = 0; i < n; ++i) {
    const int64_t c = labels[static_cast<size_t>(i)];
    if (c < 0 || c >= k) continue;
    ++cnt[static_cast<size_t>(c)];
    float* dst = sum.data() + c * dim;
    const float* src = x + i * dim;
    for (int64_t d = 0; d < dim; ++d) dst[d] += src[d];
  }
  for (int32_t c = 0; c < k; ++c) {
    if (cnt[static_cast<size_t>(c)] == 0) continue;
    float* dst = centroids + static_cast<size_t>(c) * dim;
    const float* src = sum.data() + static_cast<size_t>(c) * dim;
    const float inv = 1.f / static_cast<float>(cnt[static_cast<size_t>(c)]);
    for (int64_t d = 0; d < dim; ++d) dst[d] = src[d] * inv;
  }
  if (labels_out) std::memcpy(labels_out, labels.data(), static_cast<size_t>(n) * sizeof(int64_t));
  if (dist_out) std::memcpy(dist_out, dist.data(), static_cast<size_t>(n) * sizeof(float));
}

int32_t oracle_kmeans_fit(const float* x, int64_t n, int64_t dim, int32_t k, int32_t iters,
                          float* centroids, int32_t nthreads) {
  /* mixer.cpp:868-871 validation. */
  if (!x || n <= 0 || dim <= 0 || k <= 0 || iters < 0 || n > INT32_MAX) return -1;
  std::vector<int64_t> rows(static_cast<size_t>(k));
  const int32_t keff = oracle_kmeans_init_rows(n, k, rows.data());
  for (int32_t c = 0; c < keff; ++c)
    std::memcpy(centroids + static_cast<size_t>(c) * dim, x + rows[static_cast<size_t>(c)] * dim,
                static_cast<size_t>(dim) * sizeof(float));
  for (int32_t it = 0; it < iters; ++it)
    oracle_kmeans_step(x, n, dim, keff, centroids, nullptr, nullptr, nthreads);
  return keff;
}

int32_t oracle_bitset_from_allow_list(int64_t n, const int64_t* ids, int64_t nids,
                                      uint8_t* bitset) {
  if (!bitset || n <= 0 || nids < 0) return 2;
  const int64_t nbytes = (n + 7) / 8;
  std::memset(bitset, 0, static_cast<size_t>(nbytes));
  if (!ids || nids == 0) return 0;
  for (int64_t i = 0; i < nids; ++i) {
    const int64_t id = ids[i];
    if (id < 0 || id >= n) continue;
    bitset[id >> 3] = static_cast<uint8_t>(bitset[id >> 3] | (1u << (id & 7)));
  }
  return 0;
}

/* indexes.cpp:281-300 ovvsIvfFlatBuild + build_ivf_lists (indexes.cpp:50-57). */
int32_t oracle_ivf_flat_build(const float* x, int64_t n, int64_t dim, int32_t nlist,
                              float* centroids, int64_t* list_sizes, int64_t* list_ids,
                              int32_t nthreads) {
  if (!x || n <= 0 || dim <= 0 || nlist <= 0) return -1;
  nlist = static_cast<int32_t>(std::min<int64_t>(nlist, n));
  const int32_t keff = oracle_kmeans_fit(x, n, dim, nlist, 12, centroids, nthreads);
  if (keff < 0) return -1;
  std::vector<int64_t> labels(static_cast<size_t>(n));
  oracle_kmeans_predict(centroids, keff, dim, x, n, labels.data(), nullptr, nthreads);
  std::vector<std::vector<int64_t>> lists(static_cast<size_t>(keff));
  for (int64_t i = 0; i < n; ++i) {
    const int64_t a = labels[static_cast<size_t>(i)];
    if (a >= 0 && a < keff) lists[static_cast<size_t>(a)].push_back(i);
  }
  int64_t at = 0;
  for (int32_t c = 0; c < keff; ++c) {
    list_sizes[c] = static_cast<int64_t>(lists[static_cast<size_t>(c)].size());
    for (int64_t id : lists[static_cast<size_t>(c)]) list_ids[at++] = id;
  }
  return keff;
}

/* indexes.cpp:302-358 ovvsIvfFlatSearch over an index given by its parts (the dataset in row
   order, centroids, and the lists concatenated with their sizes). Filtered rows score +inf; a
   list id outside [0, n) is gathered as a zero row (cpu_gather_rows) and counts as filtered when
   a bitset is given (the reference would read past the bitset). */
void oracle_ivf_flat_search(const float* x, int64_t n, int64_t dim, int32_t metric,
                            const float* centroids, int32_t nlist, const int64_t* list_sizes,
                            const int64_t* list_ids, const float* queries, int64_t nq, int64_t k,
                            int32_t nprobe, const uint8_t* bitset, int64_t* neighbors,
                            float* distances, int32_t nthreads) {
  const float inf = std::numeric_limits<float>::infinity();
  std::vector<int64_t> off(static_cast<size_t>(nlist) + 1, 0);
  for (int32_t c = 0; c < nlist; ++c) off[c + 1] = off[c] + list_sizes[c];
  std::vector<float> cnorm(static_cast<size_t>(nlist));
  for (int32_t c = 0; c < nlist; ++c) cnorm[static_cast<size_t>(c)] = nrm2sq_seq(centroids + c * dim, dim);
  nprobe = std::max(1, std::min(nprobe, nlist));
  parallel_for(nq, nthreads, [&](int64_t q0, int64_t q1) {
    std::vector<float> cs(static_cast<size_t>(nlist));
    std::vector<int64_t> cl(static_cast<size_t>(nprobe));
    std::vector<float> cd(static_cast<size_t>(nprobe));
    for (int64_t q = q0; q < q1; ++q) {
      const float* qr = queries + q * dim;
      std::vector<int64_t> ids;
      if (nlist > 0) {
        pairwise_block(kL2, qr, 1, centroids, nlist, dim, cnorm.data(), cs.data(), 2.f);
        topk_rows(cs.data(), 1, nlist, nprobe, cl.data(), cd.data(), false);
        for (int32_t p = 0; p < nprobe; ++p) {
          const int64_t c = cl[static_cast<size_t>(p)];
          if (c < 0 || c >= nlist) continue;
          ids.insert(ids.end(), list_ids + off[c], list_ids + off[c + 1]);
        }
      }
      if (ids.empty()) {
        for (int64_t t = 0; t < k; ++t) {
          neighbors[q * k + t] = -1;
          distances[q * k + t] = inf;
        }
        continue;
      }
      const int64_t m = static_cast<int64_t>(ids.size());
      std::vector<float> g(static_cast<size_t>(m * dim));
      oracle_gather_rows(x, n, dim, ids.data(), m, g.data());
      std::vector<float> gn(static_cast<size_t>(m));
      for (int64_t j = 0; j < m; ++j) gn[static_cast<size_t>(j)] = nrm2sq_seq(g.data() + j * dim, dim);
      std::vector<float> sc(static_cast<size_t>(m));
      pairwise_block(metric, qr, 1, g.data(), m, dim, gn.data(), sc.data(), 2.f);
      if (bitset) {
        for (int64_t j = 0; j < m; ++j) {
          const int64_t id = ids[static_cast<size_t>(j)];
          const bool ok = id >= 0 && id < n && ((bitset[id >> 3] >> (id & 7)) & 1);
          if (!ok) sc[static_cast<size_t>(j)] = inf;
        }
      }
      const int64_t kk = std::min(k, m);
      std::vector<int64_t> ti(static_cast<size_t>(kk));
      std::vector<float> tv(static_cast<size_t>(kk));
      topk_rows(sc.data(), 1, m, kk, ti.data(), tv.data(), false);
      for (int64_t t = 0; t < k; ++t) {
        if (t < kk) {
          neighbors[q * k + t] = ids[static_cast<size_t>(ti[static_cast<size_t>(t)])];
          float d = tv[static_cast<size_t>(t)];
          if (metric == kIP) d = -d;
          distances[q * k + t] = d;
        } else {
          neighbors[q * k + t] = -1;
          distances[q * k + t] = inf;
        }
      }
    }
  });
}

}  // extern "C"

