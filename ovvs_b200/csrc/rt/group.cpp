// One Resources over several GPUs of one process (see group.hpp).
#include "group.hpp"

#include <algorithm>
#include <cstring>
#include <memory>
#include <set>

#include "../cluster/kmeans.hpp"
#include "../neighbors/brute_force.hpp"
#include "../prim/prep.cuh"

namespace ovvs {
namespace rt {

namespace {

// Below this many rows per device a dataset stays whole on the primary device: shards of a few
// tiles would spend more on the exchange than they save.
constexpr int64_t kMinShardRows = 4096;

size_t elem_bytes(int dtype) {
  if (dtype == 0) return 4;  // F32
  if (dtype == 1) return 2;  // F16
  return 1;                  // I8, U8 and the byte-read F8/F4 types
}

}  // namespace

Workers::Workers(int n) : results_(static_cast<size_t>(n), OVVS_STATUS_SUCCESS) {
  for (int g = 0; g < n; ++g) threads_.emplace_back([this, g] { loop(g); });
}

Workers::~Workers() {
  {
    std::lock_guard<std::mutex> lk(mu_);
    stop_ = true;
  }
  start_cv_.notify_all();
  for (auto& t : threads_) t.join();
}

void Workers::loop(int g) {
  uint64_t seen = 0;
  for (;;) {
    const std::function<ovvsStatus(int)>* job = nullptr;
    {
      std::unique_lock<std::mutex> lk(mu_);
      start_cv_.wait(lk, [&] { return stop_ || generation_ != seen; });
      if (stop_) return;
      seen = generation_;
      job = job_;
    }
    ovvsStatus st = OVVS_STATUS_ERROR;
    try {
      st = (*job)(g);
    } catch (...) {
      st = OVVS_STATUS_ERROR;
    }
    std::lock_guard<std::mutex> lk(mu_);
    results_[static_cast<size_t>(g)] = st;
    if (--pending_ == 0) done_cv_.notify_all();
  }
}

ovvsStatus Workers::run(const std::function<ovvsStatus(int)>& fn) {
  std::unique_lock<std::mutex> lk(mu_);
  job_ = &fn;
  pending_ = static_cast<int>(threads_.size());
  ++generation_;
  start_cv_.notify_all();
  done_cv_.wait(lk, [&] { return pending_ == 0; });
  job_ = nullptr;
  for (ovvsStatus st : results_)
    if (st != OVVS_STATUS_SUCCESS) return st;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus create_group(Resources& r, const std::vector<int>& devices) {
  const int G = static_cast<int>(devices.size());
  if (G < 2 || std::set<int>(devices.begin(), devices.end()).size() != devices.size())
    return OVVS_STATUS_INVALID_ARGUMENT;
  const NcclApi* nc = nccl();
  if (!nc) return OVVS_STATUS_DEVICE_UNAVAILABLE;
  for (int g = 0; g < G; ++g) {
    auto m = std::make_unique<Resources>();
    probe_device(*m, devices[static_cast<size_t>(g)]);
    if (!m->gpu_available) return OVVS_STATUS_DEVICE_UNAVAILABLE;
    m->rank = g;
    m->world = G;
    m->nccl_timeout_ms = r.nccl_timeout_ms;
    r.group.push_back(std::move(m));
  }
  ncclUniqueId id;
  OVVS_TRY(status_of(nc->GetUniqueId(&id)));
  r.workers = std::make_unique<Workers>(G);
  // Every rank initialises its communicator on its own thread (non-blocking, bounded).
  return r.workers->run([&](int g) {
    Resources& m = *r.group[static_cast<size_t>(g)];
    OVVS_TRY(m.activate());
    return init_comm(m, id);
  });
}

ovvsStatus group_build(Resources& r, nb::BruteIndex& top, const void* data, int dtype, int64_t n,
                       int64_t dim, int metric_raw) {
  const int G = static_cast<int>(r.group.size());
  top.device = r.device;
  top.n = n;
  top.n_total = n;
  top.row_offset = 0;
  top.sharded = false;
  top.dim = dim;
  top.metric_raw = metric_raw;
  top.metric = prim::normalize_metric(metric_raw);
  top.dtype = dtype;
  top.shards.clear();
  if (n < kMinShardRows * G) {  // small: whole on the primary device
    top.shards.push_back(std::make_unique<nb::BruteIndex>());
    OVVS_TRY(r.activate());
    return nb::build_from_host(r, *top.shards[0], data, dtype, n, dim, metric_raw, 0, false);
  }
  for (int g = 0; g < G; ++g) top.shards.push_back(std::make_unique<nb::BruteIndex>());
  const size_t row_bytes = static_cast<size_t>(dim) * elem_bytes(dtype);
  return r.workers->run([&](int g) {
    Resources& m = *r.group[static_cast<size_t>(g)];
    OVVS_TRY(m.activate());
    int64_t lo = 0, hi = 0;
    shard_rows(n, g, G, &lo, &hi);
    // collective: the shards' row counts are all-reduced into n_total
    return nb::build_from_host(m, *top.shards[static_cast<size_t>(g)],
                               static_cast<const char*>(data) + lo * row_bytes, dtype, hi - lo,
                               dim, metric_raw, lo, true);
  });
}

ovvsStatus group_search(Resources& r, const nb::BruteIndex& top, const float* queries, int64_t nq,
                        int64_t k, const uint8_t* bitset, int64_t* neighbors, float* distances,
                        int64_t* k_eff_out) {
  if (top.shards.size() == 1) {
    OVVS_TRY(r.activate());
    return nb::search_from_host(r, *top.shards[0], queries, nq, k, bitset, neighbors, distances,
                                k_eff_out);
  }
  if (top.shards.size() != r.group.size()) return OVVS_STATUS_INVALID_ARGUMENT;
  // Every rank searches all queries against its shard; the exchange leaves the merged result on
  // every rank, and rank 0 copies it out.
  return r.workers->run([&](int g) {
    Resources& m = *r.group[static_cast<size_t>(g)];
    OVVS_TRY(m.activate());
    int64_t ke = 0;
    const ovvsStatus st = nb::search_from_host(m, *top.shards[static_cast<size_t>(g)], queries, nq,
                                               k, bitset, g == 0 ? neighbors : nullptr,
                                               g == 0 ? distances : nullptr, &ke);
    if (g == 0) *k_eff_out = ke;
    return st;
  });
}

ovvsStatus group_kmeans_fit(Resources& r, const float* x, int64_t n, int64_t dim,
                            int32_t nclusters, int32_t iters, km::KMeansModel& model) {
  const int G = static_cast<int>(r.group.size());
  if (n < kMinShardRows * G) {
    OVVS_TRY(r.activate());
    return km::fit(r, x, n, 0, n, dim, nclusters, iters, model);
  }
  // Every rank fits on its shard with replicated centroids (fp64 sums all-reduced per
  // iteration), so all ranks end with the same centroids; rank 0's model is kept (it lives on the
  // primary device), the others are released.
  std::vector<std::unique_ptr<km::KMeansModel>> others(static_cast<size_t>(G));
  const ovvsStatus st = r.workers->run([&](int g) {
    Resources& m = *r.group[static_cast<size_t>(g)];
    OVVS_TRY(m.activate());
    km::KMeansModel* mm = &model;
    if (g > 0) {
      others[static_cast<size_t>(g)] = std::make_unique<km::KMeansModel>();
      mm = others[static_cast<size_t>(g)].get();
      mm->k_reported = model.k_reported;
      mm->dim = dim;
      mm->device = m.device;
    }
    int64_t lo = 0, hi = 0;
    shard_rows(n, g, G, &lo, &hi);
    return km::fit(m, x + lo * dim, hi - lo, lo, n, dim, nclusters, iters, *mm);
  });
  r.workers->run([&](int g) {  // each rank releases its own model's device memory
    others[static_cast<size_t>(g)].reset();
    return OVVS_STATUS_SUCCESS;
  });
  return st;
}

}  // namespace rt
}  // namespace ovvs
