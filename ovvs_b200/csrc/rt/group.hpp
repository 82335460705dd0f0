// One Resources over several GPUs of one process (the plain ovvs C ABI on many devices).
//
// ovvsResourcesCreate reads OVVS_CUDA_DEVICES; when it names more than one device, the Resources
// is an ordinary single-device Resources on the first one (everything off the hot path runs
// there unchanged) plus a group: one member Resources per device (rank g of G, sharing one NCCL
// communicator, non-blocking) and one persistent host thread per member. The hot-path entry
// points then shard exactly like the one-process-per-GPU deployment: ovvsBruteForceBuild* splits
// the rows into G contiguous shards, ovvsBruteForceSearch runs every shard's search and merges
// the shards' exact top-k lists after an NCCL all-gather, ovvsKMeansFit sums every shard's
// assignments in fp64 and all-reduces them each iteration. Results equal one GPU's bit for bit.
//
// The reference has one Resources per caller holding its devices and scratch
// (src/internal.hpp:459-562) and routes each operation to a single device
// (src/prim/mixer.cpp:24-45); spreading one operation over several devices is this library's.
#pragma once

#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include "runtime.hpp"

namespace ovvs {
namespace nb {
struct BruteIndex;
}
namespace km {
struct KMeansModel;
}
namespace rt {

// One host thread per group member. run(fn) calls fn(g) on thread g for every member at once and
// returns the first non-success status (an exception in fn counts as OVVS_STATUS_ERROR).
class Workers {
 public:
  explicit Workers(int n);
  ~Workers();
  Workers(const Workers&) = delete;
  Workers& operator=(const Workers&) = delete;
  ovvsStatus run(const std::function<ovvsStatus(int)>& fn);
  int size() const { return static_cast<int>(threads_.size()); }

 private:
  void loop(int g);
  std::vector<std::thread> threads_;
  std::mutex mu_;
  std::condition_variable start_cv_, done_cv_;
  const std::function<ovvsStatus(int)>* job_ = nullptr;
  uint64_t generation_ = 0;
  int pending_ = 0;
  bool stop_ = false;
  std::vector<ovvsStatus> results_;
};

// Makes r (already probed on devices[0]) the primary of a group over `devices` (two or more,
// distinct): members, workers and their communicator (bounded by r.nccl_timeout_ms).
ovvsStatus create_group(Resources& r, const std::vector<int>& devices);

// Row range of shard g of G over n rows: [n*g/G, n*(g+1)/G) (the same partition as the one-process-
// per-GPU deployment's).
inline void shard_rows(int64_t n, int g, int G, int64_t* lo, int64_t* hi) {
  *lo = n * g / G;
  *hi = n * (g + 1) / G;
}

// The group forms of the hot path (r.group non-empty). Datasets smaller than the group's minimum
// shard size stay whole on the primary device, where `top` then holds a single shard.
ovvsStatus group_build(Resources& r, nb::BruteIndex& top, const void* data, int dtype, int64_t n,
                       int64_t dim, int metric_raw);
ovvsStatus group_search(Resources& r, const nb::BruteIndex& top, const float* queries, int64_t nq,
                        int64_t k, const uint8_t* bitset, int64_t* neighbors, float* distances,
                        int64_t* k_eff_out);
ovvsStatus group_kmeans_fit(Resources& r, const float* x, int64_t n, int64_t dim,
                            int32_t nclusters, int32_t iters, km::KMeansModel& model);

}  // namespace rt
}  // namespace ovvs
