#pragma once

/* C++ RAII wrappers over the ovvs C ABI for the brute-force / k-means surface.
 *
 * Same class names and member signatures as the reference's include/ovvs/ovvs.hpp
 * (Resources, BruteForceIndex, KMeans, Batcher, bitset_from_allow_list), so C++ consumers of
 * those classes compile unchanged. Failures throw std::runtime_error with the status text. */

#include "ovvs.h"

#include <stdexcept>
#include <string>

namespace ovvs {

inline void check(ovvsStatus s) {
  if (s != OVVS_STATUS_SUCCESS) throw std::runtime_error(ovvsStatusString(s));
}

class Resources {
 public:
  Resources() { check(ovvsResourcesCreate(&res_)); }
  ~Resources() {
    if (res_) ovvsResourcesDestroy(res_);
  }
  Resources(const Resources&) = delete;
  Resources& operator=(const Resources&) = delete;
  ovvsResources_t get() const { return res_; }
  void set_policy(ovvsPolicy p) { check(ovvsResourcesSetPolicy(res_, p)); }
  ovvsDevice last_device() const {
    ovvsDevice d = OVVS_DEVICE_CPU;
    check(ovvsResourcesLastDevice(res_, &d));
    return d;
  }
  ovvsDType last_compute_dtype() const {
    ovvsDType t = OVVS_DTYPE_F32;
    check(ovvsResourcesLastComputeDtype(res_, &t));
    return t;
  }
  ovvsCagraBuildStatsV1 cagra_build_stats() const {
    ovvsCagraBuildStatsV1 stats{};
    check(ovvsResourcesCagraBuildStatsV1(res_, &stats));
    return stats;
  }

 private:
  ovvsResources_t res_ = nullptr;
};

class BruteForceIndex {
 public:
  BruteForceIndex(Resources& res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric)
      : res_(&res) {
    check(ovvsBruteForceBuild(res.get(), dataset, n, dim, metric, &ix_));
  }
  BruteForceIndex(Resources& res, const void* dataset, int64_t n, int64_t dim, ovvsMetric metric,
                  ovvsDType dtype)
      : res_(&res) {
    check(ovvsBruteForceBuildTyped(res.get(), dataset, n, dim, metric, dtype, &ix_));
  }
  ~BruteForceIndex() {
    if (ix_) ovvsBruteForceDestroy(ix_);
  }
  BruteForceIndex(const BruteForceIndex&) = delete;
  BruteForceIndex& operator=(const BruteForceIndex&) = delete;

  void search(const float* queries, int64_t nq, int64_t k, int64_t* neighbors, float* distances,
              const uint8_t* bitset = nullptr) {
    check(ovvsBruteForceSearch(res_->get(), ix_, queries, nq, k, bitset, neighbors, distances));
  }
  ovvsBruteForceIndex_t get() const { return ix_; }

 private:
  Resources* res_ = nullptr;
  ovvsBruteForceIndex_t ix_ = nullptr;
};

class KMeans {
 public:
  KMeans(Resources& res, const float* dataset, int64_t n, int64_t dim, int32_t nclusters,
         int32_t iters)
      : res_(&res) {
    check(ovvsKMeansFit(res.get(), dataset, n, dim, nclusters, iters, &m_));
  }
  ~KMeans() {
    if (m_) ovvsKMeansDestroy(m_);
  }
  KMeans(const KMeans&) = delete;
  KMeans& operator=(const KMeans&) = delete;
  void predict(const float* x, int64_t n, int64_t* labels, float* distances) {
    check(ovvsKMeansPredict(res_->get(), m_, x, n, labels, distances));
  }
  /* Borrowed pointer valid until this object is destroyed. */
  const float* centroids(int32_t* nclusters, int64_t* dim) const {
    const float* p = nullptr;
    check(ovvsKMeansCentroids(m_, &p, nclusters, dim));
    return p;
  }

 private:
  Resources* res_ = nullptr;
  ovvsKMeansModel_t m_ = nullptr;
};

class Batcher {
 public:
  Batcher(Resources& res, BruteForceIndex& index, int32_t max_batch, int32_t max_wait_ms) {
    check(ovvsBatcherCreate(res.get(), index.get(), max_batch, max_wait_ms, &b_));
  }
  ~Batcher() {
    if (b_) ovvsBatcherDestroy(b_);
  }
  Batcher(const Batcher&) = delete;
  Batcher& operator=(const Batcher&) = delete;
  void search(const float* queries, int64_t nq, int64_t k, int64_t* neighbors, float* distances) {
    check(ovvsBatcherSearch(b_, queries, nq, k, neighbors, distances));
  }

 private:
  ovvsBatcher_t b_ = nullptr;
};

inline void bitset_from_allow_list(int64_t n, const int64_t* ids, int64_t nids, uint8_t* bitset) {
  check(ovvsBitsetFromAllowList(n, ids, nids, bitset));
}

}  // namespace ovvs
