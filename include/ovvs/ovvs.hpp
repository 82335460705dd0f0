#pragma once

/* C++ RAII wrappers over the ovvs C ABI.
 *
 * Every class of the reference's C++ header (include/ovvs/ovvs.hpp: Resources, BruteForceIndex,
 * IvfFlatIndex, IvfPqIndex, IvfRabitqIndex, CagraIndex, VamanaIndex, ScannIndex, HnswIndex,
 * KMeans, Batcher, bitset_from_allow_list) with the same constructors and member signatures, so
 * C++ written against the reference compiles unchanged. Each wrapper owns one C handle; a
 * non-success status throws ovvs::Error, a std::runtime_error whose what() is the status text
 * (what the reference throws) and which also carries the status code. Indexes outside this
 * library's path (IVF-PQ, IVF-RaBitQ, CAGRA, Vamana, ScaNN, HNSW) construct through C entry points
 * that return OVVS_STATUS_UNSUPPORTED, so they throw "unsupported" at run time. */

#include "ovvs.h"

#include <stdexcept>
#include <string>
#include <utility>

namespace ovvs {

class Error : public std::runtime_error {
 public:
  explicit Error(ovvsStatus s) : std::runtime_error(ovvsStatusString(s)), status_(s) {}
  ovvsStatus status() const noexcept { return status_; }

 private:
  ovvsStatus status_;
};

inline void check(ovvsStatus s) {
  if (s != OVVS_STATUS_SUCCESS) throw Error(s);
}

namespace detail {

// Sole owner of a C handle, released with Destroy (movable, not copyable).
template <class H, ovvsStatus (*Destroy)(H)>
class Owned {
 public:
  Owned() = default;
  ~Owned() { reset(); }
  Owned(const Owned&) = delete;
  Owned& operator=(const Owned&) = delete;
  Owned(Owned&& o) noexcept : h_(std::exchange(o.h_, nullptr)) {}
  Owned& operator=(Owned&& o) noexcept {
    if (this != &o) {
      reset();
      h_ = std::exchange(o.h_, nullptr);
    }
    return *this;
  }
  H* out() { return &h_; }
  H get() const { return h_; }
  void reset() {
    if (h_) Destroy(std::exchange(h_, nullptr));
  }

 private:
  H h_ = nullptr;
};

}  // namespace detail

class Resources {
 public:
  Resources() { check(ovvsResourcesCreate(h_.out())); }
  ovvsResources_t get() const { return h_.get(); }
  void set_policy(ovvsPolicy p) { check(ovvsResourcesSetPolicy(get(), p)); }
  ovvsDevice last_device() const {
    ovvsDevice d = OVVS_DEVICE_CPU;
    check(ovvsResourcesLastDevice(get(), &d));
    return d;
  }
  ovvsDType last_compute_dtype() const {
    ovvsDType t = OVVS_DTYPE_F32;
    check(ovvsResourcesLastComputeDtype(get(), &t));
    return t;
  }
  ovvsCagraBuildStatsV1 cagra_build_stats() const {
    ovvsCagraBuildStatsV1 s{};
    check(ovvsResourcesCagraBuildStatsV1(get(), &s));
    return s;
  }

 private:
  detail::Owned<ovvsResources_t, ovvsResourcesDestroy> h_;
};

class BruteForceIndex {
 public:
  BruteForceIndex(Resources& res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric)
      : res_(&res) {
    check(ovvsBruteForceBuild(res.get(), dataset, n, dim, metric, h_.out()));
  }
  // Typed datasets (F16 / I8 / U8 ...): ovvsBruteForceBuildTyped.
  BruteForceIndex(Resources& res, const void* dataset, int64_t n, int64_t dim, ovvsMetric metric,
                  ovvsDType dtype)
      : res_(&res) {
    check(ovvsBruteForceBuildTyped(res.get(), dataset, n, dim, metric, dtype, h_.out()));
  }
  void search(const float* queries, int64_t nq, int64_t k, int64_t* neighbors, float* distances,
              const uint8_t* bitset = nullptr) {
    check(ovvsBruteForceSearch(res_->get(), h_.get(), queries, nq, k, bitset, neighbors,
                               distances));
  }
  ovvsBruteForceIndex_t get() const { return h_.get(); }

 private:
  Resources* res_;
  detail::Owned<ovvsBruteForceIndex_t, ovvsBruteForceDestroy> h_;
};

class IvfFlatIndex {
 public:
  IvfFlatIndex(Resources& res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric,
               int32_t nlist)
      : res_(&res) {
    check(ovvsIvfFlatBuild(res.get(), dataset, n, dim, metric, nlist, h_.out()));
  }
  IvfFlatIndex(Resources& res, const char* path) : res_(&res) {
    check(ovvsIvfFlatDeserialize(res.get(), path, h_.out()));
  }
  void search(const float* queries, int64_t nq, int64_t k, int32_t nprobe, int64_t* neighbors,
              float* distances, const uint8_t* bitset = nullptr) {
    check(ovvsIvfFlatSearch(res_->get(), h_.get(), queries, nq, k, nprobe, bitset, neighbors,
                            distances));
  }
  void serialize(const char* path) { check(ovvsIvfFlatSerialize(h_.get(), path)); }
  void extend(const float* extra, int64_t nextra) {
    check(ovvsIvfFlatExtend(res_->get(), h_.get(), extra, nextra));
  }

 private:
  Resources* res_;
  detail::Owned<ovvsIvfFlatIndex_t, ovvsIvfFlatDestroy> h_;
};

class IvfPqIndex {
 public:
  IvfPqIndex(Resources& res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric,
             int32_t nlist, int32_t pq_m, int32_t pq_nbits)
      : res_(&res) {
    check(ovvsIvfPqBuild(res.get(), dataset, n, dim, metric, nlist, pq_m, pq_nbits, h_.out()));
  }
  IvfPqIndex(Resources& res, const char* path) : res_(&res) {
    check(ovvsIvfPqDeserialize(res.get(), path, h_.out()));
  }
  void search(const float* queries, int64_t nq, int64_t k, int32_t nprobe, int32_t krefine,
              int64_t* neighbors, float* distances, const uint8_t* bitset = nullptr) {
    check(ovvsIvfPqSearch(res_->get(), h_.get(), queries, nq, k, nprobe, krefine, bitset,
                          neighbors, distances));
  }
  void serialize(const char* path) { check(ovvsIvfPqSerialize(h_.get(), path)); }
  void extend(const float* extra, int64_t nextra) {
    check(ovvsIvfPqExtend(res_->get(), h_.get(), extra, nextra));
  }

 private:
  Resources* res_;
  detail::Owned<ovvsIvfPqIndex_t, ovvsIvfPqDestroy> h_;
};

class IvfRabitqIndex {
 public:
  IvfRabitqIndex(Resources& res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric,
                 int32_t nlist)
      : res_(&res) {
    check(ovvsIvfRabitqBuild(res.get(), dataset, n, dim, metric, nlist, h_.out()));
  }
  IvfRabitqIndex(Resources& res, const char* path) : res_(&res) {
    check(ovvsIvfRabitqDeserialize(res.get(), path, h_.out()));
  }
  void search(const float* queries, int64_t nq, int64_t k, int32_t nprobe, int32_t krefine,
              int64_t* neighbors, float* distances, const uint8_t* bitset = nullptr) {
    check(ovvsIvfRabitqSearch(res_->get(), h_.get(), queries, nq, k, nprobe, krefine, bitset,
                              neighbors, distances));
  }
  void serialize(const char* path) { check(ovvsIvfRabitqSerialize(h_.get(), path)); }
  void extend(const float* extra, int64_t nextra) {
    check(ovvsIvfRabitqExtend(res_->get(), h_.get(), extra, nextra));
  }

 private:
  Resources* res_;
  detail::Owned<ovvsIvfRabitqIndex_t, ovvsIvfRabitqDestroy> h_;
};

class CagraIndex {
 public:
  CagraIndex(Resources& res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric,
             int32_t graph_degree, int32_t intermediate_degree)
      : res_(&res) {
    check(ovvsCagraBuild(res.get(), dataset, n, dim, metric, graph_degree, intermediate_degree,
                         h_.out()));
  }
  CagraIndex(Resources& res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric,
             int32_t graph_degree, int32_t intermediate_degree, ovvsCagraBuildAlgo algo)
      : res_(&res) {
    check(ovvsCagraBuildEx(res.get(), dataset, n, dim, metric, graph_degree,
                           intermediate_degree, algo, h_.out()));
  }
  CagraIndex(Resources& res, const char* path) : res_(&res) {
    check(ovvsCagraDeserialize(res.get(), path, h_.out()));
  }
  void search(const float* queries, int64_t nq, int64_t k, int32_t itopk, int32_t search_width,
              int64_t* neighbors, float* distances, const uint8_t* bitset = nullptr) {
    check(ovvsCagraSearch(res_->get(), h_.get(), queries, nq, k, itopk, search_width, bitset,
                          neighbors, distances));
  }
  void serialize(const char* path) { check(ovvsCagraSerialize(h_.get(), path)); }
  void extend(const float* extra, int64_t nextra) {
    check(ovvsCagraExtend(res_->get(), h_.get(), extra, nextra));
  }
  ovvsCagraIndex_t get() const { return h_.get(); }

 private:
  Resources* res_;
  detail::Owned<ovvsCagraIndex_t, ovvsCagraDestroy> h_;
};

class VamanaIndex {
 public:
  VamanaIndex(Resources& res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric,
              int32_t graph_degree, float alpha)
      : res_(&res) {
    check(ovvsVamanaBuild(res.get(), dataset, n, dim, metric, graph_degree, alpha, h_.out()));
  }
  VamanaIndex(Resources& res, const char* path) : res_(&res) {
    check(ovvsVamanaDeserialize(res.get(), path, h_.out()));
  }
  void search(const float* queries, int64_t nq, int64_t k, int32_t beam, int64_t* neighbors,
              float* distances, const uint8_t* bitset = nullptr) {
    check(ovvsVamanaSearch(res_->get(), h_.get(), queries, nq, k, beam, bitset, neighbors,
                           distances));
  }

 private:
  Resources* res_;
  detail::Owned<ovvsVamanaIndex_t, ovvsVamanaDestroy> h_;
};

class ScannIndex {
 public:
  ScannIndex(Resources& res, const float* dataset, int64_t n, int64_t dim, ovvsMetric metric,
             int32_t nlist, int32_t pq_m)
      : res_(&res) {
    check(ovvsScannBuild(res.get(), dataset, n, dim, metric, nlist, pq_m, h_.out()));
  }
  void search(const float* queries, int64_t nq, int64_t k, int32_t nprobe, int32_t krefine,
              int64_t* neighbors, float* distances) {
    check(ovvsScannSearch(res_->get(), h_.get(), queries, nq, k, nprobe, krefine, neighbors,
                          distances));
  }

 private:
  Resources* res_;
  detail::Owned<ovvsScannIndex_t, ovvsScannDestroy> h_;
};

class HnswIndex {
 public:
  HnswIndex(Resources& res, CagraIndex& cagra) : res_(&res) {
    check(ovvsHnswFromCagra(res.get(), cagra.get(), h_.out()));
  }
  void search(const float* queries, int64_t nq, int64_t k, int32_t ef, int64_t* neighbors,
              float* distances) {
    check(ovvsHnswSearch(res_->get(), h_.get(), queries, nq, k, ef, neighbors, distances));
  }
  void serialize(const char* path) { check(ovvsHnswSerialize(h_.get(), path)); }

 private:
  Resources* res_;
  detail::Owned<ovvsHnswIndex_t, ovvsHnswDestroy> h_;
};

class KMeans {
 public:
  KMeans(Resources& res, const float* dataset, int64_t n, int64_t dim, int32_t nclusters,
         int32_t iters)
      : res_(&res) {
    check(ovvsKMeansFit(res.get(), dataset, n, dim, nclusters, iters, h_.out()));
  }
  void predict(const float* x, int64_t n, int64_t* labels, float* distances) {
    check(ovvsKMeansPredict(res_->get(), h_.get(), x, n, labels, distances));
  }

 private:
  Resources* res_;
  detail::Owned<ovvsKMeansModel_t, ovvsKMeansDestroy> h_;
};

class Batcher {
 public:
  Batcher(Resources& res, BruteForceIndex& index, int32_t max_batch, int32_t max_wait_ms) {
    check(ovvsBatcherCreate(res.get(), index.get(), max_batch, max_wait_ms, h_.out()));
  }
  void search(const float* queries, int64_t nq, int64_t k, int64_t* neighbors, float* distances) {
    check(ovvsBatcherSearch(h_.get(), queries, nq, k, neighbors, distances));
  }

 private:
  detail::Owned<ovvsBatcher_t, ovvsBatcherDestroy> h_;
};

inline void bitset_from_allow_list(int64_t n, const int64_t* ids, int64_t nids, uint8_t* bitset) {
  check(ovvsBitsetFromAllowList(n, ids, nids, bitset));
}

}  // namespace ovvs
