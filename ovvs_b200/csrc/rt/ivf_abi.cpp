// The ovvs IVF-Flat entry points (reference src/neighbors/indexes.cpp:281-457) on the B200 path,
// plus the device-pointer search extension of ovvs_cuda.h. Validation follows the reference's
// entry points; where the reference would crash (negative nq or k, sizes past its own limits) the
// call returns an error status instead.
#include <cuda_runtime.h>

#include <algorithm>
#include <new>

#include "../neighbors/ivf_flat.hpp"
#include "ovvs/ovvs.h"
#include "ovvs/ovvs_cuda.h"
#include "runtime.hpp"

using ovvs::ivf::IvfFlatIndex;
using ovvs::rt::Resources;
using ovvs::rt::from_handle;

namespace {

template <class F>
ovvsStatus guarded(F&& f) {
  try {
    return f();
  } catch (const std::bad_alloc&) {
    return OVVS_STATUS_OOM;
  } catch (...) {
    return OVVS_STATUS_ERROR;
  }
}

IvfFlatIndex* as_ivf(ovvsIvfFlatIndex_t ix) { return reinterpret_cast<IvfFlatIndex*>(ix); }

bool mul_overflows(int64_t a, int64_t b, int64_t limit) { return a > 0 && b > limit / a; }

}  // namespace

extern "C" {

ovvsStatus ovvsIvfFlatBuild(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim,
                            ovvsMetric metric, int32_t nlist, ovvsIvfFlatIndex_t* index) {
  if (!res || !dataset || !index || n <= 0 || dim <= 0 || nlist <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    if (mul_overflows(n, dim, INT64_MAX / 8)) return OVVS_STATUS_SHAPE_MISMATCH;
    auto* ix = new IvfFlatIndex();
    const ovvsStatus st = ovvs::ivf::build(r, *ix, dataset, n, dim, static_cast<int>(metric), nlist);
    if (st != OVVS_STATUS_SUCCESS) {
      delete ix;
      return st;
    }
    *index = reinterpret_cast<ovvsIvfFlatIndex_t>(ix);
    r.last_device = OVVS_DEVICE_GPU;
    r.last_compute_dtype = OVVS_DTYPE_F32;
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsIvfFlatSearch(ovvsResources_t res, ovvsIvfFlatIndex_t index, const float* queries,
                             int64_t nq, int64_t k, int32_t nprobe, const uint8_t* bitset,
                             int64_t* neighbors, float* distances) {
  if (!res || !index || !queries || !neighbors || !distances) return OVVS_STATUS_INVALID_ARGUMENT;
  if (nq < 0 || k < 0) return OVVS_STATUS_INVALID_ARGUMENT;
  if (nq == 0 || k == 0) return OVVS_STATUS_SUCCESS;  // nothing to write (as the reference)
  Resources& r = *from_handle(res);
  IvfFlatIndex& ix = *as_ivf(index);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    if (ix.device != r.device) return OVVS_STATUS_INVALID_ARGUMENT;
    if (mul_overflows(nq, ix.dim, INT64_MAX / 8) || mul_overflows(nq, k, INT64_MAX / 16))
      return OVVS_STATUS_SHAPE_MISMATCH;
    float* dq = nullptr;
    OVVS_TRY(r.scratch(ovvs::rt::kWsQueries, static_cast<size_t>(nq) * ix.dim, &dq));
    OVVS_TRY_CUDA(cudaMemcpyAsync(dq, queries, static_cast<size_t>(nq) * ix.dim * sizeof(float),
                                  cudaMemcpyHostToDevice, r.stream));
    uint8_t* db = nullptr;
    if (bitset) {
      const int64_t bytes = (ix.n + 7) / 8;
      OVVS_TRY(r.scratch(ovvs::rt::kWsBitset, static_cast<size_t>(std::max<int64_t>(bytes, 1)), &db));
      if (bytes > 0)
        OVVS_TRY_CUDA(cudaMemcpyAsync(db, bitset, static_cast<size_t>(bytes),
                                      cudaMemcpyHostToDevice, r.stream));
    }
    int64_t* dn = nullptr;
    float* dd = nullptr;
    OVVS_TRY(r.scratch(ovvs::rt::kWsNeighbors, static_cast<size_t>(nq) * k, &dn));
    OVVS_TRY(r.scratch(ovvs::rt::kWsDistances, static_cast<size_t>(nq) * k, &dd));
    OVVS_TRY(ovvs::ivf::search_device(r, ix, dq, nq, k, nprobe, db, dn, dd));
    OVVS_TRY_CUDA(cudaMemcpyAsync(neighbors, dn, static_cast<size_t>(nq) * k * sizeof(int64_t),
                                  cudaMemcpyDeviceToHost, r.stream));
    OVVS_TRY_CUDA(cudaMemcpyAsync(distances, dd, static_cast<size_t>(nq) * k * sizeof(float),
                                  cudaMemcpyDeviceToHost, r.stream));
    OVVS_TRY(r.finish());
    r.last_device = OVVS_DEVICE_GPU;
    r.last_compute_dtype = OVVS_DTYPE_F32;
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsIvfFlatSearchDevice(ovvsResources_t res, ovvsIvfFlatIndex_t index,
                                   const float* d_queries, int64_t nq, int64_t k, int32_t nprobe,
                                   const uint8_t* d_bitset, int64_t* d_neighbors,
                                   float* d_distances) {
  if (!res || !index || !d_queries || !d_neighbors || !d_distances || nq <= 0 || k <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  IvfFlatIndex& ix = *as_ivf(index);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    if (ix.device != r.device) return OVVS_STATUS_INVALID_ARGUMENT;
    if (mul_overflows(nq, k, INT64_MAX / 16)) return OVVS_STATUS_SHAPE_MISMATCH;
    OVVS_TRY(ovvs::ivf::search_device(r, ix, d_queries, nq, k, nprobe, d_bitset, d_neighbors,
                                      d_distances));
    r.last_device = OVVS_DEVICE_GPU;
    r.last_compute_dtype = OVVS_DTYPE_F32;
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsIvfFlatSerialize(ovvsIvfFlatIndex_t index, const char* path) {
  if (!index || !path) return OVVS_STATUS_INVALID_ARGUMENT;
  return guarded([&] { return ovvs::ivf::serialize(*as_ivf(index), path); });
}

ovvsStatus ovvsIvfFlatDeserialize(ovvsResources_t res, const char* path,
                                  ovvsIvfFlatIndex_t* index) {
  if (!res || !path || !index) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    auto* ix = new IvfFlatIndex();
    const ovvsStatus st = ovvs::ivf::deserialize(r, path, *ix);
    if (st != OVVS_STATUS_SUCCESS) {
      delete ix;
      return st;
    }
    *index = reinterpret_cast<ovvsIvfFlatIndex_t>(ix);
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsIvfFlatExtend(ovvsResources_t res, ovvsIvfFlatIndex_t index, const float* extra,
                             int64_t nextra) {
  if (!res || !index || !extra || nextra <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  IvfFlatIndex& ix = *as_ivf(index);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    if (ix.device != r.device) return OVVS_STATUS_INVALID_ARGUMENT;
    if (mul_overflows(nextra, ix.dim, INT64_MAX / 8)) return OVVS_STATUS_SHAPE_MISMATCH;
    OVVS_TRY(ovvs::ivf::extend(r, ix, extra, nextra));
    r.last_device = OVVS_DEVICE_GPU;
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsIvfFlatDestroy(ovvsIvfFlatIndex_t index) {
  auto* ix = as_ivf(index);
  if (ix) {
    cudaSetDevice(ix->device);
    delete ix;
  }
  return OVVS_STATUS_SUCCESS;
}

}  // extern "C"
