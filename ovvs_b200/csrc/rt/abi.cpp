// The exported ovvs C ABI: validation, policy handling and host<->device staging around the
// device code. Validation order and return codes follow the reference entry points cited
// beside each function; no C++ exception crosses the boundary (allocation failures map to
// OVVS_STATUS_OOM).
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "../cluster/kmeans.hpp"
#include "../neighbors/brute_force.hpp"
#include "../prim/watchdog.cuh"
#include "group.hpp"
#include "ovvs/ovvs.h"
#include "ovvs/ovvs_cuda.h"
#include "runtime.hpp"

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

ovvs::nb::BruteIndex* as_index(ovvsBruteForceIndex_t ix) {
  return reinterpret_cast<ovvs::nb::BruteIndex*>(ix);
}

ovvs::km::KMeansModel* as_model(ovvsKMeansModel_t m) {
  return reinterpret_cast<ovvs::km::KMeansModel*>(m);
}

bool mul_overflows(int64_t a, int64_t b, int64_t limit) { return a > 0 && b > limit / a; }

// Host-buffer search through the device path (one device, or every device of a group).
ovvsStatus search_host(Resources& r, ovvs::nb::BruteIndex& ix, const float* queries, int64_t nq,
                       int64_t k, const uint8_t* bitset, int64_t* neighbors, float* distances) {
  OVVS_TRY(r.check_policy());
  OVVS_TRY(r.activate());
  if (mul_overflows(nq, ix.dim, INT64_MAX / 8) || mul_overflows(nq, k, INT64_MAX / 8))
    return OVVS_STATUS_SHAPE_MISMATCH;
  int64_t ke = 0;
  if (!ix.shards.empty()) {
    if (ix.shards.size() > 1 && r.group.size() != ix.shards.size())
      return OVVS_STATUS_INVALID_ARGUMENT;  // searched through the group that built it
    OVVS_TRY(ovvs::rt::group_search(r, ix, queries, nq, k, bitset, neighbors, distances, &ke));
  } else {
    OVVS_TRY(ovvs::nb::search_from_host(r, ix, queries, nq, k, bitset, neighbors, distances, &ke));
  }
  // mixer.cpp:860-862: for INNER_PRODUCT the reference negates nq*k entries although only
  // nq*min(k,n) were written; entries past that are caller memory it flips in place.
  if (ix.metric == OVVS_METRIC_INNER_PRODUCT && k > ke) {
    for (int64_t i = nq * ke; i < nq * k; ++i) distances[i] = -distances[i];
  }
  r.last_device = OVVS_DEVICE_GPU;
  r.last_compute_dtype = OVVS_DTYPE_F32;
  return OVVS_STATUS_SUCCESS;
}

}  // namespace

extern "C" {

// ---- version / status (reference src/rt/status.cpp:3-28) ----------------------------------

const char* ovvsGetVersion(void) { return OVVS_VERSION_STRING; }

const char* ovvsStatusString(ovvsStatus status) {
  switch (status) {
    case OVVS_STATUS_SUCCESS:
      return "success";
    case OVVS_STATUS_ERROR:
      return "error";
    case OVVS_STATUS_INVALID_ARGUMENT:
      return "invalid argument";
    case OVVS_STATUS_UNSUPPORTED:
      return "unsupported";
    case OVVS_STATUS_OOM:
      return "out of memory";
    case OVVS_STATUS_COMPILE_FAIL:
      return "compile fail";
    case OVVS_STATUS_SHAPE_MISMATCH:
      return "shape mismatch";
    case OVVS_STATUS_DEVICE_UNAVAILABLE:
      return "device unavailable";
    case OVVS_STATUS_IO:
      return "io error";
    default:
      return "unknown";
  }
}

// ---- Resources (reference src/rt/resources.cpp:14-94) ------------------------------------

// One device (OVVS_CUDA_DEVICE, else 0), or, when OVVS_CUDA_DEVICES names several, a group over
// them: the hot path then shards over every listed device (group.hpp).
ovvsStatus ovvsResourcesCreate(ovvsResources_t* res) {
  if (!res) return OVVS_STATUS_INVALID_ARGUMENT;
  auto* r = new (std::nothrow) Resources();
  if (!r) return OVVS_STATUS_OOM;
  const ovvsStatus st = guarded([&] {
    const std::vector<int> devices = ovvs::rt::default_devices();
    ovvs::rt::probe_device(*r, devices[0]);
    r->nccl_timeout_ms = ovvs::rt::nccl_timeout_ms_default();
    if (devices.size() > 1 && r->gpu_available) {
      OVVS_TRY(r->activate());
      OVVS_TRY(ovvs::rt::create_group(*r, devices));
    }
    return OVVS_STATUS_SUCCESS;
  });
  if (st != OVVS_STATUS_SUCCESS) {
    delete r;
    return st;
  }
  *res = ovvs::rt::to_handle(r);
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesDestroy(ovvsResources_t res) {
  delete from_handle(res);
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesSetPolicy(ovvsResources_t res, ovvsPolicy policy) {
  if (!res) return OVVS_STATUS_INVALID_ARGUMENT;
  from_handle(res)->policy = policy;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesGetPolicy(ovvsResources_t res, ovvsPolicy* policy) {
  if (!res || !policy) return OVVS_STATUS_INVALID_ARGUMENT;
  *policy = from_handle(res)->policy;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesNpuAvailable(ovvsResources_t res, int32_t* available) {
  if (!res || !available) return OVVS_STATUS_INVALID_ARGUMENT;
  *available = 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesGpuAvailable(ovvsResources_t res, int32_t* available) {
  if (!res || !available) return OVVS_STATUS_INVALID_ARGUMENT;
  *available = from_handle(res)->gpu_available ? 1 : 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesSku(ovvsResources_t res, char* buf, int32_t len) {
  if (!res || !buf || len <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  std::snprintf(buf, static_cast<size_t>(len), "%s", from_handle(res)->device_name.c_str());
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesNpuCompileFails(ovvsResources_t res, int32_t* count) {
  if (!res || !count) return OVVS_STATUS_INVALID_ARGUMENT;
  *count = 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesNpuFallbacks(ovvsResources_t res, int32_t* count) {
  if (!res || !count) return OVVS_STATUS_INVALID_ARGUMENT;
  *count = 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesLastDevice(ovvsResources_t res, ovvsDevice* device) {
  if (!res || !device) return OVVS_STATUS_INVALID_ARGUMENT;
  *device = from_handle(res)->last_device;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesLastComputeDtype(ovvsResources_t res, ovvsDType* dtype) {
  if (!res || !dtype) return OVVS_STATUS_INVALID_ARGUMENT;
  *dtype = from_handle(res)->last_compute_dtype;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesSetCagraWalkCounters(ovvsResources_t res, int32_t enable) {
  if (!res) return OVVS_STATUS_INVALID_ARGUMENT;
  from_handle(res)->cagra_walk_counters = enable != 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesCagraWalkCounters(ovvsResources_t res, int64_t* out, int32_t count) {
  if (!res || !out || count < 0 || count > OVVS_CAGRA_WALK_COUNTER_COUNT)
    return OVVS_STATUS_INVALID_ARGUMENT;
  for (int32_t i = 0; i < count; ++i) out[i] = 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesResetCagraWalkCounters(ovvsResources_t res) {
  return res ? OVVS_STATUS_SUCCESS : OVVS_STATUS_INVALID_ARGUMENT;
}

ovvsStatus ovvsResourcesCagraTransferStats(ovvsResources_t res, int64_t* walks,
                                           int64_t* direct_walks, int64_t* upload_calls,
                                           int64_t* upload_bytes) {
  if (!res || !walks || !direct_walks || !upload_calls || !upload_bytes)
    return OVVS_STATUS_INVALID_ARGUMENT;
  *walks = *direct_walks = *upload_calls = *upload_bytes = 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesIvfPqSearchStatsV1(ovvsResources_t res, ovvsIvfPqSearchStatsV1* stats) {
  if (!res || !stats) return OVVS_STATUS_INVALID_ARGUMENT;
  std::memset(stats, 0, sizeof(*stats));
  stats->abi_version = OVVS_IVF_PQ_SEARCH_STATS_ABI_V1;
  stats->struct_size = static_cast<uint32_t>(sizeof(*stats));
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesCagraBuildStatsV1(ovvsResources_t res, ovvsCagraBuildStatsV1* stats) {
  if (!res || !stats) return OVVS_STATUS_INVALID_ARGUMENT;
  std::memset(stats, 0, sizeof(*stats));
  stats->abi_version = OVVS_CAGRA_BUILD_STATS_ABI_V1;
  stats->struct_size = static_cast<uint32_t>(sizeof(*stats));
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesSetNpuBusy(ovvsResources_t res, int32_t busy) {
  (void)busy;
  return res ? OVVS_STATUS_SUCCESS : OVVS_STATUS_INVALID_ARGUMENT;
}

int32_t ovvsSyclEnabled(void) { return 0; }

int32_t ovvsGpuHasXmx(void) { return -1; }

ovvsStatus ovvsResourcesEnergyUj(ovvsResources_t res, int64_t* uj) {
  (void)res;
  if (!uj) return OVVS_STATUS_INVALID_ARGUMENT;
  *uj = 0;
  return OVVS_STATUS_UNSUPPORTED;
}

// compiler/shave/topk.c:4-26: k repeated minimum scans; unused slots get id -1, value 3.4e38.
void ovvsShaveTopkSmallest(const float* scores, int32_t cols, int32_t k, int32_t* idx, float* val) {
  for (int32_t t = 0; t < k; ++t) {
    int32_t best = -1;
    float bv = 3.4e38f;
    for (int32_t j = 0; j < cols; ++j) {
      bool taken = false;
      for (int32_t u = 0; u < t && !taken; ++u) taken = idx[u] == j;
      if (!taken && scores[j] < bv) {
        bv = scores[j];
        best = j;
      }
    }
    idx[t] = best;
    val[t] = bv;
  }
}

// compiler/shave/adc.c:4-10: sum over sub-quantizers of table[m][code[m]].
float ovvsShavePqAdc(const float* tables, const uint8_t* code, int32_t pq_m, int32_t ks) {
  float s = 0.f;
  for (int32_t m = 0; m < pq_m; ++m) s += tables[m * ks + code[m]];
  return s;
}

ovvsStatus ovvsPqAdcBatch(ovvsResources_t res, const float* tables, int32_t pq_m, int32_t ks,
                          const uint8_t* codes, int64_t ncodes, float* out) {
  (void)tables, (void)pq_m, (void)ks, (void)codes, (void)ncodes, (void)out;
  if (!res) return OVVS_STATUS_INVALID_ARGUMENT;
  return OVVS_STATUS_UNSUPPORTED;
}

ovvsStatus ovvsProbeJson(char* buf, int32_t len) {
  if (!buf || len <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    (void)cudaGetLastError();
    count = 0;
  }
  std::string s = "{\n  \"backend\": \"cuda-sm100a\",\n  \"devices\": [";
  for (int d = 0; d < count; ++d) {
    cudaDeviceProp p{};
    if (cudaGetDeviceProperties(&p, d) != cudaSuccess) continue;
    char item[256];
    std::snprintf(item, sizeof(item), "%s{\"index\": %d, \"name\": \"%s\", \"sm\": \"%d.%d\"}",
                  d ? ", " : "", d, p.name, p.major, p.minor);
    s += item;
  }
  s += "],\n  \"version\": \"" OVVS_VERSION_STRING "\"\n}\n";
  if (static_cast<int32_t>(s.size()) + 1 > len) return OVVS_STATUS_SHAPE_MISMATCH;
  std::memcpy(buf, s.c_str(), s.size() + 1);
  return OVVS_STATUS_SUCCESS;
}

// ---- brute force (reference src/neighbors/indexes.cpp:236-268) -----------------------------

ovvsStatus ovvsBruteForceBuild(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim,
                               ovvsMetric metric, ovvsBruteForceIndex_t* index) {
  return ovvsBruteForceBuildTyped(res, dataset, n, dim, metric, OVVS_DTYPE_F32, index);
}

ovvsStatus ovvsBruteForceBuildTyped(ovvsResources_t res, const void* dataset, int64_t n,
                                    int64_t dim, ovvsMetric metric, ovvsDType dtype,
                                    ovvsBruteForceIndex_t* index) {
  if (!res || !dataset || !index || n <= 0 || dim <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  if (r.group.empty()) return ovvsBruteForceBuildShard(res, dataset, n, dim, metric, dtype, 0, index);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    if (mul_overflows(n, dim, INT64_MAX / 8)) return OVVS_STATUS_SHAPE_MISMATCH;
    auto ix = std::make_unique<ovvs::nb::BruteIndex>();
    OVVS_TRY(ovvs::rt::group_build(r, *ix, dataset, static_cast<int>(dtype), n, dim,
                                   static_cast<int>(metric)));
    *index = reinterpret_cast<ovvsBruteForceIndex_t>(ix.release());
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsBruteForceSearch(ovvsResources_t res, ovvsBruteForceIndex_t index,
                                const float* queries, int64_t nq, int64_t k, const uint8_t* bitset,
                                int64_t* neighbors, float* distances) {
  if (!res || !index || !queries || !neighbors || !distances || nq <= 0 || k <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    return search_host(r, *as_index(index), queries, nq, k, bitset, neighbors, distances);
  });
}

ovvsStatus ovvsBruteForceDestroy(ovvsBruteForceIndex_t index) {
  auto* ix = as_index(index);
  if (ix) {
    cudaSetDevice(ix->device);
    delete ix;
  }
  return OVVS_STATUS_SUCCESS;
}

// ---- allow-list bitset (reference src/rt/resources.cpp:218-229) ---------------------------

ovvsStatus ovvsBitsetFromAllowList(int64_t n, const int64_t* ids, int64_t nids, uint8_t* bitset) {
  if (!bitset || n <= 0 || nids < 0) return OVVS_STATUS_INVALID_ARGUMENT;
  const int64_t nbytes = (n + 7) / 8;
  std::memset(bitset, 0, static_cast<size_t>(nbytes));
  if (!ids || nids == 0) return OVVS_STATUS_SUCCESS;
  for (int64_t i = 0; i < nids; ++i) {
    const int64_t id = ids[i];
    if (id < 0 || id >= n) continue;
    bitset[id >> 3] = static_cast<uint8_t>(bitset[id >> 3] | (1u << (id & 7)));
  }
  return OVVS_STATUS_SUCCESS;
}

// ---- k-means (reference src/cluster/cluster.cpp:46-84) ------------------------------------

ovvsStatus ovvsKMeansFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim,
                         int32_t nclusters, int32_t iters, ovvsKMeansModel_t* model) {
  if (!res || !dataset || !model || n <= 0 || dim <= 0 || nclusters <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  if (r.group.empty()) return ovvsKMeansFitShard(res, dataset, n, 0, n, dim, nclusters, iters, model);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    auto m = std::make_unique<ovvs::km::KMeansModel>();
    m->k_reported = nclusters;
    m->dim = dim;
    m->device = r.device;
    // cluster.cpp:54 runs max(4, iters) iterations; n > INT32_MAX leaves the model empty, as in
    // the single-device path.
    if (n <= INT32_MAX)
      OVVS_TRY(ovvs::rt::group_kmeans_fit(r, dataset, n, dim, nclusters, std::max(4, iters), *m));
    *model = reinterpret_cast<ovvsKMeansModel_t>(m.release());
    r.last_device = OVVS_DEVICE_GPU;
    r.last_compute_dtype = OVVS_DTYPE_F32;
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsKMeansPredict(ovvsResources_t res, ovvsKMeansModel_t model, const float* x,
                             int64_t n, int64_t* labels, float* distances) {
  if (!res || !model || !x || !labels || n <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    if (as_model(model)->dim <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
    OVVS_TRY(ovvs::km::predict(r, *as_model(model), x, n, labels, distances));
    r.last_device = OVVS_DEVICE_GPU;
    r.last_compute_dtype = OVVS_DTYPE_F32;
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsKMeansCentroids(ovvsKMeansModel_t model, const float** data, int32_t* nclusters,
                               int64_t* dim) {
  if (!model || !data || !nclusters || !dim) return OVVS_STATUS_INVALID_ARGUMENT;
  auto* m = as_model(model);
  *data = m->host.data();
  *nclusters = m->k_reported;
  *dim = m->dim;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsKMeansDestroy(ovvsKMeansModel_t model) {
  auto* m = as_model(model);
  if (m) {
    cudaSetDevice(m->device);
    delete m;
  }
  return OVVS_STATUS_SUCCESS;
}

// ---- extensions (ovvs_cuda.h) ---------------------------------------------------------------

ovvsStatus ovvsResourcesStream(ovvsResources_t res, void** stream) {
  if (!res || !stream) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  std::lock_guard<std::mutex> lk(r.mu);
  OVVS_TRY(r.activate());
  *stream = r.stream;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesSynchronize(ovvsResources_t res) {
  if (!res) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  std::lock_guard<std::mutex> lk(r.mu);
  OVVS_TRY(r.activate());
  return r.finish();
}

ovvsStatus ovvsResourcesDevice(ovvsResources_t res, int32_t* device) {
  if (!res || !device) return OVVS_STATUS_INVALID_ARGUMENT;
  *device = from_handle(res)->device;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsBruteForceSearchDevice(ovvsResources_t res, ovvsBruteForceIndex_t index,
                                      const float* d_queries, int64_t nq, int64_t k,
                                      const uint8_t* d_bitset, int64_t* d_neighbors,
                                      float* d_distances) {
  if (!res || !index || !d_queries || !d_neighbors || !d_distances || nq <= 0 || k <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    int64_t ke = 0;
    OVVS_TRY(ovvs::nb::search_device(r, *as_index(index), d_queries, nq, k, d_bitset,
                                     d_neighbors, d_distances, &ke));
    r.last_device = OVVS_DEVICE_GPU;
    r.last_compute_dtype = OVVS_DTYPE_F32;
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsResourcesSetProfiling(ovvsResources_t res, int32_t enable) {
  if (!res) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  std::lock_guard<std::mutex> lk(r.mu);
  r.profiling = enable != 0;
  r.phase_valid = false;
  r.hist_next = 0;
  r.hist_count = 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesPhaseHistoryMs(ovvsResources_t res, float* ms, int32_t max_searches,
                                       int32_t* count) {
  if (!res || !ms || !count || max_searches < 0) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  std::lock_guard<std::mutex> lk(r.mu);
  const int n = std::min(r.hist_count, max_searches);
  *count = 0;
  if (n > 0) {
    constexpr int H = Resources::kPhaseHistory;
    OVVS_TRY_CUDA(cudaEventSynchronize(r.hist_ev[(r.hist_next - 1 + H) % H][Resources::kPhases]));
    for (int s = 0; s < n; ++s) {
      const int slot = (r.hist_next - n + s + H) % H;
      for (int i = 0; i < Resources::kPhases; ++i) {
        float v = 0.f;
        OVVS_TRY_CUDA(cudaEventElapsedTime(&v, r.hist_ev[slot][i], r.hist_ev[slot][i + 1]));
        ms[s * Resources::kPhases + i] = v;
      }
    }
  }
  *count = n;
  r.hist_count = 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesLastPhaseMs(ovvsResources_t res, float* ms, int32_t count) {
  if (!res || !ms || count < 0) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  std::lock_guard<std::mutex> lk(r.mu);
  if (!r.phase_valid) return OVVS_STATUS_INVALID_ARGUMENT;
  OVVS_TRY_CUDA(cudaEventSynchronize(r.phase_ev[Resources::kPhases]));
  for (int32_t i = 0; i < count && i < Resources::kPhases; ++i) {
    float v = 0.f;
    OVVS_TRY_CUDA(cudaEventElapsedTime(&v, r.phase_ev[i], r.phase_ev[i + 1]));
    ms[i] = v;
  }
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesLastKernelError(ovvsResources_t res, int32_t* code) {
  if (!res || !code) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  std::lock_guard<std::mutex> lk(r.mu);
  *code = r.last_kernel_error;
  r.last_kernel_error = 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesPeerBounds(ovvsResources_t res, int32_t* active) {
  if (!res || !active) return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  std::lock_guard<std::mutex> lk(r.mu);
  // A one-process group reports its members (they share bounds with each other or none do).
  const Resources& m = r.group.empty() ? r : *r.group.front();
  *active = m.peer_bounds == 1 ? 1 : 0;
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsWatchdogSelfTest(ovvsResources_t res, int64_t limit_ns, int32_t* code) {
  if (!res || !code || limit_ns < 1000000 || limit_ns > 5000000000LL)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  std::lock_guard<std::mutex> lk(r.mu);
  OVVS_TRY(r.check_policy());
  OVVS_TRY(r.activate());
  *code = 0;
  OVVS_TRY_CUDA(ovvs::prim::launch_watchdog_selftest(r.d_err, static_cast<uint64_t>(limit_ns),
                                                     r.stream));
  const ovvsStatus st = r.finish();  // the wait ran out: ERROR, with the code recorded
  *code = r.last_kernel_error;
  r.last_kernel_error = 0;
  if (st == OVVS_STATUS_ERROR && *code == ovvs::prim::kErrSelfTest) return OVVS_STATUS_SUCCESS;
  return st == OVVS_STATUS_SUCCESS ? OVVS_STATUS_ERROR : st;
}

int32_t ovvsNcclUniqueIdSize(void) { return static_cast<int32_t>(sizeof(ncclUniqueId)); }

ovvsStatus ovvsNcclUniqueId(uint8_t* id, int32_t len) {
  if (!id || len < static_cast<int32_t>(sizeof(ncclUniqueId))) return OVVS_STATUS_INVALID_ARGUMENT;
  if (!ovvs::rt::nccl()) return OVVS_STATUS_DEVICE_UNAVAILABLE;
  ncclUniqueId u;
  OVVS_TRY(ovvs::rt::status_of(ovvs::rt::nccl()->GetUniqueId(&u)));
  std::memcpy(id, &u, sizeof(u));
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsResourcesCreateSharded(ovvsResources_t* res, int32_t device, int32_t rank,
                                      int32_t world, const uint8_t* nccl_id, int32_t len) {
  if (!res || world <= 0 || rank < 0 || rank >= world) return OVVS_STATUS_INVALID_ARGUMENT;
  if (world > 1 && (!nccl_id || len < static_cast<int32_t>(sizeof(ncclUniqueId))))
    return OVVS_STATUS_INVALID_ARGUMENT;
  auto* r = new (std::nothrow) Resources();
  if (!r) return OVVS_STATUS_OOM;
  ovvs::rt::probe_device(*r, device);
  r->rank = rank;
  r->world = world;
  r->nccl_timeout_ms = ovvs::rt::nccl_timeout_ms_default();
  ovvsStatus st = r->activate();
  if (st == OVVS_STATUS_SUCCESS && world > 1 && !ovvs::rt::nccl()) st = OVVS_STATUS_DEVICE_UNAVAILABLE;
  if (st == OVVS_STATUS_SUCCESS && world > 1) {
    ncclUniqueId u;
    std::memcpy(&u, nccl_id, sizeof(u));
    st = guarded([&] { return ovvs::rt::init_comm(*r, u); });  // non-blocking, bounded
  }
  if (st != OVVS_STATUS_SUCCESS) {
    delete r;
    return st;
  }
  *res = ovvs::rt::to_handle(r);
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsBruteForceBuildShard(ovvsResources_t res, const void* dataset, int64_t n_local,
                                    int64_t dim, ovvsMetric metric, ovvsDType dtype,
                                    int64_t row_offset, ovvsBruteForceIndex_t* index) {
  if (!res || !dataset || !index || n_local <= 0 || dim <= 0 || row_offset < 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    if (mul_overflows(n_local, dim, INT64_MAX / 8)) return OVVS_STATUS_SHAPE_MISMATCH;
    // Reference quirk kept: dtype is not validated; unknown values are read as bytes.
    auto* ix = new ovvs::nb::BruteIndex();
    const ovvsStatus st = ovvs::nb::build_from_host(r, *ix, dataset, static_cast<int>(dtype),
                                                    n_local, dim, static_cast<int>(metric),
                                                    row_offset, r.world > 1);
    if (st != OVVS_STATUS_SUCCESS) {
      delete ix;
      return st;
    }
    *index = reinterpret_cast<ovvsBruteForceIndex_t>(ix);
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsKMeansFitShard(ovvsResources_t res, const float* dataset, int64_t n_local,
                              int64_t row_offset, int64_t n_total, int64_t dim, int32_t nclusters,
                              int32_t iters, ovvsKMeansModel_t* model) {
  if (!res || !dataset || !model || n_local <= 0 || dim <= 0 || nclusters <= 0 ||
      row_offset < 0 || n_total < row_offset + n_local)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded([&] {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    auto* m = new ovvs::km::KMeansModel();
    m->k_reported = nclusters;
    m->dim = dim;
    m->device = r.device;
    // cluster.cpp:54 runs max(4, iters) iterations; mixer.cpp:869 rejects n > INT32_MAX inside
    // the fit, which the ABI ignores: the model then has no centroids.
    ovvsStatus st = OVVS_STATUS_SUCCESS;
    if (n_total <= INT32_MAX) {
      st = ovvs::km::fit(r, dataset, n_local, row_offset, n_total, dim, nclusters,
                         std::max(4, iters), *m);
    }
    if (st != OVVS_STATUS_SUCCESS) {
      delete m;
      return st;
    }
    *model = reinterpret_cast<ovvsKMeansModel_t>(m);
    r.last_device = OVVS_DEVICE_GPU;
    r.last_compute_dtype = OVVS_DTYPE_F32;
    return OVVS_STATUS_SUCCESS;
  });
}

}  // extern "C"
