// k-means fit / predict (see kmeans.hpp).
#include "kmeans.hpp"

#include <cub/device/device_radix_sort.cuh>
#include <cub/device/device_scan.cuh>

#include <algorithm>
#include <random>

#include "../prim/keys.cuh"
#include "../prim/prep.cuh"

namespace ovvs {
namespace km {
namespace {

constexpr int kDTypeF32 = 0;

__global__ void label_keys_kernel(const int64_t* __restrict__ labels, int64_t n,
                                  uint32_t* __restrict__ keys, uint32_t* __restrict__ idx,
                                  int* __restrict__ counts) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t c = static_cast<uint32_t>(labels[i]);
  keys[i] = c;
  idx[i] = static_cast<uint32_t>(i);
  atomicAdd(&counts[c], 1);
}

// Upper bound on each point's nearest-centroid ranking key for the next assignment: the point's
// value against its previous centroid under the new centroids, v = |c|^2 - 2 x.c (the fused
// kernel's L2 ranking value, without |x|^2), plus a relative margin of 1e-4 that covers the
// rounding of this warp-parallel sum and of the kernel's own values. The true nearest centroid
// has a value no larger, so seeding the kernel's shared bound with it filters from the first
// tile without excluding it.
__global__ void kmeans_bound_kernel(const float* __restrict__ x, const int64_t* __restrict__ labels,
                                    const float* __restrict__ centroids, int dim, int64_t n,
                                    uint64_t* __restrict__ bound) {
  // Four points per warp, eight lanes per point; with rows 16-byte aligned (dim % 4 == 0) each
  // lane reads its columns four at a time, so a warp has eight 16-byte loads in flight per lane.
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const int64_t i = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 4 +
                    (lane >> 3);
  const bool active = i < n;
  const int64_t lab = active ? labels[i] : -1;
  const float* xr = x + (active ? i : 0) * dim;
  const float* cr = centroids + (lab < 0 ? 0 : lab) * dim;
  float ip = 0.f, yn = 0.f;
  if (active) {
    if ((dim & 3) == 0) {
      const float4* x4 = reinterpret_cast<const float4*>(xr);
      const float4* c4 = reinterpret_cast<const float4*>(cr);
#pragma unroll 4
      for (int f = sub; f < dim / 4; f += 8) {
        const float4 a = __ldg(x4 + f), c = c4[f];
        ip = fmaf(a.x, c.x, fmaf(a.y, c.y, fmaf(a.z, c.z, fmaf(a.w, c.w, ip))));
        yn = fmaf(c.x, c.x, fmaf(c.y, c.y, fmaf(c.z, c.z, fmaf(c.w, c.w, yn))));
      }
    } else {
      for (int d = sub; d < dim; d += 8) {
        const float c = cr[d];
        ip = fmaf(xr[d], c, ip);
        yn = fmaf(c, c, yn);
      }
    }
  }
#pragma unroll
  for (int off = 4; off; off >>= 1) {
    ip += __shfl_xor_sync(0xffffffffu, ip, off);
    yn += __shfl_xor_sync(0xffffffffu, yn, off);
  }
  if (active && sub == 0) {
    const float v = yn - 2.f * ip;
    const float margin = 1e-4f * (fabsf(yn) + 2.f * fabsf(ip)) + 1e-30f;
    const bool ok = lab >= 0 && v == v && fabsf(v) < __int_as_float(0x7f800000);
    bound[i] = ok ? keys::make_key(v + margin, static_cast<uint32_t>(lab)) : keys::kEmptyKey;
  }
}

// mixer.cpp:902-918: per centroid, fp32 sum of its rows in ascending row order, then
// centroid = sum * (1 / count); a centroid without rows keeps its previous value. One block per
// centroid, one thread per dimension; the cluster's row ids are staged in shared memory 256 at a
// time so that each thread keeps kUpdateDepth independent row loads in flight (the additions stay
// in row order).
constexpr int kUpdateIdx = 256;
constexpr int kUpdateDepth = 16;

__global__ void centroid_update_kernel(const float* __restrict__ x, int dim,
                                       const uint32_t* __restrict__ sorted_idx,
                                       const int* __restrict__ counts,
                                       const int* __restrict__ offsets,
                                       float* __restrict__ centroids) {
  __shared__ uint32_t s_idx[kUpdateIdx];
  const int c = blockIdx.x;
  const int cnt = counts[c];
  if (cnt == 0) return;
  const int beg = offsets[c];
  const float inv = __fdiv_rn(1.f, static_cast<float>(cnt));
  for (int d0 = 0; d0 < dim; d0 += blockDim.x) {
    const int d = d0 + static_cast<int>(threadIdx.x);
    float s = 0.f;
    for (int j0 = 0; j0 < cnt; j0 += kUpdateIdx) {
      const int m = min(kUpdateIdx, cnt - j0);
      __syncthreads();
      for (int t = threadIdx.x; t < m; t += blockDim.x) s_idx[t] = sorted_idx[beg + j0 + t];
      __syncthreads();
      if (d < dim) {
        int j = 0;
        for (; j + kUpdateDepth <= m; j += kUpdateDepth) {
          float v[kUpdateDepth];
#pragma unroll
          for (int u = 0; u < kUpdateDepth; ++u)
            v[u] = __ldg(x + static_cast<int64_t>(s_idx[j + u]) * dim + d);
#pragma unroll
          for (int u = 0; u < kUpdateDepth; ++u) s = __fadd_rn(s, v[u]);
        }
        for (; j < m; ++j) s = __fadd_rn(s, x[static_cast<int64_t>(s_idx[j]) * dim + d]);
      }
    }
    if (d < dim) centroids[static_cast<int64_t>(c) * dim + d] = __fmul_rn(s, inv);
  }
}

// Sharded variant: this shard's per-centroid sums in fp64 (all-reduced afterwards), with the
// cluster's row ids staged in shared memory like centroid_update_kernel.
__global__ void centroid_partial_kernel(const float* __restrict__ x, int dim,
                                        const uint32_t* __restrict__ sorted_idx,
                                        const int* __restrict__ counts,
                                        const int* __restrict__ offsets,
                                        double* __restrict__ sum64, double* __restrict__ cnt64) {
  __shared__ uint32_t s_idx[kUpdateIdx];
  const int c = blockIdx.x;
  const int cnt = counts[c];
  const int beg = offsets[c];
  for (int d0 = 0; d0 < dim; d0 += blockDim.x) {
    const int d = d0 + static_cast<int>(threadIdx.x);
    double s = 0.0;
    for (int j0 = 0; j0 < cnt; j0 += kUpdateIdx) {
      const int m = min(kUpdateIdx, cnt - j0);
      __syncthreads();
      for (int t = threadIdx.x; t < m; t += blockDim.x) s_idx[t] = sorted_idx[beg + j0 + t];
      __syncthreads();
      if (d < dim) {
        int j = 0;
        for (; j + kUpdateDepth <= m; j += kUpdateDepth) {
          float v[kUpdateDepth];
#pragma unroll
          for (int u = 0; u < kUpdateDepth; ++u)
            v[u] = __ldg(x + static_cast<int64_t>(s_idx[j + u]) * dim + d);
#pragma unroll
          for (int u = 0; u < kUpdateDepth; ++u) s += v[u];
        }
        for (; j < m; ++j) s += x[static_cast<int64_t>(s_idx[j]) * dim + d];
      }
    }
    if (d < dim) sum64[static_cast<int64_t>(c) * dim + d] = s;
  }
  if (threadIdx.x == 0) cnt64[c] = static_cast<double>(cnt);
}

__global__ void centroid_finish_kernel(const double* __restrict__ sum64,
                                       const double* __restrict__ cnt64, int k, int dim,
                                       float* __restrict__ centroids) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(k) * dim) return;
  const int c = static_cast<int>(i / dim);
  const double cnt = cnt64[c];
  if (cnt == 0.0) return;
  const float inv = __fdiv_rn(1.f, static_cast<float>(cnt));
  centroids[i] = __fmul_rn(static_cast<float>(sum64[i]), inv);
}

}  // namespace

std::vector<int64_t> init_rows(int64_t n, int32_t k) {
  std::mt19937 rng(42u);
  std::uniform_int_distribution<int64_t> pick(0, n - 1);
  std::vector<int64_t> used;
  used.reserve(static_cast<size_t>(k));
  for (int32_t c = 0; c < k; ++c) {
    int64_t i = pick(rng);
    for (int t = 0; t < 8 && std::find(used.begin(), used.end(), i) != used.end(); ++t)
      i = pick(rng);
    used.push_back(i);
  }
  return used;
}

ovvsStatus fit(rt::Resources& r, const float* x, int64_t n_local, int64_t row_offset,
               int64_t n_total, int64_t dim, int32_t nclusters, int32_t iters, KMeansModel& m) {
  cudaStream_t s = r.stream;
  if (r.world > 1) OVVS_TRY(r.comm_ready());  // after a communicator failure: fail at once
  m.device = r.device;
  m.k_reported = nclusters;
  m.dim = dim;
  const int32_t k = static_cast<int32_t>(std::max<int64_t>(1, std::min<int64_t>(nclusters, n_total)));
  m.k_eff = k;
  const size_t cbytes = static_cast<size_t>(k) * dim * sizeof(float);
  // Profiling phases of a fit: [0] upload + seeding, [1] the Lloyd iterations, [2] download.
  r.mark(0);

  // Seeding (mixer.cpp:880-890) over the global row numbering: each centroid row is copied by
  // the shard that owns it, the others contribute zeros, and a sum all-reduce assembles them.
  const std::vector<int64_t> rows = init_rows(n_total, k);
  std::vector<float> init(static_cast<size_t>(k) * dim, 0.f);
  for (int32_t c = 0; c < k; ++c) {
    const int64_t g = rows[static_cast<size_t>(c)] - row_offset;
    if (g >= 0 && g < n_local)
      std::copy(x + g * dim, x + (g + 1) * dim, init.begin() + static_cast<size_t>(c) * dim);
  }
  OVVS_TRY_CUDA(m.d_centroids.reserve(cbytes));
  OVVS_TRY_CUDA(cudaMemcpyAsync(m.d_centroids.get(), init.data(), cbytes, cudaMemcpyHostToDevice, s));
  if (r.world > 1) {
    OVVS_TRY(r.comm_ready());
    OVVS_TRY(r.collective(ovvs::rt::nccl()->AllReduce(m.d_centroids.get(), m.d_centroids.get(),
                                                      static_cast<size_t>(k) * dim, ncclFloat32,
                                                      ncclSum, r.comm, s)));
  }
  const size_t xbytes = static_cast<size_t>(n_local) * dim * sizeof(float);
  OVVS_TRY_CUDA(m.d_x.reserve(xbytes + 16));
  OVVS_TRY(rt::upload(r, m.d_x.get(), x, xbytes));
  OVVS_TRY(r.finish());  // `init` is a host temporary (bounded wait: the seeding all-reduce)

  const int64_t n = n_local;
  OVVS_TRY_CUDA(m.labels.reserve(n * sizeof(int64_t) + 16));
  OVVS_TRY_CUDA(m.bound_keys.reserve(n * sizeof(uint64_t) + 16));
  OVVS_TRY_CUDA(m.dist.reserve(n * sizeof(float) + 16));
  OVVS_TRY_CUDA(m.sort_keys.reserve(n * sizeof(uint32_t) + 16));
  OVVS_TRY_CUDA(m.sorted_keys.reserve(n * sizeof(uint32_t) + 16));
  OVVS_TRY_CUDA(m.idx.reserve(n * sizeof(uint32_t) + 16));
  OVVS_TRY_CUDA(m.sorted_idx.reserve(n * sizeof(uint32_t) + 16));
  OVVS_TRY_CUDA(m.counts.reserve(static_cast<size_t>(k) * sizeof(int)));
  OVVS_TRY_CUDA(m.offsets.reserve(static_cast<size_t>(k) * sizeof(int)));
  int end_bit = 1;
  while ((1ll << end_bit) < k) ++end_bit;
  size_t sort_bytes = 0, scan_bytes = 0;
  OVVS_TRY_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, sort_bytes, m.sort_keys.as<uint32_t>(),
                                                m.sorted_keys.as<uint32_t>(), m.idx.as<uint32_t>(),
                                                m.sorted_idx.as<uint32_t>(), static_cast<int>(n),
                                                0, end_bit, s));
  OVVS_TRY_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, scan_bytes, m.counts.as<int>(),
                                              m.offsets.as<int>(), k, s));
  OVVS_TRY_CUDA(m.cub_tmp.reserve(std::max(sort_bytes, scan_bytes) + 16));
  if (r.world > 1) {
    OVVS_TRY_CUDA(m.sum64.reserve(static_cast<size_t>(k) * dim * sizeof(double)));
    OVVS_TRY_CUDA(m.cnt64.reserve(static_cast<size_t>(k) * sizeof(double)));
  }

  r.mark(1);
  r.mark_hold = true;
  struct Release {
    rt::Resources& r;
    ~Release() { r.mark_hold = false; }
  } release_marks{r};
  for (int32_t it = 0; it < iters; ++it) {
    OVVS_TRY(nb::build_from_device(r, m.index, m.d_centroids.get(), kDTypeF32, k, dim,
                                   OVVS_METRIC_L2_EXPANDED, 0));
    int64_t k_eff = 0;
    // From the second iteration on, each point's previous centroid bounds its assignment.
    if (it > 0 && n > 0) {
      kmeans_bound_kernel<<<static_cast<unsigned>((n + 31) / 32), 256, 0, s>>>(
          m.d_x.as<float>(), m.labels.as<int64_t>(), m.d_centroids.as<float>(),
          static_cast<int>(dim), n, m.bound_keys.as<uint64_t>());
      OVVS_TRY_CUDA(cudaGetLastError());
    }
    // The points' query operands (fp16 split, norms) are the same every iteration.
    if (it == 0 && n > 0) OVVS_TRY(nb::prepare_queries(r, m.index, m.d_x.as<float>(), n, m.prepared));
    OVVS_TRY(nb::search_device(r, m.index, m.d_x.as<float>(), n, 1, nullptr,
                               m.labels.as<int64_t>(), m.dist.as<float>(), &k_eff,
                               it > 0 ? m.bound_keys.as<uint64_t>() : nullptr, &m.prepared,
                               /*labels_only=*/true));
    OVVS_TRY_CUDA(cudaMemsetAsync(m.counts.get(), 0, static_cast<size_t>(k) * sizeof(int), s));
    if (n > 0) {
      label_keys_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, s>>>(
          m.labels.as<int64_t>(), n, m.sort_keys.as<uint32_t>(), m.idx.as<uint32_t>(),
          m.counts.as<int>());
      OVVS_TRY_CUDA(cudaGetLastError());
      size_t tb = sort_bytes;
      OVVS_TRY_CUDA(cub::DeviceRadixSort::SortPairs(
          m.cub_tmp.get(), tb, m.sort_keys.as<uint32_t>(), m.sorted_keys.as<uint32_t>(),
          m.idx.as<uint32_t>(), m.sorted_idx.as<uint32_t>(), static_cast<int>(n), 0, end_bit, s));
    }
    size_t sb = scan_bytes;
    OVVS_TRY_CUDA(cub::DeviceScan::ExclusiveSum(m.cub_tmp.get(), sb, m.counts.as<int>(),
                                                m.offsets.as<int>(), k, s));
    const int threads = static_cast<int>(std::min<int64_t>(128, (dim + 31) / 32 * 32));
    if (r.world <= 1) {
      centroid_update_kernel<<<k, threads, 0, s>>>(m.d_x.as<float>(), static_cast<int>(dim),
                                                   m.sorted_idx.as<uint32_t>(), m.counts.as<int>(),
                                                   m.offsets.as<int>(), m.d_centroids.as<float>());
      OVVS_TRY_CUDA(cudaGetLastError());
    } else {
      centroid_partial_kernel<<<k, threads, 0, s>>>(
          m.d_x.as<float>(), static_cast<int>(dim), m.sorted_idx.as<uint32_t>(),
          m.counts.as<int>(), m.offsets.as<int>(), m.sum64.as<double>(), m.cnt64.as<double>());
      OVVS_TRY_CUDA(cudaGetLastError());
      // Non-blocking communicator: the group's enqueue is settled (bounded) before the kernel
      // that reads the sums is launched behind it.
      const rt::NcclApi* nc = ovvs::rt::nccl();
      OVVS_TRY(r.comm_ready());
      OVVS_TRY(rt::status_of(nc->GroupStart()));
      OVVS_TRY(r.collective(nc->AllReduce(m.sum64.get(), m.sum64.get(),
                                          static_cast<size_t>(k) * dim, ncclFloat64, ncclSum,
                                          r.comm, s)));
      OVVS_TRY(r.collective(nc->AllReduce(m.cnt64.get(), m.cnt64.get(), static_cast<size_t>(k),
                                          ncclFloat64, ncclSum, r.comm, s)));
      OVVS_TRY(r.collective(nc->GroupEnd()));
      const int64_t total = static_cast<int64_t>(k) * dim;
      centroid_finish_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, s>>>(
          m.sum64.as<double>(), m.cnt64.as<double>(), k, static_cast<int>(dim),
          m.d_centroids.as<float>());
      OVVS_TRY_CUDA(cudaGetLastError());
    }
  }
  r.mark_hold = false;
  // Sharded: the last iteration's all-reduce is waited for with a bound before anything below
  // (frees, copies into pageable host memory) could wait on it without one.
  if (r.world > 1) OVVS_TRY(r.finish());
  r.mark(2);
  // free the per-fit query operands
  m.prepared.a16.release();
  m.prepared.xn.release();
  m.prepared.e_q.release();
  m.prepared.nq = 0;
  OVVS_TRY(nb::build_from_device(r, m.index, m.d_centroids.get(), kDTypeF32, k, dim,
                                 OVVS_METRIC_L2_EXPANDED, 0));
  m.host.assign(static_cast<size_t>(std::max(k, nclusters)) * dim, 0.f);
  OVVS_TRY_CUDA(cudaMemcpyAsync(m.host.data(), m.d_centroids.get(), cbytes, cudaMemcpyDeviceToHost, s));
  r.mark(3);
  r.mark(4);
  m.d_x.release();
  return r.finish();
}

ovvsStatus predict(rt::Resources& r, KMeansModel& m, const float* x, int64_t n, int64_t* labels,
                   float* distances) {
  if (m.k_eff <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  if (m.device != r.device) return OVVS_STATUS_INVALID_ARGUMENT;
  cudaStream_t s = r.stream;
  float* dq = nullptr;
  int64_t* dl = nullptr;
  float* dd = nullptr;
  OVVS_TRY(r.scratch(rt::kWsQueries, static_cast<size_t>(n) * m.dim, &dq));
  OVVS_TRY(r.scratch(rt::kWsNeighbors, static_cast<size_t>(n), &dl));
  OVVS_TRY(r.scratch(rt::kWsDistances, static_cast<size_t>(n), &dd));
  OVVS_TRY(rt::upload(r, dq, x, static_cast<size_t>(n) * m.dim * sizeof(float)));
  int64_t k_eff = 0;
  OVVS_TRY(nb::search_device(r, m.index, dq, n, 1, nullptr, dl, dd, &k_eff));
  OVVS_TRY_CUDA(cudaMemcpyAsync(labels, dl, static_cast<size_t>(n) * sizeof(int64_t),
                                cudaMemcpyDeviceToHost, s));
  if (distances)
    OVVS_TRY_CUDA(cudaMemcpyAsync(distances, dd, static_cast<size_t>(n) * sizeof(float),
                                  cudaMemcpyDeviceToHost, s));
  return r.finish();
}

}  // namespace km
}  // namespace ovvs
