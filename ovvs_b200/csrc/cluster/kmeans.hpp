// k-means (Lloyd) on the GPU, reusing the brute-force kernels with k = 1.
//
// Reference: src/cluster/cluster.cpp:7-84 (model, ABI) and src/prim/mixer.cpp:866-921
// (kmeans_fit_impl). Per iteration: assignment = fused distance/top-1 kernel + exact re-rank
// (ties to the lower centroid id), update = stable sort of row ids by label, then per centroid
// a sequential fp32 sum in ascending row order and centroid = sum * (1/count), empty clusters
// unchanged -- the reference's own operation order, so a single-GPU fit reproduces its centroids
// bit for bit whenever the assignments agree. Sharded fits (one process per GPU) sum in fp64 per
// shard and all-reduce sums and counts over NCCL.
#pragma once

#include <cstdint>
#include <vector>

#include "../neighbors/brute_force.hpp"
#include "../rt/runtime.hpp"

namespace ovvs {
namespace km {

struct KMeansModel {
  int32_t k_reported = 0;  // nclusters as passed to fit (what ovvsKMeansCentroids reports)
  int32_t k_eff = 0;       // centroids actually fitted: clamp(nclusters, 1, n)
  int64_t dim = 0;
  int device = 0;
  std::vector<float> host;  // [max(k_reported, k_eff) x dim] mirror returned by Centroids
  rt::DeviceBuffer d_centroids;
  nb::BruteIndex index;     // centroids as an L2 brute-force index (replicated)
  // iteration scratch
  rt::DeviceBuffer d_x, labels, dist, sort_keys, sorted_keys, idx, sorted_idx, counts, offsets,
      cub_tmp, sum64, cnt64, bound_keys;
  nb::PreparedQueries prepared;  // the points as query operands, during a fit
};

// Rows [row_offset, row_offset + n_local) of a dataset with n_total rows (world == 1:
// row_offset = 0, n_local = n_total).
ovvsStatus fit(rt::Resources& r, const float* x, int64_t n_local, int64_t row_offset,
               int64_t n_total, int64_t dim, int32_t nclusters, int32_t iters, KMeansModel& m);

ovvsStatus predict(rt::Resources& r, KMeansModel& m, const float* x, int64_t n, int64_t* labels,
                   float* distances);

// mixer.cpp:879-890: rows chosen by std::mt19937(42) and uniform_int_distribution<int64_t>(0,
// n-1), redrawing up to 8 times when a row was already used.
std::vector<int64_t> init_rows(int64_t n, int32_t k);

}  // namespace km
}  // namespace ovvs
