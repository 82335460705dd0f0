// IVF-Flat index on one CUDA device: the first approximate index built on the k-means path.
//
// Reference: src/neighbors/indexes.cpp:27-32 (IvfFlat), 281-300 (build), 302-358 (search),
// 366-434 (serialize / deserialize, the 'IVF1' file format), 436-457 (extend),
// 50-57 (build_ivf_lists).
//   build:   nlist = min(nlist, n); Lloyd k-means with 12 iterations (the k-means fit of this
//            library, cluster/kmeans.cu); every row assigned to its nearest centroid (squared L2,
//            top-1 -- the fused brute-force search with k = 1); list c = the rows labelled c in
//            ascending row order.
//   search:  coarse squared-L2 scores of each query against the centroids (sequential fp32 on
//            CUDA cores, the reference's prim_pairwise arithmetic) and its nprobe nearest lists;
//            then the list scan: for the L2 metrics and k <= 10 on the tensor
//            cores (the fused brute-force kernel over (list, 256 probing pairs) items, then an
//            exact re-score of each pair's candidates: the reference's results except where a
//            row ties with a pair's k-th within the approximate scores' error, as for the
//            brute-force search), otherwise the exact CUDA-core scan of prim/ivf_scan.cu.
// Device layout: the dataset in original row order (kept for serialisation and extension) and a
// copy in list order (the scan's operand) with each row's squared norm and original id; the
// centroids and their norms; list offsets. The lists themselves are mirrored on the host, as in
// the reference.
#pragma once

#include <cstdint>
#include <vector>

#include "../rt/runtime.hpp"
#include "brute_force.hpp"

namespace ovvs {
namespace ivf {

struct IvfFlatIndex {
  int device = 0;
  int64_t n = 0;    // dataset rows
  int64_t dim = 0;
  int metric = 0;   // ovvsMetric as given (the lists' scores use it; the coarse step is L2)
  int32_t nlist = 0;
  std::vector<float> centroids;     // [nlist x dim]
  std::vector<int64_t> list_off;    // [nlist + 1]
  std::vector<int64_t> list_ids;    // the lists concatenated (ids in list order)
  rt::DeviceBuffer d_x;             // [n x dim] fp32, original order
  rt::DeviceBuffer d_rows, d_rnorm, d_ids, d_loff;  // list order
  rt::DeviceBuffer d_cent, d_cnorm;
  nb::BruteIndex cindex;            // the centroids as an L2 brute-force index (assignment)
  // Tensor-core list scan (L2 family): the list-ordered rows with every list padded to whole
  // 256-row tiles, as an in-order brute-force index; pos_row[pos] = the list-order row of a
  // padded position (-1: padding); list_tiles[c] = (first tile, end tile) of list c.
  nb::BruteIndex tc;
  rt::DeviceBuffer d_pos_row, d_list_tiles;
  bool tc_ready = false;
};

ovvsStatus build(rt::Resources& r, IvfFlatIndex& ix, const float* x, int64_t n, int64_t dim,
                 int metric, int32_t nlist);

// Device-pointer search on r.stream; outputs [nq x k] (row stride k).
ovvsStatus search_device(rt::Resources& r, const IvfFlatIndex& ix, const float* d_queries,
                         int64_t nq, int64_t k, int32_t nprobe, const uint8_t* d_bitset,
                         int64_t* d_neighbors, float* d_distances);

ovvsStatus extend(rt::Resources& r, IvfFlatIndex& ix, const float* extra, int64_t nextra);

ovvsStatus serialize(const IvfFlatIndex& ix, const char* path);
ovvsStatus deserialize(rt::Resources& r, const char* path, IvfFlatIndex& ix);

}  // namespace ivf
}  // namespace ovvs
