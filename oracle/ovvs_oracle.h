#pragma once
/* CPU restatement of the reference's brute-force kNN, k-means and IVF-Flat path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the GPU library is compared against; the product
 * (libovvs.so) never links, loads or calls it. Every function follows the reference's arithmetic
 * operation for operation (sequential fp32, no FMA contraction), so its outputs are bit-identical
 * to the reference's FORCE_CPU path. It is pinned against outputs of the reference itself
 * (oracle/_ref/libovvs_ref.so, built from the reference sources) by tests/golden.
 *
 * Layouts: row-major float32 [rows x dim]; ids int64; bitset LSB-first bytes. */

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* internal.hpp:842-862 convert_to_f32 (F16 decoded exactly; I8; everything else read as U8). */
void oracle_convert_to_f32(int32_t dtype, const void* src, int64_t n, int64_t dim, float* out);

/* internal.hpp:831-840 truncating fp32 -> fp16 used by the reference tests' data prep. */
uint16_t oracle_f32_to_f16_trunc(float f);
/* internal.hpp:83-106 round-to-nearest-even fp32 -> fp16. */
uint16_t oracle_f32_to_f16_rne(float f);
/* internal.hpp:804-829 exact fp16 -> fp32. */
float oracle_f16_to_f32(uint16_t h);

/* mixer.cpp:174-221 prim_pairwise + cpu_prims.cpp:120-149 + internal.hpp:240-272 distance_one. */
void oracle_pairwise(int32_t metric, const float* x, int64_t nx, const float* y, int64_t ny,
                     int64_t dim, float* out, float metric_arg);

/* cpu_prims.cpp:61-106 cpu_topk with the total order of cpu_prims.cpp:24-32. Output rows have
   stride min(k, cols). */
void oracle_topk(const float* scores, int64_t rows, int64_t cols, int64_t k, int64_t* indices,
                 float* values, int32_t largest);

/* cpu_prims.cpp:48-58 cpu_gemm (the naive loop: sequential fp32, separate multiply and add).
   round_f16: operands rounded to half first (the F16 compute type of ovvsGemmEx). */
void oracle_gemm(const float* a, const float* b, float* c, int64_t m, int64_t n, int64_t k,
                 int32_t trans_b, int32_t round_f16);

/* cpu_prims.cpp:108-118 cpu_gather_rows (out-of-range index -> zero row). */
void oracle_gather_rows(const float* src, int64_t src_rows, int64_t dim, const int64_t* idx,
                        int64_t nidx, float* out);

/* graphs.cpp:3384-3396 ovvsAllNeighbors; outputs [n x min(k, n - 1)]. */
void oracle_all_neighbors(const float* data, int64_t n, int64_t dim, int32_t metric, int32_t k,
                          int64_t* neighbors, float* distances, int32_t nthreads);

/* mixer.cpp:843-864 brute_search_impl (blocked over queries; same per-element arithmetic).
   nthreads > 1 splits queries across threads, or, for few queries against many rows, rows into
   shards whose top-k lists merge in the reference's total order (results identical). */
void oracle_brute_search(const float* data, int64_t n, int64_t dim, int32_t metric,
                         const float* queries, int64_t nq, int64_t k, const uint8_t* bitset,
                         int64_t* neighbors, float* distances, int32_t nthreads);

/* mixer.cpp:866-921 kmeans_fit_impl. centroids: [min(max(k,1),n) x dim]. Returns the number of
   centroids written, or -1 for invalid arguments. iters is used as given (the ABI wrapper
   cluster.cpp:54 passes max(4, iters)). */
int32_t oracle_kmeans_fit(const float* x, int64_t n, int64_t dim, int32_t k, int32_t iters,
                          float* centroids, int32_t nthreads);

/* One Lloyd step as mixer.cpp:894-918: assign with prim_pairwise(L2) + top-1, then update.
   labels/dist may be NULL. centroids updated in place. */
void oracle_kmeans_step(const float* x, int64_t n, int64_t dim, int32_t k, float* centroids,
                        int64_t* labels, float* dist, int32_t nthreads);

/* cluster.cpp:59-69 ovvsKMeansPredict. */
void oracle_kmeans_predict(const float* centroids, int32_t k, int64_t dim, const float* x,
                           int64_t n, int64_t* labels, float* distances, int32_t nthreads);

/* The rows kmeans_fit_impl seeds from (mixer.cpp:880-890): k_eff row indices. */
int32_t oracle_kmeans_init_rows(int64_t n, int32_t k, int64_t* rows);

/* resources.cpp:218-229. */
int32_t oracle_bitset_from_allow_list(int64_t n, const int64_t* ids, int64_t nids,
                                      uint8_t* bitset);

/* indexes.cpp:281-300 ovvsIvfFlatBuild: nlist_eff = min(nlist, n) centroids (12 Lloyd
   iterations), list_sizes [nlist_eff] and list_ids [n] (the lists concatenated, ascending ids).
   Returns nlist_eff, or -1 for invalid arguments. */
int32_t oracle_ivf_flat_build(const float* x, int64_t n, int64_t dim, int32_t nlist,
                              float* centroids, int64_t* list_sizes, int64_t* list_ids,
                              int32_t nthreads);

/* indexes.cpp:302-358 ovvsIvfFlatSearch over an index given by its parts; outputs [nq x k]. */
void oracle_ivf_flat_search(const float* x, int64_t n, int64_t dim, int32_t metric,
                            const float* centroids, int32_t nlist, const int64_t* list_sizes,
                            const int64_t* list_ids, const float* queries, int64_t nq, int64_t k,
                            int32_t nprobe, const uint8_t* bitset, int64_t* neighbors,
                            float* distances, int32_t nthreads);

#ifdef __cplusplus
}
#endif
