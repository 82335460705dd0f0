#pragma once

/* ovvs C ABI, B200 implementation.
 *
 * Every type, enum value and function signature below is ABI-identical to the reference's
 * include/ovvs/ovvs.h, so C, C++, Python (ctypes), Go, Rust and Java consumers load this
 * libovvs.so in place of the reference one without recompiling.
 *
 * What runs on the GPU: the exact brute-force kNN path (build, typed build, search, destroy),
 * the allow-list bitset helper, k-means fit/predict/centroids/destroy, IVF-Flat (build, search,
 * serialize, deserialize, extend, destroy), the dynamic batcher on top of brute-force search,
 * the dense primitives and all-neighbors, and the Resources/status/version plumbing. Every other
 * entry point is
 * exported so that existing binaries still link and `import ovvs` still succeeds, and returns
 * OVVS_STATUS_UNSUPPORTED (see the "Outside this library's scope" section). There is no CPU
 * fallback: without a usable B200 the hot path returns OVVS_STATUS_DEVICE_UNAVAILABLE.
 *
 * Extensions with no counterpart in the reference (device-pointer search, one-process-per-GPU
 * sharding) are declared in ovvs_cuda.h. */

#include "export.h"
#include "status.h"
#include "version.h"

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------------------------ */
/* Enums (values are ABI)                                                                      */
/* ------------------------------------------------------------------------------------------ */

typedef enum ovvsDevice {
  OVVS_DEVICE_AUTO = 0,
  OVVS_DEVICE_CPU = 1,
  OVVS_DEVICE_NPU = 2,
  OVVS_DEVICE_GPU = 3, /* every computation in this library reports GPU */
  OVVS_DEVICE_HETERO = 4
} ovvsDevice;

/* AUTO, the *_IF_FASTER policies, HETERO and FORCE_GPU all run on the B200. FORCE_CPU and
   FORCE_NPU make the hot path return OVVS_STATUS_DEVICE_UNAVAILABLE: a forced device never
   falls back to another one. */
typedef enum ovvsPolicy {
  OVVS_POLICY_AUTO = 0,
  OVVS_POLICY_NPU_IF_FASTER = 1,
  OVVS_POLICY_GPU_IF_FASTER = 2,
  OVVS_POLICY_HETERO = 3,
  OVVS_POLICY_FORCE_NPU = 4,
  OVVS_POLICY_FORCE_GPU = 5,
  OVVS_POLICY_FORCE_CPU = 6
} ovvsPolicy;

/* Reported distances, per metric, for query x and row y:
     L2_EXPANDED        (|x|^2 + |y|^2) - 2 x.y          (may be slightly negative, never clamped)
     L2_SQRT_EXPANDED   sqrt(sum_d (x_d - y_d)^2)
     INNER_PRODUCT      x.y   (neighbours are the LARGEST dot products)
     COSINE_EXPANDED    1 - x.y / (sqrt(max(|x|^2,1e-12)) * sqrt(max(|y|^2,1e-12)))
     BITWISE_HAMMING    number of d where (x_d >= 0) != (y_d >= 0)
     LP_UNEXPANDED      (sum_d |x_d - y_d|^2)^(1/2)   (brute force always uses p = 2)
   Any other value behaves like sum_d (x_d - y_d)^2. */
typedef enum ovvsMetric {
  OVVS_METRIC_L2_EXPANDED = 0,
  OVVS_METRIC_L2_SQRT_EXPANDED = 1,
  OVVS_METRIC_INNER_PRODUCT = 2,
  OVVS_METRIC_COSINE_EXPANDED = 3,
  OVVS_METRIC_BITWISE_HAMMING = 4,
  OVVS_METRIC_LP_UNEXPANDED = 5
} ovvsMetric;

/* Element type of a typed brute-force dataset. F8E4M3, F8E5M2 and F4E2M1 datasets are read as
   raw unsigned bytes, as the reference does. */
typedef enum ovvsDType {
  OVVS_DTYPE_F32 = 0,
  OVVS_DTYPE_F16 = 1,
  OVVS_DTYPE_I8 = 2,
  OVVS_DTYPE_U8 = 3,
  OVVS_DTYPE_F8E4M3 = 4,
  OVVS_DTYPE_F8E5M2 = 5,
  OVVS_DTYPE_F4E2M1 = 6
} ovvsDType;

typedef enum ovvsCagraBuildAlgo {
  OVVS_CAGRA_BUILD_NN_DESCENT = 0,
  OVVS_CAGRA_BUILD_IVF_PQ = 1,
  OVVS_CAGRA_BUILD_ITERATIVE = 2
} ovvsCagraBuildAlgo;

typedef enum ovvsCagraStorage {
  OVVS_CAGRA_STORAGE_AUTO = 0,
  OVVS_CAGRA_STORAGE_FP32 = 1,
  OVVS_CAGRA_STORAGE_FP16 = 2,
  OVVS_CAGRA_STORAGE_FP16_IF_LOSSLESS = 3
} ovvsCagraStorage;

/* ------------------------------------------------------------------------------------------ */
/* Opaque handles                                                                               */
/* ------------------------------------------------------------------------------------------ */

typedef struct ovvsResourcesImpl* ovvsResources_t;
typedef struct ovvsBruteForceIndexImpl* ovvsBruteForceIndex_t;
typedef struct ovvsIvfFlatIndexImpl* ovvsIvfFlatIndex_t;
typedef struct ovvsIvfPqIndexImpl* ovvsIvfPqIndex_t;
typedef struct ovvsIvfRabitqIndexImpl* ovvsIvfRabitqIndex_t;
typedef struct ovvsCagraIndexImpl* ovvsCagraIndex_t;
typedef struct ovvsNnDescentGraphImpl* ovvsNnDescentGraph_t;
typedef struct ovvsVamanaIndexImpl* ovvsVamanaIndex_t;
typedef struct ovvsScannIndexImpl* ovvsScannIndex_t;
typedef struct ovvsHnswIndexImpl* ovvsHnswIndex_t;
typedef struct ovvsKMeansModelImpl* ovvsKMeansModel_t;
typedef struct ovvsSlinkModelImpl* ovvsSlinkModel_t;
typedef struct ovvsSpectralModelImpl* ovvsSpectralModel_t;
typedef struct ovvsPcaModelImpl* ovvsPcaModel_t;
typedef struct ovvsPqModelImpl* ovvsPqModel_t;
typedef struct ovvsSqModelImpl* ovvsSqModel_t;
typedef struct ovvsBinaryQuantizerImpl* ovvsBinaryQuantizer_t;
typedef struct ovvsSpectralEmbedImpl* ovvsSpectralEmbed_t;
typedef struct ovvsBatcherImpl* ovvsBatcher_t;

/* ------------------------------------------------------------------------------------------ */
/* Frozen telemetry structures (sizes and field offsets are ABI: 200 and 256 bytes). This      */
/* library runs no IVF-PQ or CAGRA, so their counters stay zero; the query functions still     */
/* fill abi_version and struct_size as consumers check them.                                   */
/* ------------------------------------------------------------------------------------------ */

#define OVVS_IVF_PQ_SEARCH_STATS_ABI_V1 1u

typedef struct ovvsIvfPqSearchStatsV1 {
  uint32_t abi_version;
  uint32_t struct_size;
  int64_t successful_calls;
  int64_t blocks;
  int64_t queries;
  int64_t tasks;
  int64_t candidate_rows;
  int64_t selected_rows;
  int64_t total_wall_ns;
  int64_t coarse_pairwise_ns;
  int64_t coarse_topk_ns;
  int64_t planning_ns;
  int64_t lut_build_ns;
  int64_t adc_scan_select_ns;
  int64_t shortlist_select_validate_ns;
  int64_t refine_gather_ns;
  int64_t refine_distance_ns;
  int64_t refine_topk_ns;
  int64_t gpu_allocation_calls;
  int64_t gpu_allocation_bytes;
  int64_t gpu_h2d_calls;
  int64_t gpu_h2d_bytes;
  int64_t gpu_d2h_calls;
  int64_t gpu_d2h_bytes;
  int64_t gpu_kernel_launches;
  int64_t gpu_wait_calls;
} ovvsIvfPqSearchStatsV1;

#define OVVS_CAGRA_BUILD_STATS_ABI_V1 1u

typedef struct ovvsCagraBuildStatsV1 {
  uint32_t abi_version;
  uint32_t struct_size;
  int64_t successful_calls;
  int64_t rows;
  int64_t dataset_copy_bytes;
  int64_t initializer_graph_payload_bytes;
  int64_t published_graph_copy_bytes;
  int64_t nndescent_initializer_calls;
  int64_t ivfpq_initializer_calls;
  int64_t iterative_initializer_calls;
  int64_t total_wall_ns;
  int64_t dataset_copy_ns;
  int64_t initializer_ns;
  int64_t optimizer_prune_merge_ns;
  int64_t index_materialize_ns;
  int64_t initializer_final_cpu_calls;
  int64_t initializer_final_gpu_calls;
  int64_t initializer_final_npu_calls;
  int64_t nndescent_gpu_iterations;
  int64_t nndescent_gpu_converged_calls;
  int64_t nndescent_gpu_final_changed_edges;
  int64_t nndescent_gpu_final_pending_new_edges;
  int64_t nndescent_gpu_instrumented_calls;
  int64_t nndescent_gpu_allocation_calls;
  int64_t nndescent_gpu_allocation_bytes;
  int64_t nndescent_gpu_h2d_calls;
  int64_t nndescent_gpu_h2d_bytes;
  int64_t nndescent_gpu_d2h_calls;
  int64_t nndescent_gpu_d2h_bytes;
  int64_t nndescent_gpu_kernel_launches;
  int64_t nndescent_gpu_submission_calls;
  int64_t nndescent_gpu_wait_calls;
  int64_t nndescent_gpu_peak_owned_bytes_max;
} ovvsCagraBuildStatsV1;

#define OVVS_CAGRA_WALK_COUNTER_QUERIES 0
#define OVVS_CAGRA_WALK_COUNTER_EVALS 1
#define OVVS_CAGRA_WALK_COUNTER_SEED_EVALS 2
#define OVVS_CAGRA_WALK_COUNTER_ITERATIONS 3
#define OVVS_CAGRA_WALK_COUNTER_MAX_ITERATIONS 4
#define OVVS_CAGRA_WALK_COUNTER_TABLE_FULL 5
#define OVVS_CAGRA_WALK_COUNTER_ADMITS 6
#define OVVS_CAGRA_WALK_COUNTER_SURVIVORS 7
#define OVVS_CAGRA_WALK_COUNTER_COUNT 8

/* Threading: concurrent searches may share one immutable index when each thread uses its own
   Resources object (each Resources owns its CUDA stream and workspace). Do not destroy an
   index while it is being searched. */

/* ------------------------------------------------------------------------------------------ */
/* Version, status, Resources  (reference src/rt/status.cpp:3-28, src/rt/resources.cpp:14-94) */
/* ------------------------------------------------------------------------------------------ */

OVVS_API const char* ovvsGetVersion(void);
OVVS_API const char* ovvsStatusString(ovvsStatus status);

/* Create: binds the calling thread's Resources to one CUDA device (OVVS_CUDA_DEVICE, default 0)
   and creates its stream lazily. Succeeds without a GPU; GpuAvailable then reports 0 and the hot
   path returns OVVS_STATUS_DEVICE_UNAVAILABLE. */
OVVS_API ovvsStatus ovvsResourcesCreate(ovvsResources_t* res);
OVVS_API ovvsStatus ovvsResourcesDestroy(ovvsResources_t res);
OVVS_API ovvsStatus ovvsResourcesSetPolicy(ovvsResources_t res, ovvsPolicy policy);
OVVS_API ovvsStatus ovvsResourcesGetPolicy(ovvsResources_t res, ovvsPolicy* policy);
OVVS_API ovvsStatus ovvsResourcesNpuAvailable(ovvsResources_t res, int32_t* available);
OVVS_API ovvsStatus ovvsResourcesGpuAvailable(ovvsResources_t res, int32_t* available);
/* Writes the CUDA device name (e.g. "NVIDIA B200"), or "no-cuda-device". */
OVVS_API ovvsStatus ovvsResourcesSku(ovvsResources_t res, char* buf, int32_t len);
OVVS_API ovvsStatus ovvsResourcesNpuCompileFails(ovvsResources_t res, int32_t* count);
OVVS_API ovvsStatus ovvsResourcesNpuFallbacks(ovvsResources_t res, int32_t* count);
OVVS_API ovvsStatus ovvsResourcesLastDevice(ovvsResources_t res, ovvsDevice* device);
OVVS_API ovvsStatus ovvsResourcesLastComputeDtype(ovvsResources_t res, ovvsDType* dtype);
OVVS_API ovvsStatus ovvsResourcesSetCagraWalkCounters(ovvsResources_t res, int32_t enable);
OVVS_API ovvsStatus ovvsResourcesCagraWalkCounters(ovvsResources_t res, int64_t* out,
                                                   int32_t count);
OVVS_API ovvsStatus ovvsResourcesResetCagraWalkCounters(ovvsResources_t res);
OVVS_API ovvsStatus ovvsResourcesCagraTransferStats(ovvsResources_t res, int64_t* walks,
                                                    int64_t* direct_walks,
                                                    int64_t* upload_calls,
                                                    int64_t* upload_bytes);
OVVS_API ovvsStatus ovvsResourcesIvfPqSearchStatsV1(ovvsResources_t res,
                                                    ovvsIvfPqSearchStatsV1* stats);
OVVS_API ovvsStatus ovvsResourcesCagraBuildStatsV1(ovvsResources_t res,
                                                   ovvsCagraBuildStatsV1* stats);
OVVS_API ovvsStatus ovvsResourcesSetNpuBusy(ovvsResources_t res, int32_t busy);
OVVS_API int32_t ovvsSyclEnabled(void);  /* always 0 */
OVVS_API int32_t ovvsGpuHasXmx(void);    /* always -1: no Intel GPU */
OVVS_API ovvsStatus ovvsResourcesEnergyUj(ovvsResources_t res, int64_t* uj); /* UNSUPPORTED */

/* Scalar helpers kept for link compatibility (plain host C, same results as the reference's
   compiler/shave/topk.c and adc.c). */
OVVS_API void ovvsShaveTopkSmallest(const float* scores, int32_t cols, int32_t k, int32_t* idx,
                                    float* val);
OVVS_API float ovvsShavePqAdc(const float* tables, const uint8_t* code, int32_t pq_m, int32_t ks);
OVVS_API ovvsStatus ovvsPqAdcBatch(ovvsResources_t res, const float* tables, int32_t pq_m,
                                   int32_t ks, const uint8_t* codes, int64_t ncodes, float* out);

/* JSON description of the CUDA devices this library sees. */
OVVS_API ovvsStatus ovvsProbeJson(char* buf, int32_t len);

/* ------------------------------------------------------------------------------------------ */
/* Primitives (reference src/rt/resources.cpp:178-216) on the device. Host buffers in and out.  */
/* Results equal the reference's CPU path bit for bit: every output element sums its products  */
/* in k order with separately rounded multiply and add (Lp distances use the device powf and    */
/* may differ by an ulp). Null pointers or non-positive sizes: OVVS_STATUS_INVALID_ARGUMENT.    */
/* ------------------------------------------------------------------------------------------ */

/* C[m x n] = A[m x k] * (trans_b ? B[n x k]^T : B[k x n]), row-major, fp32. */
OVVS_API ovvsStatus ovvsGemm(ovvsResources_t res, const float* a, const float* b, float* c,
                             int64_t m, int64_t n, int64_t k, int32_t trans_b);
/* compute F16 rounds A and B to half before the products (the products are exact in fp32);
   any other type computes in F32. ovvsResourcesLastComputeDtype reports which ran. */
OVVS_API ovvsStatus ovvsGemmEx(ovvsResources_t res, const float* a, const float* b, float* c,
                               int64_t m, int64_t n, int64_t k, int32_t trans_b,
                               ovvsDType compute);
/* Per row the min(k, cols) smallest (largest != 0: largest) scores, ascending (descending),
   ties by lower column, NaN after every number; indices / values are [rows][min(k, cols)]. */
OVVS_API ovvsStatus ovvsTopk(ovvsResources_t res, const float* scores, int64_t rows,
                             int64_t cols, int64_t k, int64_t* indices, float* values,
                             int32_t largest);
/* out[i] = src[idx[i]]; an idx outside [0, src_rows) gives a row of zeros. */
OVVS_API ovvsStatus ovvsGatherRows(ovvsResources_t res, const float* src, int64_t src_rows,
                                   int64_t dim, const int64_t* idx, int64_t nidx, float* out);
/* out[nx][ny]: L2_EXPANDED (squared), INNER_PRODUCT (negated dot), COSINE_EXPANDED through
   norms and the GEMM; L2_SQRT, HAMMING (sign-bit mismatches), LP (p = metric_arg > 0 ?
   metric_arg : 2) per pair. */
OVVS_API ovvsStatus ovvsPairwiseDistance(ovvsResources_t res, ovvsMetric metric, const float* x,
                                         int64_t nx, const float* y, int64_t ny, int64_t dim,
                                         float* out, float metric_arg);
/* Same as ovvsTopk. */
OVVS_API ovvsStatus ovvsKSelection(ovvsResources_t res, const float* scores, int64_t rows,
                                   int64_t cols, int64_t k, int64_t* indices, float* values,
                                   int32_t largest);

/* Exact all-pairs kNN graph on the device (reference src/neighbors/graphs.cpp:3384-3396): per
   row the min(k, n - 1) nearest other rows under ovvsPairwiseDistance's scores (LP with p = 2),
   ascending, ties by lower row; INNER_PRODUCT distances are the dot products. n <= 1 or k <= 0:
   OVVS_STATUS_INVALID_ARGUMENT. */
OVVS_API ovvsStatus ovvsAllNeighbors(ovvsResources_t res, const float* dataset, int64_t n,
                                     int64_t dim, ovvsMetric metric, int32_t k,
                                     int64_t* neighbors, float* distances);

/* ------------------------------------------------------------------------------------------ */
/* Exact brute-force kNN  (reference src/neighbors/indexes.cpp:236-268)                         */
/* ------------------------------------------------------------------------------------------ */

/* Copies the dataset to the GPU (the caller may free it afterwards). F32 rows are kept exact
   for the final distances; F16 rows stay fp16 (decoded exactly); I8/U8 rows are widened. */
OVVS_API ovvsStatus ovvsBruteForceBuild(ovvsResources_t res, const float* dataset, int64_t n,
                                        int64_t dim, ovvsMetric metric,
                                        ovvsBruteForceIndex_t* index);
OVVS_API ovvsStatus ovvsBruteForceBuildTyped(ovvsResources_t res, const void* dataset, int64_t n,
                                             int64_t dim, ovvsMetric metric, ovvsDType dtype,
                                             ovvsBruteForceIndex_t* index);
/* queries: host fp32 [nq x dim]; bitset: NULL or (n+7)/8 bytes, bit j (LSB first) = row j
   allowed; neighbors/distances: host [nq x min(k, n)], each row ascending by distance (descending
   by dot product for INNER_PRODUCT), ties by lower row id, NaN last. Filtered rows are returned
   with distance +inf (-inf for INNER_PRODUCT) only when fewer than k rows are allowed. */
OVVS_API ovvsStatus ovvsBruteForceSearch(ovvsResources_t res, ovvsBruteForceIndex_t index,
                                         const float* queries, int64_t nq, int64_t k,
                                         const uint8_t* bitset, int64_t* neighbors,
                                         float* distances);
OVVS_API ovvsStatus ovvsBruteForceDestroy(ovvsBruteForceIndex_t index);

/* ------------------------------------------------------------------------------------------ */
/* IVF-Flat  (reference src/neighbors/indexes.cpp:281-457)                                      */
/* ------------------------------------------------------------------------------------------ */

/* Build: nlist = min(nlist, n) lists from a 12-iteration k-means fit (squared L2) and each row's
   nearest centroid; the dataset is copied. Search: per query the nprobe nearest lists (nprobe
   clamped to [1, nlist]) are scored exactly with the index metric; neighbors/distances are host
   [nq x k], ties go to the earlier row in probe order, and -1 / +inf fill the rows past a query's
   candidates. Serialize/Deserialize use the reference's 'IVF1' file format. Extend appends rows
   (ids n, n+1, ...) to the lists of their nearest centroids. */
OVVS_API ovvsStatus ovvsIvfFlatBuild(ovvsResources_t res, const float* dataset, int64_t n,
                                     int64_t dim, ovvsMetric metric, int32_t nlist,
                                     ovvsIvfFlatIndex_t* index);
OVVS_API ovvsStatus ovvsIvfFlatSearch(ovvsResources_t res, ovvsIvfFlatIndex_t index,
                                      const float* queries, int64_t nq, int64_t k,
                                      int32_t nprobe, const uint8_t* bitset, int64_t* neighbors,
                                      float* distances);
OVVS_API ovvsStatus ovvsIvfFlatSerialize(ovvsIvfFlatIndex_t index, const char* path);
OVVS_API ovvsStatus ovvsIvfFlatDeserialize(ovvsResources_t res, const char* path,
                                           ovvsIvfFlatIndex_t* index);
OVVS_API ovvsStatus ovvsIvfFlatExtend(ovvsResources_t res, ovvsIvfFlatIndex_t index,
                                      const float* extra, int64_t nextra);
OVVS_API ovvsStatus ovvsIvfFlatDestroy(ovvsIvfFlatIndex_t index);

/* ------------------------------------------------------------------------------------------ */
/* Outside this library's scope: exported, return OVVS_STATUS_UNSUPPORTED.                      */
/* ------------------------------------------------------------------------------------------ */

OVVS_API ovvsStatus ovvsIvfPqBuild(ovvsResources_t res, const float* dataset, int64_t n,
                                   int64_t dim, ovvsMetric metric, int32_t nlist, int32_t pq_m,
                                   int32_t pq_nbits, ovvsIvfPqIndex_t* index);
OVVS_API ovvsStatus ovvsIvfPqSearch(ovvsResources_t res, ovvsIvfPqIndex_t index,
                                    const float* queries, int64_t nq, int64_t k, int32_t nprobe,
                                    int32_t krefine, const uint8_t* bitset, int64_t* neighbors,
                                    float* distances);
OVVS_API ovvsStatus ovvsIvfPqSerialize(ovvsIvfPqIndex_t index, const char* path);
OVVS_API ovvsStatus ovvsIvfPqDeserialize(ovvsResources_t res, const char* path,
                                         ovvsIvfPqIndex_t* index);
OVVS_API ovvsStatus ovvsIvfPqExtend(ovvsResources_t res, ovvsIvfPqIndex_t index,
                                    const float* extra, int64_t nextra);
OVVS_API ovvsStatus ovvsIvfPqDestroy(ovvsIvfPqIndex_t index);

OVVS_API ovvsStatus ovvsIvfRabitqBuild(ovvsResources_t res, const float* dataset, int64_t n,
                                       int64_t dim, ovvsMetric metric, int32_t nlist,
                                       ovvsIvfRabitqIndex_t* index);
OVVS_API ovvsStatus ovvsIvfRabitqSearch(ovvsResources_t res, ovvsIvfRabitqIndex_t index,
                                        const float* queries, int64_t nq, int64_t k,
                                        int32_t nprobe, int32_t krefine, const uint8_t* bitset,
                                        int64_t* neighbors, float* distances);
OVVS_API ovvsStatus ovvsIvfRabitqSerialize(ovvsIvfRabitqIndex_t index, const char* path);
OVVS_API ovvsStatus ovvsIvfRabitqDeserialize(ovvsResources_t res, const char* path,
                                             ovvsIvfRabitqIndex_t* index);
OVVS_API ovvsStatus ovvsIvfRabitqExtend(ovvsResources_t res, ovvsIvfRabitqIndex_t index,
                                        const float* extra, int64_t nextra);
OVVS_API ovvsStatus ovvsIvfRabitqDestroy(ovvsIvfRabitqIndex_t index);

OVVS_API ovvsStatus ovvsNnDescentBuild(ovvsResources_t res, const float* dataset, int64_t n,
                                       int64_t dim, ovvsMetric metric, int32_t graph_degree,
                                       int32_t iterations, ovvsNnDescentGraph_t* graph);
OVVS_API ovvsStatus ovvsNnDescentNeighbors(ovvsNnDescentGraph_t graph, const int32_t** ids,
                                           int64_t* n, int32_t* degree);
OVVS_API ovvsStatus ovvsNnDescentDestroy(ovvsNnDescentGraph_t graph);

OVVS_API ovvsStatus ovvsCagraBuild(ovvsResources_t res, const float* dataset, int64_t n,
                                   int64_t dim, ovvsMetric metric, int32_t graph_degree,
                                   int32_t intermediate_degree, ovvsCagraIndex_t* index);
OVVS_API ovvsStatus ovvsCagraBuildEx(ovvsResources_t res, const float* dataset, int64_t n,
                                     int64_t dim, ovvsMetric metric, int32_t graph_degree,
                                     int32_t intermediate_degree, ovvsCagraBuildAlgo algo,
                                     ovvsCagraIndex_t* index);
OVVS_API ovvsStatus ovvsCagraBuildEx2(ovvsResources_t res, const float* dataset, int64_t n,
                                      int64_t dim, ovvsMetric metric, int32_t graph_degree,
                                      int32_t intermediate_degree, ovvsCagraBuildAlgo algo,
                                      ovvsCagraStorage storage, ovvsCagraIndex_t* index);
OVVS_API ovvsStatus ovvsCagraSearch(ovvsResources_t res, ovvsCagraIndex_t index,
                                    const float* queries, int64_t nq, int64_t k,
                                    int32_t itopk_size, int32_t search_width,
                                    const uint8_t* bitset, int64_t* neighbors, float* distances);
OVVS_API ovvsStatus ovvsCagraWalOpen(ovvsResources_t res, ovvsCagraIndex_t index,
                                     const char* path, int32_t fsync_every);
OVVS_API ovvsStatus ovvsCagraWalClose(ovvsCagraIndex_t index);
OVVS_API ovvsStatus ovvsCagraCalibrate(ovvsResources_t res, ovvsCagraIndex_t index,
                                       float target_recall, int64_t k, int32_t* itopk,
                                       int32_t* width, float* achieved);
OVVS_API ovvsStatus ovvsCagraQuantize(ovvsResources_t res, ovvsCagraIndex_t index, int32_t pq_m,
                                      int32_t pq_nbits);
OVVS_API ovvsStatus ovvsCagraDetachDataset(ovvsCagraIndex_t index);
OVVS_API ovvsStatus ovvsCagraAttachDataset(ovvsCagraIndex_t index, const float* dataset,
                                           int64_t n, int64_t dim);
OVVS_API ovvsStatus ovvsCagraSerialize(ovvsCagraIndex_t index, const char* path);
OVVS_API ovvsStatus ovvsCagraSerializeEx(ovvsCagraIndex_t index, const char* path,
                                         int32_t include_dataset);
OVVS_API ovvsStatus ovvsCagraDeserialize(ovvsResources_t res, const char* path,
                                         ovvsCagraIndex_t* index);
OVVS_API ovvsStatus ovvsCagraExtend(ovvsResources_t res, ovvsCagraIndex_t index,
                                    const float* extra, int64_t nextra);
OVVS_API ovvsStatus ovvsCagraExtendEx(ovvsResources_t res, ovvsCagraIndex_t index,
                                      const float* extra, int64_t nextra, int64_t* out_ids);
OVVS_API ovvsStatus ovvsCagraDelete(ovvsResources_t res, ovvsCagraIndex_t index,
                                    const int64_t* ids, int64_t nids);
OVVS_API ovvsStatus ovvsCagraUpdate(ovvsResources_t res, ovvsCagraIndex_t index,
                                    const int64_t* ids, const float* vectors, int64_t nids);
OVVS_API ovvsStatus ovvsCagraCounts(ovvsCagraIndex_t index, int64_t* live, int64_t* deleted);
OVVS_API ovvsStatus ovvsCagraDestroy(ovvsCagraIndex_t index);

OVVS_API ovvsStatus ovvsHnswFromCagra(ovvsResources_t res, ovvsCagraIndex_t cagra,
                                      ovvsHnswIndex_t* index);
OVVS_API ovvsStatus ovvsHnswSearch(ovvsResources_t res, ovvsHnswIndex_t index,
                                   const float* queries, int64_t nq, int64_t k, int32_t ef,
                                   int64_t* neighbors, float* distances);
OVVS_API ovvsStatus ovvsHnswSerialize(ovvsHnswIndex_t index, const char* path);
OVVS_API ovvsStatus ovvsHnswDeserialize(ovvsResources_t res, const char* path,
                                        ovvsHnswIndex_t* index);
OVVS_API ovvsStatus ovvsHnswDestroy(ovvsHnswIndex_t index);

OVVS_API ovvsStatus ovvsVamanaBuild(ovvsResources_t res, const float* dataset, int64_t n,
                                    int64_t dim, ovvsMetric metric, int32_t graph_degree,
                                    float alpha, ovvsVamanaIndex_t* index);
OVVS_API ovvsStatus ovvsVamanaSearch(ovvsResources_t res, ovvsVamanaIndex_t index,
                                     const float* queries, int64_t nq, int64_t k, int32_t beam,
                                     const uint8_t* bitset, int64_t* neighbors,
                                     float* distances);
OVVS_API ovvsStatus ovvsVamanaSerialize(ovvsVamanaIndex_t index, const char* path);
OVVS_API ovvsStatus ovvsVamanaDeserialize(ovvsResources_t res, const char* path,
                                          ovvsVamanaIndex_t* index);
OVVS_API ovvsStatus ovvsVamanaMmap(ovvsResources_t res, const char* path,
                                   ovvsVamanaIndex_t* index);
OVVS_API ovvsStatus ovvsVamanaDestroy(ovvsVamanaIndex_t index);

OVVS_API ovvsStatus ovvsScannBuild(ovvsResources_t res, const float* dataset, int64_t n,
                                   int64_t dim, ovvsMetric metric, int32_t nlist, int32_t pq_m,
                                   ovvsScannIndex_t* index);
OVVS_API ovvsStatus ovvsScannSearch(ovvsResources_t res, ovvsScannIndex_t index,
                                    const float* queries, int64_t nq, int64_t k, int32_t nprobe,
                                    int32_t krefine, int64_t* neighbors, float* distances);
OVVS_API ovvsStatus ovvsScannDestroy(ovvsScannIndex_t index);

/* ------------------------------------------------------------------------------------------ */
/* Allow-list bitset  (reference src/rt/resources.cpp:218-229)                                 */
/* ------------------------------------------------------------------------------------------ */

/* Writes (n+7)/8 bytes: bit id (LSB first) set for every id in [0, n) listed in ids; ids outside
   the range are ignored. Host-only, no GPU needed. */
OVVS_API ovvsStatus ovvsBitsetFromAllowList(int64_t n, const int64_t* ids, int64_t nids,
                                            uint8_t* bitset);

/* ------------------------------------------------------------------------------------------ */
/* k-means (Lloyd)  (reference src/cluster/cluster.cpp:46-84, src/prim/mixer.cpp:866-921)     */
/* ------------------------------------------------------------------------------------------ */

/* Runs max(4, iters) Lloyd iterations with min(nclusters, n) centroids seeded from rows chosen
   by std::mt19937(42), exactly as the reference. Assignment ties go to the lower centroid id;
   empty clusters keep their previous centroid. */
OVVS_API ovvsStatus ovvsKMeansFit(ovvsResources_t res, const float* dataset, int64_t n,
                                  int64_t dim, int32_t nclusters, int32_t iters,
                                  ovvsKMeansModel_t* model);
/* labels: host int64 [n]; distances: NULL or host fp32 [n] squared L2 to the chosen centroid. */
OVVS_API ovvsStatus ovvsKMeansPredict(ovvsResources_t res, ovvsKMeansModel_t model,
                                      const float* x, int64_t n, int64_t* labels,
                                      float* distances);
/* *data stays valid until ovvsKMeansDestroy (a host mirror owned by the model). */
OVVS_API ovvsStatus ovvsKMeansCentroids(ovvsKMeansModel_t model, const float** data,
                                        int32_t* nclusters, int64_t* dim);
OVVS_API ovvsStatus ovvsKMeansDestroy(ovvsKMeansModel_t model);

/* Outside this library's scope: exported, return OVVS_STATUS_UNSUPPORTED. */
OVVS_API ovvsStatus ovvsSlinkFit(ovvsResources_t res, const float* dataset, int64_t n,
                                 int64_t dim, int32_t nclusters, int32_t knn,
                                 ovvsSlinkModel_t* model);
OVVS_API ovvsStatus ovvsSlinkLabels(ovvsSlinkModel_t model, const int64_t** labels, int64_t* n);
OVVS_API ovvsStatus ovvsSlinkDestroy(ovvsSlinkModel_t model);
OVVS_API ovvsStatus ovvsSpectralFit(ovvsResources_t res, const float* dataset, int64_t n,
                                    int64_t dim, int32_t nclusters, int32_t knn,
                                    ovvsSpectralModel_t* model);
OVVS_API ovvsStatus ovvsSpectralLabels(ovvsSpectralModel_t model, const int64_t** labels,
                                       int64_t* n);
OVVS_API ovvsStatus ovvsSpectralDestroy(ovvsSpectralModel_t model);
OVVS_API ovvsStatus ovvsSqFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim,
                              ovvsSqModel_t* model);
OVVS_API ovvsStatus ovvsSqEncode(ovvsSqModel_t model, const float* x, int64_t n, uint8_t* codes);
OVVS_API ovvsStatus ovvsSqDecode(ovvsSqModel_t model, const uint8_t* codes, int64_t n, float* x);
OVVS_API ovvsStatus ovvsSqDestroy(ovvsSqModel_t model);
OVVS_API ovvsStatus ovvsPqFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim,
                              int32_t pq_m, int32_t pq_nbits, ovvsPqModel_t* model);
OVVS_API ovvsStatus ovvsPqEncode(ovvsPqModel_t model, const float* x, int64_t n, uint8_t* codes);
OVVS_API ovvsStatus ovvsPqDecode(ovvsPqModel_t model, const uint8_t* codes, int64_t n, float* x);
OVVS_API ovvsStatus ovvsPqDestroy(ovvsPqModel_t model);
OVVS_API ovvsStatus ovvsBinaryFit(ovvsResources_t res, const float* dataset, int64_t n,
                                  int64_t dim, ovvsBinaryQuantizer_t* model);
OVVS_API ovvsStatus ovvsBinaryEncode(ovvsBinaryQuantizer_t model, const float* x, int64_t n,
                                     uint8_t* codes);
OVVS_API ovvsStatus ovvsBinaryDestroy(ovvsBinaryQuantizer_t model);
OVVS_API ovvsStatus ovvsPcaFit(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim,
                               int32_t ncomp, ovvsPcaModel_t* model);
OVVS_API ovvsStatus ovvsPcaTransform(ovvsPcaModel_t model, const float* x, int64_t n,
                                     float* out);
OVVS_API ovvsStatus ovvsPcaDestroy(ovvsPcaModel_t model);
OVVS_API ovvsStatus ovvsSpectralEmbedFit(ovvsResources_t res, const float* dataset, int64_t n,
                                         int64_t dim, int32_t ncomp, int32_t knn,
                                         ovvsSpectralEmbed_t* model);
OVVS_API ovvsStatus ovvsSpectralEmbedData(ovvsSpectralEmbed_t model, const float** data,
                                          int64_t* n, int32_t* ncomp);
OVVS_API ovvsStatus ovvsSpectralEmbedDestroy(ovvsSpectralEmbed_t model);

/* ------------------------------------------------------------------------------------------ */
/* Dynamic batcher over a brute-force index  (reference src/rt/batcher.cpp:65-138)              */
/* ------------------------------------------------------------------------------------------ */

/* Concurrent small searches are queued and issued as one ovvsBruteForceSearch once max_batch
   queries are queued, the requested k changes, or max_wait_ms has passed. Results equal the
   eager search's. */
OVVS_API ovvsStatus ovvsBatcherCreate(ovvsResources_t res, ovvsBruteForceIndex_t index,
                                      int32_t max_batch, int32_t max_wait_ms,
                                      ovvsBatcher_t* out);
OVVS_API ovvsStatus ovvsBatcherSearch(ovvsBatcher_t batcher, const float* queries, int64_t nq,
                                      int64_t k, int64_t* neighbors, float* distances);
OVVS_API ovvsStatus ovvsBatcherLastBatchSize(ovvsBatcher_t batcher, int32_t* nq);
OVVS_API ovvsStatus ovvsBatcherDestroy(ovvsBatcher_t batcher);

#ifdef __cplusplus
}
#endif
