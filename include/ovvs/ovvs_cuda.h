#pragma once

/* B200 extensions to the ovvs C ABI.
 *
 * None of these entry points has a counterpart in the reference (its ABI is single-process,
 * host-pointer only). They exist for two kinds of caller:
 *   - callers whose queries and results already live in GPU memory (device-pointer search), and
 *   - one-process-per-GPU deployments that shard the database rows across GPUs and merge the
 *     per-shard candidates with an NCCL all-gather.
 * Everything here uses the same handles and status codes as ovvs.h. */

#include "ovvs.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- streams and errors ------------------------------------------------------------------ */

/* The cudaStream_t (as void*) that this Resources enqueues its work on. Created on first use. */
OVVS_API ovvsStatus ovvsResourcesStream(ovvsResources_t res, void** stream);

/* Waits for all work enqueued through this Resources and reports what the kernels recorded:
   OVVS_STATUS_ERROR if a kernel's bounded wait gave up (its watchdog), or a CUDA error. */
OVVS_API ovvsStatus ovvsResourcesSynchronize(ovvsResources_t res);

/* CUDA device ordinal this Resources is bound to. */
OVVS_API ovvsStatus ovvsResourcesDevice(ovvsResources_t res, int32_t* device);

/* Per-phase device timing. When enabled, each search records CUDA events on the Resources'
   stream at its phase boundaries; ovvsResourcesLastPhaseMs waits for the last search and writes
   up to `count` durations in milliseconds: [0] query preparation (+ allow bits), [1] fused
   distance / top-k kernel, [2] candidate merge + exact re-rank, [3] cross-shard all-gather and
   merge (0 on one GPU). After a k-means fit the phases are the fit's: [0] dataset upload and
   seeding, [1] the Lloyd iterations, [2] centroid download, [3] 0. After ovvsGemm / ovvsGemmEx /
   ovvsPairwiseDistance: [0] the uploads before the first output block's kernels, [1] those
   kernels (the whole call when the output fits one block, 1 GiB), [2] the rest (downloads and
   any further blocks), [3] 0. */
OVVS_API ovvsStatus ovvsResourcesSetProfiling(ovvsResources_t res, int32_t enable);
OVVS_API ovvsStatus ovvsResourcesLastPhaseMs(ovvsResources_t res, float* ms, int32_t count);

/* The same four phase durations for each of the last searches run while profiling was enabled (up
   to 64, oldest first), so back-to-back searches can be timed without synchronising after each:
   waits for the most recent one, writes min(recorded, max_searches) rows of 4 floats (ms) to `ms`
   and their number to *count, then clears the record (enabling profiling also clears it). Not in
   the reference. */
OVVS_API ovvsStatus ovvsResourcesPhaseHistoryMs(ovvsResources_t res, float* ms,
                                                int32_t max_searches, int32_t* count);

/* ---- kernel watchdog ---------------------------------------------------------------------- */

/* Every wait inside this library's kernels (on a copy, an MMA, another warp or another GPU) is
   bounded in time. A wait that runs out writes a watchdog code into the Resources' error word and
   the kernel unwinds and returns, so the device context stays usable; the next synchronising call
   on the Resources (a search, ovvsResourcesSynchronize) then returns OVVS_STATUS_ERROR. This call
   writes the code that call saw (0 if none) and clears it. Codes: 0x101-0x109 waits of the fused
   kernel (query tile, ring slot empty/full, TMEM buffer empty/full, query tile empty, unwinding,
   side slot empty/full), 0x201 the self test below. Not in the reference. */
OVVS_API ovvsStatus ovvsResourcesLastKernelError(ovvsResources_t res, int32_t* code);

/* 1 when sharded searches on this Resources share each query's bound with the other ranks: the
   fused kernel of every rank min-writes its current k-th best key for a query into every
   rank's bound array (mapped over NVLink from a CUDA virtual-memory allocation each rank
   exports to its peers), so each rank filters with the best bound found on any rank. 0 before
   the first sharded search, when peer memory cannot be shared, for cosine and large-k searches
   (which keep their bound on their own rank), or when OVVS_PEER_BOUNDS=0 is set (on every
   rank). Results are the same either way. Not in the reference. */
OVVS_API ovvsStatus ovvsResourcesPeerBounds(ovvsResources_t res, int32_t* active);

/* Runs a one-block kernel whose bounded wait is never satisfied, with a limit of `limit_ns`
   nanoseconds (1e6..5e9), and checks that the watchdog fired: the kernel returns, the
   synchronising call reports OVVS_STATUS_ERROR and the code is 0x201. Returns
   OVVS_STATUS_SUCCESS and *code = 0x201 when that is what happened. Not in the reference. */
OVVS_API ovvsStatus ovvsWatchdogSelfTest(ovvsResources_t res, int64_t limit_ns, int32_t* code);

/* ---- device-pointer search ---------------------------------------------------------------- */

/* Same contract as ovvsBruteForceSearch, but queries, bitset, neighbors and distances are device
   pointers on the Resources' device, and the call only enqueues work on the Resources' stream
   (no host synchronisation), except for k above the register lists (k beyond 28), where it waits
   for its own work once per pass to check the candidate buffers for overflow. Output rows have
   stride min(k, n). Call ovvsResourcesSynchronize
   (or synchronise the stream) before reading the results. On a sharded Resources the call is
   collective: every rank passes the same queries and receives the global result. */
OVVS_API ovvsStatus ovvsBruteForceSearchDevice(ovvsResources_t res, ovvsBruteForceIndex_t index,
                                               const float* d_queries, int64_t nq, int64_t k,
                                               const uint8_t* d_bitset, int64_t* d_neighbors,
                                               float* d_distances);

/* Same search as ovvsBruteForceSearchDevice for callers that cannot let a library allocate GPU
   memory -- e.g. a process whose free device memory is already reserved by another allocator
   (a framework's caching pool), or a latency-critical request loop where cudaMalloc/cudaFree and
   their implicit device synchronisation are not acceptable. This entry point has no counterpart
   in the reference. It allocates nothing: all intermediate buffers come from a fixed 32 MiB
   device array built into the library, which lives until the process exits. The runtime creates
   the array on a device when it loads that part of the library there; with CUDA's default lazy
   module loading this is the first call on the device, which also looks up the array's address
   (the one-time set-up). So make that first call at start-up, before another allocator takes the
   device's free memory (or set CUDA_MODULE_LOADING=EAGER). Work runs on
   `stream` (NULL = the default stream) and the call returns after it has finished. Sizes whose
   buffers do not fit the array (about 4*dim + 16 + 8*list bytes per query, list = k plus a small
   margin rounded up to 4/8/12/16/32: some 50k queries of dim 128 at k = 10) are rejected with
   OVVS_STATUS_SHAPE_MISMATCH;
   sharded indexes and k above the register-list limit return OVVS_STATUS_UNSUPPORTED. All calls on
   a device share the array and keep the last call's contents; the library clears what must start
   empty and serialises its own calls per device, because calls whose GPU work overlapped on the
   same array would race. */
OVVS_API ovvsStatus ovvsBruteForceSearchDeviceNoAlloc(ovvsResources_t res,
                                                      ovvsBruteForceIndex_t index,
                                                      const float* d_queries, int64_t nq,
                                                      int64_t k, const uint8_t* d_bitset,
                                                      int64_t* d_neighbors, float* d_distances,
                                                      void* stream);

/* Device-pointer IVF-Flat search: the contract of ovvsIvfFlatSearch (reference
   src/neighbors/indexes.cpp:302-358; outputs [nq x k], -1 / +inf past a query's candidates) with
   queries, bitset (indexed by row id, covering the index's rows), neighbors and distances in GPU
   memory on the Resources' device. Enqueues work on the Resources' stream; synchronise before
   reading the results. With the L2 metrics and k <= 10 (the tensor-core list scan) the call also
   waits once per query block for the stream's work so far, to size the scan's work items from
   the probe counts. Not in the reference. */
OVVS_API ovvsStatus ovvsIvfFlatSearchDevice(ovvsResources_t res, ovvsIvfFlatIndex_t index,
                                            const float* d_queries, int64_t nq, int64_t k,
                                            int32_t nprobe, const uint8_t* d_bitset,
                                            int64_t* d_neighbors, float* d_distances);

/* ---- one process per GPU ------------------------------------------------------------------ */

/* Size in bytes of the NCCL unique id that ovvsNcclUniqueId writes (128). */
OVVS_API int32_t ovvsNcclUniqueIdSize(void);

/* Rank 0 calls this once and shares the bytes with every other rank (any transport). */
OVVS_API ovvsStatus ovvsNcclUniqueId(uint8_t* id, int32_t len);

/* Creates a Resources bound to CUDA device `device` that is rank `rank` of `world` ranks. With
   world > 1 it owns an NCCL communicator built from `nccl_id` (collective: all ranks must call).
   Searches and k-means fits through it are collective over the ranks. */
OVVS_API ovvsStatus ovvsResourcesCreateSharded(ovvsResources_t* res, int32_t device,
                                               int32_t rank, int32_t world,
                                               const uint8_t* nccl_id, int32_t len);

/* Builds this rank's shard: `n_local` rows that are rows [row_offset, row_offset + n_local) of
   the global dataset. Search results report global row ids, and a search bitset is indexed by
   global row id. */
OVVS_API ovvsStatus ovvsBruteForceBuildShard(ovvsResources_t res, const void* dataset,
                                             int64_t n_local, int64_t dim, ovvsMetric metric,
                                             ovvsDType dtype, int64_t row_offset,
                                             ovvsBruteForceIndex_t* index);

/* Collective k-means over row shards: rank r passes rows [row_offset, row_offset + n_local) of a
   dataset with n_total rows. Seeding picks the same global rows as ovvsKMeansFit would on the
   whole dataset; per-iteration sums and counts are all-reduced, so every rank ends with the same
   centroids. */
OVVS_API ovvsStatus ovvsKMeansFitShard(ovvsResources_t res, const float* dataset, int64_t n_local,
                                       int64_t row_offset, int64_t n_total, int64_t dim,
                                       int32_t nclusters, int32_t iters,
                                       ovvsKMeansModel_t* model);

#ifdef __cplusplus
}
#endif
