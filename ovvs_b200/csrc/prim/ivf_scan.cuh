// IVF-Flat list scan on the device (reference src/neighbors/indexes.cpp:302-358).
//
// The reference searches one query at a time: it concatenates the rows of the query's nprobe
// probed lists in probe order, scores them with prim_pairwise (the index metric, sequential
// fp32), sets filtered rows to +inf and keeps the k smallest in cpu_topk's total order, whose
// ties go to the lower position in the concatenation. Here the same scores are computed per
// (list, batch of queries that probe it) tile -- a list's rows are read once for up to 64
// queries -- with every score accumulated in the reference's order on CUDA cores, so the results
// are bit-identical. Candidate keys are (order bits of the score, position in the query's
// concatenation), so any split of the work keeps the reference's order exactly.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ovvs {
namespace prim {

constexpr int kIvfPairs = 64;      // (query, probe) pairs per scan work item
constexpr int kIvfRows = 64;       // list rows per tile
constexpr int kIvfMaxSelect = 256; // largest k kept in shared-memory lists (larger k: sort path)

// probe [nq x nprobe] list ids (int64, from the coarse top-k). Writes cum [nq x (nprobe + 1)]:
// cum[q][p] = position of probe p's first row in the query's concatenation, cum[q][nprobe] =
// total rows; list_q_count[c] += number of (q, p) pairs probing list c (zeroed by the caller).
cudaError_t launch_ivf_probe_offsets(const int64_t* probe, int64_t nq, int nprobe,
                                     const int64_t* list_off, int nlist, uint32_t* cum,
                                     int* list_q_count, cudaStream_t stream);

// Groups the (q, p) pairs by list: pair_of[list_q_off[c] + i] = q * nprobe + p for the pairs
// probing list c, in any order (cursor [nlist] zeroed by the caller counts them off).
cudaError_t launch_ivf_group_pairs(const int64_t* probe, int64_t nq, int nprobe, int nlist,
                                   const int* list_q_off, int* cursor, int* pair_of,
                                   cudaStream_t stream);
// item_count[c] = ceil(list_q_count[c] / kIvfPairs) for c < nlist, item_count[nlist] = 0 (an
// exclusive scan of nlist + 1 entries then gives each list's first item and the total).
cudaError_t launch_ivf_item_counts(const int* list_q_count, int nlist, int* item_count,
                                   cudaStream_t stream);

// Scan parameters shared by both modes.
struct IvfScanParams {
  const float* queries;     // [nq x dim] fp32
  const float* q_norm;      // [nq] nrm2sq of each query
  const float* rows;        // [n x dim] fp32 rows in list order
  const float* row_norm;    // [n] nrm2sq of each row (list order)
  const int64_t* row_ids;   // [n] original id of each row (list order)
  const int64_t* list_off;  // [nlist + 1]
  const uint8_t* bitset;    // by original id, or null
  int64_t bitset_bits;      // ids the bitset covers (the dataset rows); others are filtered
  const int* list_q_off;    // [nlist + 1] first pair of each list in pair_of
  const int* pair_of;       // [nq * nprobe] q * nprobe + p, grouped by list
  const int* item_off;      // [nlist + 1] first work item of each list
  const uint32_t* cum;      // [nq x (nprobe + 1)]
  const int64_t* probe;     // [nq x nprobe] probed list ids
  int64_t nq;
  int nprobe;
  int nlist;
  int dim;
  int metric;               // ovvsMetric value
  // select mode: per pair the k_sel smallest keys, [nq * nprobe x k_sel]
  int k_sel;
  uint64_t* cand;
  // sort mode: every candidate's key at keys[seg_base[q] + position]
  const int64_t* seg_base;
  uint64_t* keys;
};

// Upper bound on the number of work items (the grid size): nq * nprobe / kIvfPairs + nlist.
int64_t ivf_max_items(int64_t nq, int nprobe, int nlist);
// Shared memory of the select-mode kernel for a list size k_sel.
size_t ivf_select_smem(int k_sel);

cudaError_t launch_ivf_scan_select(const IvfScanParams& p, int64_t grid, cudaStream_t stream);
cudaError_t launch_ivf_scan_sort(const IvfScanParams& p, int64_t grid, cudaStream_t stream);

// Final top-k per query: merges the nprobe sorted lists of k_sel keys (select mode) -- or takes
// the first k keys of the query's sorted segment (sort mode: merged = null, sorted_keys +
// seg_base) -- decodes positions to ids and re-evaluates each result's score exactly. Writes
// neighbors / distances [nq x k]: -1 / +inf past the query's candidate count, and the negated
// score for inner product (indexes.cpp:346-355).
cudaError_t launch_ivf_emit(const IvfScanParams& p, const uint64_t* sorted_keys, int64_t k,
                            int64_t* neighbors, float* distances, cudaStream_t stream);
// Shared memory of the select-mode emit kernel for k results per query.
size_t ivf_emit_smem(int64_t k);

// Coarse probe selection: for each of `rows` score rows [rows x cols], the ids of its K smallest
// scores in the top-k total order (ties to the lower column), K <= kIvfMaxSelect, written to
// probe [rows x K] (int64). Equal to cpu_topk's first K indices.
cudaError_t launch_ivf_coarse_select(const float* scores, int64_t rows, int cols, int K,
                                     int64_t* probe, cudaStream_t stream);

// Sort mode segments: totals[q] = cum[q][nprobe] for q < nq and totals[nq] = 0 (an exclusive
// scan gives seg_base); then seg_begin/seg_end [nq] = seg_base[q] and seg_base[q] + total.
cudaError_t launch_ivf_totals(const uint32_t* cum, int64_t nq, int nprobe, int64_t* totals,
                              cudaStream_t stream);
cudaError_t launch_ivf_seg_bounds(const int64_t* seg_base, const uint32_t* cum, int64_t nq,
                                  int nprobe, int* seg_begin, int* seg_end, cudaStream_t stream);

// Layout kernels: rows[g] = x[ids[g]] (zero row when the id is outside [0, n_x)) and
// row_norm[g] = nrm2sq(rows[g]), for g < n_rows.
cudaError_t launch_ivf_gather_rows(const float* x, int64_t n_x, int dim, const int64_t* ids,
                                   int64_t n_rows, float* rows, float* row_norm,
                                   cudaStream_t stream);

}  // namespace prim
}  // namespace ovvs
