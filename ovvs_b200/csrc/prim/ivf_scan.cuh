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

// ---- tensor-core list scan (L2 family, k up to 10) --------------------------------------------
// The (query, probe) pairs of each list get "slots": list c's pairs occupy slots
// [slot_off[c], slot_off[c] + list_q_count[c]) of a range padded to whole 256-slot pair tiles, and
// the fused brute-force kernel runs one item per (list, pair tile) over the list's database tiles
// (an item table). Then every pair's two candidate lists are re-scored exactly and written as the
// select-mode candidate lists that launch_ivf_emit merges.

// slot_count[c] = list_q_count[c] rounded up to 256 (0 for an empty list, whose pairs get no
// slot), item_count[c] = slot_count[c] / 256 for c < nlist, and both 0 at c = nlist (exclusive
// scans of nlist + 1 entries give the offsets).
cudaError_t launch_ivf_tc_counts(const int* list_q_count, const int2* list_tiles, int nlist,
                                 int* slot_count, int* item_count, cudaStream_t stream);

// slot_pair[s] = q * nprobe + p of slot s (-1 for padding slots), pair_slot[q * nprobe + p] = s
// (pairs of empty lists keep the caller's -1),
// and item_tab[i] = (pair tile of the slots, first database tile, end database tile, 0) for the
// items of every list; list_tiles[c] = (first tile, end tile) of list c in the padded operand.
cudaError_t launch_ivf_tc_fill(const int* list_q_count, const int* list_q_off, const int* pair_of,
                               const int* slot_off, const int* item_off, const int2* list_tiles,
                               int nlist, int* slot_pair, int* pair_slot, int4* item_tab,
                               cudaStream_t stream);

// Allow bits by padded position for a bitset by original id (allow_pos[w] bit b = position
// 32 w + b; padding positions are not allowed).
cudaError_t launch_ivf_tc_allow(const uint8_t* bitset, int64_t bits, const int64_t* pos_row,
                                const int64_t* row_ids, int64_t n_pos, uint32_t* allow_pos,
                                cudaStream_t stream);

// The fused kernel's query operand per slot: row s of a16_slot = row (slot_pair[s] / nprobe) of
// a16_query (zeros for padding slots), row_halves fp16 values each; q_mul_slot likewise (-1 for
// padding).
cudaError_t launch_ivf_tc_gather(const void* a16_query, const float* q_mul_query,
                                 const int* slot_pair, int nprobe, int64_t slots, int row_halves,
                                 void* a16_slot, float* q_mul_slot, cudaStream_t stream);

// Per pair: its slot's two candidate lists of kl keys (approximate value, padded position) from
// the fused kernel, re-scored exactly (the scan's arithmetic) and keyed by (score, position in
// the query's concatenation); the k_sel smallest, ascending, go to p.cand[pair * k_sel ...].
// pos_row[pos] = the list-order row of a padded position.
cudaError_t launch_ivf_tc_refine(const IvfScanParams& p, const uint64_t* tc_cand, int kl,
                                 const int* pair_slot, const int64_t* pos_row,
                                 cudaStream_t stream);

// Layout kernels: rows[g] = x[ids[g]] (zero row when the id is outside [0, n_x)) and
// row_norm[g] = nrm2sq(rows[g]), for g < n_rows.
cudaError_t launch_ivf_gather_rows(const float* x, int64_t n_x, int dim, const int64_t* ids,
                                   int64_t n_rows, float* rows, float* row_norm,
                                   cudaStream_t stream);

}  // namespace prim
}  // namespace ovvs
