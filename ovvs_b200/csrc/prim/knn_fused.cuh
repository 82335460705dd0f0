// Fused distance + top-k kernel (sm_100a).
//
// Replaces the reference's dense pairwise + top-k pipeline (src/prim/mixer.cpp:843-864 with
// prim_pairwise 174-221 and cpu_topk src/prim/cpu/cpu_prims.cpp:61-106): the nq x n score matrix
// never exists. One CTA per SM loops over work items (query tile of 128, super-chunk of database
// tiles of 256 rows):
//
//   warp 8  TMA producer   loads the query tile once per item (resident A) and streams database
//                          K-chunks (<= 64 fp16 columns x 256 rows) through an smem ring, plus
//                          per tile the rows' aux values, ids and allow bits (2 KB) into a
//                          4-deep side ring that the epilogue reads on its exact path;
//   warp 9  MMA issuer     tcgen05.mma kind::f16, M=128 (queries) x N=256 (rows), fp32
//                          accumulators in TMEM, double-buffered (2 x 256 columns);
//   warps 0-7 epilogue     warps w and w+4 share TMEM lane quarter w (32 queries, one per
//                          thread) and take 128 of the 256 columns each: four tcgen05.ld of 32
//                          columns issued back to back, one wait, then per 32 columns a 3-input
//                          max tree against the query's current threshold and, rarely, an exact
//                          per-column check + insertion into the thread's sorted register list
//                          of the KL best (value, row id) keys. Each half keeps its own list.
//
// Ranking values ("v", smaller is better) per query q and database position j, from the MMA dot
// product s (queries and rows pre-scaled by powers of two, split into fp16 hi/lo parts when the
// data is not fp16-exact):
//   kRankAffine        v = s * m_q + aux_j     (L2 family: m_q = -2 * 2^-(e_q+e_db), aux = |y|^2)
//   kRankScaled        v = s * m_q             (inner product / Hamming: m_q = -2^-(e_q+e_db))
//   kRankColumnScaled  v = s * aux_j           (cosine: aux = -1/max(|y|, 1e-6))
// Database rows are stored sorted by aux, so the per-tile range [aux_min, aux_max] turns the
// exact test into a column-independent bound on s. Final distances are recomputed exactly from
// the original values by the merge kernel; v only selects candidates.
#pragma once

#include <cstdint>
#include <cuda.h>

#include "keys.cuh"
#include "ptx.cuh"

namespace ovvs {
namespace prim {

constexpr int kTileQ = 128;                // queries per tile: MMA M, TMEM lanes
constexpr int kTileN = 256;                // database rows per tile: MMA N
constexpr int kUnitBytes = kTileN * 128;   // one smem slot: a 64-column fp16 chunk of a tile
constexpr int kEpiWarps = 8;               // two warps per TMEM lane quarter, 128 columns each
constexpr int kListsPerItem = 2;           // list-mode output: one sorted list per column half
constexpr int kFusedThreads = 320;         // warps 0-7 epilogue, 8 TMA, 9 MMA
constexpr int kMaxChunks = 8;              // padded dim <= 512 per part
constexpr int kTmemCols = 512;             // two 256-column fp32 accumulators
constexpr int kSideBufs = 4;               // side ring depth (tiles)
constexpr int kSideAuxOff = 0;             // side slot: aux[256] fp32
constexpr int kSideIdOff = 1024;           //            row id[256] u32
constexpr int kSideAllowOff = 2048;        //            allow bits[256] (8 words)
constexpr int kSideBytes = 2176;           // slot stride (multiple of 128 bytes)

enum RankKind : int { kRankAffine = 0, kRankScaled = 1, kRankColumnScaled = 2 };

// Watchdog codes written to the kernel error word.
enum WatchdogCode : int {
  kErrNone = 0,
  kErrWaitA = 0x101,
  kErrWaitSlotEmpty = 0x102,
  kErrWaitSlotFull = 0x103,
  kErrWaitTmemEmpty = 0x104,
  kErrWaitTmemFull = 0x105,
  kErrWaitAEmpty = 0x106,
  kErrDrain = 0x107,
  kErrWaitSideEmpty = 0x108,
  kErrWaitSideFull = 0x109,
};

struct FusedParams {
  int dp;                          // padded dim per part (multiple of 16)
  int nchunk;                      // K chunks per part
  int chunk_x[kMaxChunks];         // first column of each chunk within a part
  int chunk_w[kMaxChunks];         // chunk width in fp16 elements: 64, 32 or 16
  int a_off[2][kMaxChunks];        // smem byte offset of query chunk (part, chunk)
  int a_tx_bytes[2];               // bytes of one query part (all chunks)
  int b_parts;                     // 1: rows fp16-exact; 2: rows split hi + lo
  int nunits;                      // smem units per database tile = b_parts * nchunk
  int nstages;                     // smem ring slots
  int stage_off;                   // smem byte offset of slot 0
  int side_off;                    // smem byte offset of the side ring
  int bar_off;                     // smem byte offset of the mbarriers
  int smem_bytes;                  // dynamic smem requested (includes 1 KB alignment slack)
  int query_split;                 // 1: the query lo part is used when *q_lo_flag != 0
  const int* q_lo_flag;            // set by the query-prep kernel
  int num_qtiles;
  int num_dbtiles;
  int tiles_per_item;
  int num_sc;                      // super-chunks (items per query tile)
  int num_items;
  int64_t n_rows;                  // valid database rows (positions >= n_rows are padding)
  const float* row_aux;            // [n_pad] aux by position
  const float2* tile_aux;          // [num_dbtiles] (min, max) of aux over the tile's valid rows
  const uint32_t* row_id;          // [n_pad] position -> row id
  const float* q_mul;              // [q_pad] m_q
  const uint32_t* allow;           // [n_pad / 32] allow bits by position, or null
  int rank_kind;
  int64_t nq;                      // real queries (lanes >= nq are padding and never select)
  int k_pub;                       // rank (1-based) whose key a list publishes as a bound
  uint64_t* q_bound;               // [q_pad] smallest published k_pub-th key per query
  uint64_t* out;                   // [q_pad][num_sc][2][KL] sorted keys (list mode; one list per
                                   // column half)
  int* err;                        // watchdog word
  int tile_stride = 1;             // item tile ranges count every tile_stride-th database tile
  // Append mode (KL = 0): every column whose key is within the query's bound q_tau_key[q] is
  // appended to the query's buffer app_buf[q * app_cap + i]; app_count[q] counts them (it may
  // exceed app_cap: the caller then tightens the bound and runs again). With a finite bound value
  // the test is value <= bound value (+ relative slack 1e-5, so near-ties survive for the exact
  // re-rank); otherwise, or with app_exact, it is key <= bound key (kEmptyKey keeps everything).
  const uint64_t* q_tau_key;
  int app_exact;
  uint32_t* app_count;
  uint64_t* app_buf;
  int app_cap;
};

// Every kBoundPeriod tiles each epilogue thread publishes its list's k_pub-th key to q_bound
// (atomicMin) and re-reads the minimum. Any list's k_pub-th key is an upper bound on the
// k_pub-th best key of the whole database for that query, so lists of other work items (which
// start empty) filter with it from their first tile on.
constexpr int kBoundPeriod = 16;

struct FusedMaps {
  CUtensorMap a64, a32, a16;  // queries [q_pad, 2 * dp] fp16, boxes {64|32|16, 128}
  CUtensorMap b64, b32, b16;  // rows    [n_pad, b_parts * dp] fp16, boxes {64|32|16, 256}
};

// Host-side launcher (knn_fused.cu). `kl` in {4, 8, 16, 32} (sorted register lists), or 0 for
// append mode.
cudaError_t launch_knn_fused(const FusedMaps& maps, const FusedParams& p, int kl, int grid,
                             cudaStream_t stream);

// Fills the smem layout fields of `p` (offsets, stages) for dim `dp` split into chunks.
// Returns false if the query tile does not fit in shared memory.
bool plan_fused_smem(FusedParams& p, int max_smem_optin);

}  // namespace prim
}  // namespace ovvs
