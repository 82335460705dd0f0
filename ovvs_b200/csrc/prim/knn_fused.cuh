// Fused distance + top-k kernel (sm_100a).
//
// Replaces the reference's dense pairwise + top-k pipeline (src/prim/mixer.cpp:843-864 with
// prim_pairwise 174-221 and cpu_topk src/prim/cpu/cpu_prims.cpp:61-106): the nq x n score matrix
// never exists. CTAs work in pairs (clusters of 2, one CTA per SM): a pair loops over work items
// (query pair-tile of 256 = 128 per CTA, super-chunk of database tiles of 256 rows) and shares
// one tcgen05 MMA of M=256 x N=256, so each SM stores and reads only half of every database tile
// (halving each SM's share of the database traffic and of the MMA instruction stream):
//
//   warp 8  TMA producer   (each CTA) loads its 128 queries once per item (resident A) and
//                          streams its 128-row half of each database K-chunk (<= 64 fp16
//                          columns) through an smem ring, completion counted on the leader
//                          CTA's barriers; plus per tile the 256 rows' aux values, ids and
//                          allow bits (2 KB) into a 4-deep side ring that its epilogue reads
//                          on the exact path;
//   warp 9  MMA issuer     (leader CTA only) tcgen05.mma.cta_group::2 kind::f16, M=256 x N=256,
//                          fp32 accumulators in both CTAs' TMEM (each CTA: its 128 queries x
//                          the 256 rows), double-buffered (2 x 256 columns);
//   warps 0-7 epilogue     warps w, w+4 share TMEM lane quarter w % 4 (32 queries, one per
//                          thread) and take columns [0,128) and [128,256): per 32
//                          columns one tcgen05.ld and a 3-input max tree against the query's
//                          current threshold. A lane whose chunk may hold a candidate (on
//                          config 3: 0.14% of a lane's chunks; some lane of the warp in 2.9%
//                          of a warp's chunks) copies it to its private deferred row in shared
//                          memory;
//                          the exact per-column checks + insertions into the thread's sorted
//                          register list of the KL best (value, row id) keys run after the
//                          TMEM buffer is handed back, so with 16 epilogue warps per pair tile
//                          the MMA never waits for the slowest one. Each column part keeps its
//                          own list.
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

constexpr int kTileQ = 128;                // queries per CTA tile: TMEM lanes
constexpr int kPairQ = 2 * kTileQ;         // queries per pair tile: MMA M
constexpr int kTileN = 256;                // database rows per tile: MMA N
constexpr int kHalfN = kTileN / 2;         // rows of each tile held by one CTA of the pair
constexpr int kUnitBytes = kHalfN * 128;   // one smem slot: a 64-column fp16 chunk, 128 rows
constexpr int kEpiWarps = 8;               // two warps per TMEM lane quarter
constexpr int kPartCols = 128;             // columns per epilogue warp (a part of the tile)
constexpr int kListsPerItem = kEpiWarps / 4;  // list-mode output: one sorted list per column part
constexpr int kFusedThreads = 32 * (kEpiWarps + 2);  // epilogue warps, then TMA, then MMA
constexpr int kMaxStages = 16;             // smem ring slots at most
constexpr int kMaxChunks = 66;             // padded dim <= 4096 per part (64 + 32/16 tails)
constexpr int kResChunks = 8;              // resident query tile: at most 8 chunks per part
constexpr int kTmemCols = 512;             // two 256-column fp32 accumulators
constexpr int kMaxPeers = 15;              // other ranks a sharded search shares bounds with
constexpr int kSideBufs = 4;               // side ring depth (tiles)
constexpr int kSideAuxOff = 0;             // side slot: aux[256] fp32
constexpr int kSideIdOff = 1024;           //            row id[256] u32
constexpr int kSideAllowOff = 2048;        //            allow bits[256] (8 words)
constexpr int kSideBytes = 2176;           // slot stride (multiple of 128 bytes)
constexpr int kDeferStride = 33;           // floats per deferred row (32 values + candidate mask;
                                           // 33 keeps the lanes' rows on distinct banks)

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
  int a_off[2][kResChunks];        // resident mode: smem byte offset of query chunk (part, chunk)
  // Streamed mode (a_stream = 1, when the resident query tile does not fit shared memory, i.e.
  // large dims): each ring slot holds a database chunk at +0, the matching query hi chunk at
  // slot_a_off and lo chunk at slot_alo_off, slots slot_bytes apart; no resident query tile.
  int a_stream;
  int slot_bytes;
  int slot_a_off;
  int slot_alo_off;
  int a_tx_bytes[2];               // bytes of one query part (all chunks)
  int b_parts;                     // 1: rows fp16-exact; 2: rows split hi + lo
  int nunits;                      // smem units per database tile = b_parts * nchunk
  int nstages;                     // smem ring slots
  int stage_off;                   // smem byte offset of slot 0
  int side_off;                    // smem byte offset of the side ring
  int defer_off;                   // smem byte offset of the epilogue's deferred rows
  int bar_off;                     // smem byte offset of the mbarriers
  int smem_bytes;                  // dynamic smem requested (includes 1 KB alignment slack)
  int query_split;                 // 1: the query lo part is used when *q_lo_flag != 0
  const int* q_lo_flag;            // set by the query-prep kernel
  int num_qtiles;                  // 128-query tiles (even: queries are padded to kPairQ)
  int num_dbtiles;
  int tiles_per_item;
  int num_sc;                      // super-chunks (items per query pair-tile)
  int num_items;                   // fused_items(num_qtiles, num_sc)
  int64_t n_rows;                  // valid database rows (positions >= n_rows are padding)
  const float* row_aux;            // [n_pad] aux by position
  const float2* group_aux;         // (min, max) of aux per group of 8 consecutive tiles (by
                                   // position: group of tile t = (t * tile_stride) >> 3)
  const uint32_t* row_id;          // [n_pad] position -> row id
  const float* q_mul;              // [q_pad] m_q
  const uint32_t* allow;           // [n_pad / 32] allow bits by position, or null
  int rank_kind;
  int64_t nq;                      // real queries (lanes >= nq are padding and never select)
  int k_pub;                       // rank (1-based) whose key a list publishes as a bound
  uint64_t* q_bound;               // [q_pad] smallest published k_pub-th key per query
  // Sharded searches: the q_bound arrays of the other ranks, mapped from their GPUs. A list
  // whose k_pub-th key beats the bound it last read also min-writes it there, so every rank
  // filters with the best bound found on any rank (rank values are in the same units on every
  // rank: not used for cosine, whose values carry each shard's scale).
  uint64_t* peer_bound[kMaxPeers] = {};
  int n_peers = 0;
  // List mode, L2 / cosine over few rows (k-means centroids, coarse quantisers): the filter
  // compares every column's ranking value with the list's threshold instead of the tile group's
  // conservative bound on s. Rows are sorted by aux, but a group of 8 tiles of a small database
  // spans a wide aux range, so the conservative bound lets many columns through to the exact
  // path; computing each value (one FMA per column with aux from shared memory) costs less.
  int exact_filter = 0;
  // Item table (IVF-Flat list scan): item i = (query pair-tile, first and end database tile),
  // instead of query pair-tiles x equal super-chunks; num_sc = 1. Query rows ("slots") whose
  // slot_pair entry is negative are padding and never select.
  const int4* item_tab = nullptr;
  const int* slot_pair = nullptr;
  uint64_t* out;                   // [q_pad][num_sc][kListsPerItem][KL] sorted keys (list mode;
                                   // one list per column part)
  int* err;                        // watchdog word
  int tile_stride = 1;             // item tile ranges count every tile_stride-th database tile
  int tile_base = 0;               // first database tile of this launch (the launch covers tiles
                                   // [tile_base, tile_base + num_dbtiles))
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
  CUtensorMap b64, b32, b16;  // rows    [n_pad, b_parts * dp] fp16, boxes {64|32|16, 128}
};

// Query rows are padded to whole pair tiles.
inline int64_t pad_queries(int64_t nq) { return (nq + kPairQ - 1) / kPairQ * kPairQ; }
// Work items: query pair-tiles x super-chunks.
inline int fused_items(int num_qtiles, int num_sc) { return num_qtiles / 2 * num_sc; }
// Grid: one CTA pair per two SMs, at most one pair per item.
inline int fused_grid(int num_items, int num_sms) {
  const int pairs = num_items < num_sms / 2 ? num_items : num_sms / 2;
  return 2 * (pairs > 0 ? pairs : 1);
}

// Host-side launcher (knn_fused.cu). `kl` in {4, 8, 12, 16, 32} (sorted register lists), or 0 for
// append mode. `grid` is even (clusters of 2).
cudaError_t launch_knn_fused(const FusedMaps& maps, const FusedParams& p, int kl, int grid,
                             cudaStream_t stream);

// CTA pairs of the fused kernel that can be resident at once on the current device with
// `smem_bytes` of dynamic shared memory per CTA (a pair needs two SMs of one GPC). Cached.
int fused_max_pairs(int smem_bytes);

// Fills the smem layout fields of `p` (offsets, stages) for dim `dp` split into chunks.
// Returns false if the query tile does not fit in shared memory.
bool plan_fused_smem(FusedParams& p, int max_smem_optin);

}  // namespace prim
}  // namespace ovvs
