// Fused distance + top-k kernel. Design notes in knn_fused.cuh.
#include "knn_fused.cuh"
#include "prep.cuh"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

namespace ovvs {
namespace prim {
namespace {

using keys::kEmptyKey;

constexpr float kInf = __builtin_huge_valf();

struct Smem {
  uint8_t* base;
  uint64_t* full;    // [nstages] TMA -> MMA
  uint64_t* empty;   // [nstages] MMA -> TMA
  uint64_t* tfull;   // [2] MMA -> epilogue
  uint64_t* tempty;  // [2] epilogue -> MMA (one arrival per epilogue warp)
  uint64_t* afull;   // query tile landed
  uint64_t* aempty;  // MMA done with the query tile
  uint64_t* drain;   // final MMA completion
  uint64_t* side_full;   // [kSideBufs] side data landed
  uint64_t* side_empty;  // [kSideBufs] epilogue done with the slot (one arrival per warp)
  uint8_t* side;         // [kSideBufs][kSideBytes]
  float* defer;          // [kEpiWarps * 32][kDeferStride] one deferred chunk row per epilogue lane
  uint32_t* tmem_slot;
  volatile int* abort;
};

__device__ __forceinline__ Smem carve(const FusedParams& p, uint8_t* raw) {
  Smem s;
  s.base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(s.base + p.bar_off);
  s.full = bars;
  s.empty = bars + p.nstages;
  s.tfull = s.empty + p.nstages;
  s.tempty = s.tfull + 2;
  s.afull = s.tempty + 2;
  s.aempty = s.afull + 1;
  s.drain = s.aempty + 1;
  s.side_full = s.drain + 1;
  s.side_empty = s.side_full + kSideBufs;
  s.side = s.base + p.side_off;
  s.defer = reinterpret_cast<float*>(s.base + p.defer_off);
  s.tmem_slot = reinterpret_cast<uint32_t*>(s.side_empty + kSideBufs);
  s.abort = reinterpret_cast<volatile int*>(s.tmem_slot + 1);
  return s;
}

__device__ __forceinline__ const CUtensorMap* pick_map(int w, const CUtensorMap* m64,
                                                       const CUtensorMap* m32,
                                                       const CUtensorMap* m16) {
  return w == 64 ? m64 : (w == 32 ? m32 : m16);
}

// Work item -> (query pair-tile, super-chunk, tile range); this CTA's query tile is
// qt = 2 * pair-tile + rank. Items are ordered super-chunk-major so that pairs running at the
// same time stream the same database tiles (L2 reuse). Pair c of the grid runs items c, c +
// pairs, c + 2 * pairs, ...
struct Item {
  int qt, sc, t0, t1;
};
__device__ __forceinline__ Item item_of(const FusedParams& p, int item, uint32_t rank) {
  Item it;
  if (p.item_tab != nullptr) {
    const int4 e = p.item_tab[item];
    it.qt = 2 * e.x + static_cast<int>(rank);
    it.sc = 0;
    it.t0 = e.y;
    it.t1 = e.z;
    return it;
  }
  const int num_qpairs = p.num_qtiles >> 1;
  const int qp = item % num_qpairs;
  it.qt = 2 * qp + static_cast<int>(rank);
  it.sc = item / num_qpairs;
  it.t0 = p.tile_base + it.sc * p.tiles_per_item;
  it.t1 = min(it.t0 + p.tiles_per_item, p.tile_base + p.num_dbtiles);
  return it;
}
__device__ __forceinline__ int first_item() { return static_cast<int>(blockIdx.x >> 1); }
__device__ __forceinline__ int item_step() { return static_cast<int>(gridDim.x >> 1); }

// Bounded wait used only while unwinding: ignores the abort flag (the copies or MMAs it waits
// for complete on their own), still gives up after the time limit: the normal limit when the
// CTA finished its work, 20 ms after an abort (in-flight copies land within microseconds; the
// phase may never complete because the other role stopped).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, int* err,
                                           volatile int* abort) {
  if (ptx::mbar_try_wait(bar, parity)) return;
  const uint64_t limit = *abort ? 20000000ull : ptx::kWaitLimitNs;
  const uint64_t t0 = ptx::globaltimer();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::globaltimer() - t0 > limit) {
      atomicCAS(err, 0, kErrDrain);
      return;
    }
  }
}

// ------------------------------------------------------------------------------------------
// TMA producer (one thread)
// ------------------------------------------------------------------------------------------
// Per tile: the 256 rows' aux values, ids and allow bits into side slot tile % kSideBufs, once
// the epilogue has released it. Returns false when the wait gave up.
__device__ __forceinline__ bool load_side(const FusedParams& p, const Smem& s, int t,
                                          uint32_t tile, bool need_aux, uint32_t side_tx) {
  const uint32_t sb = tile % kSideBufs, suse = tile / kSideBufs;
  if (suse > 0 && !ptx::mbar_wait(&s.side_empty[sb], (suse - 1) & 1, s.abort, p.err,
                                  kErrWaitSideEmpty))
    return false;
  const int64_t pos0 = static_cast<int64_t>(t) * p.tile_stride * kTileN;
  uint8_t* slot_side = s.side + sb * kSideBytes;
  ptx::mbar_arrive_expect_tx(&s.side_full[sb], side_tx);
  if (need_aux) ptx::bulk_load(slot_side + kSideAuxOff, p.row_aux + pos0, 1024, &s.side_full[sb]);
  ptx::bulk_load(slot_side + kSideIdOff, p.row_id + pos0, 1024, &s.side_full[sb]);
  if (p.allow) ptx::bulk_load(slot_side + kSideAllowOff, p.allow + pos0 / 32, 32, &s.side_full[sb]);
  return true;
}

// Both CTAs of the pair run a producer: each loads its own 128 queries and its own 128-row half
// of every database chunk into its own shared memory. The copies are counted on the leader's
// full / afull barriers (the leader arms them with the bytes of both CTAs); each producer learns
// that a slot may be refilled from its own empty / aempty barrier, which the leader's MMA
// commits reach in both CTAs.
__device__ void run_producer(const FusedParams& p, const FusedMaps& maps, const Smem& s, bool lo,
                             uint32_t rank) {
  const bool leader = rank == 0;
  const uint32_t full_l = ptx::peer_addr(s.full, 0);  // leader's full[0]
  const uint32_t afull_l = ptx::peer_addr(s.afull, 0);
  uint32_t unit = 0, tile = 0;
  uint32_t slot = 0, phase = 0;  // ring position; `phase` = parity of the current pass
  bool wrapped = false;          // a slot is refilled only after its previous use was consumed
  const bool need_aux = p.rank_kind != kRankScaled;
  const uint32_t side_tx = (need_aux ? 1024u : 0u) + 1024u + (p.allow ? 32u : 0u);
  int a_loads = 0;
  int cur_qt = -1;
  bool ok = true;
  for (int item = first_item(); item < p.num_items && ok; item += item_step()) {
    const Item it = item_of(p, item, rank);
    if (it.qt != cur_qt) {
      if (a_loads > 0 &&
          !ptx::mbar_wait(s.aempty, (a_loads - 1) & 1, s.abort, p.err, kErrWaitAEmpty)) {
        ok = false;
        break;
      }
      if (leader)
        ptx::mbar_arrive_expect_tx(s.afull, 2 * (p.a_tx_bytes[0] + (lo ? p.a_tx_bytes[1] : 0)));
      for (int part = 0; part < (lo ? 2 : 1); ++part) {
        for (int c = 0; c < p.nchunk; ++c) {
          const int w = p.chunk_w[c];
          ptx::tma_load_2d_pair(s.base + p.a_off[part][c],
                                pick_map(w, &maps.a64, &maps.a32, &maps.a16),
                                part * p.dp + p.chunk_x[c], it.qt * kTileQ, afull_l);
        }
      }
      ++a_loads;
      cur_qt = it.qt;
    }
    for (int t = it.t0; t < it.t1 && ok; ++t) {
      // Side data first: the epilogue needs it only after this tile's MMAs.
      if (!load_side(p, s, t, tile, need_aux, side_tx)) {
        ok = false;
        break;
      }
      ++tile;
      // Units in MMA order: database part bp major, chunk c minor. The chunk loop is unrolled so
      // the per-chunk parameters are static-index loads, and the ring position is tracked
      // without division (like the MMA thread's).
      const int row = t * p.tile_stride * kTileN + static_cast<int>(rank) * kHalfN;
      for (int bp = 0; bp < p.b_parts && ok; ++bp) {
#pragma unroll
        for (int c = 0; c < kResChunks; ++c) {
          if (c >= p.nchunk) break;
          if (wrapped &&
              !ptx::mbar_wait(&s.empty[slot], phase ^ 1u, s.abort, p.err, kErrWaitSlotEmpty)) {
            ok = false;
            break;
          }
          const int w = p.chunk_w[c];
          if (leader)
            ptx::mbar_arrive_expect_tx(&s.full[slot], static_cast<uint32_t>(kTileN * w * 2));
          ptx::tma_load_2d_pair(s.base + p.stage_off + slot * kUnitBytes,
                                pick_map(w, &maps.b64, &maps.b32, &maps.b16),
                                bp * p.dp + p.chunk_x[c], row, full_l + slot * 8);
          ++unit;
          if (++slot == static_cast<uint32_t>(p.nstages)) {
            slot = 0;
            phase ^= 1u;
            wrapped = true;
          }
        }
      }
    }
  }
  // Unwind: every copy this thread issued must have landed before the CTA exits. B copies count
  // on the leader's barriers, so this CTA waits for their consumption instead: the MMA commit
  // that frees the last use of each slot (empty, phase of that use), and the final MMA
  // completion for the query tile. Side copies count on this CTA's own barriers.
  const uint32_t issued = unit;
  for (uint32_t slot = 0; slot < static_cast<uint32_t>(p.nstages) && slot < issued; ++slot) {
    const uint32_t last = ((issued - 1 - slot) / p.nstages) * p.nstages + slot;
    drain_wait(&s.empty[slot], (last / p.nstages) & 1, p.err, s.abort);
  }
  if (a_loads > 0) drain_wait(s.drain, 0, p.err, s.abort);
  for (uint32_t sb = 0; sb < static_cast<uint32_t>(kSideBufs) && sb < tile; ++sb) {
    const uint32_t last = ((tile - 1 - sb) / kSideBufs) * kSideBufs + sb;
    drain_wait(&s.side_full[sb], (last / kSideBufs) & 1, p.err, s.abort);
  }
}

// ------------------------------------------------------------------------------------------
// MMA issuer (one thread)
// ------------------------------------------------------------------------------------------
// One thread feeds the tensor core: at D=128 a tile is 8 MMAs of 128 cycles each, so the whole
// per-tile loop (waits, fences, commits, descriptor arithmetic) has to stay under 1,024 cycles or
// the tensor core idles. The loop therefore carries no branch between the MMAs of a unit: the
// query-lo pass (LO) and the K steps per chunk (KS: 4, 2 or 1 for chunks of 64, 32 or 16
// columns; 0 = chunks of mixed widths, dispatched once per chunk) are template parameters, and
// run_mma_dispatch picks the instance once per launch. Descriptors are built once per chunk and
// kept in registers (the chunk loop is unrolled over kResChunks so every index is static); the
// ring position is tracked without division.
constexpr uint32_t kIdesc = ptx::idesc_f16_f32(kPairQ, kTileN);
// Descriptor address fields count 16-byte units; a K step of 16 fp16 values is 32 bytes.
constexpr uint64_t kStepDesc = 32 >> 4;
constexpr uint64_t kSlotDesc = kUnitBytes >> 4;

// The MMAs of one unit (one chunk of one database part): K steps of 16, each against the query's
// hi part and, with LO, its lo part. `acc` = 0 only for the first unit of a tile.
template <bool LO, int KS>
__device__ __forceinline__ void issue_unit(uint32_t d_tmem, uint64_t a_hi, uint64_t a_lo,
                                           uint64_t bd, uint32_t acc) {
  ptx::mma_f16_pair(d_tmem, a_hi, bd, kIdesc, acc);
  if constexpr (LO) ptx::mma_f16_pair(d_tmem, a_lo, bd, kIdesc, 1);
#pragma unroll
  for (int ks = 1; ks < KS; ++ks) {
    ptx::mma_f16_pair(d_tmem, a_hi + ks * kStepDesc, bd + ks * kStepDesc, kIdesc, 1);
    if constexpr (LO) ptx::mma_f16_pair(d_tmem, a_lo + ks * kStepDesc, bd + ks * kStepDesc, kIdesc, 1);
  }
}

template <bool LO, int KS>
__device__ __forceinline__ void issue_chunk(uint32_t d_tmem, uint64_t a_hi, uint64_t a_lo,
                                            uint64_t bd, uint32_t acc, int ksteps) {
  if constexpr (KS > 0) {
    issue_unit<LO, KS>(d_tmem, a_hi, a_lo, bd, acc);
  } else if (ksteps == 4) {
    issue_unit<LO, 4>(d_tmem, a_hi, a_lo, bd, acc);
  } else if (ksteps == 2) {
    issue_unit<LO, 2>(d_tmem, a_hi, a_lo, bd, acc);
  } else {
    issue_unit<LO, 1>(d_tmem, a_hi, a_lo, bd, acc);
  }
}

template <bool LO, int KS>
__device__ void run_mma(const FusedParams& p, const Smem& s, uint32_t tmem_base) {
  const uint32_t base_addr = ptx::smem_addr(s.base);
  // Equal chunk widths (KS > 0): the chunks' query regions are evenly spaced, so descriptors are
  // a base plus a constant per chunk (three registers). Mixed widths (KS == 0): each chunk's
  // descriptors are rebuilt at use from the kernel parameters (static indices after unrolling),
  // which keeps them out of registers.
  constexpr uint64_t kAStep = KS > 0 ? static_cast<uint64_t>(kTileQ * 32 * KS) >> 4 : 0;
  constexpr uint32_t kRowBytes = KS > 0 ? 32 * KS : 0;
  const uint64_t a_hi0 = ptx::smem_desc(base_addr + p.a_off[0][0], kRowBytes ? kRowBytes : 128);
  const uint64_t a_lo0 = ptx::smem_desc(base_addr + p.a_off[1][0], kRowBytes ? kRowBytes : 128);
  const uint64_t b0 = ptx::smem_desc(base_addr + p.stage_off, kRowBytes ? kRowBytes : 128);
  uint32_t slot = 0, phase = 0;
  uint32_t tile = 0;
  int a_waits = 0, cur_qt = -1;
  bool ok = true;
  for (int item = first_item(); item < p.num_items && ok; item += item_step()) {
    const Item it = item_of(p, item, 0);
    if (it.qt != cur_qt) {
      if (!ptx::mbar_wait(s.afull, a_waits & 1, s.abort, p.err, kErrWaitA)) {
        ok = false;
        break;
      }
      ++a_waits;
      cur_qt = it.qt;
      ptx::tc_fence_after();
    }
    for (int t = it.t0; t < it.t1 && ok; ++t) {
      const uint32_t buf = tile & 1, use = tile >> 1;
      if (use > 0 &&
          !ptx::mbar_wait(&s.tempty[buf], (use - 1) & 1, s.abort, p.err, kErrWaitTmemEmpty)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * kTileN;
      uint32_t acc = 0;
      // Units arrive in the producer's order: database part bp major, chunk c minor. The query's
      // lo part meets only the database hi part (bp == 0).
      for (int bp = 0; bp < p.b_parts && ok; ++bp) {
#pragma unroll
        for (int c = 0; c < kResChunks; ++c) {
          if (c >= p.nchunk) break;
          if (!ptx::mbar_wait(&s.full[slot], phase, s.abort, p.err, kErrWaitSlotFull)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          uint64_t ah, al, bd;
          int ksteps = KS;
          if constexpr (KS > 0) {
            ah = a_hi0 + c * kAStep;
            al = a_lo0 + c * kAStep;
            bd = b0 + slot * kSlotDesc;
          } else {
            const uint32_t row_bytes = static_cast<uint32_t>(p.chunk_w[c] * 2);
            ah = ptx::smem_desc(base_addr + p.a_off[0][c], row_bytes);
            al = ptx::smem_desc(base_addr + p.a_off[1][c], row_bytes);
            bd = ptx::smem_desc(base_addr + p.stage_off + slot * kUnitBytes, row_bytes);
            ksteps = p.chunk_w[c] / 16;
          }
          if (LO && bp == 0)
            issue_chunk<true, KS>(d_tmem, ah, al, bd, acc, ksteps);
          else
            issue_chunk<false, KS>(d_tmem, ah, al, bd, acc, ksteps);
          acc = 1;
          ptx::mma_commit_pair(&s.empty[slot]);  // both CTAs' slot reusable once read
          if (++slot == static_cast<uint32_t>(p.nstages)) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) break;
      ptx::mma_commit_pair(&s.tfull[buf]);
      ++tile;
    }
    if (!ok) break;
    const int next = item + item_step();
    if (next < p.num_items && item_of(p, next, 0).qt != it.qt) ptx::mma_commit_pair(s.aempty);
  }
  // Unwind: every MMA issued by this thread completes before either CTA releases TMEM or shared
  // memory (both CTAs wait for `drain`).
  ptx::mma_commit_pair(s.drain);
  drain_wait(s.drain, 0, p.err, s.abort);
}

// ------------------------------------------------------------------------------------------
// Streamed query mode (large dims): every ring slot carries a database chunk together with the
// matching chunk of this CTA's queries (hi, and lo for the database hi part when the lo pass
// runs), so no query tile is resident. The query chunks are re-read per tile (from L2: the query
// operand array is small next to the database), which doubles the shared-memory fill but keeps
// any dim up to 4096 on the same kernel.
// ------------------------------------------------------------------------------------------
__device__ void run_producer_stream(const FusedParams& p, const FusedMaps& maps, const Smem& s,
                                    bool lo, uint32_t rank) {
  const bool leader = rank == 0;
  const uint32_t full_l = ptx::peer_addr(s.full, 0);
  uint32_t unit = 0, tile = 0;
  uint32_t slot = 0, phase = 0;
  bool wrapped = false;
  const bool need_aux = p.rank_kind != kRankScaled;
  const uint32_t side_tx = (need_aux ? 1024u : 0u) + 1024u + (p.allow ? 32u : 0u);
  bool ok = true;
  for (int item = first_item(); item < p.num_items && ok; item += item_step()) {
    const Item it = item_of(p, item, rank);
    for (int t = it.t0; t < it.t1 && ok; ++t) {
      if (!load_side(p, s, t, tile, need_aux, side_tx)) {
        ok = false;
        break;
      }
      ++tile;
      const int row = t * p.tile_stride * kTileN + static_cast<int>(rank) * kHalfN;
      for (int bp = 0; bp < p.b_parts && ok; ++bp) {
        const bool with_lo = lo && bp == 0;
        for (int c = 0; c < p.nchunk; ++c) {
          if (wrapped &&
              !ptx::mbar_wait(&s.empty[slot], phase ^ 1u, s.abort, p.err, kErrWaitSlotEmpty)) {
            ok = false;
            break;
          }
          const int w = p.chunk_w[c];
          const uint32_t a_bytes = 2u * static_cast<uint32_t>(kTileQ * w * 2);  // both CTAs
          if (leader)
            ptx::mbar_arrive_expect_tx(
                &s.full[slot], static_cast<uint32_t>(kTileN * w * 2) + a_bytes * (with_lo ? 2 : 1));
          uint8_t* sb = s.base + p.stage_off + slot * p.slot_bytes;
          const uint32_t bar = full_l + slot * 8;
          ptx::tma_load_2d_pair(sb, pick_map(w, &maps.b64, &maps.b32, &maps.b16),
                                bp * p.dp + p.chunk_x[c], row, bar);
          const CUtensorMap* am = pick_map(w, &maps.a64, &maps.a32, &maps.a16);
          ptx::tma_load_2d_pair(sb + p.slot_a_off, am, p.chunk_x[c], it.qt * kTileQ, bar);
          if (with_lo)
            ptx::tma_load_2d_pair(sb + p.slot_alo_off, am, p.dp + p.chunk_x[c], it.qt * kTileQ,
                                  bar);
          ++unit;
          if (++slot == static_cast<uint32_t>(p.nstages)) {
            slot = 0;
            phase ^= 1u;
            wrapped = true;
          }
        }
      }
    }
  }
  // Unwind as run_producer: every copy landed before the CTA exits (the MMA consumed each slot's
  // last use; side copies on this CTA's barriers).
  const uint32_t issued = unit;
  for (uint32_t sl = 0; sl < static_cast<uint32_t>(p.nstages) && sl < issued; ++sl) {
    const uint32_t last = ((issued - 1 - sl) / p.nstages) * p.nstages + sl;
    drain_wait(&s.empty[sl], (last / p.nstages) & 1, p.err, s.abort);
  }
  for (uint32_t sb = 0; sb < static_cast<uint32_t>(kSideBufs) && sb < tile; ++sb) {
    const uint32_t last = ((tile - 1 - sb) / kSideBufs) * kSideBufs + sb;
    drain_wait(&s.side_full[sb], (last / kSideBufs) & 1, p.err, s.abort);
  }
}

template <bool LO>
__device__ void run_mma_stream(const FusedParams& p, const Smem& s, uint32_t tmem_base) {
  const uint32_t base_addr = ptx::smem_addr(s.base);
  uint32_t slot = 0, phase = 0, tile = 0;
  bool ok = true;
  for (int item = first_item(); item < p.num_items && ok; item += item_step()) {
    const Item it = item_of(p, item, 0);
    for (int t = it.t0; t < it.t1 && ok; ++t) {
      const uint32_t buf = tile & 1, use = tile >> 1;
      if (use > 0 &&
          !ptx::mbar_wait(&s.tempty[buf], (use - 1) & 1, s.abort, p.err, kErrWaitTmemEmpty)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * kTileN;
      uint32_t acc = 0;
      for (int bp = 0; bp < p.b_parts && ok; ++bp) {
        for (int c = 0; c < p.nchunk; ++c) {
          if (!ptx::mbar_wait(&s.full[slot], phase, s.abort, p.err, kErrWaitSlotFull)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t sb = base_addr + p.stage_off + slot * p.slot_bytes;
          const uint32_t row_bytes = static_cast<uint32_t>(p.chunk_w[c] * 2);
          const uint64_t ah = ptx::smem_desc(sb + p.slot_a_off, row_bytes);
          const uint64_t al = ptx::smem_desc(sb + p.slot_alo_off, row_bytes);
          const uint64_t bd = ptx::smem_desc(sb, row_bytes);
          if (LO && bp == 0)
            issue_chunk<true, 0>(d_tmem, ah, al, bd, acc, p.chunk_w[c] / 16);
          else
            issue_chunk<false, 0>(d_tmem, ah, al, bd, acc, p.chunk_w[c] / 16);
          acc = 1;
          ptx::mma_commit_pair(&s.empty[slot]);
          if (++slot == static_cast<uint32_t>(p.nstages)) {
            slot = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) break;
      ptx::mma_commit_pair(&s.tfull[buf]);
      ++tile;
    }
  }
  ptx::mma_commit_pair(s.drain);
  drain_wait(s.drain, 0, p.err, s.abort);
}

// Picks the run_mma instance: LO from the launch's query-split flag, KS from the chunk widths
// when they are all equal (0 = mixed).
__device__ void run_mma_dispatch(const FusedParams& p, const Smem& s, uint32_t tmem_base, bool lo) {
  int ks = p.chunk_w[0] / 16;
  for (int c = 1; c < p.nchunk; ++c)
    if (p.chunk_w[c] / 16 != ks) ks = 0;
  if (lo) {
    if (ks == 4) return run_mma<true, 4>(p, s, tmem_base);
    if (ks == 2) return run_mma<true, 2>(p, s, tmem_base);
    if (ks == 1) return run_mma<true, 1>(p, s, tmem_base);
    return run_mma<true, 0>(p, s, tmem_base);
  }
  if (ks == 4) return run_mma<false, 4>(p, s, tmem_base);
  if (ks == 2) return run_mma<false, 2>(p, s, tmem_base);
  if (ks == 1) return run_mma<false, 1>(p, s, tmem_base);
  return run_mma<false, 0>(p, s, tmem_base);
}

// ------------------------------------------------------------------------------------------
// Epilogue (warps 0-3, one query per thread)
// ------------------------------------------------------------------------------------------
template <int KL>
__device__ __forceinline__ void list_insert(uint64_t (&L)[KL], uint64_t c) {
#pragma unroll
  for (int i = 0; i < KL; ++i) {
    const uint64_t lo = c < L[i] ? c : L[i];
    const uint64_t hi = c < L[i] ? L[i] : c;
    L[i] = lo;
    c = hi;
  }
}

// Smallest s that can still produce a ranking value <= w for any column of the tile; -inf
// accepts everything (w = +inf or NaN: nothing to compare against yet).
//   affine:  v = s*m + aux <= w with m < 0 and aux >= aux_min  =>  s >= (w - aux_min) / m
//   scaled:  v = s*m <= w with m < 0                           =>  s >= w / m
//   column:  v = s*aux <= w with aux in [aux_min, aux_max] < 0  =>  s >= w / aux_min (w < 0)
//                                                                   s >= w / aux_max (w >= 0)
// The slack (1e-5 of the magnitudes involved) keeps the bound conservative against the rounding
// of the exact per-column evaluation in the slow path, and against the 1.5 ulp of dividing by m
// through its reciprocal inv_m = 1/m (computed once per query).
__device__ __forceinline__ float s_threshold(float w, float inv_m, float2 ta, int kind) {
  if (!(w < kInf)) return -kInf;
  float t, mag;
  if (kind == kRankAffine) {
    t = (w - ta.x) * inv_m;
    mag = fabsf(t) + (fabsf(w) + fabsf(ta.x)) * fabsf(inv_m);
  } else if (kind == kRankScaled) {
    t = w * inv_m;
    mag = fabsf(t);
  } else {
    t = (w < 0.f) ? w / ta.x : w / ta.y;
    mag = fabsf(t);
  }
  if (!(t == t) || !(mag < kInf)) return -kInf;
  return t - mag * 1e-5f - 1e-30f;
}

__device__ __forceinline__ float max32(const float (&r)[32]) {
  float a0 = ptx::fmax3(r[0], r[1], r[2]);
  float a1 = ptx::fmax3(r[3], r[4], r[5]);
  float a2 = ptx::fmax3(r[6], r[7], r[8]);
  float a3 = ptx::fmax3(r[9], r[10], r[11]);
  float a4 = ptx::fmax3(r[12], r[13], r[14]);
  float a5 = ptx::fmax3(r[15], r[16], r[17]);
  float a6 = ptx::fmax3(r[18], r[19], r[20]);
  float a7 = ptx::fmax3(r[21], r[22], r[23]);
  float a8 = ptx::fmax3(r[24], r[25], r[26]);
  float a9 = ptx::fmax3(r[27], r[28], r[29]);
  float b0 = ptx::fmax3(a0, a1, a2);
  float b1 = ptx::fmax3(a3, a4, a5);
  float b2 = ptx::fmax3(a6, a7, a8);
  float b3 = ptx::fmax3(a9, r[30], r[31]);
  return fmaxf(ptx::fmax3(b0, b1, b2), b3);
}

template <int KL>
struct EpiState {
  uint64_t L[KL > 0 ? KL : 1];
  float m;
  float inv_m;    // 1 / m
  float thr;      // s-space threshold for the current tile
  float gw;       // ranking value of the shared per-query bound (+ slack), NaN when none
  float2 ta;
  bool real;      // this lane holds a real query
  int64_t qi;     // this lane's query index
  uint64_t gkey;  // append mode: the query's bound key
  bool by_key;    // append mode: compare keys (bound value not finite, or exact mode)
  int kpub;       // 4-entry lists: index of the entry that bounds the query (k_pub - 1), or -1
  bool xf;        // exact filter: thr is a ranking value (candidates: v <= thr), not a bound on s
};

// Ranking value the filter compares against: the list's own worst entry, tightened by the
// shared per-query bound and, for 4-entry lists (k <= 2: k-means and coarse assignment, k = 1),
// by the list's own k_pub-th entry. Both bounds get a relative slack of 1e-5 of the magnitudes
// involved so that rows tied with them within the ranking values' rounding still pass (the exact
// re-rank then orders them). The own k_pub-th entry is the bound this list publishes every
// kBoundPeriod tiles; applying it at once matters where the list is much longer than k and items
// are short (a k-means item spans all centroids in a few tiles). With longer lists the extra
// selection on every refresh cost more than it saved (config 3: 26.3 instead of 25.1 ms).
template <int KL>
__device__ __forceinline__ void refresh_threshold(EpiState<KL>& st, int kind) {
  if (!st.real) {
    st.thr = st.xf ? -kInf : kInf;  // padding lanes never select
    return;
  }
  if constexpr (KL == 0) {  // append mode: fixed per-query threshold (already has its slack)
    st.thr = s_threshold(st.gw, st.inv_m, st.ta, kind);
  } else {
    float w = fminf(keys::key_value(st.L[KL - 1]), st.gw);  // NaN entries: not full yet
    if (KL == 4 && st.kpub >= 0) {
      // Branch-free selection keeps the list in registers.
      uint64_t kth = 0;
#pragma unroll
      for (int i = 0; i < KL; ++i) kth |= st.L[i] & (0ull - static_cast<uint64_t>(i == st.kpub));
      const float kv = keys::key_value(kth);  // NaN while that rank is empty
      w = fminf(w, kv + (fabsf(kv) + fabsf(st.ta.x) + fabsf(st.ta.y)) * 1e-5f);
    }
    st.thr = st.xf ? w : s_threshold(w, st.inv_m, st.ta, kind);
  }
}

// Append-mode threshold in ranking-value space: the bound value plus a relative slack of 1e-5.
__device__ __forceinline__ float append_limit(float tau, float2 ta) {
  if (!(tau < kInf)) return tau;
  return tau + (fabsf(tau) + fabsf(ta.x) + fabsf(ta.y)) * 1e-5f;
}

template <int KL>
__device__ __forceinline__ void apply_bound(uint64_t b, EpiState<KL>& st) {
  const float w = keys::key_value(b);
  const float mag = fabsf(w) + fabsf(st.ta.x) + fabsf(st.ta.y);
  st.gw = w + mag * 1e-5f;
}

// Min-writes `kth` into every other rank's bound array. Out of line, and compiled only into the
// kernels of sharded searches: inlined into the epilogue's tile loop (even never executed) it
// slowed config 3 by 12 %, and as a call by 1.5 %.
__device__ __noinline__ void publish_to_peers(const FusedParams& p, int64_t q, uint64_t kth) {
  for (int i = 0; i < p.n_peers; ++i)
    atomicMin_system(reinterpret_cast<unsigned long long*>(p.peer_bound[i] + q), kth);
}

// `seen` is the bound this lane read last: a key that beats it is news to the other ranks too.
template <int KL, bool PEER>
__device__ __forceinline__ void publish_bound(const FusedParams& p, int64_t q,
                                              const EpiState<KL>& st, uint64_t seen) {
  if (p.k_pub < 1 || p.k_pub > KL) return;  // the list cannot bound that rank
  // Branch-free selection keeps the list in registers (a select chain would be turned into an
  // indexed load, which moves the whole list to local memory).
  uint64_t kth = 0;
#pragma unroll
  for (int i = 0; i < KL; ++i) kth |= st.L[i] & (0ull - static_cast<uint64_t>(i == p.k_pub - 1));
  if (kth == kEmptyKey) return;
  atomicMin(reinterpret_cast<unsigned long long*>(p.q_bound + q), kth);
  if constexpr (PEER) {
    if (kth < seen) publish_to_peers(p, q, kth);
  }
}

// r[j] for a run-time j through a tree of selects on statically indexed registers (an indexed
// access would move the array to local memory).
__device__ __forceinline__ float pick32(const float (&r)[32], int j) {
  float a[16], b[8], c[4], d[2];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = (j & 16) ? r[i + 16] : r[i];
#pragma unroll
  for (int i = 0; i < 8; ++i) b[i] = (j & 8) ? a[i + 8] : a[i];
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = (j & 4) ? b[i + 4] : b[i];
#pragma unroll
  for (int i = 0; i < 2; ++i) d[i] = (j & 2) ? c[i + 2] : c[i];
  return (j & 1) ? d[1] : d[0];
}

template <int KL>
__device__ __forceinline__ void slow_path(const FusedParams& p, const float (&r)[32],
                                          int64_t col0, int ct0, const uint8_t* side,
                                          EpiState<KL>& st) {
  // Per-column data of this tile, staged in shared memory by the producer (column ct of the
  // tile: aux[ct], id[ct], allow bit ct).
  const float* aux = reinterpret_cast<const float*>(side + kSideAuxOff);
  const uint32_t* ids = reinterpret_cast<const uint32_t*>(side + kSideIdOff);
  const uint32_t* allow = reinterpret_cast<const uint32_t*>(side + kSideAllowOff);
  // Visit only the columns that pass the conservative bound (NaN passes: its exact key is
  // decided below).
  uint32_t mask = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) mask |= static_cast<uint32_t>(!(r[j] < st.thr)) << j;
  while (mask) {
    const int j = __ffs(mask) - 1;
    mask &= mask - 1;
    const float sv = pick32(r, j);
    if (sv < st.thr) continue;  // threshold tightened by an earlier insertion
    const int64_t pos = col0 + j;
    if (pos >= p.n_rows) break;
    float v;
    const int ct = ct0 + j;
    const bool allowed = p.allow == nullptr || ((allow[ct >> 5] >> (ct & 31)) & 1u);
    if (!allowed) {
      v = kInf;
    } else if (p.rank_kind == kRankAffine) {
      v = fmaf(sv, st.m, aux[ct]);
    } else if (p.rank_kind == kRankScaled) {
      v = sv * st.m;
    } else {
      v = sv * aux[ct];
    }
    const uint64_t key = keys::make_key(v, ids[ct]);
    if constexpr (KL == 0) {
      if (st.by_key ? key <= st.gkey : v <= st.gw) {
        const uint32_t slot = atomicAdd(p.app_count + st.qi, 1u);
        if (slot < static_cast<uint32_t>(p.app_cap))
          p.app_buf[static_cast<size_t>(st.qi) * p.app_cap + slot] = key;
      }
    } else {
      if (key < st.L[KL - 1]) {
        list_insert<KL>(st.L, key);
        refresh_threshold<KL>(st, p.rank_kind);
      }
    }
  }
}


// The exact path for a deferred chunk: `row` = this lane's 32 values in shared memory and
// row[32] = the bits of the columns that passed the threshold when it was saved (a superset of
// those that pass now: thresholds only tighten). Only those columns are read back.
template <int KL>
__device__ __forceinline__ void check_row(const FusedParams& p, const float* row, int64_t col0,
                                          int ct0, const uint8_t* side, EpiState<KL>& st) {
  const float* aux = reinterpret_cast<const float*>(side + kSideAuxOff);
  const uint32_t* ids = reinterpret_cast<const uint32_t*>(side + kSideIdOff);
  const uint32_t* allow = reinterpret_cast<const uint32_t*>(side + kSideAllowOff);
  uint32_t mask = __float_as_uint(row[32]);
  while (mask) {
    const int j = __ffs(mask) - 1;
    mask &= mask - 1;
    const float sv = row[j];
    if (sv < st.thr) continue;  // threshold tightened by an earlier insertion
    const int64_t pos = col0 + j;
    if (pos >= p.n_rows) break;
    float v;
    const int ct = ct0 + j;
    const bool allowed = p.allow == nullptr || ((allow[ct >> 5] >> (ct & 31)) & 1u);
    if (!allowed) {
      v = kInf;
    } else if (p.rank_kind == kRankAffine) {
      v = fmaf(sv, st.m, aux[ct]);
    } else if (p.rank_kind == kRankScaled) {
      v = sv * st.m;
    } else {
      v = sv * aux[ct];
    }
    const uint64_t key = keys::make_key(v, ids[ct]);
    if constexpr (KL == 0) {
      if (st.by_key ? key <= st.gkey : v <= st.gw) {
        const uint32_t slot = atomicAdd(p.app_count + st.qi, 1u);
        if (slot < static_cast<uint32_t>(p.app_cap))
          p.app_buf[static_cast<size_t>(st.qi) * p.app_cap + slot] = key;
      }
    } else {
      if (key < st.L[KL - 1]) {
        list_insert<KL>(st.L, key);
        refresh_threshold<KL>(st, p.rank_kind);
      }
    }
  }
}

__device__ __forceinline__ float min32(const float (&r)[32]) {
  float a[10];
#pragma unroll
  for (int i = 0; i < 10; ++i) a[i] = ptx::fmin3(r[3 * i], r[3 * i + 1], r[3 * i + 2]);
  const float b0 = ptx::fmin3(a[0], a[1], a[2]), b1 = ptx::fmin3(a[3], a[4], a[5]);
  const float b2 = ptx::fmin3(a[6], a[7], a[8]), b3 = ptx::fmin3(a[9], r[30], r[31]);
  return fminf(ptx::fmin3(b0, b1, b2), b3);
}

// Exact filter: turns a chunk's 32 dot products into ranking values in place, with the same
// arithmetic as the slow path (aux = the chunk's 32 columns in shared memory, 16-byte aligned).
__device__ __forceinline__ void chunk_values(float (&r)[32], const float* aux, float m, int kind) {
  if (kind == kRankScaled) {
#pragma unroll
    for (int j = 0; j < 32; ++j) r[j] = r[j] * m;
    return;
  }
#pragma unroll
  for (int j4 = 0; j4 < 8; ++j4) {
    const float4 a = reinterpret_cast<const float4*>(aux)[j4];
    const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float& v = r[4 * j4 + i];
      v = kind == kRankAffine ? fmaf(v, m, av[i]) : v * av[i];
    }
  }
}

// Exact filter: the columns of one chunk whose ranking value v (in r) is within the threshold,
// inserted into the list in column order, re-checked against the threshold as it tightens.
template <int KL>
__device__ __forceinline__ void exact_chunk(const FusedParams& p, const float (&r)[32],
                                            int64_t col0, int ct0, const uint8_t* side,
                                            EpiState<KL>& st) {
  const uint32_t* ids = reinterpret_cast<const uint32_t*>(side + kSideIdOff);
  const uint32_t* allow = reinterpret_cast<const uint32_t*>(side + kSideAllowOff);
  uint32_t mask = 0;
#pragma unroll
  for (int j = 0; j < 32; ++j) mask |= static_cast<uint32_t>(!(r[j] > st.thr)) << j;
  while (mask) {
    const int j = __ffs(mask) - 1;
    mask &= mask - 1;
    const float v = pick32(r, j);
    if (v > st.thr) continue;  // threshold tightened by an earlier insertion
    const int64_t pos = col0 + j;
    if (pos >= p.n_rows) break;
    const int ct = ct0 + j;
    // a row outside the allow list ranks as +inf (it still fills a list that has room)
    const bool allowed = p.allow == nullptr || ((allow[ct >> 5] >> (ct & 31)) & 1u);
    const uint64_t key = keys::make_key(allowed ? v : kInf, ids[ct]);
    if (key < st.L[KL - 1]) {
      list_insert<KL>(st.L, key);
      refresh_threshold<KL>(st, p.rank_kind);
    }
  }
}

template <int KL, bool XF, bool PEER>
__device__ void run_epilogue(const FusedParams& p, const Smem& s, uint32_t tmem_base, uint32_t rank) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // TMEM buffers are handed back to the leader's MMA thread: its tempty barrier counts the
  // arrivals of both CTAs' epilogue warps.
  const uint32_t tempty_l = ptx::peer_addr(s.tempty, 0);
  // Warp w reads TMEM lane quarter w % 4 (the hardware ties a warp to its quarter) and owns
  // columns [kPartCols * part, kPartCols * part + kPartCols) of every tile, part = w / 4.
  const int quarter = warp & 3, part = warp >> 2;
  constexpr int nchunks = kPartCols / 32;
  float* my_row = s.defer + threadIdx.x * kDeferStride;  // this lane's deferred chunk
  const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
  uint32_t tile = 0;
  EpiState<KL> st;
  st.kpub = (p.k_pub >= 1 && p.k_pub <= KL) ? p.k_pub - 1 : -1;
  st.xf = XF;
  for (int item = first_item(); item < p.num_items; item += item_step()) {
    const Item it = item_of(p, item, rank);
    const int64_t q = static_cast<int64_t>(it.qt) * kTileQ + quarter * 32 + lane;
    st.m = p.q_mul[q];
    st.inv_m = 1.0f / st.m;
    st.real = q < p.nq && (p.slot_pair == nullptr || p.slot_pair[q] >= 0);
    st.qi = q;
    // The filter threshold is computed against the aux range of the tile's group of
    // kGroupTiles consecutive tiles (rows are sorted by aux, so the group range is barely wider
    // than a tile's, and it stays conservative). It is therefore recomputed only when the group
    // changes, when the shared bound is re-read, or after an insertion, not on every tile. The
    // next group's range is loaded one tile before it is needed.
    int g_cur = (it.t0 * p.tile_stride) >> kGroupShift, g_pf = -1;
    uint64_t bound_pf = kEmptyKey;
    float2 ta_pf = make_float2(0.f, 0.f);
    st.ta = p.group_aux[g_cur];
    if constexpr (KL > 0) {
      bound_pf = __ldcg(reinterpret_cast<const unsigned long long*>(p.q_bound + q));
      apply_bound<KL>(bound_pf, st);
#pragma unroll
      for (int i = 0; i < KL; ++i) st.L[i] = kEmptyKey;
    } else {
      st.gkey = p.q_tau_key[q];
    }
    // Everything tile t's filter needs (aux range, shared bound, threshold) is known once tile
    // t-1 is done, so it is prepared then, while the next TMEM buffer is still being filled:
    // after the buffer fills, this warp goes straight to reading it and hands it back sooner,
    // which is what lets the MMA of tile t+2 start before the tensor core runs dry.
    auto prepare = [&](int t, bool refresh) {
      const int g = (t * p.tile_stride) >> kGroupShift;
      if (g != g_cur) {
        st.ta = g == g_pf ? ta_pf : p.group_aux[g];
        g_cur = g;
        refresh = true;
      }
      if (t + 1 < it.t1) {
        const int gn = ((t + 1) * p.tile_stride) >> kGroupShift;
        if (gn != g_cur && gn != g_pf) {
          ta_pf = p.group_aux[gn];
          g_pf = gn;
        }
      }
      if constexpr (KL > 0) {
        // The shared bound is read a tile before it is used, so the load's latency is hidden.
        const int phase_t = (t - it.t0) & (kBoundPeriod - 1);
        if (phase_t == kBoundPeriod - 2 && st.real)
          bound_pf = __ldcg(reinterpret_cast<const unsigned long long*>(p.q_bound + q));
        if (phase_t == kBoundPeriod - 1 && st.real) {
          publish_bound<KL, PEER>(p, q, st, bound_pf);
          apply_bound<KL>(bound_pf, st);
          refresh = true;
        }
      } else if (refresh) {
        const float tv = keys::key_value(st.gkey);
        st.by_key = p.app_exact || !(tv < kInf);
        st.gw = st.by_key ? tv : append_limit(tv, st.ta);
      }
      if (refresh) refresh_threshold<KL>(st, p.rank_kind);
    };
    prepare(it.t0, true);
    bool ok = true;
    for (int t = it.t0; t < it.t1; ++t) {
      const uint32_t buf = tile & 1, use = tile >> 1;
      // Warp-uniform decision: tcgen05.ld below is warp-collective, so either every lane
      // proceeds or every lane unwinds.
      const uint32_t sb = tile % kSideBufs, suse = tile / kSideBufs;
      bool got = ptx::mbar_wait(&s.tfull[buf], use & 1, s.abort, p.err, kErrWaitTmemFull);
      got = got && ptx::mbar_wait(&s.side_full[sb], suse & 1, s.abort, p.err, kErrWaitSideFull);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      ptx::tc_fence_after();
      const uint8_t* side = s.side + sb * kSideBytes;
      const int ct0 = part * kPartCols;  // this warp's first column within the tile
      const int tile_pos = t * p.tile_stride;
      const uint32_t taddr = lane_base + buf * kTileN + ct0;
      const int64_t col0 = static_cast<int64_t>(tile_pos) * kTileN + ct0;
      // One 32-column chunk in registers at a time, a 3-input max tree against the threshold.
      // A lane whose chunk may hold a candidate saves it to its deferred row (the first such
      // chunk of the tile) or flags it (any further one: item starts, lists still empty). The
      // exact checks run after the loop: flagged chunks first, re-read from TMEM while the
      // buffer is still held; then the buffer goes back to the MMA, then the deferred row.
      uint32_t flagged = 0;  // chunks this lane must re-read
      int saved = -1;        // chunk index in the deferred row, or -1
      if constexpr (XF) {
        // Exact filter: every column's ranking value against the list's threshold; the few
        // candidates are inserted before the buffer is handed back.
        const float* aux = reinterpret_cast<const float*>(side + kSideAuxOff) + ct0;
#pragma unroll 1
        for (int c = 0; c < nchunks; ++c) {
          float r0[32];
          ptx::tmem_ld32(taddr + 32 * c, r0);
          ptx::tmem_wait_ld();
          chunk_values(r0, aux + 32 * c, st.m, p.rank_kind);
          if (!(min32(r0) > st.thr)) exact_chunk<KL>(p, r0, col0 + 32 * c, ct0 + 32 * c, side, st);
          __syncwarp();
        }
      } else {
#pragma unroll
        for (int c = 0; c < nchunks; ++c) {
          float r0[32];
          ptx::tmem_ld32(taddr + 32 * c, r0);
          ptx::tmem_wait_ld();
          if (!(max32(r0) < st.thr)) {
            if (saved < 0) {
              uint32_t cand = 0;
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                my_row[j] = r0[j];
                cand |= static_cast<uint32_t>(!(r0[j] < st.thr)) << j;
              }
              my_row[32] = __uint_as_float(cand);
              saved = c;
            } else {
              flagged |= 1u << c;
            }
          }
          __syncwarp();
        }
        if (__any_sync(0xffffffffu, flagged != 0)) {
          for (int c = 0; c < nchunks; ++c) {
            if (!__any_sync(0xffffffffu, (flagged >> c) & 1u)) continue;
            float r0[32];
            ptx::tmem_ld32(taddr + 32 * c, r0);
            ptx::tmem_wait_ld();
            if ((flagged >> c) & 1u) slow_path<KL>(p, r0, col0 + 32 * c, ct0 + 32 * c, side, st);
            __syncwarp();
          }
        }
      }  // exact filter or conservative bound
      // Every chunk of this warp is read: hand its share of the buffer back.
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(tempty_l + buf * 8);
      if (saved >= 0) check_row<KL>(p, my_row, col0 + 32 * saved, ct0 + 32 * saved, side, st);
      // Side slot released once this warp's exact checks of the tile are done.
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&s.side_empty[sb]);
      ++tile;
      if (t + 1 < it.t1) prepare(t + 1, false);
    }
    if (!ok) return;
    if constexpr (KL > 0) {
      if (st.real) publish_bound<KL, PEER>(p, q, st, bound_pf);
      uint64_t* dst =
          p.out + ((static_cast<size_t>(q) * p.num_sc + it.sc) * kListsPerItem + part) * KL;
#pragma unroll
      for (int i = 0; i < KL; ++i) dst[i] = st.L[i];
    }
  }
}

template <int KL, bool XF, bool PEER>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kFusedThreads, 1)
    knn_fused_kernel(const __grid_constant__ FusedMaps maps, const __grid_constant__ FusedParams p) {
  extern __shared__ uint8_t smem_raw[];
  const Smem s = carve(p, smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_rank();

  if (threadIdx.x == 0) {
    for (int i = 0; i < p.nstages; ++i) {
      ptx::mbar_init(&s.full[i], 1);
      ptx::mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      ptx::mbar_init(&s.tfull[i], 1);
      ptx::mbar_init(&s.tempty[i], 2 * kEpiWarps);  // leader's: both CTAs' epilogue warps
    }
    ptx::mbar_init(s.afull, 1);
    ptx::mbar_init(s.aempty, 1);
    ptx::mbar_init(s.drain, 1);
    for (int i = 0; i < kSideBufs; ++i) {
      ptx::mbar_init(&s.side_full[i], 1);
      ptx::mbar_init(&s.side_empty[i], kEpiWarps);
    }
    *s.abort = 0;
    ptx::fence_barrier_init();
  }
  if (warp == kEpiWarps && lane == 0) {
    ptx::tma_prefetch_desc(&maps.a64);
    ptx::tma_prefetch_desc(&maps.b64);
  }
  if (warp == kEpiWarps + 1) ptx::tmem_alloc_pair(s.tmem_slot, kTmemCols);
  // Both CTAs' barriers are initialised (and TMEM allocated) before either CTA touches the
  // other's barriers or shared memory.
  ptx::tc_fence_before();
  ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *s.tmem_slot;
  const bool lo = p.query_split != 0 && *p.q_lo_flag != 0;

  if (warp == kEpiWarps) {
    if (lane == 0) {
      if (p.a_stream)
        run_producer_stream(p, maps, s, lo, rank);
      else
        run_producer(p, maps, s, lo, rank);
    }
  } else if (warp == kEpiWarps + 1) {
    if (lane == 0 && rank == 0) {
      if (!p.a_stream)
        run_mma_dispatch(p, s, tmem_base, lo);
      else if (lo)
        run_mma_stream<true>(p, s, tmem_base);
      else
        run_mma_stream<false>(p, s, tmem_base);
    }
    __syncwarp();
  } else {
    run_epilogue<KL, XF, PEER>(p, s, tmem_base, rank);
  }

  // The leader's MMAs read the other CTA's shared memory and write its TMEM: that CTA waits for
  // their completion (`drain`) before it may leave, but only once its own roles are done (its
  // epilogue has consumed every tile), so the wait is short. Waiting from the start would span
  // the whole launch and trip the watchdog on launches longer than its limit.
  __syncthreads();
  if (rank != 0 && warp == kEpiWarps + 1 && lane == 0) drain_wait(s.drain, 0, p.err, s.abort);

  // Neither CTA leaves (or frees TMEM) while the other may still arrive on its barriers.
  ptx::tc_fence_before();
  ptx::cluster_sync();
  if (warp == kEpiWarps + 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, kTmemCols);
  }
}

template <int KL, bool XF = false, bool PEER = false>
cudaError_t launch_kl(const FusedMaps& maps, const FusedParams& p, int grid, cudaStream_t stream) {
  auto kern = knn_fused_kernel<KL, XF, PEER>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem_bytes);
  if (e != cudaSuccess) return e;
  kern<<<grid, kFusedThreads, p.smem_bytes, stream>>>(maps, p);
  return cudaGetLastError();
}

}  // namespace

int fused_max_pairs(int smem_bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, int>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 1;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_pair(dev, smem_bytes);
  auto hit = cache.find(key);
  if (hit != cache.end()) return hit->second;
  auto kern = knn_fused_kernel<16, false, false>;  // every instance: same threads, smem, cluster
  int pairs = 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) ==
      cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2, 1, 1);
    cfg.blockDim = dim3(kFusedThreads, 1, 1);
    cfg.dynamicSmemBytes = static_cast<size_t>(smem_bytes);
    if (cudaOccupancyMaxActiveClusters(&pairs, kern, &cfg) != cudaSuccess) pairs = 0;
  }
  (void)cudaGetLastError();
  if (pairs < 1) pairs = 1;
  cache[key] = pairs;
  return pairs;
}

bool plan_fused_smem(FusedParams& p, int max_smem_optin) {
  const int budget = max_smem_optin - 1024;  // alignment slack
  auto bar_bytes = [](int stages) { return (2 * stages + 7 + 2 * kSideBufs) * 8 + 16; };
  // Side ring + deferred rows, then the ring (1024-aligned for the 128-byte swizzle).
  auto tail_from = [&](int off) {
    p.side_off = off;
    off += kSideBufs * kSideBytes;
    p.defer_off = off;
    off += kEpiWarps * 32 * kDeferStride * 4;
    return (off + 1023) & ~1023;
  };
  auto ring = [&](int off, int slot_bytes) {
    int stages = kMaxStages;
    while (stages >= 2 && off + stages * slot_bytes + bar_bytes(stages) > budget) --stages;
    return stages;
  };
  // Resident query tile (both parts) when it fits with at least two ring slots.
  if (p.nchunk <= kResChunks) {
    int off = 0;
    for (int part = 0; part < 2; ++part) {
      p.a_tx_bytes[part] = 0;
      for (int c = 0; c < p.nchunk; ++c) {
        const int bytes = kTileQ * p.chunk_w[c] * 2;
        p.a_off[part][c] = off;
        off += (bytes + 1023) & ~1023;
        p.a_tx_bytes[part] += bytes;
      }
    }
    off = tail_from(off);
    const int stages = ring(off, kUnitBytes);
    if (stages >= 2) {
      p.a_stream = 0;
      p.slot_bytes = kUnitBytes;
      p.slot_a_off = p.slot_alo_off = 0;
      p.stage_off = off;
      p.nstages = stages;
      p.bar_off = off + stages * kUnitBytes;
      p.smem_bytes = p.bar_off + bar_bytes(stages) + 1024;
      return true;
    }
  }
  // Streamed: each slot = database chunk + query hi chunk + query lo chunk (16 KB each).
  const int off = tail_from(0);
  const int slot_bytes = kUnitBytes + 2 * (kTileQ * 64 * 2);
  const int stages = ring(off, slot_bytes);
  if (stages < 2) return false;
  p.a_stream = 1;
  p.slot_bytes = slot_bytes;
  p.slot_a_off = kUnitBytes;
  p.slot_alo_off = kUnitBytes + kTileQ * 64 * 2;
  p.a_tx_bytes[0] = p.a_tx_bytes[1] = 0;
  p.stage_off = off;
  p.nstages = stages;
  p.bar_off = off + stages * slot_bytes;
  p.smem_bytes = p.bar_off + bar_bytes(stages) + 1024;
  return true;
}

cudaError_t launch_knn_fused(const FusedMaps& maps, const FusedParams& p, int kl, int grid,
                             cudaStream_t stream) {
  if (p.n_peers > 0) {  // sharded search sharing its bounds (list mode, conservative filter)
    switch (kl) {
      case 4:
        return launch_kl<4, false, true>(maps, p, grid, stream);
      case 8:
        return launch_kl<8, false, true>(maps, p, grid, stream);
      case 12:
        return launch_kl<12, false, true>(maps, p, grid, stream);
      case 16:
        return launch_kl<16, false, true>(maps, p, grid, stream);
      case 32:
        return launch_kl<32, false, true>(maps, p, grid, stream);
      default:
        break;  // append mode has no lists to publish
    }
  }
  if (p.exact_filter && p.rank_kind != kRankScaled) {
    switch (kl) {
      case 4:
        return launch_kl<4, true>(maps, p, grid, stream);
      case 8:
        return launch_kl<8, true>(maps, p, grid, stream);
      case 12:
        return launch_kl<12, true>(maps, p, grid, stream);
      default:
        break;  // longer lists: the conservative filter
    }
  }
  switch (kl) {
    case 4:
      return launch_kl<4>(maps, p, grid, stream);
    case 8:
      return launch_kl<8>(maps, p, grid, stream);
    case 12:
      return launch_kl<12>(maps, p, grid, stream);
    case 16:
      return launch_kl<16>(maps, p, grid, stream);
    case 32:
      return launch_kl<32>(maps, p, grid, stream);
    case 0:
      return launch_kl<0>(maps, p, grid, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace prim
}  // namespace ovvs
