// IVF-Flat list scan kernels (see ivf_scan.cuh).
#include "ivf_scan.cuh"

#include <math.h>

#include "keys.cuh"

namespace ovvs {
namespace prim {
namespace {

constexpr int kThreads = 256;  // 16 x 16 threads, 4 x 4 (pair, row) scores each (strided by 16)
constexpr int kTK = 32;        // K slab staged in shared memory (row-major, 8 float4 per row)
constexpr int kSlabStride = kTK + 4;  // floats per staged row: 16-byte aligned, float4 reads of
                                      // 16 consecutive rows fall on distinct bank groups
constexpr int kPadR = kIvfRows + 1;

// ovvsMetric values (ovvs.h)
constexpr int kRawL2 = 0, kRawL2Sqrt = 1, kRawIp = 2, kRawCosine = 3, kRawHamming = 4, kRawLp = 5;

// How a metric accumulates over the dimensions (prim_pairwise, mixer.cpp:174-197: the three
// expanded metrics go through the dot product; every other one through distance_one,
// internal.hpp:240-272, whose default is the squared L2 of l2sq).
enum AccKind : int { kAccDot = 0, kAccL2 = 1, kAccHamming = 2, kAccLp = 3 };

__host__ __device__ inline int acc_kind(int metric) {
  switch (metric) {
    case kRawL2:
    case kRawIp:
    case kRawCosine:
      return kAccDot;
    case kRawHamming:
      return kAccHamming;
    case kRawLp:
      return kAccLp;
    default:
      return kAccL2;
  }
}

// The IVF search calls prim_pairwise with metric_arg = 2 (indexes.cpp:334).
constexpr float kLpP = 2.f;

template <int ACC>
__device__ __forceinline__ void accumulate(float& acc, int& cnt, float x, float y) {
  if constexpr (ACC == kAccDot) {
    acc = __fadd_rn(acc, __fmul_rn(x, y));
  } else if constexpr (ACC == kAccL2) {
    const float d = __fsub_rn(x, y);
    acc = __fadd_rn(acc, __fmul_rn(d, d));
  } else if constexpr (ACC == kAccHamming) {
    cnt += static_cast<int>((x >= 0.f) != (y >= 0.f));
  } else {
    const float p = kLpP;
    acc = __fadd_rn(acc, powf(fabsf(__fsub_rn(x, y)), p));
  }
}

// The score of one (query, row) pair from its accumulated value: the reference's epilogue
// (mixer.cpp:184-197) for the expanded metrics, distance_one's last step for the others.
template <int ACC>
__device__ __forceinline__ float finish(int metric, float acc, int cnt, float qn, float yn) {
  if constexpr (ACC == kAccDot) {
    if (metric == kRawIp) return -acc;
    if (metric == kRawCosine) {
      const float nxv = __fsqrt_rn(qn < 1e-12f ? 1e-12f : qn);
      const float nyv = __fsqrt_rn(yn < 1e-12f ? 1e-12f : yn);
      return __fsub_rn(1.f, __fdiv_rn(acc, __fmul_rn(nxv, nyv)));
    }
    return __fsub_rn(__fadd_rn(qn, yn), __fmul_rn(2.f, acc));
  } else if constexpr (ACC == kAccL2) {
    return metric == kRawL2Sqrt ? __fsqrt_rn(acc) : acc;
  } else if constexpr (ACC == kAccHamming) {
    return static_cast<float>(cnt);
  } else {
    const float p = kLpP;
    return powf(acc, __fdiv_rn(1.f, p));
  }
}

// allowed() of internal.hpp:274-277. Ids outside the dataset occur only in a hand-made index
// file; the reference would read past the bitset for them, here they count as filtered.
__device__ __forceinline__ bool allowed(const uint8_t* bitset, int64_t bits, int64_t id) {
  if (!bitset) return true;
  if (id < 0 || id >= bits) return false;
  return (bitset[id >> 3] >> (id & 7)) & 1u;
}

// The exact score of one pair, sequential over the dimensions (used for the reported
// distances; it repeats the scan's arithmetic operation for operation).
__device__ float exact_score(int metric, const float* q, float qn, const float* y, float yn,
                             int dim) {
  float acc = 0.f;
  int cnt = 0;
  switch (acc_kind(metric)) {
    case kAccDot:
      for (int d = 0; d < dim; ++d) accumulate<kAccDot>(acc, cnt, q[d], y[d]);
      return finish<kAccDot>(metric, acc, cnt, qn, yn);
    case kAccHamming:
      for (int d = 0; d < dim; ++d) accumulate<kAccHamming>(acc, cnt, q[d], y[d]);
      return finish<kAccHamming>(metric, acc, cnt, qn, yn);
    case kAccLp:
      for (int d = 0; d < dim; ++d) accumulate<kAccLp>(acc, cnt, q[d], y[d]);
      return finish<kAccLp>(metric, acc, cnt, qn, yn);
    default:
      for (int d = 0; d < dim; ++d) accumulate<kAccL2>(acc, cnt, q[d], y[d]);
      return finish<kAccL2>(metric, acc, cnt, qn, yn);
  }
}

// Inserts key x into the ascending list[0..K) held in shared memory (its last entry drops out).
// Lane l owns entries [l*S, l*S + S), S = ceil(K / 32) <= 8. Keys are unique, so the insertion
// point is the count of smaller entries.
__device__ __forceinline__ void warp_insert(uint64_t* list, int K, uint64_t x, int lane) {
  const int S = (K + 31) >> 5;
  const int base = lane * S;
  uint64_t vals[kIvfMaxSelect / 32];
  int less = 0;
#pragma unroll
  for (int s = 0; s < kIvfMaxSelect / 32; ++s) {
    if (s < S) {
      const int i = base + s;
      vals[s] = i < K ? list[i] : keys::kEmptyKey;
      less += static_cast<int>(i < K && vals[s] < x);
    }
  }
  const uint64_t prev = (base > 0 && base - 1 < K) ? list[base - 1] : keys::kEmptyKey;
  const int pos = __reduce_add_sync(0xffffffffu, less);
  __syncwarp();
#pragma unroll
  for (int s = 0; s < kIvfMaxSelect / 32; ++s) {
    if (s < S) {
      const int i = base + s;
      if (i < K && i >= pos) list[i] = i == pos ? x : (s == 0 ? prev : vals[s - 1]);
    }
  }
  __syncwarp();
}

// warp_insert for K <= 32: one entry per lane.
__device__ __forceinline__ void warp_insert_small(uint64_t* list, int K, uint64_t x, int lane) {
  const uint64_t v = lane < K ? list[lane] : keys::kEmptyKey;
  const int pos = __popc(__ballot_sync(0xffffffffu, v < x));
  const uint64_t up = __shfl_up_sync(0xffffffffu, v, 1);
  __syncwarp();
  if (lane < K && lane >= pos) list[lane] = lane == pos ? x : up;
  __syncwarp();
}

__device__ __forceinline__ void insert_key(uint64_t* list, int K, uint64_t x, int lane) {
  if (K <= 32)
    warp_insert_small(list, K, x, lane);
  else
    warp_insert(list, K, x, lane);
}

// Work item -> list: the largest c with item_off[c] <= item.
__device__ __forceinline__ int list_of_item(const int* item_off, int nlist, int item) {
  int lo = 0, hi = nlist - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (item_off[mid] <= item)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

// One work item = one list c and up to kIvfPairs (query, probe) pairs that probe it. The list's
// rows are scored in tiles of kIvfRows against all the item's queries (4 x 4 per thread, every
// score accumulated over d = 0, 1, ... with separately rounded operations; zero padding past dim
// adds +0 products, which leave every metric's sum unchanged).
//   SORT = false: each pair keeps its k_sel smallest keys in shared memory, written to cand.
//   SORT = true:  every candidate's key is written to its place in the query's segment.
// Staging of one K slab: the item's query rows (by index) and the tile's list rows, row-major
// with kSlabStride floats per row, zero outside the matrices. VEC: 16-byte loads (dim a multiple
// of 4 and both bases 16-byte aligned); the slab is fetched into registers first (`fetch`) so its
// global latency overlaps the previous slab's arithmetic, then stored (`store`).
template <bool VEC>
struct Stager {
  static constexpr int kPer = VEC ? 2 : 8;  // float4 / float elements per thread per matrix
  float4 ra[VEC ? 2 : 1], rb[VEC ? 2 : 1];
  float sa[VEC ? 1 : 8], sb[VEC ? 1 : 8];
  __device__ __forceinline__ void fetch(const IvfScanParams& p, const int* s_q, int64_t row0,
                                        int64_t j0, int64_t L, int t0, int tid) {
    const int dim = p.dim;
    if constexpr (VEC) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int e = tid + kThreads * i, r = e >> 3, c = (e & 7) * 4;
        const int q = s_q[r];
        const bool in = t0 + c < dim;
        ra[i] = (q >= 0 && in)
                    ? *reinterpret_cast<const float4*>(p.queries + static_cast<int64_t>(q) * dim + t0 + c)
                    : make_float4(0.f, 0.f, 0.f, 0.f);
        const int64_t j = j0 + r;
        rb[i] = (j < L && in) ? *reinterpret_cast<const float4*>(p.rows + (row0 + j) * dim + t0 + c)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int e = tid + kThreads * i, r = e >> 5, c = e & 31;
        const int q = s_q[r];
        const bool in = t0 + c < dim;
        sa[i] = (q >= 0 && in) ? p.queries[static_cast<int64_t>(q) * dim + t0 + c] : 0.f;
        const int64_t j = j0 + r;
        sb[i] = (j < L && in) ? p.rows[(row0 + j) * dim + t0 + c] : 0.f;
      }
    }
  }
  __device__ __forceinline__ void store(float* As, float* Bs, int tid) {
    if constexpr (VEC) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int e = tid + kThreads * i, r = e >> 3, c = (e & 7) * 4;
        *reinterpret_cast<float4*>(As + r * kSlabStride + c) = ra[i];
        *reinterpret_cast<float4*>(Bs + r * kSlabStride + c) = rb[i];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int e = tid + kThreads * i, r = e >> 5, c = e & 31;
        As[r * kSlabStride + c] = sa[i];
        Bs[r * kSlabStride + c] = sb[i];
      }
    }
  }
};

// Three CTAs per SM (at most 85 registers): the k loop is not unrolled, which keeps the main
// variants free of spills and measured 4 % faster than two CTAs per SM with the loop unrolled.
template <int ACC, bool SORT, bool VEC>
__global__ void __launch_bounds__(kThreads, 3)
    ivf_scan_kernel(const __grid_constant__ IvfScanParams p) {
  extern __shared__ __align__(16) uint8_t dyn[];
  uint64_t* lists = reinterpret_cast<uint64_t*>(dyn);
  __shared__ __align__(16) float As[kIvfPairs * kSlabStride];
  __shared__ __align__(16) float Bs[kIvfRows * kSlabStride];
  __shared__ float S[SORT ? 1 : kIvfPairs][kPadR];
  __shared__ int s_q[kIvfPairs];
  __shared__ int s_pair[kIvfPairs];
  __shared__ uint32_t s_cum[kIvfPairs];
  __shared__ float s_qn[kIvfPairs];
  __shared__ int64_t s_seg[SORT ? kIvfPairs : 1];

  const int item = static_cast<int>(blockIdx.x);
  if (item >= p.item_off[p.nlist]) return;
  const int c = list_of_item(p.item_off, p.nlist, item);
  const int chunk = item - p.item_off[c];
  const int pair0 = p.list_q_off[c] + chunk * kIvfPairs;
  const int npairs = min(kIvfPairs, p.list_q_off[c + 1] - pair0);
  const int64_t row0 = p.list_off[c];
  const int64_t L = p.list_off[c + 1] - row0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tx = tid & 15, ty = tid >> 4;
  const int dim = p.dim;

  if (tid < kIvfPairs) {
    if (tid < npairs) {
      const int pr = p.pair_of[pair0 + tid];
      const int q = pr / p.nprobe, pp = pr - q * p.nprobe;
      s_q[tid] = q;
      s_pair[tid] = pr;
      s_cum[tid] = p.cum[static_cast<int64_t>(q) * (p.nprobe + 1) + pp];
      s_qn[tid] = p.q_norm[q];
      if constexpr (SORT) s_seg[tid] = p.seg_base[q];
    } else {
      s_q[tid] = -1;
      s_pair[tid] = -1;
      s_cum[tid] = 0;
      s_qn[tid] = 0.f;
    }
  }
  if constexpr (!SORT) {
    for (int e = tid; e < npairs * p.k_sel; e += kThreads) lists[e] = keys::kEmptyKey;
  }
  __syncthreads();

  for (int64_t j0 = 0; j0 < L; j0 += kIvfRows) {
    float acc[4][4];
    int cnt[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        acc[a][b] = 0.f;
        cnt[a][b] = 0;
      }
    Stager<VEC> st;
    st.fetch(p, s_q, row0, j0, L, 0, tid);
    for (int t0 = 0; t0 < dim; t0 += kTK) {
      __syncthreads();  // the previous slab's reads are done
      st.store(As, Bs, tid);
      __syncthreads();
      if (t0 + kTK < dim) st.fetch(p, s_q, row0, j0, L, t0 + kTK, tid);
      // every score sums its products in k order: float4 reads along k, then the four steps
#pragma unroll 1
      for (int t = 0; t < kTK; t += 4) {
        float4 av[4], bv[4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
          av[a] = *reinterpret_cast<const float4*>(As + (ty + 16 * a) * kSlabStride + t);
#pragma unroll
        for (int b = 0; b < 4; ++b)
          bv[b] = *reinterpret_cast<const float4*>(Bs + (tx + 16 * b) * kSlabStride + t);
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            accumulate<ACC>(acc[a][b], cnt[a][b], av[a].x, bv[b].x);
            accumulate<ACC>(acc[a][b], cnt[a][b], av[a].y, bv[b].y);
            accumulate<ACC>(acc[a][b], cnt[a][b], av[a].z, bv[b].z);
            accumulate<ACC>(acc[a][b], cnt[a][b], av[a].w, bv[b].w);
          }
      }
    }
    // scores (+inf for filtered rows, indexes.cpp:336-339)
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const int pi = ty + 16 * a;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int rj = tx + 16 * b;
        const int64_t j = j0 + rj;
        if (pi < npairs && j < L) {
          float v = finish<ACC>(p.metric, acc[a][b], cnt[a][b], s_qn[pi], p.row_norm[row0 + j]);
          if (p.bitset && !allowed(p.bitset, p.bitset_bits, p.row_ids[row0 + j]))
            v = __int_as_float(0x7f800000);
          if constexpr (SORT) {
            const uint32_t pos = s_cum[pi] + static_cast<uint32_t>(j);
            p.keys[s_seg[pi] + pos] = keys::make_key(v, pos);
          } else {
            S[pi][rj] = v;
          }
        }
      }
    }
    if constexpr (!SORT) {
      __syncthreads();
      // warp w keeps the lists of pairs 8w .. 8w+7
      for (int i = 0; i < kIvfPairs / 8; ++i) {
        const int pi = warp * (kIvfPairs / 8) + i;
        if (pi >= npairs) break;
        uint64_t* list = lists + static_cast<size_t>(pi) * p.k_sel;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int rj = lane + 32 * half;
          const int64_t j = j0 + rj;
          const uint64_t key = j < L ? keys::make_key(S[pi][rj], s_cum[pi] + static_cast<uint32_t>(j))
                                     : keys::kEmptyKey;
          uint32_t mask = __ballot_sync(0xffffffffu, key < list[p.k_sel - 1]);
          while (mask) {
            const int src = __ffs(mask) - 1;
            mask &= mask - 1;
            const uint64_t x = __shfl_sync(0xffffffffu, key, src);
            if (x < list[p.k_sel - 1]) insert_key(list, p.k_sel, x, lane);
          }
        }
      }
      __syncthreads();
    }
  }
  if constexpr (!SORT) {
    for (int e = tid; e < npairs * p.k_sel; e += kThreads) {
      const int pi = e / p.k_sel, i = e - pi * p.k_sel;
      p.cand[static_cast<size_t>(s_pair[pi]) * p.k_sel + i] = lists[e];
    }
  }
}

__global__ void probe_offsets_kernel(const int64_t* __restrict__ probe, int64_t nq, int nprobe,
                                     const int64_t* __restrict__ list_off, int nlist,
                                     uint32_t* __restrict__ cum, int* __restrict__ list_q_count) {
  const int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  uint32_t acc = 0;
  uint32_t* out = cum + q * (nprobe + 1);
  for (int pp = 0; pp < nprobe; ++pp) {
    const int64_t c = probe[q * nprobe + pp];
    out[pp] = acc;
    if (c >= 0 && c < nlist) {
      acc += static_cast<uint32_t>(list_off[c + 1] - list_off[c]);
      atomicAdd(&list_q_count[c], 1);
    }
  }
  out[nprobe] = acc;
}

__global__ void group_pairs_kernel(const int64_t* __restrict__ probe, int64_t nq, int nprobe,
                                   int nlist, const int* __restrict__ list_q_off,
                                   int* __restrict__ cursor, int* __restrict__ pair_of) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= nq * nprobe) return;
  const int64_t c = probe[e];
  if (c < 0 || c >= nlist) return;
  const int slot = atomicAdd(&cursor[c], 1);
  pair_of[list_q_off[c] + slot] = static_cast<int>(e);
}

__global__ void item_counts_kernel(const int* __restrict__ list_q_count, int nlist,
                                   int* __restrict__ item_count) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c > nlist) return;
  item_count[c] = c < nlist ? (list_q_count[c] + kIvfPairs - 1) / kIvfPairs : 0;
}

// One warp per query: the k smallest keys of its candidates (merged from the per-pair lists in
// select mode, the head of its sorted segment in sort mode), then ids and exact distances.
__global__ void ivf_emit_kernel(const __grid_constant__ IvfScanParams p,
                                const uint64_t* __restrict__ sorted_keys, int64_t k,
                                int64_t* __restrict__ neighbors, float* __restrict__ distances) {
  extern __shared__ __align__(16) uint8_t dyn[];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + wib;
  if (q >= p.nq) return;
  const int np = p.nprobe;
  const uint32_t* cum = p.cum + q * (np + 1);
  const uint32_t total = cum[np];
  const uint64_t* best;
  if (sorted_keys == nullptr) {
    uint64_t* list = reinterpret_cast<uint64_t*>(dyn) + static_cast<size_t>(wib) * k;
    for (int64_t i = lane; i < k; i += 32) list[i] = keys::kEmptyKey;
    __syncwarp();
    const int K = static_cast<int>(k);
    const int64_t n_in = static_cast<int64_t>(np) * p.k_sel;
    const uint64_t* in = p.cand + q * n_in;
    for (int64_t b = 0; b < n_in; b += 32) {
      const uint64_t key = b + lane < n_in ? in[b + lane] : keys::kEmptyKey;
      uint32_t mask = __ballot_sync(0xffffffffu, key < list[K - 1]);
      while (mask) {
        const int src = __ffs(mask) - 1;
        mask &= mask - 1;
        const uint64_t x = __shfl_sync(0xffffffffu, key, src);
        if (x < list[K - 1]) insert_key(list, K, x, lane);
      }
    }
    best = list;
  } else {
    best = sorted_keys + p.seg_base[q];
  }
  const int64_t kk = static_cast<int64_t>(total) < k ? static_cast<int64_t>(total) : k;
  const float inf = __int_as_float(0x7f800000);
  for (int64_t t = lane; t < k; t += 32) {
    int64_t id = -1;
    float d = inf;
    const uint64_t key = t < kk ? best[t] : keys::kEmptyKey;
    if (t < kk && key != keys::kEmptyKey) {
      const uint32_t pos = keys::key_id(key);
      // probe of this position: the last pp with cum[pp] <= pos
      int lo = 0, hi = np - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (cum[mid] <= pos)
          lo = mid;
        else
          hi = mid - 1;
      }
      const int64_t c = p.probe[q * np + lo];
      const int64_t g = p.list_off[c] + (pos - cum[lo]);
      id = p.row_ids[g];
      const float* qr = p.queries + q * p.dim;
      float v = exact_score(p.metric, qr, p.q_norm[q], p.rows + g * p.dim, p.row_norm[g], p.dim);
      if (p.bitset && !allowed(p.bitset, p.bitset_bits, id)) v = inf;
      d = p.metric == kRawIp ? -v : v;
    }
    neighbors[q * k + t] = id;
    distances[q * k + t] = d;
  }
}

__global__ void gather_list_rows_kernel(const float* __restrict__ x, int64_t n_x, int dim,
                                        const int64_t* __restrict__ ids, int64_t n_rows,
                                        float* __restrict__ rows, float* __restrict__ row_norm) {
  const int lane = threadIdx.x & 31;
  const int64_t g = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (g >= n_rows) return;
  const int64_t id = ids[g];
  const bool ok = id >= 0 && id < n_x;
  float* dst = rows + g * dim;
  for (int d = lane; d < dim; d += 32) dst[d] = ok ? x[id * dim + d] : 0.f;
  __syncwarp();
  if (lane == 0) {
    float s = 0.f;  // nrm2sq (internal.hpp:221-225): sequential
    for (int d = 0; d < dim; ++d) s = __fadd_rn(s, __fmul_rn(dst[d], dst[d]));
    row_norm[g] = s;
  }
}

// One warp per score row: the K smallest (score, column) keys by warp insertion into a list in
// shared memory, then their columns.
__global__ void coarse_select_kernel(const float* __restrict__ scores, int64_t rows, int cols,
                                     int K, int64_t* __restrict__ probe) {
  extern __shared__ __align__(16) uint8_t dyn[];
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + wib;
  if (r >= rows) return;
  uint64_t* list = reinterpret_cast<uint64_t*>(dyn) + static_cast<size_t>(wib) * K;
  for (int i = lane; i < K; i += 32) list[i] = keys::kEmptyKey;
  __syncwarp();
  const float* row = scores + r * cols;
  for (int b = 0; b < cols; b += 32) {
    const int j = b + lane;
    const uint64_t key = j < cols ? keys::make_key(row[j], static_cast<uint32_t>(j)) : keys::kEmptyKey;
    uint32_t mask = __ballot_sync(0xffffffffu, key < list[K - 1]);
    while (mask) {
      const int src = __ffs(mask) - 1;
      mask &= mask - 1;
      const uint64_t x = __shfl_sync(0xffffffffu, key, src);
      if (x < list[K - 1]) insert_key(list, K, x, lane);
    }
  }
  for (int i = lane; i < K; i += 32) {
    const uint64_t key = list[i];
    probe[r * K + i] = key == keys::kEmptyKey ? -1 : static_cast<int64_t>(keys::key_id(key));
  }
}

__global__ void totals_kernel(const uint32_t* __restrict__ cum, int64_t nq, int nprobe,
                              int64_t* __restrict__ totals) {
  const int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q > nq) return;
  totals[q] = q < nq ? static_cast<int64_t>(cum[q * (nprobe + 1) + nprobe]) : 0;
}

__global__ void seg_bounds_kernel(const int64_t* __restrict__ seg_base,
                                  const uint32_t* __restrict__ cum, int64_t nq, int nprobe,
                                  int* __restrict__ seg_begin, int* __restrict__ seg_end) {
  const int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= nq) return;
  seg_begin[q] = static_cast<int>(seg_base[q]);
  seg_end[q] = static_cast<int>(seg_base[q] + cum[q * (nprobe + 1) + nprobe]);
}

template <bool SORT>
cudaError_t launch_scan(const IvfScanParams& p, int64_t grid, cudaStream_t stream) {
  if (grid <= 0) return cudaSuccess;
  if (grid > 0x7fffffffLL) return cudaErrorInvalidValue;
  const size_t dyn = SORT ? 0 : static_cast<size_t>(kIvfPairs) * p.k_sel * sizeof(uint64_t);
  const dim3 g(static_cast<unsigned>(grid));
  auto run = [&](auto kern) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(dyn));
    if (e != cudaSuccess) return e;
    kern<<<g, kThreads, dyn, stream>>>(p);
    return cudaGetLastError();
  };
  const bool vec = p.dim % 4 == 0 && (reinterpret_cast<uintptr_t>(p.queries) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(p.rows) & 15) == 0;
  switch (acc_kind(p.metric)) {
    case kAccDot:
      return vec ? run(ivf_scan_kernel<kAccDot, SORT, true>)
                 : run(ivf_scan_kernel<kAccDot, SORT, false>);
    case kAccHamming:
      return vec ? run(ivf_scan_kernel<kAccHamming, SORT, true>)
                 : run(ivf_scan_kernel<kAccHamming, SORT, false>);
    case kAccLp:
      return vec ? run(ivf_scan_kernel<kAccLp, SORT, true>)
                 : run(ivf_scan_kernel<kAccLp, SORT, false>);
    default:
      return vec ? run(ivf_scan_kernel<kAccL2, SORT, true>)
                 : run(ivf_scan_kernel<kAccL2, SORT, false>);
  }
}

// ---- tensor-core list scan helpers ---------------------------------------------------------
constexpr int kTcSlots = 256;  // slots per pair tile of the fused kernel

__global__ void tc_counts_kernel(const int* __restrict__ list_q_count,
                                 const int2* __restrict__ list_tiles, int nlist,
                                 int* __restrict__ slot_count, int* __restrict__ item_count) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c > nlist) return;
  // an empty list gets no slots (its pairs have no candidates)
  const int cnt = c < nlist && list_tiles[c].y > list_tiles[c].x ? list_q_count[c] : 0;
  const int padded = (cnt + kTcSlots - 1) / kTcSlots * kTcSlots;
  slot_count[c] = padded;
  item_count[c] = padded / kTcSlots;
}

// Allow bits by padded position (bit b of word w = position 32 w + b): the bitset bit of the
// position's original id; padding positions and ids outside the bitset are not allowed.
__global__ void tc_allow_kernel(const uint8_t* __restrict__ bitset, int64_t bits,
                                const int64_t* __restrict__ pos_row,
                                const int64_t* __restrict__ row_ids, int64_t n_pos,
                                uint32_t* __restrict__ allow_pos) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w * 32 >= n_pos) return;
  uint32_t word = 0;
  for (int b = 0; b < 32; ++b) {
    const int64_t pos = w * 32 + b;
    const int64_t g = pos < n_pos ? pos_row[pos] : -1;
    if (g >= 0 && allowed(bitset, bits, row_ids[g])) word |= 1u << b;
  }
  allow_pos[w] = word;
}

// One block per list.
__global__ void tc_fill_kernel(const int* __restrict__ list_q_count,
                               const int* __restrict__ list_q_off, const int* __restrict__ pair_of,
                               const int* __restrict__ slot_off, const int* __restrict__ item_off,
                               const int2* __restrict__ list_tiles, int* __restrict__ slot_pair,
                               int* __restrict__ pair_slot, int4* __restrict__ item_tab) {
  const int c = blockIdx.x;
  const int cnt = list_q_count[c];
  const int s0 = slot_off[c], ns = slot_off[c + 1] - s0;
  for (int i = threadIdx.x; i < ns; i += blockDim.x) {
    const int pair = i < cnt ? pair_of[list_q_off[c] + i] : -1;
    slot_pair[s0 + i] = pair;
    if (pair >= 0) pair_slot[pair] = s0 + i;
  }
  const int i0 = item_off[c], ni = item_off[c + 1] - i0;
  const int2 tiles = list_tiles[c];
  for (int j = threadIdx.x; j < ni; j += blockDim.x)
    item_tab[i0 + j] = make_int4(s0 / kTcSlots + j, tiles.x, tiles.y, 0);
}

// One warp per slot; rows of row_halves fp16 values copied as 16-byte words.
__global__ void tc_gather_kernel(const uint4* __restrict__ a16_query,
                                 const float* __restrict__ q_mul_query,
                                 const int* __restrict__ slot_pair, int nprobe, int64_t slots,
                                 int words, uint4* __restrict__ a16_slot,
                                 float* __restrict__ q_mul_slot) {
  const int lane = threadIdx.x & 31;
  const int64_t s = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (s >= slots) return;
  const int pair = slot_pair[s];
  const int64_t q = pair >= 0 ? pair / nprobe : 0;
  for (int w = lane; w < words; w += 32)
    a16_slot[s * words + w] = pair >= 0 ? a16_query[q * words + w] : make_uint4(0, 0, 0, 0);
  if (lane == 0) q_mul_slot[s] = pair >= 0 ? q_mul_query[q] : -1.f;
}

// exact_score with the row read four columns at a time (rows 16-byte aligned, dim % 4 == 0);
// the same operations in the same order.
template <int ACC>
__device__ float exact_score_v4(int metric, const float* q, float qn, const float* y, float yn,
                                int dim) {
  float acc = 0.f;
  int cnt = 0;
  const float4* y4 = reinterpret_cast<const float4*>(y);
  for (int d4 = 0; d4 < dim / 4; ++d4) {
    const float4 v = __ldg(y4 + d4);
    accumulate<ACC>(acc, cnt, q[4 * d4], v.x);
    accumulate<ACC>(acc, cnt, q[4 * d4 + 1], v.y);
    accumulate<ACC>(acc, cnt, q[4 * d4 + 2], v.z);
    accumulate<ACC>(acc, cnt, q[4 * d4 + 3], v.w);
  }
  return finish<ACC>(metric, acc, cnt, qn, yn);
}

__device__ __forceinline__ uint64_t warp_sort_asc(uint64_t key, int lane) {
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, key, stride);
      const bool up = (lane & size) == 0;
      const bool lower = (lane & stride) == 0;
      key = (lower == up) ? (other < key ? other : key) : (other > key ? other : key);
    }
  }
  return key;
}

// One warp per (query, probe) pair; kl <= 16, so its 2 * kl candidates fit one per lane. Only
// the candidates that can reach the pair's exact top k_sel are re-scored: those whose
// approximate value is within the error margin of the k_sel-th best approximate value (the
// approximate values v = |y|^2 - 2 q.y are within ~1e-6 of their magnitudes of the exact ones;
// the margin is 1e-5 of the magnitudes of both values).
__global__ void tc_refine_kernel(const __grid_constant__ IvfScanParams p,
                                 const uint64_t* __restrict__ tc_cand, int kl,
                                 const int* __restrict__ pair_slot,
                                 const int64_t* __restrict__ pos_row) {
  const int lane = threadIdx.x & 31;
  const int64_t pair = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pair >= p.nq * p.nprobe) return;
  const int64_t q = pair / p.nprobe;
  const int pr = static_cast<int>(pair % p.nprobe);
  const int slot = pair_slot[pair];
  uint64_t approx = keys::kEmptyKey;
  int64_t g = -1;
  if (slot >= 0 && lane < 2 * kl) {
    approx = tc_cand[static_cast<int64_t>(slot) * 2 * kl + lane];
    // a list shorter than kl may hold padding positions (ranking value +inf): dropped
    g = approx != keys::kEmptyKey ? pos_row[keys::key_id(approx)] : -1;
    if (g < 0) approx = keys::kEmptyKey;
  }
  approx = warp_sort_asc(approx, lane);
  g = approx != keys::kEmptyKey ? pos_row[keys::key_id(approx)] : -1;
  const float qn = p.q_norm[q];
  const float yn = g >= 0 ? p.row_norm[g] : 0.f;
  const float va = keys::key_value(approx);  // NaN for an empty entry
  const float scale = g >= 0 ? fabsf(va) + qn + yn + 2.f * sqrtf(qn * yn) : 0.f;
  const float vk = __shfl_sync(0xffffffffu, va, p.k_sel - 1);
  float smax = lane < p.k_sel ? scale : 0.f;
#pragma unroll
  for (int off = 16; off; off >>= 1) smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, off));
  // rescore when the k_sel-th is empty or not finite, or when within the margin of it
  const bool rescore = g >= 0 && (lane < p.k_sel || !(fabsf(vk) < __int_as_float(0x7f800000)) ||
                                  !(va > vk + 1e-5f * (scale + smax)));
  uint64_t key = keys::kEmptyKey;
  if (rescore) {
    const int64_t list = p.probe[pair];
    const uint32_t concat =
        p.cum[q * (p.nprobe + 1) + pr] + static_cast<uint32_t>(g - p.list_off[list]);
    const float* qr = p.queries + q * p.dim;
    const float* yr = p.rows + g * p.dim;
    float v;
    if (p.bitset && !allowed(p.bitset, p.bitset_bits, p.row_ids[g])) {
      v = __int_as_float(0x7f800000);  // filtered: +inf, ordered by position (indexes.cpp:346-355)
    } else if ((p.dim & 3) == 0) {
      v = acc_kind(p.metric) == kAccDot
              ? exact_score_v4<kAccDot>(p.metric, qr, qn, yr, yn, p.dim)
              : exact_score_v4<kAccL2>(p.metric, qr, qn, yr, yn, p.dim);
    } else {
      v = exact_score(p.metric, qr, qn, yr, yn, p.dim);
    }
    key = keys::make_key(v, concat);
  }
  key = warp_sort_asc(key, lane);
  if (lane < p.k_sel) p.cand[pair * p.k_sel + lane] = key;
}

}  // namespace

int64_t ivf_max_items(int64_t nq, int nprobe, int nlist) {
  return nq * nprobe / kIvfPairs + nlist;
}

size_t ivf_select_smem(int k_sel) {
  return static_cast<size_t>(kIvfPairs) * k_sel * sizeof(uint64_t);
}

cudaError_t launch_ivf_probe_offsets(const int64_t* probe, int64_t nq, int nprobe,
                                     const int64_t* list_off, int nlist, uint32_t* cum,
                                     int* list_q_count, cudaStream_t stream) {
  probe_offsets_kernel<<<static_cast<unsigned>((nq + 127) / 128), 128, 0, stream>>>(
      probe, nq, nprobe, list_off, nlist, cum, list_q_count);
  return cudaGetLastError();
}

cudaError_t launch_ivf_group_pairs(const int64_t* probe, int64_t nq, int nprobe, int nlist,
                                   const int* list_q_off, int* cursor, int* pair_of,
                                   cudaStream_t stream) {
  const int64_t n = nq * nprobe;
  if (n <= 0) return cudaSuccess;
  group_pairs_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
      probe, nq, nprobe, nlist, list_q_off, cursor, pair_of);
  return cudaGetLastError();
}

cudaError_t launch_ivf_item_counts(const int* list_q_count, int nlist, int* item_count,
                                   cudaStream_t stream) {
  item_counts_kernel<<<static_cast<unsigned>((nlist + 1 + 255) / 256), 256, 0, stream>>>(
      list_q_count, nlist, item_count);
  return cudaGetLastError();
}

cudaError_t launch_ivf_scan_select(const IvfScanParams& p, int64_t grid, cudaStream_t stream) {
  if (p.k_sel < 1 || p.k_sel > kIvfMaxSelect) return cudaErrorInvalidValue;
  return launch_scan<false>(p, grid, stream);
}

cudaError_t launch_ivf_scan_sort(const IvfScanParams& p, int64_t grid, cudaStream_t stream) {
  return launch_scan<true>(p, grid, stream);
}

constexpr int kEmitWarps = 8;

size_t ivf_emit_smem(int64_t k) { return static_cast<size_t>(kEmitWarps) * k * sizeof(uint64_t); }

cudaError_t launch_ivf_emit(const IvfScanParams& p, const uint64_t* sorted_keys, int64_t k,
                            int64_t* neighbors, float* distances, cudaStream_t stream) {
  constexpr int kWarps = kEmitWarps;
  const size_t dyn = sorted_keys ? 0 : ivf_emit_smem(k);
  cudaError_t e = cudaFuncSetAttribute(ivf_emit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(dyn));
  if (e != cudaSuccess) return e;
  ivf_emit_kernel<<<static_cast<unsigned>((p.nq + kWarps - 1) / kWarps), kWarps * 32, dyn,
                    stream>>>(p, sorted_keys, k, neighbors, distances);
  return cudaGetLastError();
}

cudaError_t launch_ivf_coarse_select(const float* scores, int64_t rows, int cols, int K,
                                     int64_t* probe, cudaStream_t stream) {
  if (K < 1 || K > kIvfMaxSelect) return cudaErrorInvalidValue;
  if (rows <= 0) return cudaSuccess;
  constexpr int kWarps = 8;
  const size_t dyn = static_cast<size_t>(kWarps) * K * sizeof(uint64_t);
  cudaError_t e = cudaFuncSetAttribute(coarse_select_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(dyn));
  if (e != cudaSuccess) return e;
  coarse_select_kernel<<<static_cast<unsigned>((rows + kWarps - 1) / kWarps), kWarps * 32, dyn,
                         stream>>>(scores, rows, cols, K, probe);
  return cudaGetLastError();
}

cudaError_t launch_ivf_totals(const uint32_t* cum, int64_t nq, int nprobe, int64_t* totals,
                              cudaStream_t stream) {
  totals_kernel<<<static_cast<unsigned>((nq + 1 + 255) / 256), 256, 0, stream>>>(cum, nq, nprobe,
                                                                                totals);
  return cudaGetLastError();
}

cudaError_t launch_ivf_seg_bounds(const int64_t* seg_base, const uint32_t* cum, int64_t nq,
                                  int nprobe, int* seg_begin, int* seg_end, cudaStream_t stream) {
  if (nq <= 0) return cudaSuccess;
  seg_bounds_kernel<<<static_cast<unsigned>((nq + 255) / 256), 256, 0, stream>>>(
      seg_base, cum, nq, nprobe, seg_begin, seg_end);
  return cudaGetLastError();
}

cudaError_t launch_ivf_tc_counts(const int* list_q_count, const int2* list_tiles, int nlist,
                                 int* slot_count, int* item_count, cudaStream_t stream) {
  tc_counts_kernel<<<static_cast<unsigned>((nlist + 1 + 255) / 256), 256, 0, stream>>>(
      list_q_count, list_tiles, nlist, slot_count, item_count);
  return cudaGetLastError();
}

cudaError_t launch_ivf_tc_allow(const uint8_t* bitset, int64_t bits, const int64_t* pos_row,
                                const int64_t* row_ids, int64_t n_pos, uint32_t* allow_pos,
                                cudaStream_t stream) {
  const int64_t words = (n_pos + 31) / 32;
  if (words <= 0) return cudaSuccess;
  tc_allow_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, stream>>>(
      bitset, bits, pos_row, row_ids, n_pos, allow_pos);
  return cudaGetLastError();
}

cudaError_t launch_ivf_tc_fill(const int* list_q_count, const int* list_q_off, const int* pair_of,
                               const int* slot_off, const int* item_off, const int2* list_tiles,
                               int nlist, int* slot_pair, int* pair_slot, int4* item_tab,
                               cudaStream_t stream) {
  if (nlist <= 0) return cudaSuccess;
  tc_fill_kernel<<<static_cast<unsigned>(nlist), 256, 0, stream>>>(
      list_q_count, list_q_off, pair_of, slot_off, item_off, list_tiles, slot_pair, pair_slot,
      item_tab);
  return cudaGetLastError();
}

cudaError_t launch_ivf_tc_gather(const void* a16_query, const float* q_mul_query,
                                 const int* slot_pair, int nprobe, int64_t slots, int row_halves,
                                 void* a16_slot, float* q_mul_slot, cudaStream_t stream) {
  if (slots <= 0) return cudaSuccess;
  if (row_halves % 8 != 0) return cudaErrorInvalidValue;  // whole 16-byte words per row
  tc_gather_kernel<<<static_cast<unsigned>((slots + 7) / 8), 256, 0, stream>>>(
      static_cast<const uint4*>(a16_query), q_mul_query, slot_pair, nprobe, slots, row_halves / 8,
      static_cast<uint4*>(a16_slot), q_mul_slot);
  return cudaGetLastError();
}

cudaError_t launch_ivf_tc_refine(const IvfScanParams& p, const uint64_t* tc_cand, int kl,
                                 const int* pair_slot, const int64_t* pos_row,
                                 cudaStream_t stream) {
  if (kl < 1 || kl > 16 || p.k_sel < 1 || p.k_sel > 2 * kl) return cudaErrorInvalidValue;
  const int64_t pairs = p.nq * p.nprobe;
  if (pairs <= 0) return cudaSuccess;
  tc_refine_kernel<<<static_cast<unsigned>((pairs + 7) / 8), 256, 0, stream>>>(p, tc_cand, kl,
                                                                              pair_slot, pos_row);
  return cudaGetLastError();
}

cudaError_t launch_ivf_gather_rows(const float* x, int64_t n_x, int dim, const int64_t* ids,
                                   int64_t n_rows, float* rows, float* row_norm,
                                   cudaStream_t stream) {
  if (n_rows <= 0) return cudaSuccess;
  gather_list_rows_kernel<<<static_cast<unsigned>((n_rows + 7) / 8), 256, 0, stream>>>(
      x, n_x, dim, ids, n_rows, rows, row_norm);
  return cudaGetLastError();
}

}  // namespace prim
}  // namespace ovvs
