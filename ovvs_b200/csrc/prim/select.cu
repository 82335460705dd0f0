// Candidate merge + exact re-ranking (see select.cuh).
#include "select.cuh"

#include "keys.cuh"
#include "prep.cuh"

namespace ovvs {
namespace prim {
namespace {

using keys::kEmptyKey;
constexpr unsigned kFull = 0xffffffffu;
constexpr int kMergeWarps = 4;

__device__ __forceinline__ void warp_argmin(uint64_t& k, int& l) {
#pragma unroll
  for (int off = 16; off; off >>= 1) {
    const uint64_t ok = __shfl_xor_sync(kFull, k, off);
    const int ol = __shfl_xor_sync(kFull, l, off);
    if (ok < k || (ok == k && ol < l)) {
      k = ok;
      l = ol;
    }
  }
}

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

// The reference's arithmetic for one (query, row) pair, in its operation order:
//   L2_EXPANDED   (xn + yn) - 2*ip             mixer.cpp:194 / cpu_prims.cpp:138
//   INNER_PRODUCT -ip                          mixer.cpp:186 (negated back for output)
//   COSINE        1 - ip / (sqrt(max(xn,1e-12)) * sqrt(max(yn,1e-12)))   mixer.cpp:188-190
//   L2_SQRT       sqrt(sum (x-y)^2)            internal.hpp:247-248
//   HAMMING       #{d : (x_d >= 0) != (y_d >= 0)}   internal.hpp:256-264
//   LP (p = 2)    sqrt(sum |x-y|^2)            internal.hpp:265-268 (pow(.,2) and pow(.,1/2))
//   other         sum (x-y)^2                  internal.hpp:269-270
// Sums are sequential over d with separately rounded multiply and add, like the reference's
// scalar loops; ip is cpu_gemm's sequential dot product (cpu_prims.cpp:48-58).
// The sums stay strictly sequential (the reference's order); only the loads are batched: 16
// elements of each row are loaded before their 16 in-order multiply/adds, so a query pays one
// memory latency per 16 dimensions instead of one per dimension.
constexpr int kSeqBlock = 16;

template <class Y>
__device__ __forceinline__ float seq_dot(const float* __restrict__ x, Y y, int D) {
  float ip = 0.f;
  int d = 0;
  for (; d + kSeqBlock <= D; d += kSeqBlock) {
    float xv[kSeqBlock], yv[kSeqBlock];
#pragma unroll
    for (int i = 0; i < kSeqBlock; ++i) {
      xv[i] = x[d + i];
      yv[i] = y(d + i);
    }
#pragma unroll
    for (int i = 0; i < kSeqBlock; ++i) ip = __fadd_rn(ip, __fmul_rn(xv[i], yv[i]));
  }
  for (; d < D; ++d) ip = __fadd_rn(ip, __fmul_rn(x[d], y(d)));
  return ip;
}

template <class Y>
__device__ __forceinline__ float seq_sqdiff(const float* __restrict__ x, Y y, int D) {
  float s = 0.f;
  int d = 0;
  for (; d + kSeqBlock <= D; d += kSeqBlock) {
    float xv[kSeqBlock], yv[kSeqBlock];
#pragma unroll
    for (int i = 0; i < kSeqBlock; ++i) {
      xv[i] = x[d + i];
      yv[i] = y(d + i);
    }
#pragma unroll
    for (int i = 0; i < kSeqBlock; ++i) {
      const float t = __fsub_rn(xv[i], yv[i]);
      s = __fadd_rn(s, __fmul_rn(t, t));
    }
  }
  for (; d < D; ++d) {
    const float t = __fsub_rn(x[d], y(d));
    s = __fadd_rn(s, __fmul_rn(t, t));
  }
  return s;
}

template <class Y>
__device__ __forceinline__ float exact_rank_with(const MergeParams& p, const float* __restrict__ x,
                                                 float xn, int64_t pos, Y y_at) {
  const int D = p.dim;
  switch (p.metric) {
    case kMetricL2:
    case kMetricInnerProduct:
    case kMetricCosine: {
      const float ip = seq_dot(x, y_at, D);
      if (p.metric == kMetricInnerProduct) return -ip;
      const float yn = p.norm_sorted[pos];
      if (p.metric == kMetricL2) return __fsub_rn(__fadd_rn(xn, yn), __fmul_rn(2.f, ip));
      const float nxv = __fsqrt_rn(xn < 1e-12f ? 1e-12f : xn);
      const float nyv = __fsqrt_rn(yn < 1e-12f ? 1e-12f : yn);
      return __fsub_rn(1.f, __fdiv_rn(ip, __fmul_rn(nxv, nyv)));
    }
    case kMetricHamming: {
      int c = 0;
      for (int d = 0; d < D; ++d) c += static_cast<int>((x[d] >= 0.f) != (y_at(d) >= 0.f));
      return static_cast<float>(c);
    }
    default: {
      const float s = seq_sqdiff(x, y_at, D);
      if (p.metric == kMetricL2Sqrt || p.metric == kMetricLp) return __fsqrt_rn(s);
      return s;
    }
  }
}

// Sums are sequential over d with separately rounded multiply and add, like the reference's
// scalar loops; ip is cpu_gemm's sequential dot product (cpu_prims.cpp:48-58).
__device__ float exact_rank(const MergeParams& p, const float* __restrict__ x, float xn,
                            int64_t pos) {
  if (p.exact32) {
    const float* __restrict__ y32 = p.exact32 + pos * p.dim;
    return exact_rank_with(p, x, xn, pos, [&](int d) { return y32[d]; });
  }
  const __half* __restrict__ y16 = p.rows16 + pos * p.rows16_stride;
  return exact_rank_with(p, x, xn, pos, [&](int d) { return __half2float(y16[d]); });
}

// The k = 1 assignment's shortcut (labels_only): when the best candidate's approximate value is
// below the second's by more than their error bound, the best id is the exact argmin. The
// approximate ranking values v = |y|^2 - 2 x.y differ from the exact ones by at most ~1e-6
// (|x| |y| + |v|) (split fp16 products, fp32 sums); the margin is 10x wider, so ties never take
// it. Writes the result and returns true when it applies.
__device__ __forceinline__ bool assign_shortcut(const MergeParams& p, int64_t q, float xn,
                                                uint64_t k0, uint64_t k1) {
  if (k0 == kEmptyKey) return false;
  const float v0 = keys::key_value(k0);
  const float v1 = k1 == kEmptyKey ? __int_as_float(0x7f800000) : keys::key_value(k1);
  const float yn0 = p.norm_sorted[p.inv_perm[keys::key_id(k0)]];
  const float yn1 = k1 == kEmptyKey ? 0.f : p.norm_sorted[p.inv_perm[keys::key_id(k1)]];
  const float fin = __int_as_float(0x7f800000);
  const bool finite = fabsf(v0) < fin && fabsf(xn) < fin && fabsf(yn0) < fin &&
                      fabsf(yn1) < fin && !(v1 != v1);
  const float margin =
      1e-5f * (fabsf(v0) + (k1 == kEmptyKey ? 0.f : fabsf(v1)) + xn + yn0 + yn1 +
               2.f * sqrtf(xn * yn0) + 2.f * sqrtf(xn * yn1)) + 1e-30f;
  if (!(finite && v1 - v0 > margin)) return false;
  p.neighbors[q] = p.row_offset + static_cast<int64_t>(keys::key_id(k0));
  p.distances[q] = __fadd_rn(xn, v0);
  return true;
}

__host__ __device__ inline bool use_assign_shortcut(const MergeParams& p) {
  return p.labels_only && p.k_eff == 1 && p.neighbors && p.allow == nullptr &&
         p.metric == kMetricL2;
}

// Merge + exact re-rank of query q by one warp (lists: this warp's KL x 32 keys of shared
// memory).
template <int KL>
__device__ void merge_query(const MergeParams& p, int64_t q, uint64_t* lists) {
  const int lane = threadIdx.x & 31;
  const uint64_t* c = p.cand + static_cast<size_t>(q) * p.num_sc * KL;
  const int total = p.num_sc * KL;
  uint64_t sel = kEmptyKey;
  if (total <= 32) {
    // Few candidates (small k, few lists, e.g. a k-means assignment): one per lane, a 32-key
    // bitonic sort, lane r keeps the r-th best.
    uint64_t key = lane < total ? c[lane] : kEmptyKey;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
      for (int stride = size >> 1; stride > 0; stride >>= 1) {
        const uint64_t other = __shfl_xor_sync(kFull, key, stride);
        const bool up = (lane & size) == 0;
        const bool lower = (lane & stride) == 0;
        const bool take_min = lower == up;
        key = take_min ? (other < key ? other : key) : (other > key ? other : key);
      }
    }
    sel = lane < KL ? key : kEmptyKey;
  } else {
    // 1. Each lane keeps the KL best keys of a strided share of the candidates.
    uint64_t L[KL];
#pragma unroll
    for (int i = 0; i < KL; ++i) L[i] = kEmptyKey;
    for (int e = lane; e < total; e += 32) {
      const uint64_t key = c[e];
      if (key < L[KL - 1]) list_insert<KL>(L, key);
    }
#pragma unroll
    for (int i = 0; i < KL; ++i) lists[lane * KL + i] = L[i];
    __syncwarp();

    // 2. Merge the 32 sorted lane lists: lane r receives the r-th best key overall.
    int ptr = 0;
    for (int r = 0; r < KL; ++r) {
      uint64_t k = ptr < KL ? lists[lane * KL + ptr] : kEmptyKey;
      int l = lane;
      warp_argmin(k, l);
      if (lane == l) ++ptr;
      if (lane == r) sel = k;
    }
  }

  // 3. Exact distance of each survivor.
  const float* x = p.queries + q * p.dim;
  const float xn = p.xn[q];
  if (use_assign_shortcut(p)) {
    const uint64_t k0 = __shfl_sync(kFull, sel, 0), k1 = __shfl_sync(kFull, sel, 1);
    bool done = false;
    if (lane == 0) done = assign_shortcut(p, q, xn, k0, k1);
    if (__shfl_sync(kFull, done, 0)) return;
  }
  float rank = __int_as_float(0x7fffffff);
  uint64_t key = kEmptyKey;
  if (sel != kEmptyKey) {
    const uint32_t id = keys::key_id(sel);
    const int64_t pos = p.inv_perm[id];
    const bool allowed = p.allow == nullptr || ((p.allow[pos >> 5] >> (pos & 31)) & 1u);
    rank = allowed ? exact_rank(p, x, xn, pos) : __int_as_float(0x7f800000);
    key = keys::make_key(rank, id);
  }

  // 4. Bitonic sort of the 32 (key, rank) pairs, ascending.
#pragma unroll
  for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      const uint64_t ok = __shfl_xor_sync(kFull, key, stride);
      const float orank = __shfl_xor_sync(kFull, rank, stride);
      const bool up = (lane & size) == 0;
      const bool lower = (lane & stride) == 0;
      const bool swap = (lower == up) ? (ok < key) : (ok > key);
      if (swap) {
        key = ok;
        rank = orank;
      }
    }
  }

  // 5. Emit the first k_eff.
  if (lane < p.k_eff) {
    const size_t o = static_cast<size_t>(q) * p.k_eff + lane;
    const bool empty = key == kEmptyKey;
    const int64_t gid = p.row_offset + static_cast<int64_t>(keys::key_id(key));
    if (p.neighbors) {
      p.neighbors[o] = empty ? -1 : gid;
      p.distances[o] = p.negate_output ? -rank : rank;
    } else {
      p.shard_rank[o] = rank;
      p.shard_gid[o] = empty ? INT64_MAX : gid;
    }
  }
}

template <int KL>
__global__ void __launch_bounds__(kMergeWarps * 32)
    merge_rerank_kernel(const MergeParams p) {
  extern __shared__ uint64_t merge_smem[];
  const int warp = threadIdx.x >> 5;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * kMergeWarps + warp;
  if (q >= p.nq) return;
  merge_query<KL>(p, q, merge_smem + warp * 32 * KL);
}

// k-means assignment (use_assign_shortcut, at most kAssignMaxCand candidates per point): one
// thread per point finds its two best candidate keys and takes the shortcut; the points where it
// does not apply (near-ties) are merged and re-ranked exactly by the whole warp, one at a time.
constexpr int kAssignMaxCand = 64;

template <int KL>
__global__ void __launch_bounds__(kMergeWarps * 32)
    assign_kernel(const MergeParams p) {
  extern __shared__ uint64_t merge_smem[];
  const int warp = threadIdx.x >> 5;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  bool slow = false;
  if (q < p.nq) {
    const int total = p.num_sc * KL;
    const uint64_t* c = p.cand + static_cast<size_t>(q) * total;
    uint64_t k0 = kEmptyKey, k1 = kEmptyKey;
    for (int e = 0; e < total; ++e) {
      const uint64_t key = c[e];
      if (key < k0) {
        k1 = k0;
        k0 = key;
      } else if (key < k1) {
        k1 = key;
      }
    }
    slow = !assign_shortcut(p, q, p.xn[q], k0, k1);
  }
  uint32_t pending = __ballot_sync(kFull, slow);
  while (pending) {
    const int src = __ffs(pending) - 1;
    pending &= pending - 1;
    merge_query<KL>(p, __shfl_sync(kFull, q, src), merge_smem + warp * 32 * KL);
  }
}

__global__ void shard_merge_kernel(const float* __restrict__ rank, const int64_t* __restrict__ gid,
                                   int world, int64_t nq, int k_eff, int negate,
                                   int64_t* __restrict__ neighbors, float* __restrict__ distances) {
  const int lane = threadIdx.x & 31;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (q >= nq) return;
  const size_t stride = static_cast<size_t>(nq) * k_eff;
  int ptr = 0;
  for (int r = 0; r < k_eff; ++r) {
    uint32_t ord = 0xFFFFFFFFu;
    int64_t g = INT64_MAX;
    float v = __int_as_float(0x7fffffff);
    if (lane < world && ptr < k_eff) {
      const size_t o = lane * stride + static_cast<size_t>(q) * k_eff + ptr;
      v = rank[o];
      g = gid[o];
      ord = keys::order_bits(v);
    }
    uint32_t bo = ord;
    int64_t bg = g;
    int bl = lane;
#pragma unroll
    for (int off = 16; off; off >>= 1) {
      const uint32_t oo = __shfl_xor_sync(kFull, bo, off);
      const int64_t og = __shfl_xor_sync(kFull, bg, off);
      const int ol = __shfl_xor_sync(kFull, bl, off);
      if (oo < bo || (oo == bo && (og < bg || (og == bg && ol < bl)))) {
        bo = oo;
        bg = og;
        bl = ol;
      }
    }
    const float bv = __shfl_sync(kFull, v, bl);
    if (lane == bl) ++ptr;
    if (lane == 0) {
      const size_t o = static_cast<size_t>(q) * k_eff + r;
      neighbors[o] = bg == INT64_MAX ? -1 : bg;
      distances[o] = negate ? -bv : bv;
    }
  }
}

__global__ void kth_bound_kernel(const uint64_t* __restrict__ cand, int num_sc, int64_t nq,
                                 int k, int KL, uint64_t* __restrict__ tau_key) {
  const int lane = threadIdx.x & 31;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (q >= nq) return;
  const uint64_t* c = cand + static_cast<size_t>(q) * num_sc * KL;
  // lane l walks lists l, l+32, ...: its head is the smallest unconsumed key among them
  int ptr[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int mine = (num_sc - lane + 31) / 32;  // lists owned by this lane (<= 8: num_sc <= 256)
  uint64_t kth = kEmptyKey;
  for (int r = 0; r < k; ++r) {
    uint64_t head = kEmptyKey;
    int which = -1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j < mine && ptr[j] < KL) {
        const uint64_t v = c[(lane + 32 * j) * KL + ptr[j]];
        if (v < head) {
          head = v;
          which = j;
        }
      }
    }
    uint64_t best = head;
    int bl = lane;
    warp_argmin(best, bl);
    if (best == kEmptyKey) {
      kth = kEmptyKey;
      break;
    }
    if (lane == bl) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j == which) ++ptr[j];
    }
    kth = best;
  }
  if (lane == 0) tau_key[q] = kth;
}

// Large k, between the stages of the append pass: the need-th smallest key among the keys a
// query has appended so far bounds its need-th best key overall (they are real rows), so it
// replaces tau_key[q] when smaller. Each lane keeps the 4 smallest keys of its strided share and
// the warp takes the need-th smallest of those 128: the need-th smallest of a subset is never
// below the set's, so the result stays a valid bound (a little looser when a lane held more
// than 4 of the set's smallest need).
__global__ void tighten_tau_kernel(const uint64_t* __restrict__ app_buf,
                                   const uint32_t* __restrict__ app_count, int cap, int64_t nq,
                                   int need, uint64_t* __restrict__ tau_key) {
  const int lane = threadIdx.x & 31;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (q >= nq) return;
  const int count = static_cast<int>(min(app_count[q], static_cast<uint32_t>(cap)));
  if (count < need) return;  // too few so far to bound rank `need`
  const uint64_t* b = app_buf + static_cast<size_t>(q) * cap;
  uint64_t L[4] = {kEmptyKey, kEmptyKey, kEmptyKey, kEmptyKey};
  for (int i = lane; i < count; i += 32) {
    const uint64_t key = b[i];
    if (key < L[3]) list_insert<4>(L, key);
  }
  int ptr = 0;
  uint64_t kth = kEmptyKey;
  for (int r = 0; r < need; ++r) {
    uint64_t head = ptr == 0 ? L[0] : ptr == 1 ? L[1] : ptr == 2 ? L[2] : ptr == 3 ? L[3]
                                                                           : kEmptyKey;
    int bl = lane;
    warp_argmin(head, bl);
    if (head == kEmptyKey) return;  // fewer than `need` keys held: no bound
    if (lane == bl) ++ptr;
    kth = head;
  }
  if (lane == 0 && kth < tau_key[q]) tau_key[q] = kth;
}

__device__ __forceinline__ void bitonic_block(uint64_t* key, float* val, int n) {
  // Ascending bitonic sort of n (power of two) entries in shared memory by the whole block.
  for (int size = 2; size <= n; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      __syncthreads();
      for (int i = threadIdx.x; i < n / 2; i += blockDim.x) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool up = (lo & size) == 0;
        const uint64_t a = key[lo], b = key[hi];
        if ((a > b) == up) {
          key[lo] = b;
          key[hi] = a;
          if (val) {
            const float t = val[lo];
            val[lo] = val[hi];
            val[hi] = t;
          }
        }
      }
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(256) select_rerank_kernel(const SelectParams sp) {
  extern __shared__ uint64_t sel_smem[];
  const MergeParams& p = sp.m;
  const int64_t q = blockIdx.x;
  if (q >= p.nq) return;
  uint64_t* cand = sel_smem;                                    // [cap] buffered keys
  uint64_t* ekey = sel_smem + sp.cap;                           // [cap] exact keys
  float* erank = reinterpret_cast<float*>(sel_smem + 2 * sp.cap);  // [cap] exact ranking values
  const uint32_t cnt = sp.count[q];
  const int n = static_cast<int>(cnt < static_cast<uint32_t>(sp.cap) ? cnt : static_cast<uint32_t>(sp.cap));
  int P = 32;
  while (P < n) P <<= 1;
  const uint64_t* b = sp.buf + static_cast<size_t>(q) * sp.cap;
  for (int i = threadIdx.x; i < P; i += blockDim.x) cand[i] = i < n ? b[i] : kEmptyKey;
  bitonic_block(cand, nullptr, P);
  const int T = min(n, p.k_eff + sp.margin);
  if (cnt > static_cast<uint32_t>(sp.cap)) {
    // The buffer holds cap real rows, so its T-th key bounds the T-th best of the database.
    if (threadIdx.x == 0) {
      sp.tau_key[q] = cand[T - 1];
      atomicOr(sp.overflow, 1);
    }
    return;
  }
  // Exact re-rank of the T best candidates.
  const float* x = p.queries + q * p.dim;
  const float xn = p.xn[q];
  int P2 = 32;
  while (P2 < T) P2 <<= 1;
  for (int i = threadIdx.x; i < P2; i += blockDim.x) {
    uint64_t ek = kEmptyKey;
    float rank = __int_as_float(0x7fffffff);
    if (i < T && cand[i] != kEmptyKey) {
      const uint32_t id = keys::key_id(cand[i]);
      const int64_t pos = p.inv_perm[id];
      const bool allowed = p.allow == nullptr || ((p.allow[pos >> 5] >> (pos & 31)) & 1u);
      rank = allowed ? exact_rank(p, x, xn, pos) : __int_as_float(0x7f800000);
      ek = keys::make_key(rank, id);
    }
    ekey[i] = ek;
    erank[i] = rank;
  }
  bitonic_block(ekey, erank, P2);
  for (int i = threadIdx.x; i < p.k_eff; i += blockDim.x) {
    const size_t o = static_cast<size_t>(q) * p.k_eff + i;
    const uint64_t key = i < P2 ? ekey[i] : kEmptyKey;
    const float rank = i < P2 ? erank[i] : __int_as_float(0x7fffffff);
    const bool empty = key == kEmptyKey;
    const int64_t gid = p.row_offset + static_cast<int64_t>(keys::key_id(key));
    if (p.neighbors) {
      p.neighbors[o] = empty ? -1 : gid;
      p.distances[o] = p.negate_output ? -rank : rank;
    } else {
      p.shard_rank[o] = rank;
      p.shard_gid[o] = empty ? INT64_MAX : gid;
    }
  }
}

template <int KL>
cudaError_t launch_kl(const MergeParams& p, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(kMergeWarps) * 32 * KL * sizeof(uint64_t);
  const bool assign = use_assign_shortcut(p) && p.num_sc * KL <= kAssignMaxCand;
  auto kern = assign ? assign_kernel<KL> : merge_rerank_kernel<KL>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int64_t per_block = assign ? kMergeWarps * 32 : kMergeWarps;  // points or queries
  const int64_t blocks = (p.nq + per_block - 1) / per_block;
  kern<<<static_cast<unsigned>(blocks), kMergeWarps * 32, smem, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_merge_rerank(const MergeParams& p, cudaStream_t stream) {
  switch (p.kl) {
    case 4:
      return launch_kl<4>(p, stream);
    case 8:
      return launch_kl<8>(p, stream);
    case 12:
      return launch_kl<12>(p, stream);
    case 16:
      return launch_kl<16>(p, stream);
    case 32:
      return launch_kl<32>(p, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_kth_bound(const uint64_t* cand, int num_sc, int64_t nq, int k, int kl,
                             uint64_t* tau_key, cudaStream_t stream) {
  if (num_sc > 256 || kl < 1) return cudaErrorInvalidValue;
  const int wpb = 8;
  const int64_t blocks = (nq + wpb - 1) / wpb;
  kth_bound_kernel<<<static_cast<unsigned>(blocks), wpb * 32, 0, stream>>>(cand, num_sc, nq, k,
                                                                        kl, tau_key);
  return cudaGetLastError();
}

cudaError_t launch_tighten_tau(const uint64_t* app_buf, const uint32_t* app_count, int cap,
                              int64_t nq, int need, uint64_t* tau_key, cudaStream_t stream) {
  if (need < 1 || nq <= 0) return cudaSuccess;
  const int wpb = 8;
  tighten_tau_kernel<<<static_cast<unsigned>((nq + wpb - 1) / wpb), wpb * 32, 0, stream>>>(
      app_buf, app_count, cap, nq, need, tau_key);
  return cudaGetLastError();
}

cudaError_t launch_select_rerank(const SelectParams& p, cudaStream_t stream) {
  if (p.cap > kSelectMaxCap || (p.cap & (p.cap - 1)) != 0) return cudaErrorInvalidValue;
  const size_t smem = static_cast<size_t>(p.cap) * (2 * sizeof(uint64_t) + sizeof(float));
  cudaError_t e = cudaFuncSetAttribute(select_rerank_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  select_rerank_kernel<<<static_cast<unsigned>(p.m.nq), 256, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_shard_merge(const float* rank, const int64_t* gid, int world, int64_t nq,
                               int k_eff, int negate_output, int64_t* neighbors, float* distances,
                               cudaStream_t stream) {
  const int wpb = 8;
  const int64_t blocks = (nq + wpb - 1) / wpb;
  shard_merge_kernel<<<static_cast<unsigned>(blocks), wpb * 32, 0, stream>>>(
      rank, gid, world, nq, k_eff, negate_output, neighbors, distances);
  return cudaGetLastError();
}

}  // namespace prim
}  // namespace ovvs
