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
__device__ float exact_rank(const MergeParams& p, const float* __restrict__ x, float xn,
                            int64_t pos) {
  const int D = p.dim;
  const float* y32 = p.exact32 ? p.exact32 + pos * D : nullptr;
  const __half* y16 = p.rows16 + pos * p.rows16_stride;
  auto y_at = [&](int d) -> float { return y32 ? y32[d] : __half2float(y16[d]); };
  switch (p.metric) {
    case kMetricL2:
    case kMetricInnerProduct:
    case kMetricCosine: {
      float ip = 0.f;
      for (int d = 0; d < D; ++d) ip = __fadd_rn(ip, __fmul_rn(x[d], y_at(d)));
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
      float s = 0.f;
      for (int d = 0; d < D; ++d) {
        const float t = __fsub_rn(x[d], y_at(d));
        s = __fadd_rn(s, __fmul_rn(t, t));
      }
      if (p.metric == kMetricL2Sqrt || p.metric == kMetricLp) return __fsqrt_rn(s);
      return s;
    }
  }
}

template <int KL>
__global__ void __launch_bounds__(kMergeWarps * 32)
    merge_rerank_kernel(const MergeParams p) {
  extern __shared__ uint64_t merge_smem[];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * kMergeWarps + warp;
  if (q >= p.nq) return;
  uint64_t* lists = merge_smem + warp * 32 * KL;

  // 1. Each lane keeps the KL best keys of a strided share of the candidates.
  uint64_t L[KL];
#pragma unroll
  for (int i = 0; i < KL; ++i) L[i] = kEmptyKey;
  const uint64_t* c = p.cand + static_cast<size_t>(q) * p.num_sc * KL;
  const int total = p.num_sc * KL;
  for (int e = lane; e < total; e += 32) {
    const uint64_t key = c[e];
    if (key < L[KL - 1]) list_insert<KL>(L, key);
  }
#pragma unroll
  for (int i = 0; i < KL; ++i) lists[lane * KL + i] = L[i];
  __syncwarp();

  // 2. Merge the 32 sorted lane lists: lane r receives the r-th best key overall.
  int ptr = 0;
  uint64_t sel = kEmptyKey;
  for (int r = 0; r < KL; ++r) {
    uint64_t k = ptr < KL ? lists[lane * KL + ptr] : kEmptyKey;
    int l = lane;
    warp_argmin(k, l);
    if (lane == l) ++ptr;
    if (lane == r) sel = k;
  }

  // 3. Exact distance of each survivor.
  const float* x = p.queries + q * p.dim;
  const float xn = p.xn[q];
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

template <int KL>
cudaError_t launch_kl(const MergeParams& p, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(kMergeWarps) * 32 * KL * sizeof(uint64_t);
  auto kern = merge_rerank_kernel<KL>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int64_t blocks = (p.nq + kMergeWarps - 1) / kMergeWarps;
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
    case 16:
      return launch_kl<16>(p, stream);
    case 32:
      return launch_kl<32>(p, stream);
    default:
      return cudaErrorInvalidValue;
  }
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
