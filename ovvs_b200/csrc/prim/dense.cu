// Dense primitives (see dense.cuh).
#include "dense.cuh"

#include <cub/device/device_segmented_sort.cuh>
#include <cuda_fp16.h>

#include "keys.cuh"
#include "prep.cuh"

namespace ovvs {
namespace prim {
namespace {

constexpr int kTile = 64;     // 64 x 64 outputs per block
constexpr int kTileK = 16;    // K step staged in shared memory
constexpr int kThreads = 256; // 16 x 16 threads, 4 x 4 outputs each (strided by 16)

// ovvsMetric values (ovvs.h)
constexpr int kRawL2 = 0, kRawL2Sqrt = 1, kRawIp = 2, kRawCosine = 3, kRawHamming = 4, kRawLp = 5;

__device__ __forceinline__ float round_to(float v, int round) {
  if (round == kRoundF16) return __half2float(__float2half_rn(v));
  return v;
}

// Stages a kTileK x kTile slab of a row-major [rows x k] matrix (rows r0.., columns t0..) as
// S[t][r], zero outside the matrix; loads run along k (coalesced).
__device__ __forceinline__ void stage_rows(float (&S)[kTileK][kTile + 1], const float* M,
                                           int64_t rows, int64_t k, int64_t r0, int64_t t0,
                                           int round) {
  for (int e = threadIdx.x; e < kTile * kTileK; e += kThreads) {
    const int r = e / kTileK, c = e % kTileK;
    const int64_t gr = r0 + r, gt = t0 + c;
    S[c][r] = (gr < rows && gt < k) ? round_to(M[gr * k + gt], round) : 0.f;
  }
}

// Same for a row-major [k x cols] matrix read as its transpose (loads run along cols).
__device__ __forceinline__ void stage_cols(float (&S)[kTileK][kTile + 1], const float* M,
                                           int64_t cols, int64_t k, int64_t c0, int64_t t0,
                                           int round) {
  for (int e = threadIdx.x; e < kTile * kTileK; e += kThreads) {
    const int c = e / kTile, r = e % kTile;
    const int64_t gc = c0 + r, gt = t0 + c;
    S[c][r] = (gc < cols && gt < k) ? round_to(M[gt * cols + gc], round) : 0.f;
  }
}

// Every output's sum runs over t = 0, 1, ... in order with separately rounded multiply and
// add: the reference's naive loop (cpu_prims.cpp:48-58). Zero padding past k adds +0 products
// at the end, which leaves the sum unchanged.
__global__ void __launch_bounds__(kThreads)
    gemm_seq_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ C,
                    int64_t m, int64_t n, int64_t k, int trans_b, int round) {
  __shared__ float As[kTileK][kTile + 1];
  __shared__ float Bs[kTileK][kTile + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t i0 = static_cast<int64_t>(blockIdx.y) * kTile;
  const int64_t j0 = static_cast<int64_t>(blockIdx.x) * kTile;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) acc[a][b] = 0.f;
  for (int64_t t0 = 0; t0 < k; t0 += kTileK) {
    stage_rows(As, A, m, k, i0, t0, round);
    if (trans_b)
      stage_rows(Bs, B, n, k, j0, t0, round);
    else
      stage_cols(Bs, B, n, k, j0, t0, round);
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kTileK; ++t) {
      float av[4], bv[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) av[a] = As[t][ty + 16 * a];
#pragma unroll
      for (int b = 0; b < 4; ++b) bv[b] = Bs[t][tx + 16 * b];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(av[a], bv[b]));
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t i = i0 + ty + 16 * a;
    if (i >= m) continue;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int64_t j = j0 + tx + 16 * b;
      if (j < n) C[i * n + j] = acc[a][b];
    }
  }
}

// distance_one's direct metrics, one pair per (a, b) slot of the same 64 x 64 tiling; the sum
// over d is sequential like the reference's loops.
template <int M>
__global__ void __launch_bounds__(kThreads)
    pairwise_direct_kernel(const float* __restrict__ X, const float* __restrict__ Y, int64_t nx,
                           int64_t ny, int64_t dim, float p, float* __restrict__ out) {
  __shared__ float Xs[kTileK][kTile + 1];
  __shared__ float Ys[kTileK][kTile + 1];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t i0 = static_cast<int64_t>(blockIdx.y) * kTile;
  const int64_t j0 = static_cast<int64_t>(blockIdx.x) * kTile;
  float acc[4][4];
  int cnt[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      acc[a][b] = 0.f;
      cnt[a][b] = 0;
    }
  for (int64_t t0 = 0; t0 < dim; t0 += kTileK) {
    stage_rows(Xs, X, nx, dim, i0, t0, kRoundNone);
    stage_rows(Ys, Y, ny, dim, j0, t0, kRoundNone);
    __syncthreads();
    const int tn = static_cast<int>(dim - t0 < kTileK ? dim - t0 : kTileK);
    for (int t = 0; t < tn; ++t) {
      float xv[4], yv[4];
#pragma unroll
      for (int a = 0; a < 4; ++a) xv[a] = Xs[t][ty + 16 * a];
#pragma unroll
      for (int b = 0; b < 4; ++b) yv[b] = Ys[t][tx + 16 * b];
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          if constexpr (M == kRawHamming) {
            cnt[a][b] += static_cast<int>((xv[a] >= 0.f) != (yv[b] >= 0.f));
          } else if constexpr (M == kRawLp) {
            acc[a][b] = __fadd_rn(acc[a][b], powf(fabsf(__fsub_rn(xv[a], yv[b])), p));
          } else {
            const float d = __fsub_rn(xv[a], yv[b]);
            acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(d, d));
          }
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int64_t i = i0 + ty + 16 * a;
    if (i >= nx) continue;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int64_t j = j0 + tx + 16 * b;
      if (j >= ny) continue;
      float v;
      if constexpr (M == kRawHamming)
        v = static_cast<float>(cnt[a][b]);
      else if constexpr (M == kRawLp)
        v = powf(acc[a][b], __fdiv_rn(1.f, p));
      else if constexpr (M == kRawL2Sqrt)
        v = __fsqrt_rn(acc[a][b]);
      else
        v = acc[a][b];
      out[i * ny + j] = v;
    }
  }
}

__global__ void row_norms_seq_kernel(const float* __restrict__ x, int64_t rows, int64_t dim,
                                     float* __restrict__ out) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  const float* r = x + i * dim;
  float s = 0.f;
  for (int64_t d = 0; d < dim; ++d) s = __fadd_rn(s, __fmul_rn(r[d], r[d]));
  out[i] = s;
}

__global__ void pairwise_expand_kernel(float* __restrict__ out, const float* __restrict__ xn,
                                       const float* __restrict__ yn, int64_t nx, int64_t ny,
                                       int metric) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= nx * ny) return;
  const int64_t i = e / ny, j = e % ny;
  const float ip = out[e];
  if (metric == kRawIp) {
    out[e] = -ip;
  } else if (metric == kRawCosine) {
    const float a = xn[i], b = yn[j];
    const float nxv = __fsqrt_rn(a < 1e-12f ? 1e-12f : a);
    const float nyv = __fsqrt_rn(b < 1e-12f ? 1e-12f : b);
    out[e] = __fsub_rn(1.f, __fdiv_rn(ip, __fmul_rn(nxv, nyv)));
  } else {
    out[e] = __fsub_rn(__fadd_rn(xn[i], yn[j]), __fmul_rn(2.f, ip));
  }
}

__global__ void gather_rows_kernel(const float* __restrict__ src, int64_t src_rows, int64_t dim,
                                   const int64_t* __restrict__ idx, int64_t nidx,
                                   float* __restrict__ out) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= nidx * dim) return;
  const int64_t i = e / dim, d = e % dim;
  const int64_t r = idx[i];
  out[e] = (r >= 0 && r < src_rows) ? src[r * dim + d] : 0.f;
}

// One thread per row: the row's search results (queries = the dataset's own rows row0.., k_in of
// them, in the top-k total order) with the row itself replaced by a +inf score, truncated to
// k_out -- the order of a top-k over the row's scores with its diagonal set to +inf.
__global__ void exclude_self_kernel(const int64_t* __restrict__ in_ids,
                                    const float* __restrict__ in_dist, int64_t rows, int k_in,
                                    int64_t row0, int k_out, int negate,
                                    int64_t* __restrict__ out_ids, float* __restrict__ out_dist) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int64_t self = row0 + r;
  const float inf = __int_as_float(0x7f800000);
  const uint64_t self_key = keys::make_key(inf, static_cast<uint32_t>(self));
  const int64_t* ids = in_ids + r * k_in;
  const float* dist = in_dist + r * k_in;
  int64_t* oi = out_ids + r * k_out;
  float* od = out_dist + r * k_out;
  int p = 0;
  bool placed = false;
  for (int j = 0; j < k_in && p < k_out; ++j) {
    const int64_t id = ids[j];
    if (id == self) continue;
    const float d = dist[j];
    if (!placed && self_key < keys::make_key(negate ? -d : d, static_cast<uint32_t>(id))) {
      oi[p] = self;
      od[p] = negate ? -inf : inf;
      ++p;
      placed = true;
      if (p == k_out) break;
    }
    oi[p] = id;
    od[p] = d;
    ++p;
  }
  if (p < k_out && !placed) {
    oi[p] = self;
    od[p] = negate ? -inf : inf;
  }
}

// (order of the score, column) keys: ascending numbers (descending when `largest`, via the
// negated score), -0 == +0, NaN after every number, ties by lower column.
__global__ void topk_keys_kernel(const float* __restrict__ scores, int64_t rows, int64_t cols,
                                 int largest, uint64_t* __restrict__ keys,
                                 int* __restrict__ offsets) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e <= rows && e < rows + 1 && offsets) offsets[e] = static_cast<int>(e * cols);
  if (e >= rows * cols) return;
  const float v = scores[e];
  keys[e] = keys::make_key(largest ? -v : v, static_cast<uint32_t>(e % cols));
}

__global__ void topk_emit_kernel(const float* __restrict__ scores,
                                 const uint64_t* __restrict__ sorted, int64_t rows, int64_t cols,
                                 int64_t k_eff, int64_t* __restrict__ indices,
                                 float* __restrict__ values) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= rows * k_eff) return;
  const int64_t r = e / k_eff, t = e % k_eff;
  const int64_t c = static_cast<int64_t>(keys::key_id(sorted[r * cols + t]));
  indices[e] = c;
  values[e] = scores[r * cols + c];
}

unsigned blocks_for(int64_t n, int threads) {
  return static_cast<unsigned>((n + threads - 1) / threads);
}

}  // namespace

cudaError_t launch_gemm_seq(const float* a, const float* b, float* c, int64_t m, int64_t n,
                            int64_t k, bool trans_b, int round, cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>((n + kTile - 1) / kTile),
                  static_cast<unsigned>((m + kTile - 1) / kTile));
  if (grid.y > 65535u) return cudaErrorInvalidValue;
  gemm_seq_kernel<<<grid, kThreads, 0, stream>>>(a, b, c, m, n, k, trans_b ? 1 : 0, round);
  return cudaGetLastError();
}

cudaError_t launch_row_norms_seq(const float* x, int64_t rows, int64_t dim, float* out,
                                 cudaStream_t stream) {
  row_norms_seq_kernel<<<blocks_for(rows, 256), 256, 0, stream>>>(x, rows, dim, out);
  return cudaGetLastError();
}

cudaError_t launch_pairwise_expand(float* out, const float* xn, const float* yn, int64_t nx,
                                   int64_t ny, int metric_raw, cudaStream_t stream) {
  pairwise_expand_kernel<<<blocks_for(nx * ny, 256), 256, 0, stream>>>(out, xn, yn, nx, ny,
                                                                       metric_raw);
  return cudaGetLastError();
}

cudaError_t launch_pairwise_direct(const float* x, const float* y, int64_t nx, int64_t ny,
                                   int64_t dim, int metric_raw, float metric_arg, float* out,
                                   cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>((ny + kTile - 1) / kTile),
                  static_cast<unsigned>((nx + kTile - 1) / kTile));
  if (grid.y > 65535u) return cudaErrorInvalidValue;
  const float p = metric_arg > 0.f ? metric_arg : 2.f;
  switch (metric_raw) {
    case kRawL2Sqrt:
      pairwise_direct_kernel<kRawL2Sqrt><<<grid, kThreads, 0, stream>>>(x, y, nx, ny, dim, p, out);
      break;
    case kRawHamming:
      pairwise_direct_kernel<kRawHamming><<<grid, kThreads, 0, stream>>>(x, y, nx, ny, dim, p, out);
      break;
    case kRawLp:
      pairwise_direct_kernel<kRawLp><<<grid, kThreads, 0, stream>>>(x, y, nx, ny, dim, p, out);
      break;
    default:
      pairwise_direct_kernel<kRawL2><<<grid, kThreads, 0, stream>>>(x, y, nx, ny, dim, p, out);
  }
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const float* src, int64_t src_rows, int64_t dim,
                               const int64_t* idx, int64_t nidx, float* out, cudaStream_t stream) {
  gather_rows_kernel<<<blocks_for(nidx * dim, 256), 256, 0, stream>>>(src, src_rows, dim, idx,
                                                                       nidx, out);
  return cudaGetLastError();
}

cudaError_t launch_exclude_self(const int64_t* in_ids, const float* in_dist, int64_t rows,
                                int k_in, int64_t row0, int k_out, bool negate, int64_t* out_ids,
                                float* out_dist, cudaStream_t stream) {
  exclude_self_kernel<<<blocks_for(rows, 128), 128, 0, stream>>>(
      in_ids, in_dist, rows, k_in, row0, k_out, negate ? 1 : 0, out_ids, out_dist);
  return cudaGetLastError();
}

size_t topk_tmp_bytes(int64_t rows, int64_t cols) {
  size_t bytes = 0;
  cub::DeviceSegmentedSort::SortKeys(nullptr, bytes, static_cast<const uint64_t*>(nullptr),
                                     static_cast<uint64_t*>(nullptr),
                                     static_cast<int>(rows * cols), static_cast<int>(rows),
                                     static_cast<const int*>(nullptr),
                                     static_cast<const int*>(nullptr));
  return bytes;
}

cudaError_t launch_topk(const float* scores, int64_t rows, int64_t cols, int64_t k, bool largest,
                        uint64_t* keys, uint64_t* keys_sorted, int* offsets, void* tmp,
                        size_t tmp_bytes, int64_t* indices, float* values, cudaStream_t stream) {
  const int64_t total = rows * cols;
  if (total > 0x7fffffffLL) return cudaErrorInvalidValue;
  const int64_t k_eff = k < cols ? k : cols;
  topk_keys_kernel<<<blocks_for(total > rows + 1 ? total : rows + 1, 256), 256, 0, stream>>>(
      scores, rows, cols, largest ? 1 : 0, keys, offsets);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  size_t bytes = tmp_bytes;
  e = cub::DeviceSegmentedSort::SortKeys(tmp, bytes, keys, keys_sorted, static_cast<int>(total),
                                         static_cast<int>(rows), offsets, offsets + 1, stream);
  if (e != cudaSuccess) return e;
  topk_emit_kernel<<<blocks_for(rows * k_eff, 256), 256, 0, stream>>>(scores, keys_sorted, rows,
                                                                      cols, k_eff, indices, values);
  return cudaGetLastError();
}

}  // namespace prim
}  // namespace ovvs
