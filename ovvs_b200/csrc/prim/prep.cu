// Data-layout kernels around the fused kernel (see prep.cuh).
#include "prep.cuh"

#include "keys.cuh"
#include "knn_fused.cuh"

namespace ovvs {
namespace prim {
namespace {

constexpr int kDTypeF32 = 0, kDTypeF16 = 1, kDTypeI8 = 2;

// internal.hpp:842-862 convert_to_f32: F32 as is, F16 decoded exactly, I8 widened, every other
// dtype (U8, F8E4M3, F8E5M2, F4E2M1) read as unsigned bytes.
__device__ __forceinline__ float decode(const void* data, int dtype, int64_t idx) {
  if (dtype == kDTypeF32) return static_cast<const float*>(data)[idx];
  if (dtype == kDTypeF16) return __half2float(static_cast<const __half*>(data)[idx]);
  if (dtype == kDTypeI8) return static_cast<float>(static_cast<const int8_t*>(data)[idx]);
  return static_cast<float>(static_cast<const uint8_t*>(data)[idx]);
}

__device__ __forceinline__ float pow2f(int e) {
  // 2^e for e in [-149, 127], exact.
  if (e >= -126) return __int_as_float((e + 127) << 23);
  return __int_as_float(1 << (e + 149));
}

__device__ __forceinline__ float query_mul(int metric, int e, int e_db) {
  const int rk = rank_kind_of(metric);
  const float sigma = metric == kMetricHamming ? 1.f : pow2f(max(-149, -(e + e_db)));
  return rk == kRankAffine ? -2.f * sigma : (rk == kRankScaled ? -sigma : 1.f);
}

__global__ void query_prep_kernel(const float* __restrict__ queries, int64_t nq, int64_t q_pad,
                                  int dim, int dp, int metric, int e_db, __half* __restrict__ a16,
                                  float* __restrict__ q_mul, float* __restrict__ xn,
                                  int* __restrict__ lo_flag, int16_t* __restrict__ e_out) {
  const int lane = threadIdx.x & 31;
  const int64_t q = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (q >= q_pad) return;
  __half* hi_row = a16 + q * 2 * dp;
  __half* lo_row = hi_row + dp;
  const __half z = __float2half_rn(0.f);
  if (q >= nq) {
    for (int d = lane; d < dp; d += 32) {
      hi_row[d] = z;
      lo_row[d] = z;
    }
    if (lane == 0) {
      q_mul[q] = -1.f;
      xn[q] = 0.f;
      if (e_out) e_out[q] = 0;
    }
    return;
  }
  const float* x = queries + q * dim;
  float mx = 0.f;
  for (int d = lane; d < dim; d += 32) {
    const float a = fabsf(x[d]);
    if (a < __int_as_float(0x7f800000)) mx = fmaxf(mx, a);
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  const bool hamming = metric == kMetricHamming;
  int e = 0;
  if (!hamming && mx > 0.f) e = min(14 - ilogbf(mx), 127);  // scaled max in [2^14, 2^15)
  const float scale = pow2f(e);
  bool any_lo = false;
  for (int d = lane; d < dp; d += 32) {
    __half h = z, l = z;
    if (d < dim) {
      const float v = x[d];
      if (hamming) {
        h = __float2half_rn(v >= 0.f ? 1.f : -1.f);
      } else {
        const float xs = v * scale;
        h = __float2half_rn(xs);
        l = __float2half_rn(xs - __half2float(h));
        any_lo |= __half2float(l) != 0.f;
      }
    }
    hi_row[d] = h;
    lo_row[d] = l;
  }
  if (__any_sync(0xffffffffu, any_lo) && lane == 0) atomicOr(lo_flag, 1);
  if (lane == 0) {
    // internal.hpp:221-225 nrm2sq: strictly sequential sum; loads batched 16 at a time so the
    // lane waits for memory once per 16 elements.
    float s = 0.f;
    int d = 0;
    for (; d + 16 <= dim; d += 16) {
      float v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = x[d + i];
#pragma unroll
      for (int i = 0; i < 16; ++i) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
    }
    for (; d < dim; ++d) s = __fadd_rn(s, __fmul_rn(x[d], x[d]));
    xn[q] = s;
    q_mul[q] = query_mul(metric, e, e_db);
    if (e_out) e_out[q] = static_cast<int16_t>(e);
  }
}

__global__ void row_stats_kernel(const void* __restrict__ data, int dtype, int64_t n, int dim,
                                 int metric, float* __restrict__ norm,
                                 float* __restrict__ sort_key,
                                 unsigned int* __restrict__ absmax_bits) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  float mx = 0.f;
  if (i < n) {
    float s = 0.f;
    for (int d = 0; d < dim; ++d) {
      const float y = decode(data, dtype, i * dim + d);
      s = __fadd_rn(s, __fmul_rn(y, y));
      const float a = fabsf(y);
      if (a < __int_as_float(0x7f800000)) mx = fmaxf(mx, a);
    }
    norm[i] = s;
    float key = 0.f;
    const int rk = rank_kind_of(metric);
    if (rk == kRankAffine) {
      key = s;
    } else if (rk == kRankColumnScaled) {
      const float c = s < 1e-12f ? 1e-12f : s;
      key = -1.f / __fsqrt_rn(c);
    }
    sort_key[i] = key;
  }
#pragma unroll
  for (int off = 16; off; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if ((threadIdx.x & 31) == 0 && mx > 0.f) atomicMax(absmax_bits, __float_as_uint(mx));
}

__global__ void scatter_rows_kernel(const void* __restrict__ data, int dtype, int64_t n,
                                    int64_t n_pad, int dim, int dp, int b_parts, int metric,
                                    int e_db, const uint32_t* __restrict__ perm,
                                    const float* __restrict__ norm,
                                    const float* __restrict__ sort_key, __half* __restrict__ rows16,
                                    float* __restrict__ exact32, float* __restrict__ aux,
                                    float* __restrict__ norm_sorted, uint32_t* __restrict__ row_id,
                                    uint32_t* __restrict__ inv_perm) {
  const int lane = threadIdx.x & 31;
  const int64_t pos = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (pos >= n_pad) return;
  const int stride = b_parts * dp;
  __half* r16 = rows16 + pos * stride;
  const __half z = __float2half_rn(0.f);
  if (pos >= n) {
    for (int d = lane; d < stride; d += 32) r16[d] = z;
    if (exact32)
      for (int d = lane; d < dim; d += 32) exact32[pos * dim + d] = 0.f;
    if (lane == 0) {
      aux[pos] = 0.f;
      norm_sorted[pos] = 0.f;
      row_id[pos] = keys::kEmptyId;
    }
    return;
  }
  const uint32_t id = perm[pos];
  if (lane == 0) {
    row_id[pos] = id;
    inv_perm[id] = static_cast<uint32_t>(pos);
    aux[pos] = sort_key[id];
    norm_sorted[pos] = norm[id];
  }
  const bool hamming = metric == kMetricHamming;
  const float scale = pow2f(e_db);
  for (int d = lane; d < dp; d += 32) {
    __half h = z, l = z;
    if (d < dim) {
      const int64_t src = static_cast<int64_t>(id) * dim + d;
      const float y = decode(data, dtype, src);
      if (hamming) {
        h = __float2half_rn(y >= 0.f ? 1.f : -1.f);
      } else if (dtype == kDTypeF16) {
        h = static_cast<const __half*>(data)[src];  // bit-exact copy
      } else if (b_parts == 1) {
        h = __float2half_rn(y);  // small integers: exact
      } else {
        const float ys = y * scale;
        h = __float2half_rn(ys);
        l = __float2half_rn(ys - __half2float(h));
      }
      if (exact32) exact32[pos * dim + d] = y;
    }
    r16[d] = h;
    if (b_parts == 2) r16[dp + d] = l;
  }
}

__global__ void tile_bounds_kernel(const float* __restrict__ aux, int64_t n, int num_tiles,
                                   float2* __restrict__ tile_aux) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= num_tiles) return;
  const int64_t b = static_cast<int64_t>(t) * kTileN;
  const int64_t e = min(n, b + kTileN);
  float lo = __int_as_float(0x7f800000), hi = -lo;
  for (int64_t i = b; i < e; ++i) {
    lo = fminf(lo, aux[i]);
    hi = fmaxf(hi, aux[i]);
  }
  if (b >= e) lo = hi = 0.f;
  tile_aux[t] = make_float2(lo, hi);
}

__global__ void group_bounds_kernel(const float2* __restrict__ tile_aux, int num_tiles,
                                    float2* __restrict__ group_aux) {
  const int g = blockIdx.x * blockDim.x + threadIdx.x;
  const int t0 = g * kGroupTiles;
  if (t0 >= num_tiles) return;
  const int t1 = min(num_tiles, t0 + kGroupTiles);
  float2 r = tile_aux[t0];
  for (int t = t0 + 1; t < t1; ++t) {
    r.x = fminf(r.x, tile_aux[t].x);
    r.y = fmaxf(r.y, tile_aux[t].y);
  }
  group_aux[g] = r;
}

__global__ void allow_bits_kernel(const uint8_t* __restrict__ bitset, int64_t row_offset,
                                  const uint32_t* __restrict__ row_id, int64_t n, int64_t n_pad,
                                  uint32_t* __restrict__ allow_pos) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (w * 32 >= n_pad) return;
  uint32_t word = 0;
  for (int b = 0; b < 32; ++b) {
    const int64_t pos = w * 32 + b;
    if (pos < n) {
      const int64_t g = row_offset + row_id[pos];
      word |= static_cast<uint32_t>((bitset[g >> 3] >> (g & 7)) & 1u) << b;
    }
  }
  allow_pos[w] = word;
}

}  // namespace

void launch_query_prep(const float* queries, int64_t nq, int64_t q_pad, int dim, int dp,
                       int metric_code, int e_db, __half* a16, float* q_mul, float* xn,
                       int* lo_flag, cudaStream_t stream, int16_t* e_q) {
  const int wpb = 8;
  const int64_t blocks = (q_pad + wpb - 1) / wpb;
  query_prep_kernel<<<static_cast<unsigned>(blocks), wpb * 32, 0, stream>>>(
      queries, nq, q_pad, dim, dp, metric_code, e_db, a16, q_mul, xn, lo_flag, e_q);
}

namespace {
__global__ void query_mul_kernel(const int16_t* __restrict__ e_q, int64_t nq, int64_t q_pad,
                                 int metric, int e_db, float* __restrict__ q_mul) {
  const int64_t q = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (q >= q_pad) return;
  q_mul[q] = q < nq ? query_mul(metric, e_q[q], e_db) : -1.f;
}
}  // namespace

void launch_query_mul(const int16_t* e_q, int64_t nq, int64_t q_pad, int metric_code, int e_db,
                      float* q_mul, cudaStream_t stream) {
  query_mul_kernel<<<static_cast<unsigned>((q_pad + 255) / 256), 256, 0, stream>>>(
      e_q, nq, q_pad, metric_code, e_db, q_mul);
}

void launch_row_stats(const void* data, int dtype, int64_t n, int dim, int metric_code,
                      float* norm, float* sort_key, unsigned int* absmax_bits,
                      cudaStream_t stream) {
  const int64_t blocks = (n + 255) / 256;
  row_stats_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
      data, dtype, n, dim, metric_code, norm, sort_key, absmax_bits);
}

void launch_scatter_rows(const void* data, int dtype, int64_t n, int64_t n_pad, int dim, int dp,
                         int b_parts, int metric_code, int e_db, const uint32_t* perm,
                         const float* norm, const float* sort_key, __half* rows16,
                         float* exact32, float* aux, float* norm_sorted, uint32_t* row_id,
                         uint32_t* inv_perm, cudaStream_t stream) {
  const int wpb = 8;
  const int64_t blocks = (n_pad + wpb - 1) / wpb;
  scatter_rows_kernel<<<static_cast<unsigned>(blocks), wpb * 32, 0, stream>>>(
      data, dtype, n, n_pad, dim, dp, b_parts, metric_code, e_db, perm, norm, sort_key, rows16,
      exact32, aux, norm_sorted, row_id, inv_perm);
}

void launch_tile_bounds(const float* aux, int64_t n, int num_tiles, float2* tile_aux,
                        cudaStream_t stream) {
  tile_bounds_kernel<<<(num_tiles + 127) / 128, 128, 0, stream>>>(aux, n, num_tiles, tile_aux);
  const int groups = (num_tiles + kGroupTiles - 1) / kGroupTiles;
  group_bounds_kernel<<<(groups + 127) / 128, 128, 0, stream>>>(tile_aux, num_tiles,
                                                                tile_aux + num_tiles);
}

void launch_allow_bits(const uint8_t* bitset, int64_t row_offset, const uint32_t* row_id,
                       int64_t n, int64_t n_pad, uint32_t* allow_pos, cudaStream_t stream) {
  const int64_t words = n_pad / 32;
  allow_bits_kernel<<<static_cast<unsigned>((words + 255) / 256), 256, 0, stream>>>(
      bitset, row_offset, row_id, n, n_pad, allow_pos);
}

}  // namespace prim
}  // namespace ovvs
