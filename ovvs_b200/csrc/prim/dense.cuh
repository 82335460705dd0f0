// Dense primitives of the ovvs ABI on the device: GEMM, pairwise distances, top-k selection,
// row gather (reference src/rt/resources.cpp:178-216, src/prim/mixer.cpp:94-221,
// src/prim/cpu/cpu_prims.cpp:24-118).
//
// These are the hot path's stages exposed one at a time, and they reproduce the reference's own
// CPU results bit for bit rather than to a tolerance: every output element accumulates its
// products strictly in k order with separately rounded multiply and add (cpu_gemm's naive loop,
// cpu_prims.cpp:48-58; nrm2sq / dot / l2sq, internal.hpp:57-63,215-225), on CUDA cores. Top-k uses
// the same strict total order as the search (cpu_prims.cpp:24-32).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace ovvs {
namespace prim {

// Operand rounding before the products (ovvsGemmEx compute dtypes): none, or to fp16.
enum DenseRound : int { kRoundNone = 0, kRoundF16 = 1 };

// C[m x n] = A[m x k] * (trans_b ? B[n x k]^T : B[k x n]), row-major, sequential k sums.
cudaError_t launch_gemm_seq(const float* a, const float* b, float* c, int64_t m, int64_t n,
                            int64_t k, bool trans_b, int round, cudaStream_t stream);

// out[i] = sum over d of x[i][d]^2, sequential (nrm2sq).
cudaError_t launch_row_norms_seq(const float* x, int64_t rows, int64_t dim, float* out,
                                 cudaStream_t stream);

// Expanded metrics from ip = out[i][j] (in place): inner product -ip; cosine
// 1 - ip / (sqrt(max(xn,1e-12)) * sqrt(max(yn,1e-12))); otherwise (xn + yn) - 2 ip.
cudaError_t launch_pairwise_expand(float* out, const float* xn, const float* yn, int64_t nx,
                                   int64_t ny, int metric_raw, cudaStream_t stream);

// Direct metrics per pair (distance_one, internal.hpp:240-272): L2 sqrt, Hamming (sign-bit
// mismatches), Lp (p = metric_arg > 0 ? metric_arg : 2), anything else squared L2.
cudaError_t launch_pairwise_direct(const float* x, const float* y, int64_t nx, int64_t ny,
                                   int64_t dim, int metric_raw, float metric_arg, float* out,
                                   cudaStream_t stream);

// out[i][:] = src[idx[i]][:] when 0 <= idx[i] < src_rows, else zeros.
cudaError_t launch_gather_rows(const float* src, int64_t src_rows, int64_t dim,
                               const int64_t* idx, int64_t nidx, float* out, cudaStream_t stream);

// Self-exclusion for a kNN graph: in_ids / in_dist [rows x k_in] are the search results of the
// dataset's rows row0.. against the whole dataset (k_in = min(k + 1, n), the reference's top-k
// order; `negate`: distances are negated scores, as for inner product). Writes [rows x k_out]
// equal to a top-k of each row's scores with the row itself scored +inf (graphs.cpp:3390).
cudaError_t launch_exclude_self(const int64_t* in_ids, const float* in_dist, int64_t rows,
                                int k_in, int64_t row0, int k_out, bool negate, int64_t* out_ids,
                                float* out_dist, cudaStream_t stream);

// Top-k per row in the reference's order: ascending (largest: descending), NaN after every
// number, ties by lower column. indices/values [rows][min(k, cols)]. Scratch via the callbacks'
// caller: `keys` and `keys_sorted` hold rows * cols u64, `offsets` rows + 1 int, `tmp` tmp_bytes.
size_t topk_tmp_bytes(int64_t rows, int64_t cols);
cudaError_t launch_topk(const float* scores, int64_t rows, int64_t cols, int64_t k, bool largest,
                        uint64_t* keys, uint64_t* keys_sorted, int* offsets, void* tmp,
                        size_t tmp_bytes, int64_t* indices, float* values, cudaStream_t stream);

}  // namespace prim
}  // namespace ovvs
