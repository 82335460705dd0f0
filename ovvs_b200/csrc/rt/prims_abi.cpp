// The dense primitives of the ovvs ABI and ovvsAllNeighbors on the device (reference
// src/rt/resources.cpp:178-216, src/neighbors/graphs.cpp:3384-3396). Host buffers in and out,
// like the reference; argument checks in the reference's order; results bit-identical to the
// reference's CPU path (see prim/dense.cuh), except Lp distances, whose powf may differ from the
// C library's by an ulp. Large problems are processed in row blocks so that device memory stays
// bounded.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>
#include <new>

#include "../neighbors/brute_force.hpp"
#include "../prim/dense.cuh"
#include "ovvs/ovvs.h"
#include "runtime.hpp"

using ovvs::rt::DeviceBuffer;
using ovvs::rt::Resources;
using ovvs::rt::from_handle;

namespace {

constexpr size_t kBlockBytes = size_t(1) << 30;  // device bytes per output block

template <class F>
ovvsStatus guarded(Resources& r, F&& f) {
  try {
    std::lock_guard<std::mutex> lk(r.mu);
    OVVS_TRY(r.check_policy());
    OVVS_TRY(r.activate());
    return f();
  } catch (const std::bad_alloc&) {
    return OVVS_STATUS_OOM;
  } catch (...) {
    return OVVS_STATUS_ERROR;
  }
}

bool too_big(int64_t a, int64_t b) { return a > 0 && b > (INT64_MAX / 16) / a; }

ovvsStatus upload(DeviceBuffer& buf, const void* host, size_t bytes, cudaStream_t s) {
  OVVS_TRY_CUDA(buf.reserve(bytes + 16));
  OVVS_TRY_CUDA(cudaMemcpyAsync(buf.get(), host, bytes, cudaMemcpyHostToDevice, s));
  return OVVS_STATUS_SUCCESS;
}

// Rows of an output block of `cols` columns that fit kBlockBytes (at least 1), and at most what
// one launch of the 64-row tiled kernels covers (65535 row tiles).
int64_t block_rows(int64_t cols, size_t bytes_per_elem) {
  const int64_t r = static_cast<int64_t>(kBlockBytes / (static_cast<size_t>(cols) * bytes_per_elem));
  return std::min<int64_t>(std::max<int64_t>(1, r), int64_t{65535} * 64);
}

// Top-k of a device score block [rows x cols] into device indices / values [rows x k_eff].
ovvsStatus topk_device(Resources& r, const float* d_scores, int64_t rows, int64_t cols, int64_t k,
                       bool largest, int64_t* d_idx, float* d_val) {
  DeviceBuffer keys, sorted, offsets, tmp;
  OVVS_TRY_CUDA(keys.reserve(static_cast<size_t>(rows * cols) * sizeof(uint64_t)));
  OVVS_TRY_CUDA(sorted.reserve(static_cast<size_t>(rows * cols) * sizeof(uint64_t)));
  OVVS_TRY_CUDA(offsets.reserve(static_cast<size_t>(rows + 1) * sizeof(int)));
  const size_t tb = ovvs::prim::topk_tmp_bytes(rows, cols);
  OVVS_TRY_CUDA(tmp.reserve(tb + 16));
  OVVS_TRY_CUDA(ovvs::prim::launch_topk(d_scores, rows, cols, k, largest, keys.as<uint64_t>(),
                                        sorted.as<uint64_t>(), offsets.as<int>(), tmp.get(), tb,
                                        d_idx, d_val, r.stream));
  return OVVS_STATUS_SUCCESS;
}

// Pairwise scores of x rows [i0, i0 + rows) against all y rows into d_out [rows x ny]
// (prim_pairwise, mixer.cpp:174-221): expanded metrics through the sequential GEMM and the
// reference's epilogue, the others per pair.
ovvsStatus pairwise_block(Resources& r, ovvsMetric metric, const float* d_x, int64_t rows,
                          const float* d_y, int64_t ny, int64_t dim, const float* d_yn,
                          float metric_arg, float* d_xn, float* d_out) {
  const int m = static_cast<int>(metric);
  if (metric == OVVS_METRIC_L2_EXPANDED || metric == OVVS_METRIC_INNER_PRODUCT ||
      metric == OVVS_METRIC_COSINE_EXPANDED) {
    OVVS_TRY_CUDA(ovvs::prim::launch_row_norms_seq(d_x, rows, dim, d_xn, r.stream));
    OVVS_TRY_CUDA(ovvs::prim::launch_gemm_seq(d_x, d_y, d_out, rows, ny, dim, true,
                                              ovvs::prim::kRoundNone, r.stream));
    OVVS_TRY_CUDA(ovvs::prim::launch_pairwise_expand(d_out, d_xn, d_yn, rows, ny, m, r.stream));
    return OVVS_STATUS_SUCCESS;
  }
  OVVS_TRY_CUDA(ovvs::prim::launch_pairwise_direct(d_x, d_y, rows, ny, dim, m, metric_arg, d_out,
                                                   r.stream));
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus gemm_impl(ovvsResources_t res, const float* a, const float* b, float* c, int64_t m,
                     int64_t n, int64_t k, int32_t trans_b, ovvsDType compute) {
  Resources& r = *from_handle(res);
  return guarded(r, [&]() -> ovvsStatus {
    if (too_big(m, k) || too_big(k, n) || too_big(m, n)) return OVVS_STATUS_SHAPE_MISMATCH;
    // F16 rounds the operands before the products (a product of two halves is exact in fp32,
    // so the result is deterministic), as the reference's device path does
    // (backend_gpu.cpp:523-548); every other compute type runs in F32, as its CPU path does when
    // no device kernel takes the type (mixer.cpp:85-90).
    const int round = compute == OVVS_DTYPE_F16 ? ovvs::prim::kRoundF16 : ovvs::prim::kRoundNone;
    DeviceBuffer da, db, dc;
    r.mark(0);
    OVVS_TRY(upload(db, b, static_cast<size_t>(k * n) * sizeof(float), r.stream));
    const int64_t rb = std::min(m, block_rows(std::max(n, k), 2 * sizeof(float)));
    OVVS_TRY_CUDA(da.reserve(static_cast<size_t>(rb * k) * sizeof(float) + 16));
    OVVS_TRY_CUDA(dc.reserve(static_cast<size_t>(rb * n) * sizeof(float) + 16));
    for (int64_t i0 = 0; i0 < m; i0 += rb) {
      const int64_t rows = std::min(rb, m - i0);
      OVVS_TRY_CUDA(cudaMemcpyAsync(da.get(), a + i0 * k, static_cast<size_t>(rows * k) * sizeof(float),
                                    cudaMemcpyHostToDevice, r.stream));
      if (i0 == 0) r.mark(1);
      OVVS_TRY_CUDA(ovvs::prim::launch_gemm_seq(da.as<float>(), db.as<float>(), dc.as<float>(),
                                                rows, n, k, trans_b != 0, round, r.stream));
      if (i0 == 0) r.mark(2);
      OVVS_TRY_CUDA(cudaMemcpyAsync(c + i0 * n, dc.get(), static_cast<size_t>(rows * n) * sizeof(float),
                                    cudaMemcpyDeviceToHost, r.stream));
    }
    r.mark(3);
    r.mark(4);
    OVVS_TRY(r.finish());
    r.last_device = OVVS_DEVICE_GPU;
    r.last_compute_dtype = round == ovvs::prim::kRoundF16 ? OVVS_DTYPE_F16 : OVVS_DTYPE_F32;
    return OVVS_STATUS_SUCCESS;
  });
}

}  // namespace

extern "C" {

ovvsStatus ovvsGemm(ovvsResources_t res, const float* a, const float* b, float* c, int64_t m,
                    int64_t n, int64_t k, int32_t trans_b) {
  if (!res || !a || !b || !c || m <= 0 || n <= 0 || k <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  return gemm_impl(res, a, b, c, m, n, k, trans_b, OVVS_DTYPE_F32);
}

ovvsStatus ovvsGemmEx(ovvsResources_t res, const float* a, const float* b, float* c, int64_t m,
                      int64_t n, int64_t k, int32_t trans_b, ovvsDType compute) {
  if (!res || !a || !b || !c || m <= 0 || n <= 0 || k <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  return gemm_impl(res, a, b, c, m, n, k, trans_b, compute);
}

ovvsStatus ovvsTopk(ovvsResources_t res, const float* scores, int64_t rows, int64_t cols, int64_t k,
                    int64_t* indices, float* values, int32_t largest) {
  if (!res || !scores || !indices || !values || rows <= 0 || cols <= 0 || k <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded(r, [&]() -> ovvsStatus {
    if (too_big(rows, cols) || cols > 0x7fffffffLL) return OVVS_STATUS_SHAPE_MISMATCH;
    const int64_t k_eff = std::min(k, cols);  // rows are written with stride k_eff
    const int64_t rb = std::min(rows, std::min<int64_t>(block_rows(cols, 20),
                                                        0x7fffffffLL / cols));
    DeviceBuffer ds, di, dv;
    OVVS_TRY_CUDA(ds.reserve(static_cast<size_t>(rb * cols) * sizeof(float) + 16));
    OVVS_TRY_CUDA(di.reserve(static_cast<size_t>(rb * k_eff) * sizeof(int64_t) + 16));
    OVVS_TRY_CUDA(dv.reserve(static_cast<size_t>(rb * k_eff) * sizeof(float) + 16));
    for (int64_t r0 = 0; r0 < rows; r0 += rb) {
      const int64_t nr = std::min(rb, rows - r0);
      OVVS_TRY_CUDA(cudaMemcpyAsync(ds.get(), scores + r0 * cols,
                                    static_cast<size_t>(nr * cols) * sizeof(float),
                                    cudaMemcpyHostToDevice, r.stream));
      OVVS_TRY(topk_device(r, ds.as<float>(), nr, cols, k, largest != 0, di.as<int64_t>(),
                           dv.as<float>()));
      OVVS_TRY_CUDA(cudaMemcpyAsync(indices + r0 * k_eff, di.get(),
                                    static_cast<size_t>(nr * k_eff) * sizeof(int64_t),
                                    cudaMemcpyDeviceToHost, r.stream));
      OVVS_TRY_CUDA(cudaMemcpyAsync(values + r0 * k_eff, dv.get(),
                                    static_cast<size_t>(nr * k_eff) * sizeof(float),
                                    cudaMemcpyDeviceToHost, r.stream));
    }
    OVVS_TRY(r.finish());
    r.last_device = OVVS_DEVICE_GPU;
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsKSelection(ovvsResources_t res, const float* scores, int64_t rows, int64_t cols,
                          int64_t k, int64_t* indices, float* values, int32_t largest) {
  return ovvsTopk(res, scores, rows, cols, k, indices, values, largest);
}

ovvsStatus ovvsGatherRows(ovvsResources_t res, const float* src, int64_t src_rows, int64_t dim,
                          const int64_t* idx, int64_t nidx, float* out) {
  if (!res || !src || !idx || !out || src_rows <= 0 || dim <= 0 || nidx <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded(r, [&]() -> ovvsStatus {
    if (too_big(src_rows, dim) || too_big(nidx, dim)) return OVVS_STATUS_SHAPE_MISMATCH;
    DeviceBuffer ds, di, dout;
    OVVS_TRY(upload(ds, src, static_cast<size_t>(src_rows * dim) * sizeof(float), r.stream));
    OVVS_TRY(upload(di, idx, static_cast<size_t>(nidx) * sizeof(int64_t), r.stream));
    OVVS_TRY_CUDA(dout.reserve(static_cast<size_t>(nidx * dim) * sizeof(float) + 16));
    OVVS_TRY_CUDA(ovvs::prim::launch_gather_rows(ds.as<float>(), src_rows, dim,
                                                 di.as<int64_t>(), nidx, dout.as<float>(),
                                                 r.stream));
    OVVS_TRY_CUDA(cudaMemcpyAsync(out, dout.get(), static_cast<size_t>(nidx * dim) * sizeof(float),
                                  cudaMemcpyDeviceToHost, r.stream));
    OVVS_TRY(r.finish());
    r.last_device = OVVS_DEVICE_GPU;
    return OVVS_STATUS_SUCCESS;
  });
}

ovvsStatus ovvsPairwiseDistance(ovvsResources_t res, ovvsMetric metric, const float* x, int64_t nx,
                                const float* y, int64_t ny, int64_t dim, float* out,
                                float metric_arg) {
  if (!res || !x || !y || !out || nx <= 0 || ny <= 0 || dim <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded(r, [&]() -> ovvsStatus {
    if (too_big(nx, dim) || too_big(ny, dim) || too_big(nx, ny)) return OVVS_STATUS_SHAPE_MISMATCH;
    DeviceBuffer dx, dy, dyn, dxn, dout;
    r.mark(0);
    OVVS_TRY(upload(dy, y, static_cast<size_t>(ny * dim) * sizeof(float), r.stream));
    OVVS_TRY_CUDA(dyn.reserve(static_cast<size_t>(ny) * sizeof(float) + 16));
    OVVS_TRY_CUDA(ovvs::prim::launch_row_norms_seq(dy.as<float>(), ny, dim, dyn.as<float>(),
                                                   r.stream));
    const int64_t rb = std::min(nx, block_rows(std::max(ny, dim), 2 * sizeof(float)));
    OVVS_TRY_CUDA(dx.reserve(static_cast<size_t>(rb * dim) * sizeof(float) + 16));
    OVVS_TRY_CUDA(dxn.reserve(static_cast<size_t>(rb) * sizeof(float) + 16));
    OVVS_TRY_CUDA(dout.reserve(static_cast<size_t>(rb * ny) * sizeof(float) + 16));
    for (int64_t i0 = 0; i0 < nx; i0 += rb) {
      const int64_t rows = std::min(rb, nx - i0);
      OVVS_TRY_CUDA(cudaMemcpyAsync(dx.get(), x + i0 * dim,
                                    static_cast<size_t>(rows * dim) * sizeof(float),
                                    cudaMemcpyHostToDevice, r.stream));
      if (i0 == 0) r.mark(1);
      OVVS_TRY(pairwise_block(r, metric, dx.as<float>(), rows, dy.as<float>(), ny, dim,
                              dyn.as<float>(), metric_arg, dxn.as<float>(), dout.as<float>()));
      if (i0 == 0) r.mark(2);
      OVVS_TRY_CUDA(cudaMemcpyAsync(out + i0 * ny, dout.get(),
                                    static_cast<size_t>(rows * ny) * sizeof(float),
                                    cudaMemcpyDeviceToHost, r.stream));
    }
    r.mark(3);
    r.mark(4);
    OVVS_TRY(r.finish());
    r.last_device = OVVS_DEVICE_GPU;
    return OVVS_STATUS_SUCCESS;
  });
}

// graphs.cpp:3384-3396 scores every pair (prim_pairwise, metric_arg 2), sets the diagonal to
// +inf and takes the k smallest per row -- brute_search_impl (mixer.cpp:843-864) of the dataset
// against itself except for the diagonal. Here: one brute-force index over the dataset, a search
// of its own rows for min(k + 1, n) neighbours through the fused kernel, and a per-row merge that
// drops the row itself and re-inserts it with score +inf at its place in the top-k order. No
// n x n matrix is formed; rows are searched in blocks so the result buffers stay bounded.
ovvsStatus ovvsAllNeighbors(ovvsResources_t res, const float* dataset, int64_t n, int64_t dim,
                            ovvsMetric metric, int32_t k, int64_t* neighbors, float* distances) {
  if (!res || !dataset || !neighbors || !distances || n <= 1 || k <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  Resources& r = *from_handle(res);
  return guarded(r, [&]() -> ovvsStatus {
    if (too_big(n, dim) || n > 0x7fffffffLL) return OVVS_STATUS_SHAPE_MISMATCH;
    const int64_t ke = std::min<int64_t>(k, n - 1);
    const int64_t kin = std::min<int64_t>(ke + 1, n);
    DeviceBuffer dx, si, sd, oi, od;
    OVVS_TRY(upload(dx, dataset, static_cast<size_t>(n * dim) * sizeof(float), r.stream));
    ovvs::nb::BruteIndex ix;
    OVVS_TRY(ovvs::nb::build_from_device(r, ix, dx.get(), OVVS_DTYPE_F32, n, dim,
                                         static_cast<int>(metric), 0));
    const int64_t rb = std::min(n, block_rows(kin, 2 * (sizeof(int64_t) + sizeof(float))));
    OVVS_TRY_CUDA(si.reserve(static_cast<size_t>(rb * kin) * sizeof(int64_t) + 16));
    OVVS_TRY_CUDA(sd.reserve(static_cast<size_t>(rb * kin) * sizeof(float) + 16));
    OVVS_TRY_CUDA(oi.reserve(static_cast<size_t>(rb * ke) * sizeof(int64_t) + 16));
    OVVS_TRY_CUDA(od.reserve(static_cast<size_t>(rb * ke) * sizeof(float) + 16));
    const bool negate = metric == OVVS_METRIC_INNER_PRODUCT;
    for (int64_t i0 = 0; i0 < n; i0 += rb) {
      const int64_t rows = std::min(rb, n - i0);
      int64_t got = 0;
      OVVS_TRY(ovvs::nb::search_device(r, ix, dx.as<float>() + i0 * dim, rows, kin, nullptr,
                                       si.as<int64_t>(), sd.as<float>(), &got));
      if (got != kin) return OVVS_STATUS_ERROR;
      OVVS_TRY_CUDA(ovvs::prim::launch_exclude_self(si.as<int64_t>(), sd.as<float>(), rows,
                                                    static_cast<int>(kin), i0,
                                                    static_cast<int>(ke), negate,
                                                    oi.as<int64_t>(), od.as<float>(), r.stream));
      OVVS_TRY_CUDA(cudaMemcpyAsync(neighbors + i0 * ke, oi.get(),
                                    static_cast<size_t>(rows * ke) * sizeof(int64_t),
                                    cudaMemcpyDeviceToHost, r.stream));
      OVVS_TRY_CUDA(cudaMemcpyAsync(distances + i0 * ke, od.get(),
                                    static_cast<size_t>(rows * ke) * sizeof(float),
                                    cudaMemcpyDeviceToHost, r.stream));
    }
    OVVS_TRY(r.finish());
    r.last_device = OVVS_DEVICE_GPU;
    r.last_compute_dtype = OVVS_DTYPE_F32;
    return OVVS_STATUS_SUCCESS;
  });
}

}  // extern "C"
