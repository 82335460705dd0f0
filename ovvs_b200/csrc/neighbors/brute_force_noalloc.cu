// ovvsBruteForceSearchDeviceNoAlloc: the device-pointer brute-force search without any device
// allocation.
//
// Who needs it: callers that cannot let a library allocate GPU memory. Typical cases are a
// process whose free device memory is already reserved by another allocator (a framework's
// caching pool, a serving engine that pre-assigns the whole GPU), where a cudaMalloc inside the
// search would fail or fragment that pool; and latency-critical request loops, where the
// implicit device-wide synchronisation of cudaMalloc / cudaFree in the middle of a request is
// not acceptable.
//
// How: every intermediate buffer of the search (scaled query operand, per-query multipliers and
// norms, allow bits, candidate lists, the shared per-query bound, the kernel error word) is carved
// out of one file-scope __device__ array of kNoAllocScratchBytes (32 MiB). The CUDA runtime
// creates that array once per device when this module is loaded and keeps it until the process
// exits. Its device address is obtained with cudaGetSymbolAddress on the first call on each
// device (the one-time set-up); later calls reuse the cached address.
//
// The caller passes the inputs and outputs (device pointers) and a stream. Nothing here calls
// cudaMalloc, cudaFree or an allocating library routine, and no existing code path changes: the
// same kernels as ovvsBruteForceSearchDevice run on the caller's stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "../prim/prep.cuh"
#include "../prim/select.cuh"
#include "../rt/runtime.hpp"
#include "brute_force.hpp"
#include "ovvs/ovvs_cuda.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;
constexpr int kMaxDevices = 64;

// The shared scratch: every call on a device uses (and overwrites) this array.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices] = {};
// Calls on one device are serialised: they share the array, so two calls whose GPU work
// overlapped would race on it.
std::mutex g_device_mu[kMaxDevices];

// One-time, per-device set-up: the device address of the array (device must be current).
ovvsStatus scratch_address(int device, unsigned char** out) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (!g_scratch_addr[device]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      (void)cudaGetLastError();
      return e == cudaSuccess ? OVVS_STATUS_ERROR : ovvs::rt::status_of(e);
    }
    g_scratch_addr[device] = p;
  }
  *out = static_cast<unsigned char*>(g_scratch_addr[device]);
  return OVVS_STATUS_SUCCESS;
}

// Bump allocator over the scratch array (256-byte aligned pieces).
struct Carver {
  unsigned char* base;
  size_t used = 0;
  template <class T>
  T* take(size_t count) {
    T* p = reinterpret_cast<T*>(base + used);
    used += (count * sizeof(T) + 255) & ~size_t(255);
    return p;
  }
};

size_t piece(size_t bytes) { return (bytes + 255) & ~size_t(255); }

}  // namespace

extern "C" ovvsStatus ovvsBruteForceSearchDeviceNoAlloc(ovvsResources_t res,
                                                        ovvsBruteForceIndex_t index,
                                                        const float* d_queries, int64_t nq,
                                                        int64_t k, const uint8_t* d_bitset,
                                                        int64_t* d_neighbors, float* d_distances,
                                                        void* stream) {
  using namespace ovvs;
  if (!res || !index || !d_queries || !d_neighbors || !d_distances || nq <= 0 || k <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  rt::Resources& r = *rt::from_handle(res);
  const nb::BruteIndex& ix = *reinterpret_cast<const nb::BruteIndex*>(index);
  OVVS_TRY(r.check_policy());
  if (!r.gpu_available) return OVVS_STATUS_DEVICE_UNAVAILABLE;
  if (r.device < 0 || r.device >= kMaxDevices || ix.device != r.device)
    return OVVS_STATUS_INVALID_ARGUMENT;
  if (ix.sharded) return OVVS_STATUS_UNSUPPORTED;  // the cross-shard exchange needs buffers
  const int64_t k_eff = std::min<int64_t>(k, ix.n_total);
  const int kl = nb::list_size_for(k_eff);
  if (kl == 0) return OVVS_STATUS_UNSUPPORTED;

  std::lock_guard<std::mutex> device_lock(g_device_mu[r.device]);
  OVVS_TRY_CUDA(cudaSetDevice(r.device));
  unsigned char* base = nullptr;
  OVVS_TRY(scratch_address(r.device, &base));
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  // Size the pieces and reject what does not fit the fixed array.
  const int64_t q_pad = prim::pad_queries(nq);
  const int num_qtiles = static_cast<int>(q_pad / prim::kTileQ);
  const size_t fixed = piece(sizeof(int)) + piece(sizeof(int)) +
                       piece(static_cast<size_t>(q_pad) * 2 * ix.dp * sizeof(__half)) +
                       2 * piece(static_cast<size_t>(q_pad) * sizeof(float)) +
                       piece(static_cast<size_t>(q_pad) * sizeof(uint64_t)) +
                       (d_bitset ? piece(static_cast<size_t>(ix.n_pad / 32) * sizeof(uint32_t)) : 0);
  const size_t cand_per_sc = static_cast<size_t>(q_pad) * kl * prim::kListsPerItem * sizeof(uint64_t);
  if (fixed + piece(cand_per_sc) > kNoAllocScratchBytes) return OVVS_STATUS_SHAPE_MISMATCH;
  const size_t cand_budget = kNoAllocScratchBytes - fixed - 256;

  prim::FusedParams p{};
  p.dp = ix.dp;
  p.nchunk = ix.nchunk;
  for (int c = 0; c < ix.nchunk; ++c) {
    p.chunk_x[c] = ix.chunk_x[c];
    p.chunk_w[c] = ix.chunk_w[c];
  }
  p.b_parts = ix.b_parts;
  p.nunits = ix.b_parts * ix.nchunk;
  if (!prim::plan_fused_smem(p, r.max_smem_optin)) return OVVS_STATUS_UNSUPPORTED;
  // The planner caps the candidate lists at 1.5e9 bytes; scale the per-super-chunk size so that
  // its cap lands on this array's budget instead.
  const double scale = 1.5e9 / static_cast<double>(cand_budget);
  const int sms = 2 * std::min(r.num_sms / 2, prim::fused_max_pairs(p.smem_bytes));
  p.num_sc = nb::choose_num_sc(num_qtiles, ix.num_tiles, sms,
                               static_cast<int64_t>(static_cast<double>(cand_per_sc) * scale) + 1,
                               &p.tiles_per_item);
  if (static_cast<size_t>(p.num_sc) * cand_per_sc > cand_budget) return OVVS_STATUS_SHAPE_MISMATCH;

  Carver cv{base};
  int* err = cv.take<int>(1);
  int* flag = cv.take<int>(1);
  __half* a16 = cv.take<__half>(static_cast<size_t>(q_pad) * 2 * ix.dp);
  float* q_mul = cv.take<float>(q_pad);
  float* xn = cv.take<float>(q_pad);
  uint64_t* bound = cv.take<uint64_t>(q_pad);
  uint32_t* allow = d_bitset ? cv.take<uint32_t>(ix.n_pad / 32) : nullptr;
  uint64_t* cand = cv.take<uint64_t>(static_cast<size_t>(p.num_sc) * cand_per_sc / sizeof(uint64_t));
  if (cv.used > kNoAllocScratchBytes) return OVVS_STATUS_SHAPE_MISMATCH;

  // The array keeps the previous call's contents: clear what must start at zero / empty.
  OVVS_TRY_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
  OVVS_TRY_CUDA(cudaMemsetAsync(flag, 0, sizeof(int), s));
  OVVS_TRY_CUDA(cudaMemsetAsync(bound, 0xFF, static_cast<size_t>(q_pad) * sizeof(uint64_t), s));

  const int dim = static_cast<int>(ix.dim);
  prim::launch_query_prep(d_queries, nq, q_pad, dim, ix.dp, ix.metric, ix.e_db, a16, q_mul, xn,
                          flag, s);
  OVVS_TRY_CUDA(cudaGetLastError());
  if (d_bitset) {
    prim::launch_allow_bits(d_bitset, ix.row_offset, ix.row_id.as<uint32_t>(), ix.n, ix.n_pad,
                            allow, s);
    OVVS_TRY_CUDA(cudaGetLastError());
  }
  p.query_split = ix.metric != prim::kMetricHamming;
  p.q_lo_flag = flag;
  p.num_qtiles = num_qtiles;
  p.num_dbtiles = ix.num_tiles;
  p.num_items = prim::fused_items(num_qtiles, p.num_sc);
  p.n_rows = ix.n;
  p.row_aux = ix.aux.as<float>();
  p.group_aux = ix.tile_aux.as<float2>() + ix.num_tiles;
  p.row_id = ix.row_id.as<uint32_t>();
  p.q_mul = q_mul;
  p.allow = allow;
  p.rank_kind = prim::rank_kind_of(ix.metric);
  p.nq = nq;
  p.k_pub = static_cast<int>(k_eff);
  p.q_bound = bound;
  p.out = cand;
  p.err = err;
  prim::FusedMaps maps{};
  const uint64_t a_cols = static_cast<uint64_t>(2 * ix.dp);
  if (!rt::encode_f16_2d(&maps.a64, a16, a_cols, q_pad, 64, prim::kTileQ) ||
      !rt::encode_f16_2d(&maps.a32, a16, a_cols, q_pad, 32, prim::kTileQ) ||
      !rt::encode_f16_2d(&maps.a16, a16, a_cols, q_pad, 16, prim::kTileQ))
    return OVVS_STATUS_ERROR;
  maps.b64 = ix.b64;
  maps.b32 = ix.b32;
  maps.b16 = ix.b16;
  const int grid = prim::fused_grid(p.num_items, sms);
  OVVS_TRY_CUDA(prim::launch_knn_fused(maps, p, kl, grid, s));

  prim::MergeParams m{};
  m.cand = cand;
  m.num_sc = p.num_sc * prim::kListsPerItem;  // lists per query
  m.kl = kl;
  m.nq = nq;
  m.dim = dim;
  m.queries = d_queries;
  m.xn = xn;
  m.metric = ix.metric;
  m.exact32 = ix.exact32.get() ? ix.exact32.as<float>() : nullptr;
  m.rows16 = ix.rows16.as<__half>();
  m.rows16_stride = ix.b_parts * ix.dp;
  m.norm_sorted = ix.norm_sorted.as<float>();
  m.inv_perm = ix.inv_perm.as<uint32_t>();
  m.allow = allow;
  m.row_offset = ix.row_offset;
  m.k_eff = static_cast<int>(k_eff);
  m.negate_output = ix.metric == prim::kMetricInnerProduct;
  m.neighbors = d_neighbors;
  m.distances = d_distances;
  OVVS_TRY_CUDA(prim::launch_merge_rerank(m, s));

  // Synchronous: the next call may reuse the array only after this one's GPU work is done.
  OVVS_TRY_CUDA(cudaStreamSynchronize(s));
  int host_err = 0;
  OVVS_TRY_CUDA(cudaMemcpy(&host_err, err, sizeof(int), cudaMemcpyDeviceToHost));
  if (host_err != 0) return OVVS_STATUS_ERROR;
  r.last_device = OVVS_DEVICE_GPU;
  r.last_compute_dtype = OVVS_DTYPE_F32;
  return OVVS_STATUS_SUCCESS;
}
