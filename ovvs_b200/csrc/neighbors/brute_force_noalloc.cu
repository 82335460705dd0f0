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
// creates that array on a device when it loads this file's module there, and keeps it until the
// process exits. With the runtime's lazy module loading (the default since CUDA 12.2) that load
// happens at the first call on each device, whose set-up looks up the array's device address with
// cudaGetSymbolAddress (later calls reuse the cached address): the 32 MiB are reserved then, so a
// caller whose allocator will take the device's free memory makes that first call at start-up,
// before it does (or sets CUDA_MODULE_LOADING=EAGER, which loads it with the library).
//
// The caller passes the inputs and outputs (device pointers) and a stream. Nothing here calls
// cudaMalloc, cudaFree or an allocating library routine, and no existing code path changes: the
// same kernels as ovvsBruteForceSearchDevice run on the caller's stream.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <new>

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


// Holds a device's array while one call uses it. Once GPU work has been queued on the array, every
// exit (errors included) waits for the stream before the next call may take the array.
class ArrayHold {
 public:
  ArrayHold(int device, cudaStream_t s) : lock_(g_device_mu[device]), s_(s) {}
  ~ArrayHold() {
    if (queued_) (void)cudaStreamSynchronize(s_);
  }
  void queued() { queued_ = true; }

 private:
  std::lock_guard<std::mutex> lock_;
  cudaStream_t s_;
  bool queued_ = false;
};

ovvsStatus search_no_alloc(ovvs::rt::Resources& r, const ovvs::nb::BruteIndex& ix,
                           const float* d_queries, int64_t nq, int64_t k, const uint8_t* d_bitset,
                           int64_t* d_neighbors, float* d_distances, cudaStream_t s) {
  using namespace ovvs;
  OVVS_TRY(r.check_policy());
  if (!r.gpu_available) return OVVS_STATUS_DEVICE_UNAVAILABLE;
  if (r.device < 0 || r.device >= kMaxDevices || ix.device != r.device)
    return OVVS_STATUS_INVALID_ARGUMENT;
  // the cross-shard exchange (and a group's shards) need buffers of their own
  if (ix.sharded || !ix.shards.empty()) return OVVS_STATUS_UNSUPPORTED;
  const int64_t k_eff = std::min<int64_t>(k, ix.n_total);
  const int kl = nb::list_size_for(k_eff);
  if (kl == 0) return OVVS_STATUS_UNSUPPORTED;

  ArrayHold hold(r.device, s);
  OVVS_TRY_CUDA(cudaSetDevice(r.device));
  unsigned char* base = nullptr;
  OVVS_TRY(scratch_address(r.device, &base));

  // Size the pieces and reject what does not fit the fixed array.
  nb::SearchCtx c;
  c.q_pad = prim::pad_queries(nq);
  c.num_qtiles = static_cast<int>(c.q_pad / prim::kTileQ);
  const size_t fixed = piece(sizeof(int)) + piece(sizeof(int)) +
                       piece(static_cast<size_t>(c.q_pad) * 2 * ix.dp * sizeof(__half)) +
                       2 * piece(static_cast<size_t>(c.q_pad) * sizeof(float)) +
                       piece(static_cast<size_t>(c.q_pad) * sizeof(uint64_t)) +
                       (d_bitset ? piece(static_cast<size_t>(ix.n_pad / 32) * sizeof(uint32_t)) : 0);
  const size_t cand_per_sc =
      static_cast<size_t>(c.q_pad) * kl * prim::kListsPerItem * sizeof(uint64_t);
  if (fixed + piece(cand_per_sc) > kNoAllocScratchBytes) return OVVS_STATUS_SHAPE_MISMATCH;
  const size_t cand_budget = kNoAllocScratchBytes - fixed - 256;

  Carver cv{base};
  int* err = cv.take<int>(1);
  c.flag = cv.take<int>(1);
  c.a16 = cv.take<__half>(static_cast<size_t>(c.q_pad) * 2 * ix.dp);
  c.q_mul = cv.take<float>(c.q_pad);
  c.xn = cv.take<float>(c.q_pad);
  uint64_t* bound = cv.take<uint64_t>(c.q_pad);
  c.allow = d_bitset ? cv.take<uint32_t>(ix.n_pad / 32) : nullptr;

  prim::FusedParams p;
  OVVS_TRY(nb::base_params(r, ix, c, nq, &p));
  p.err = err;  // this call's own error word, in the array
  // The planner caps the candidate lists at 1.5e9 bytes; scale the per-super-chunk size so that
  // its cap lands on this array's budget instead.
  const double scale = 1.5e9 / static_cast<double>(cand_budget);
  const int sms = nb::pair_sms(r, p);
  p.num_sc = nb::choose_num_sc(c.num_qtiles, ix.num_tiles, sms,
                               static_cast<int64_t>(static_cast<double>(cand_per_sc) * scale) + 1,
                               &p.tiles_per_item);
  if (static_cast<size_t>(p.num_sc) * cand_per_sc > cand_budget) return OVVS_STATUS_SHAPE_MISMATCH;
  p.num_items = prim::fused_items(c.num_qtiles, p.num_sc);
  uint64_t* cand = cv.take<uint64_t>(static_cast<size_t>(p.num_sc) * cand_per_sc / sizeof(uint64_t));
  if (cv.used > kNoAllocScratchBytes) return OVVS_STATUS_SHAPE_MISMATCH;
  OVVS_TRY(nb::encode_query_maps(c, ix.dp));
  c.maps.b64 = ix.b64;
  c.maps.b32 = ix.b32;
  c.maps.b16 = ix.b16;
  p.q_bound = bound;
  p.k_pub = static_cast<int>(k_eff);
  p.out = cand;

  // The array keeps the previous call's contents: clear what must start at zero / empty.
  hold.queued();
  OVVS_TRY_CUDA(cudaMemsetAsync(err, 0, sizeof(int), s));
  OVVS_TRY_CUDA(cudaMemsetAsync(c.flag, 0, sizeof(int), s));
  OVVS_TRY_CUDA(cudaMemsetAsync(bound, 0xFF, static_cast<size_t>(c.q_pad) * sizeof(uint64_t), s));
  prim::launch_query_prep(d_queries, nq, c.q_pad, static_cast<int>(ix.dim), ix.dp, ix.metric,
                          ix.e_db, c.a16, c.q_mul, c.xn, c.flag, s);
  OVVS_TRY_CUDA(cudaGetLastError());
  if (d_bitset) {
    prim::launch_allow_bits(d_bitset, ix.row_offset, ix.row_id.as<uint32_t>(), ix.n, ix.n_pad,
                            c.allow, s);
    OVVS_TRY_CUDA(cudaGetLastError());
  }
  OVVS_TRY_CUDA(prim::launch_knn_fused(c.maps, p, kl, prim::fused_grid(p.num_items, sms), s));
  prim::MergeParams m = nb::merge_params(ix, c, d_queries, nq, k_eff);
  m.cand = cand;
  m.num_sc = p.num_sc * prim::kListsPerItem;  // lists per query
  m.kl = kl;
  m.neighbors = d_neighbors;
  m.distances = d_distances;
  OVVS_TRY_CUDA(prim::launch_merge_rerank(m, s));

  // Synchronous: the next call may reuse the array only after this one's GPU work is done.
  OVVS_TRY_CUDA(cudaStreamSynchronize(s));
  int host_err = 0;
  OVVS_TRY_CUDA(cudaMemcpy(&host_err, err, sizeof(int), cudaMemcpyDeviceToHost));
  std::lock_guard<std::mutex> lk(r.mu);
  if (host_err != 0) {
    r.last_kernel_error = host_err;  // which bounded wait ran out (ovvsResourcesLastKernelError)
    return OVVS_STATUS_ERROR;
  }
  r.last_device = OVVS_DEVICE_GPU;
  r.last_compute_dtype = OVVS_DTYPE_F32;
  return OVVS_STATUS_SUCCESS;
}

}  // namespace

extern "C" ovvsStatus ovvsBruteForceSearchDeviceNoAlloc(ovvsResources_t res,
                                                        ovvsBruteForceIndex_t index,
                                                        const float* d_queries, int64_t nq,
                                                        int64_t k, const uint8_t* d_bitset,
                                                        int64_t* d_neighbors, float* d_distances,
                                                        void* stream) {
  if (!res || !index || !d_queries || !d_neighbors || !d_distances || nq <= 0 || k <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  try {
    return search_no_alloc(*ovvs::rt::from_handle(res),
                           *reinterpret_cast<const ovvs::nb::BruteIndex*>(index), d_queries, nq,
                           k, d_bitset, d_neighbors, d_distances,
                           static_cast<cudaStream_t>(stream));
  } catch (const std::bad_alloc&) {
    return OVVS_STATUS_OOM;
  } catch (...) {
    return OVVS_STATUS_ERROR;
  }
}
