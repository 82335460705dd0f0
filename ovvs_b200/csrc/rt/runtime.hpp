// CUDA runtime layer behind the ovvs C ABI: the Resources object (device, stream, NCCL
// communicator, workspace, watchdog word), device/pinned buffers, tensor-map encoding and the
// mapping from CUDA/NCCL errors to ovvsStatus.
//
// Replaces the reference's ResourcesData (src/internal.hpp:459-562) and its device probing
// (src/rt/probe.cpp:132-140): one Resources = one CUDA device + one stream; there is no device
// selection between backends and no CPU fallback.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <atomic>
#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include "nccl_dl.hpp"
#include "ovvs/ovvs.h"
#include "peer_window.hpp"

struct ovvsResourcesImpl;

namespace ovvs {
namespace rt {

ovvsStatus status_of(cudaError_t e);
ovvsStatus status_of(ncclResult_t e);

#define OVVS_TRY_CUDA(expr)                                   \
  do {                                                        \
    const cudaError_t ovvs_e_ = (expr);                       \
    if (ovvs_e_ != cudaSuccess) return ::ovvs::rt::status_of(ovvs_e_); \
  } while (0)

#define OVVS_TRY(expr)                                        \
  do {                                                        \
    const ovvsStatus ovvs_s_ = (expr);                        \
    if (ovvs_s_ != OVVS_STATUS_SUCCESS) return ovvs_s_;       \
  } while (0)

// Grow-only device allocation on one device.
class DeviceBuffer {
 public:
  DeviceBuffer() = default;
  ~DeviceBuffer();
  DeviceBuffer(const DeviceBuffer&) = delete;
  DeviceBuffer& operator=(const DeviceBuffer&) = delete;
  // Ensures at least `bytes` are allocated (contents are not preserved on growth).
  cudaError_t reserve(size_t bytes);
  void release();
  // Exchanges the allocations of two buffers (used to grow a buffer while keeping its data).
  void swap(DeviceBuffer& o) noexcept {
    std::swap(ptr_, o.ptr_);
    std::swap(bytes_, o.bytes_);
    std::swap(device_, o.device_);
  }
  // Forgets the allocation without freeing it (it is returned when the process exits). Used when
  // freeing could wait on device work that may never finish (a collective whose peer is gone).
  void abandon() noexcept {
    ptr_ = nullptr;
    bytes_ = 0;
  }
  void* get() const { return ptr_; }
  size_t size() const { return bytes_; }
  template <class T>
  T* as() const {
    return static_cast<T*>(ptr_);
  }

 private:
  void* ptr_ = nullptr;
  size_t bytes_ = 0;
  int device_ = -1;
};

// Workspace slots owned by a Resources (reused across calls on that Resources).
enum WorkSlot : int {
  kWsQueries = 0,  // fp32 queries
  kWsQueryA,       // fp16 hi/lo query operand
  kWsQueryMul,
  kWsQueryNorm,
  kWsFlags,        // lo flag
  kWsBitset,       // caller bitset (host searches)
  kWsAllow,        // position-ordered allow bits
  kWsCand,         // fused-kernel candidate lists
  kWsBound,        // shared per-query bound of the fused kernel / large-k bound keys
  kWsAppCount,     // large k: per-query append counts
  kWsAppBuf,       // large k: per-query append buffers
  kWsAppBound,     // large k: shared bound of the pre-pass lists
  kWsOverflow,     // large k: append-buffer overflow flag
  kWsNeighbors,    // results (host searches)
  kWsDistances,
  kWsShardRank,    // per-shard results for the all-gather
  kWsShardGid,
  kWsGatherRank,
  kWsGatherGid,
  kWsIvfQueryNorm,  // IVF-Flat search: query norms
  kWsIvfScores,     // coarse scores [queries x nlist]
  kWsIvfProbe,      // probed lists [queries x nprobe]
  kWsIvfProbeVal,
  kWsIvfCum,        // per-query positions of the probed lists
  kWsIvfListCount,  // pairs per list, their offsets, fill cursors
  kWsIvfListOff,
  kWsIvfCursor,
  kWsIvfPairs,
  kWsIvfItemCount,
  kWsIvfItemOff,
  kWsIvfCand,       // per-pair candidate lists (select mode) / candidate keys (sort mode)
  kWsIvfCand2,
  kWsIvfSeg,        // sort mode: segment bases and bounds
  kWsIvfSegBegin,
  kWsIvfSegEnd,
  kWsIvfTmp,        // CUB temporary storage
  kWsIvfTcQueryA,   // tensor-core list scan: fp16 query operand per query, then per slot
  kWsIvfTcSlotA,
  kWsIvfTcQueryMul,
  kWsIvfTcSlotMul,
  kWsIvfTcQueryNorm,
  kWsIvfTcFlag,
  kWsIvfTcCounts,   // slot and item counts and offsets per list
  kWsIvfTcSlotPair,
  kWsIvfTcPairSlot,
  kWsIvfTcItems,
  kWsIvfTcBound,
  kWsIvfTcCand,
  kWsIvfTcAllow,
  kWsCount
};

class Workers;

struct Resources {
  int device = 0;
  bool gpu_available = false;
  int num_sms = 0;
  int max_smem_optin = 0;
  std::string device_name = "no-cuda-device";
  ovvsPolicy policy = OVVS_POLICY_AUTO;
  std::atomic<ovvsDevice> last_device{OVVS_DEVICE_CPU};
  ovvsDType last_compute_dtype = OVVS_DTYPE_F32;
  bool cagra_walk_counters = false;
  cudaStream_t stream = nullptr;
  int rank = 0;
  int world = 1;
  ncclComm_t comm = nullptr;       // non-blocking communicator of the world's ranks (world > 1)
  bool comm_failed = false;        // aborted after an NCCL error or an expired deadline
  // The abort did not finish within its bound (it waits on a departed peer): collectives may still
  // occupy the device, so this Resources leaves its device memory to the process's exit.
  bool abort_pending = false;
  int64_t nccl_timeout_ms = 60000; // deadline of NCCL set-up and of waits on collectives
  uint64_t comm_tag = 0;           // hash of the communicator's unique id (same on every rank)
  int window_seq = 0;              // peer windows created so far (names their exchanges)
  // Sharded searches share each query's bound between ranks through this window (q_pad keys
  // per rank). peer_bounds: 0 not tried yet, 1 in use, -1 unavailable or switched off
  // (OVVS_PEER_BOUNDS=0).
  PeerWindow bound_win;
  int peer_bounds = 0;
  // One process, several devices (ovvsResourcesCreate with OVVS_CUDA_DEVICES naming more than
  // one): this object is an ordinary Resources on the first device, and `group` holds one member
  // per device (rank g of world G, sharing a communicator) driven by one worker thread each.
  std::vector<std::unique_ptr<Resources>> group;
  std::unique_ptr<Workers> workers;
  int* d_err = nullptr;  // kernel watchdog word (device)
  int last_kernel_error = 0;  // last nonzero watchdog code seen by finish()
  static constexpr int kPhases = 4;
  bool profiling = false;
  bool phase_valid = false;
  cudaEvent_t phase_ev[kPhases + 1] = {};
  // While profiling, the phase boundaries of the last kPhaseHistory searches are also kept in a
  // ring, so back-to-back searches can be timed without a synchronisation after each.
  static constexpr int kPhaseHistory = 64;
  cudaEvent_t hist_ev[kPhaseHistory][kPhases + 1] = {};
  int hist_next = 0;   // ring slot of the search being recorded
  int hist_count = 0;  // completed searches in the ring (<= kPhaseHistory)
  std::mutex mu;
  DeviceBuffer ws[kWsCount];
  // Pinned staging buffers of upload() (allocated on the first large upload).
  void* stage_buf[2] = {};
  cudaEvent_t stage_ev[2] = {};
  bool stage_used[2] = {};

  ~Resources();
  // Makes `device` current on the calling thread and creates the stream / error word on first
  // use. Returns DEVICE_UNAVAILABLE without a usable sm_100 device.
  ovvsStatus activate();
  // FORCE_CPU / FORCE_NPU cannot be honoured: the forced device never falls back.
  ovvsStatus check_policy() const;
  // Waits for the stream, then reads and clears the watchdog word. With a communicator the wait
  // polls the stream and the communicator's asynchronous error against nccl_timeout_ms; an NCCL
  // error or the deadline aborts the communicator and returns ERROR.
  ovvsStatus finish();
  // Return value of an NCCL call on `comm`: settles ncclInProgress (bounded); a failure aborts
  // the communicator and gives ERROR. Calls after an abort give ERROR without touching NCCL.
  ovvsStatus collective(ncclResult_t ret);
  ovvsStatus comm_ready() const {
    return comm && !comm_failed ? OVVS_STATUS_SUCCESS : OVVS_STATUS_ERROR;
  }
  void abort_comm();
  // Records phase boundary `i` (0..kPhases) of the current search when profiling (ignored while
  // mark_hold is set: a k-means fit keeps its own phases while its searches run).
  void mark(int i);
  bool mark_hold = false;
  template <class T>
  ovvsStatus scratch(WorkSlot slot, size_t count, T** out) {
    const cudaError_t e = ws[slot].reserve(count * sizeof(T) + 16);
    if (e != cudaSuccess) return status_of(e);
    *out = ws[slot].as<T>();
    return OVVS_STATUS_SUCCESS;
  }
};

inline Resources* from_handle(ovvsResources_t r) { return reinterpret_cast<Resources*>(r); }
inline ovvsResources_t to_handle(Resources* r) { return reinterpret_cast<ovvsResources_t>(r); }

// Probes `device` and fills the device fields of `r` (no stream yet).
void probe_device(Resources& r, int device);

// 2D fp16 tensor map over a row-major [rows x cols] matrix with a {box_cols x box_rows} box and
// the swizzle that matches box_cols * 2 bytes (128/64/32).
bool encode_f16_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                   uint32_t box_cols, uint32_t box_rows);

// Enqueues a host -> device copy of `bytes` on r.stream; the host buffer may be reused as soon as
// this returns (as with a pageable cudaMemcpyAsync). Large pageable buffers go through two pinned
// staging buffers filled by several host threads while the previous chunk's DMA runs, which is
// faster than the driver's own pageable path; small or already pinned buffers are copied directly.
ovvsStatus upload(Resources& r, void* dst, const void* src, size_t bytes);

// Global row count of a sharded dataset (sum over ranks) and other small all-reduces.
ovvsStatus allreduce_i64_sum(Resources& r, int64_t* value);

// Devices for ovvsResourcesCreate: OVVS_CUDA_DEVICES (comma-separated, e.g. "0,1,2,3"), else
// OVVS_CUDA_DEVICE, else 0.
std::vector<int> default_devices();

// Creates r's communicator as rank r.rank of r.world from `id` (non-blocking, bounded by
// r.nccl_timeout_ms). r's device must be current.
ovvsStatus init_comm(Resources& r, const ncclUniqueId& id);

// Deadline for NCCL set-up and waits: OVVS_NCCL_TIMEOUT_MS, else 60 s.
int64_t nccl_timeout_ms_default();

}  // namespace rt
}  // namespace ovvs
