// CUDA runtime layer (see runtime.hpp).
#include "runtime.hpp"

#include <algorithm>
#include <atomic>
#include <chrono>
#include <memory>
#include <cstdlib>
#include <cstring>
#include <sstream>
#include <thread>
#include <vector>

#include "group.hpp"
#include "nccl_watch.hpp"

namespace ovvs {
namespace rt {

ovvsStatus status_of(cudaError_t e) {
  switch (e) {
    case cudaSuccess:
      return OVVS_STATUS_SUCCESS;
    case cudaErrorMemoryAllocation:
      return OVVS_STATUS_OOM;
    case cudaErrorNoDevice:
    case cudaErrorInsufficientDriver:
    case cudaErrorInvalidDevice:
    case cudaErrorNoKernelImageForDevice:
    case cudaErrorDevicesUnavailable:
      return OVVS_STATUS_DEVICE_UNAVAILABLE;
    default:
      return OVVS_STATUS_ERROR;
  }
}

ovvsStatus status_of(ncclResult_t e) {
  if (e == ncclSuccess) return OVVS_STATUS_SUCCESS;
  if (e == ncclInvalidArgument || e == ncclInvalidUsage) return OVVS_STATUS_INVALID_ARGUMENT;
  return OVVS_STATUS_ERROR;
}

DeviceBuffer::~DeviceBuffer() { release(); }

cudaError_t DeviceBuffer::reserve(size_t bytes) {
  if (bytes <= bytes_ && ptr_) return cudaSuccess;
  release();
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  void* p = nullptr;
  e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    return e;
  }
  ptr_ = p;
  bytes_ = bytes;
  device_ = dev;
  return cudaSuccess;
}

void DeviceBuffer::release() {
  if (!ptr_) return;
  int cur = -1;
  cudaGetDevice(&cur);
  if (device_ >= 0 && device_ != cur) cudaSetDevice(device_);
  cudaFree(ptr_);
  if (device_ >= 0 && device_ != cur && cur >= 0) cudaSetDevice(cur);
  ptr_ = nullptr;
  bytes_ = 0;
}

std::vector<int> default_devices() {
  std::vector<int> out;
  const char* list = std::getenv("OVVS_CUDA_DEVICES");
  if (list && *list) {
    std::stringstream ss(list);
    std::string item;
    while (std::getline(ss, item, ','))
      if (!item.empty()) out.push_back(std::atoi(item.c_str()));
  }
  if (out.empty()) {
    const char* one = std::getenv("OVVS_CUDA_DEVICE");
    out.push_back(one && *one ? std::atoi(one) : 0);
  }
  return out;
}

int64_t nccl_timeout_ms_default() {
  const char* s = std::getenv("OVVS_NCCL_TIMEOUT_MS");
  const long long v = s && *s ? std::atoll(s) : 0;
  return v > 0 ? v : 60000;
}

namespace {

int64_t now_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

void short_pause() { std::this_thread::sleep_for(std::chrono::microseconds(50)); }

}  // namespace

ovvsStatus init_comm(Resources& r, const ncclUniqueId& id) {
  const NcclApi* nc = nccl();
  if (!nc) return OVVS_STATUS_DEVICE_UNAVAILABLE;
  // FNV-1a of the unique id: the same on every rank, different for every communicator.
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < sizeof(id.internal); ++i) {
    h ^= static_cast<uint8_t>(id.internal[i]);
    h *= 1099511628211ull;
  }
  r.comm_tag = h;
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  const ncclResult_t ret = nc->CommInitRankConfig(&r.comm, r.world, id, r.rank, &cfg);
  return r.collective(ret);
}

void Resources::abort_comm() {
  ncclComm_t c = comm;
  comm = nullptr;
  comm_failed = true;
  if (!c) return;
  // ncclCommAbort ends the communicator's kernels still waiting for a peer, but its teardown can
  // itself wait on a peer that is gone. It runs on a helper thread; the caller waits a bounded
  // time and returns its error either way.
  auto done = std::make_shared<std::atomic<bool>>(false);
  std::thread([c, done] {
    nccl()->CommAbort(c);
    done->store(true);
  }).detach();
  const int64_t t0 = now_ms();
  while (!done->load() && now_ms() - t0 < 5000) short_pause();
  if (!done->load()) abort_pending = true;
}

ovvsStatus Resources::collective(ncclResult_t ret) {
  if (comm_failed) return OVVS_STATUS_ERROR;
  const NcclApi* nc = nccl();
  auto async_error = [&](ncclResult_t* st) {
    return comm ? nc->CommGetAsyncError(comm, st) : ncclInvalidUsage;
  };
  const WatchResult w = settle_nccl(ret, async_error, now_ms, short_pause, nccl_timeout_ms);
  if (w.abort) abort_comm();
  return w.status;
}

void probe_device(Resources& r, int device) {
  r.device = device;
  r.gpu_available = false;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    (void)cudaGetLastError();
    return;
  }
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
    (void)cudaGetLastError();
    return;
  }
  r.device_name = prop.name;
  r.num_sms = prop.multiProcessorCount;
  r.max_smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
  // The kernels are built for sm_100a only (tcgen05 / TMEM / TMA).
  r.gpu_available = prop.major == 10 && prop.minor == 0;
}

Resources::~Resources() {
  // Group members first, each from its own worker thread (their communicators are torn down
  // together), then the workers.
  if (workers) {
    workers->run([&](int g) {
      group[static_cast<size_t>(g)].reset();
      return OVVS_STATUS_SUCCESS;
    });
    workers.reset();
  }
  group.clear();
  if (abort_pending) {
    // A collective of the aborted communicator may still run: freeing could wait on it.
    for (auto& b : ws) b.abandon();
    bound_win.abandon();
    d_err = nullptr;
    stage_buf[0] = stage_buf[1] = nullptr;
  }
  if (gpu_available) cudaSetDevice(device);
  // The peer window is unmapped only once this rank's kernels are done with it.
  if (bound_win.ready() && stream) cudaStreamSynchronize(stream);
  bound_win.reset();
  for (auto& b : ws) b.release();
  if (comm) ovvs::rt::nccl()->CommDestroy(comm);
  if (d_err) cudaFree(d_err);
  for (auto& e : phase_ev)
    if (e) cudaEventDestroy(e);
  for (auto& row : hist_ev)
    for (auto& e : row)
      if (e) cudaEventDestroy(e);
  for (int b = 0; b < 2; ++b) {
    if (stage_ev[b]) {
      cudaEventSynchronize(stage_ev[b]);
      cudaEventDestroy(stage_ev[b]);
    }
    if (stage_buf[b]) cudaFreeHost(stage_buf[b]);
  }
  if (stream) cudaStreamDestroy(stream);
}

void Resources::mark(int i) {
  if (!profiling || mark_hold) return;
  if (!phase_ev[i] && cudaEventCreate(&phase_ev[i]) != cudaSuccess) {
    (void)cudaGetLastError();
    return;
  }
  cudaEventRecord(phase_ev[i], stream);
  phase_valid = true;
  cudaEvent_t& h = hist_ev[hist_next][i];
  if (!h && cudaEventCreate(&h) != cudaSuccess) {
    (void)cudaGetLastError();
    return;
  }
  cudaEventRecord(h, stream);
  if (i == kPhases) {
    hist_next = (hist_next + 1) % kPhaseHistory;
    if (hist_count < kPhaseHistory) ++hist_count;
  }
}

ovvsStatus Resources::check_policy() const {
  if (policy == OVVS_POLICY_FORCE_CPU || policy == OVVS_POLICY_FORCE_NPU) {
    return OVVS_STATUS_DEVICE_UNAVAILABLE;
  }
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus Resources::activate() {
  if (!gpu_available) return OVVS_STATUS_DEVICE_UNAVAILABLE;
  OVVS_TRY_CUDA(cudaSetDevice(device));
  if (!stream) OVVS_TRY_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  if (!d_err) {
    OVVS_TRY_CUDA(cudaMalloc(&d_err, sizeof(int)));
    OVVS_TRY_CUDA(cudaMemset(d_err, 0, sizeof(int)));
  }
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus Resources::finish() {
  if (comm || comm_failed) {
    auto stream_state = [&] {
      const cudaError_t e = cudaStreamQuery(stream);
      if (e == cudaSuccess) return StreamState::kIdle;
      if (e == cudaErrorNotReady) return StreamState::kBusy;
      return StreamState::kFailed;
    };
    auto async_error = [&](ncclResult_t* st) {
      if (!comm) {
        *st = ncclSuccess;  // already aborted: only the stream is left to drain
        return ncclSuccess;
      }
      return nccl()->CommGetAsyncError(comm, st);
    };
    const WatchResult w = watch_stream(stream_state, async_error, now_ms, short_pause,
                                       nccl_timeout_ms);
    if (w.abort) {
      abort_comm();
      // the abort ends the collectives still waiting for a peer; what remains drains quickly
      if (!abort_pending) {
        const WatchResult d = watch_stream(stream_state, async_error, now_ms, short_pause, 10000);
        (void)d;
      }
      (void)cudaGetLastError();
      return OVVS_STATUS_ERROR;
    }
    if (w.status != OVVS_STATUS_SUCCESS) return status_of(cudaStreamSynchronize(stream));
  }
  OVVS_TRY_CUDA(cudaStreamSynchronize(stream));
  int err = 0;
  OVVS_TRY_CUDA(cudaMemcpy(&err, d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (err != 0) {
    last_kernel_error = err;
    cudaMemset(d_err, 0, sizeof(int));
    return OVVS_STATUS_ERROR;
  }
  return OVVS_STATUS_SUCCESS;
}

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      (void)cudaGetLastError();
      return static_cast<EncodeTiledFn>(nullptr);
    }
    return reinterpret_cast<EncodeTiledFn>(p);
  }();
  return fn;
}

}  // namespace

bool encode_f16_2d(CUtensorMap* map, const void* base, uint64_t cols, uint64_t rows,
                   uint32_t box_cols, uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  const uint32_t row_bytes = box_cols * 2;
  const CUtensorMapSwizzle sw = row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                : row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                  : CU_TENSOR_MAP_SWIZZLE_32B;
  std::memset(map, 0, sizeof(*map));
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            elem, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

ovvsStatus allreduce_i64_sum(Resources& r, int64_t* value) {
  if (r.world <= 1) return OVVS_STATUS_SUCCESS;
  OVVS_TRY(r.comm_ready());
  int64_t* d = nullptr;
  OVVS_TRY(r.scratch<int64_t>(kWsFlags, 1, &d));
  OVVS_TRY_CUDA(cudaMemcpyAsync(d, value, sizeof(int64_t), cudaMemcpyHostToDevice, r.stream));
  OVVS_TRY(r.collective(ovvs::rt::nccl()->AllReduce(d, d, 1, ncclInt64, ncclSum, r.comm, r.stream)));
  OVVS_TRY(r.finish());  // bounded wait before the (blocking) copy into host memory
  OVVS_TRY_CUDA(cudaMemcpy(value, d, sizeof(int64_t), cudaMemcpyDeviceToHost));
  return OVVS_STATUS_SUCCESS;
}

namespace {

constexpr size_t kStageMin = size_t(16) << 20;    // smaller copies go direct
constexpr size_t kStageChunk = size_t(32) << 20;  // bytes per staging buffer

// memcpy split over `threads` host threads.
void parallel_copy(void* dst, const void* src, size_t bytes, unsigned threads) {
  if (threads <= 1 || bytes < (size_t(1) << 20)) {
    std::memcpy(dst, src, bytes);
    return;
  }
  std::vector<std::thread> pool;
  const size_t part = (bytes + threads - 1) / threads;
  for (unsigned t = 0; t < threads; ++t) {
    const size_t lo = t * part;
    if (lo >= bytes) break;
    const size_t len = std::min(part, bytes - lo);
    pool.emplace_back([=] {
      std::memcpy(static_cast<char*>(dst) + lo, static_cast<const char*>(src) + lo, len);
    });
  }
  for (auto& th : pool) th.join();
}

}  // namespace

ovvsStatus upload(Resources& r, void* dst, const void* src, size_t bytes) {
  if (bytes == 0) return OVVS_STATUS_SUCCESS;
  bool direct = bytes < kStageMin;
  if (!direct) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, src) == cudaSuccess && a.type == cudaMemoryTypeHost)
      direct = true;  // already pinned (or registered): the DMA reads it directly
    (void)cudaGetLastError();
  }
  if (!direct) {
    for (int b = 0; b < 2 && !direct; ++b) {
      if (!r.stage_buf[b] && cudaMallocHost(&r.stage_buf[b], kStageChunk) != cudaSuccess) {
        r.stage_buf[b] = nullptr;
        direct = true;  // no pinned memory to spare: the driver's pageable path
      }
      if (!direct && !r.stage_ev[b] &&
          cudaEventCreateWithFlags(&r.stage_ev[b], cudaEventDisableTiming) != cudaSuccess) {
        r.stage_ev[b] = nullptr;
        direct = true;
      }
    }
    (void)cudaGetLastError();
  }
  if (direct) {
    OVVS_TRY_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, r.stream));
    return OVVS_STATUS_SUCCESS;
  }
  const unsigned threads = std::max(1u, std::min(8u, std::thread::hardware_concurrency() / 2));
  size_t off = 0;
  for (int i = 0; off < bytes; ++i) {
    const int b = i & 1;
    const size_t len = std::min(kStageChunk, bytes - off);
    // the DMA that last read this buffer has finished before it is refilled
    if (r.stage_used[b]) OVVS_TRY_CUDA(cudaEventSynchronize(r.stage_ev[b]));
    parallel_copy(r.stage_buf[b], static_cast<const char*>(src) + off, len, threads);
    OVVS_TRY_CUDA(cudaMemcpyAsync(static_cast<char*>(dst) + off, r.stage_buf[b], len,
                                  cudaMemcpyHostToDevice, r.stream));
    OVVS_TRY_CUDA(cudaEventRecord(r.stage_ev[b], r.stream));
    r.stage_used[b] = true;
    off += len;
  }
  return OVVS_STATUS_SUCCESS;
}

}  // namespace rt
}  // namespace ovvs
