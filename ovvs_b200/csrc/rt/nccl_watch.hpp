// Failure detection for work that includes NCCL collectives: bounded host-side polling instead
// of blocking waits, so that a rank that died or left cannot hold the others forever.
//
// The reference's policy is to fail closed (src/prim/mixer.cpp:47-50: a requested device that
// cannot run returns an error, never a silent fallback). Here every collective runs on a
// non-blocking communicator; the host
//   * settles each NCCL call that returned ncclInProgress (its enqueue is still being completed)
//     by polling ncclCommGetAsyncError, and
//   * waits for a stream holding collectives by polling the stream and the communicator's
//     asynchronous error,
// both against a deadline. An NCCL error or an expired deadline returns `abort = true`: the caller
// then aborts the communicator (which ends its kernels still waiting for a peer) and reports
// OVVS_STATUS_ERROR; the communicator is not used again.
//
// The loops are templates over their probes so that tests can drive them with fakes.
#pragma once

#include <nccl.h>

#include <cstdint>

#include "ovvs/ovvs.h"

namespace ovvs {
namespace rt {

enum class StreamState { kIdle, kBusy, kFailed };

struct WatchResult {
  ovvsStatus status;
  bool abort;  // the communicator must be aborted
};

// `first` is the NCCL call's own return value. ncclSuccess: done. ncclInProgress: poll
// async_error() until it leaves ncclInProgress, or until now_ms() passes timeout_ms. Anything else
// (or an error reported while polling, or the deadline): ERROR with abort.
template <class AsyncError, class Clock, class Pause>
WatchResult settle_nccl(ncclResult_t first, AsyncError async_error, Clock now_ms, Pause pause,
                        int64_t timeout_ms) {
  if (first == ncclSuccess) return {OVVS_STATUS_SUCCESS, false};
  if (first != ncclInProgress) return {OVVS_STATUS_ERROR, true};
  const int64_t t0 = now_ms();
  for (;;) {
    ncclResult_t st = ncclInProgress;
    if (async_error(&st) != ncclSuccess) return {OVVS_STATUS_ERROR, true};
    if (st == ncclSuccess) return {OVVS_STATUS_SUCCESS, false};
    if (st != ncclInProgress) return {OVVS_STATUS_ERROR, true};
    if (now_ms() - t0 > timeout_ms) return {OVVS_STATUS_ERROR, true};
    pause();
  }
}

// Waits until stream_state() reports the stream idle. While it is busy the communicator's
// asynchronous error is checked: an NCCL error, or a deadline of timeout_ms, gives ERROR with
// abort. A CUDA error of the stream gives ERROR without abort (the communicator is not at fault).
template <class StreamQuery, class AsyncError, class Clock, class Pause>
WatchResult watch_stream(StreamQuery stream_state, AsyncError async_error, Clock now_ms,
                         Pause pause, int64_t timeout_ms) {
  const int64_t t0 = now_ms();
  for (;;) {
    const StreamState s = stream_state();
    if (s == StreamState::kIdle) return {OVVS_STATUS_SUCCESS, false};
    if (s == StreamState::kFailed) return {OVVS_STATUS_ERROR, false};
    ncclResult_t st = ncclSuccess;
    if (async_error(&st) != ncclSuccess) return {OVVS_STATUS_ERROR, true};
    if (st != ncclSuccess && st != ncclInProgress) return {OVVS_STATUS_ERROR, true};
    if (now_ms() - t0 > timeout_ms) return {OVVS_STATUS_ERROR, true};
    pause();
  }
}

}  // namespace rt
}  // namespace ovvs
