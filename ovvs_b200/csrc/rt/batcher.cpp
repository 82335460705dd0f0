// Dynamic batcher over a brute-force index: the ovvsBatcher* entry points.
//
// Observable rules kept from the reference (src/rt/batcher.cpp:82-113): concurrent
// ovvsBatcherSearch calls coalesce into one ovvsBruteForceSearch; a batch is searched as soon as it
// holds max_batch queries, when a caller with a different k arrives (the open batch goes first),
// or when a member has waited max_wait_ms (0: no wait). Every member gets its own rows and the
// batch search's status; ovvsBatcherLastBatchSize reports the size of the last batch searched.
//
// Design: each coalescing window is a Batch generation shared by its members. The caller that
// closes a window (by filling it, by changing k, or by timing out) leads it: it takes the batch
// out of the batcher, runs the search WITHOUT holding the batcher's lock, scatters the rows to the
// members' buffers and wakes them. Callers arriving meanwhile open the next window, so the host
// keeps gathering the next batch while the GPU searches the current one. On this library the
// batch search is one fused GPU launch, which turns nq = 1 traffic into tensor-core-sized work.
#include <algorithm>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <memory>
#include <mutex>
#include <new>
#include <vector>

#include "../neighbors/brute_force.hpp"
#include "ovvs/ovvs.h"

namespace {

// One member's place in a batch: its first row and its caller-owned outputs.
struct Member {
  int64_t first_row;
  int64_t rows;
  int64_t* neighbors;
  float* distances;
};

// One coalescing window.
struct Batch {
  explicit Batch(int64_t k_) : k(k_) {}
  const int64_t k;
  std::vector<float> rows;  // queries of every member, in arrival order
  std::vector<Member> members;
  int64_t nq = 0;
  bool closed = false;  // taken by its leader: no more members
  bool done = false;    // searched and scattered
  ovvsStatus status = OVVS_STATUS_SUCCESS;
};

class Batcher {
 public:
  Batcher(ovvsResources_t res, ovvsBruteForceIndex_t index, int32_t max_batch, int32_t wait_ms,
          int64_t dim)
      : res_(res), index_(index), max_batch_(max_batch), wait_(wait_ms), dim_(dim) {}

  ovvsStatus search(const float* queries, int64_t nq, int64_t k, int64_t* neighbors,
                    float* distances) {
    std::unique_lock<std::mutex> lock(mu_);
    if (dead_) return OVVS_STATUS_ERROR;
    // Counts this caller as inside until it returns (the lock is held again by then).
    struct Inside {
      Batcher* b;
      ~Inside() {
        if (--b->inside_ == 0) b->cv_.notify_all();
      }
    } inside{this};
    ++inside_;
    // A different k cannot share the open window: it is searched first, by this caller.
    while (open_ && open_->k != k) {
      lead(lock, take_open());
      if (dead_) return OVVS_STATUS_ERROR;
    }
    if (!open_) open_ = std::make_shared<Batch>(k);
    std::shared_ptr<Batch> mine = open_;
    mine->rows.insert(mine->rows.end(), queries, queries + nq * dim_);
    mine->members.push_back(Member{mine->nq, nq, neighbors, distances});
    mine->nq += nq;
    if (mine->nq >= max_batch_) {
      lead(lock, take_open());
    } else {
      // Wait for another member to close the window; past the deadline, close it here.
      const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(wait_);
      while (!mine->closed && !dead_ &&
             cv_.wait_until(lock, deadline) != std::cv_status::timeout) {
      }
      if (!mine->closed && !dead_) lead(lock, take_open());
    }
    // A closed window always completes (its leader writes into this caller's buffers), so a
    // member returns only after that; a window still open when the batcher shuts down is dropped.
    cv_.wait(lock, [&] { return mine->done || (dead_ && !mine->closed); });
    return mine->done ? mine->status : OVVS_STATUS_ERROR;
  }

  int32_t last_batch_size() {
    std::lock_guard<std::mutex> lock(mu_);
    return last_nq_;
  }

  // Fails pending members with ERROR and returns once no caller is inside any more.
  void shut_down() {
    std::unique_lock<std::mutex> lock(mu_);
    dead_ = true;
    cv_.notify_all();
    cv_.wait(lock, [&] { return inside_ == 0; });
  }

 private:
  std::shared_ptr<Batch> take_open() {
    std::shared_ptr<Batch> b = std::move(open_);
    b->closed = true;
    cv_.notify_all();
    return b;
  }

  // Runs batch `b` (already taken out of the batcher) with the lock released, then publishes it.
  void lead(std::unique_lock<std::mutex>& lock, std::shared_ptr<Batch> b) {
    lock.unlock();
    ovvsStatus st = OVVS_STATUS_SUCCESS;
    try {
      // Result buffers of nq x k filled like a caller's (the reference's batch buffers: -1 / 0);
      // the search writes rows of stride min(k, n) into them, and each member receives its rows
      // at stride k.
      std::vector<int64_t> nb(static_cast<size_t>(b->nq * b->k), -1);
      std::vector<float> ds(static_cast<size_t>(b->nq * b->k), 0.f);
      st = ovvsBruteForceSearch(res_, index_, b->rows.data(), b->nq, b->k, nullptr, nb.data(),
                                ds.data());
      for (const Member& m : b->members) {
        const size_t off = static_cast<size_t>(m.first_row * b->k);
        const size_t cnt = static_cast<size_t>(m.rows * b->k);
        std::memcpy(m.neighbors, nb.data() + off, cnt * sizeof(int64_t));
        std::memcpy(m.distances, ds.data() + off, cnt * sizeof(float));
      }
    } catch (const std::bad_alloc&) {
      st = OVVS_STATUS_OOM;
    }
    lock.lock();
    b->status = st;
    b->done = true;
    last_nq_ = static_cast<int32_t>(b->nq);
    cv_.notify_all();
  }

  const ovvsResources_t res_;
  const ovvsBruteForceIndex_t index_;
  const int64_t max_batch_;
  const int32_t wait_;
  const int64_t dim_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::shared_ptr<Batch> open_;
  int32_t last_nq_ = 0;
  int inside_ = 0;
  bool dead_ = false;
};

Batcher* as_batcher(ovvsBatcher_t b) { return reinterpret_cast<Batcher*>(b); }

}  // namespace

extern "C" {

ovvsStatus ovvsBatcherCreate(ovvsResources_t res, ovvsBruteForceIndex_t index, int32_t max_batch,
                             int32_t max_wait_ms, ovvsBatcher_t* out) {
  if (!res || !index || !out || max_batch <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  const int64_t dim = reinterpret_cast<ovvs::nb::BruteIndex*>(index)->dim;
  if (dim <= 0) return OVVS_STATUS_INVALID_ARGUMENT;
  auto* b = new (std::nothrow) Batcher(res, index, max_batch, std::max(0, max_wait_ms), dim);
  if (!b) return OVVS_STATUS_OOM;
  *out = reinterpret_cast<ovvsBatcher_t>(b);
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsBatcherSearch(ovvsBatcher_t batcher, const float* queries, int64_t nq, int64_t k,
                             int64_t* neighbors, float* distances) {
  if (!batcher || !queries || !neighbors || !distances || nq <= 0 || k <= 0)
    return OVVS_STATUS_INVALID_ARGUMENT;
  try {
    return as_batcher(batcher)->search(queries, nq, k, neighbors, distances);
  } catch (const std::bad_alloc&) {
    return OVVS_STATUS_OOM;
  } catch (...) {
    return OVVS_STATUS_ERROR;
  }
}

ovvsStatus ovvsBatcherLastBatchSize(ovvsBatcher_t batcher, int32_t* nq) {
  if (!batcher || !nq) return OVVS_STATUS_INVALID_ARGUMENT;
  *nq = as_batcher(batcher)->last_batch_size();
  return OVVS_STATUS_SUCCESS;
}

ovvsStatus ovvsBatcherDestroy(ovvsBatcher_t batcher) {
  Batcher* b = as_batcher(batcher);
  if (!b) return OVVS_STATUS_SUCCESS;
  b->shut_down();
  delete b;
  return OVVS_STATUS_SUCCESS;
}

}  // extern "C"
