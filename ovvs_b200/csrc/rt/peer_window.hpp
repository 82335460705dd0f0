// Device memory that every rank of a sharded Resources maps from every other rank (one process
// per GPU, or one worker thread per GPU in one process).
//
// Each rank allocates its buffer with the CUDA virtual memory API as an exportable allocation,
// hands a POSIX file descriptor of it to every peer (fd_exchange.hpp) and maps every peer's
// allocation into its own address space with access from its own device (over NVLink). A
// mapping holds its own reference to the peer's physical memory, so the pages stay valid even
// if that peer exits: a write into a departed peer's buffer lands in memory nobody reads, never
// in freed memory.
//
// Used for the per-query bound of sharded searches: each rank's fused kernel publishes its
// k-th best key into every rank's bound buffer (a remote atomic min), so every rank filters
// with the best bound found anywhere.
#pragma once

#include <cstddef>
#include <cstdint>
#include <vector>

#include "ovvs/ovvs.h"

namespace ovvs {
namespace rt {

struct Resources;

class PeerWindow {
 public:
  PeerWindow() = default;
  PeerWindow(const PeerWindow&) = delete;
  PeerWindow& operator=(const PeerWindow&) = delete;
  ~PeerWindow() { reset(); }

  // Collective over r's ranks (every rank calls it with the same `bytes`, in the same order
  // relative to its other windows): allocates this rank's buffer of at least `bytes` and maps
  // every peer's. `tag` identifies the exchange on the host (derived from the communicator's
  // unique id and a per-Resources sequence number); `timeout_ms` bounds the descriptor exchange.
  // Returns SUCCESS; UNSUPPORTED (on every rank alike, nothing left allocated) when some rank
  // cannot allocate, export, exchange or map; or the error of the communicator's all-reduce
  // when a rank is gone.
  ovvsStatus create(Resources& r, size_t bytes, uint64_t tag, int64_t timeout_ms);
  void reset();
  // Forgets the mappings without unmapping them (they go with the process): for a Resources
  // whose communicator abort did not finish, where a kernel may still write through them.
  void abandon() {
    maps_.clear();
    ptr_.clear();
    bytes_ = 0;
  }

  bool ready() const { return !ptr_.empty(); }
  size_t bytes() const { return bytes_; }
  // Rank p's buffer as mapped in this process (p = own rank: this rank's buffer).
  void* ptr(int p) const { return ptr_[static_cast<size_t>(p)]; }
  int world() const { return static_cast<int>(ptr_.size()); }

 private:
  struct Map {
    unsigned long long handle = 0;  // CUmemGenericAllocationHandle
    uintptr_t va = 0;
    bool mapped = false;
  };
  static bool map_handle(unsigned long long handle, size_t size, size_t align, int device,
                         Map& m);
  std::vector<Map> maps_;
  std::vector<void*> ptr_;
  size_t bytes_ = 0;
  int device_ = -1;
};

}  // namespace rt
}  // namespace ovvs
