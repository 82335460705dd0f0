// PeerWindow (see peer_window.hpp): CUDA virtual-memory allocations shared between ranks
// through POSIX file descriptors. The driver entry points are resolved through the runtime
// (cudaGetDriverEntryPoint), like the tensor-map encoder.
#include "peer_window.hpp"

#include <cuda.h>
#include <cuda_runtime.h>
#include <unistd.h>

#include "fd_exchange.hpp"
#include "runtime.hpp"

namespace ovvs {
namespace rt {
namespace {

struct VmmApi {
  CUresult (*granularity)(size_t*, const CUmemAllocationProp*, CUmemAllocationGranularity_flags);
  CUresult (*create)(CUmemGenericAllocationHandle*, size_t, const CUmemAllocationProp*,
                     unsigned long long);
  CUresult (*reserve)(CUdeviceptr*, size_t, size_t, CUdeviceptr, unsigned long long);
  CUresult (*map)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
  CUresult (*set_access)(CUdeviceptr, size_t, const CUmemAccessDesc*, size_t);
  CUresult (*export_handle)(void*, CUmemGenericAllocationHandle, CUmemAllocationHandleType,
                            unsigned long long);
  CUresult (*import_handle)(CUmemGenericAllocationHandle*, void*, CUmemAllocationHandleType);
  CUresult (*unmap)(CUdeviceptr, size_t);
  CUresult (*address_free)(CUdeviceptr, size_t);
  CUresult (*release)(CUmemGenericAllocationHandle);
};

template <class F>
bool resolve(const char* name, F* fn) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !p) {
    (void)cudaGetLastError();
    return false;
  }
  *fn = reinterpret_cast<F>(p);
  return true;
}

const VmmApi* vmm() {
  static const VmmApi* api = [] {
    static VmmApi a{};
    const bool ok = resolve("cuMemGetAllocationGranularity", &a.granularity) &&
                    resolve("cuMemCreate", &a.create) &&
                    resolve("cuMemAddressReserve", &a.reserve) && resolve("cuMemMap", &a.map) &&
                    resolve("cuMemSetAccess", &a.set_access) &&
                    resolve("cuMemExportToShareableHandle", &a.export_handle) &&
                    resolve("cuMemImportFromShareableHandle", &a.import_handle) &&
                    resolve("cuMemUnmap", &a.unmap) &&
                    resolve("cuMemAddressFree", &a.address_free) &&
                    resolve("cuMemRelease", &a.release);
    return ok ? &a : static_cast<const VmmApi*>(nullptr);
  }();
  return api;
}

CUmemAccessDesc device_access(int device) {
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  return acc;
}

CUmemAllocationProp alloc_prop(int device) {
  CUmemAllocationProp prop{};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return prop;
}

}  // namespace

// Reserves an address range for `handle` and maps it readable and writable from `device`.
bool PeerWindow::map_handle(unsigned long long handle, size_t size, size_t align, int device,
                            Map& m) {
  const VmmApi* a = vmm();
  m.handle = handle;
  CUdeviceptr va = 0;
  if (a->reserve(&va, size, align, 0, 0) != CUDA_SUCCESS) return false;
  m.va = va;
  if (a->map(va, size, 0, handle, 0) != CUDA_SUCCESS) return false;
  m.mapped = true;
  const CUmemAccessDesc acc = device_access(device);
  return a->set_access(va, size, &acc, 1) == CUDA_SUCCESS;
}

void PeerWindow::reset() {
  const VmmApi* a = vmm();
  if (a && !maps_.empty()) {
    if (device_ >= 0) cudaSetDevice(device_);
    for (Map& m : maps_) {
      if (m.mapped) a->unmap(m.va, bytes_);
      if (m.va) a->address_free(m.va, bytes_);
      if (m.handle) a->release(m.handle);
    }
  }
  maps_.clear();
  ptr_.clear();
  bytes_ = 0;
}

ovvsStatus PeerWindow::create(Resources& r, size_t bytes, uint64_t tag, int64_t timeout_ms) {
  reset();
  const VmmApi* a = vmm();
  device_ = r.device;
  const int world = r.world, rank = r.rank;
  // 1. Every rank says whether it can take part; all or none do.
  const CUmemAllocationProp prop = alloc_prop(r.device);
  size_t gran = 0;
  bool capable = a && a->granularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) ==
                          CUDA_SUCCESS && gran > 0;
  const size_t size = capable ? (bytes + gran - 1) / gran * gran : 0;
  maps_.assign(static_cast<size_t>(world), Map{});
  Map& own = maps_[static_cast<size_t>(rank)];
  int fd = -1;
  bytes_ = size;
  if (capable) {
    CUmemGenericAllocationHandle h = 0;
    capable = a->create(&h, size, &prop, 0) == CUDA_SUCCESS;
    if (capable) {
      capable = map_handle(h, size, gran, r.device, own) &&
                a->export_handle(&fd, h, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0) ==
                    CUDA_SUCCESS;
    }
  }
  int64_t votes = capable ? 1 : 0;
  ovvsStatus st = allreduce_i64_sum(r, &votes);
  if (st != OVVS_STATUS_SUCCESS || votes != world) {
    if (fd >= 0) close(fd);
    reset();
    return st != OVVS_STATUS_SUCCESS ? st : OVVS_STATUS_UNSUPPORTED;
  }
  // 2. Descriptors to and from every peer; each peer's allocation mapped here.
  std::vector<int> peer_fd;
  const bool exchanged = exchange_fds(tag, rank, world, fd, peer_fd, timeout_ms);
  bool ok = exchanged;
  close(fd);
  for (int p = 0; p < world; ++p) {
    if (p == rank) continue;
    Map& m = maps_[static_cast<size_t>(p)];
    const int pfd = peer_fd[static_cast<size_t>(p)];
    if (ok) {
      CUmemGenericAllocationHandle h = 0;
      ok = a->import_handle(&h, reinterpret_cast<void*>(static_cast<intptr_t>(pfd)),
                            CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR) == CUDA_SUCCESS;
      if (ok) ok = map_handle(h, size, gran, r.device, m);
    }
    if (pfd >= 0) close(pfd);
  }
  (void)cudaGetLastError();
  // 3. All ranks mapped every buffer, or none uses the window; every rank returns the same
  // status. This all-reduce completing shows every rank is alive, so a failed exchange (sockets
  // not reachable between the ranks, e.g. separate network namespaces) or mapping (no peer
  // access between the devices) means the window is unavailable here: UNSUPPORTED.
  int64_t votes2 = (ok ? 1 : 0) + (exchanged ? world + 1 : 0);
  st = allreduce_i64_sum(r, &votes2);
  if (st != OVVS_STATUS_SUCCESS) {
    reset();
    return st;
  }
  const int64_t n_exchanged = votes2 / (world + 1), n_mapped = votes2 % (world + 1);
  if (n_exchanged != world || n_mapped != world) {
    reset();
    return OVVS_STATUS_UNSUPPORTED;
  }
  ptr_.resize(static_cast<size_t>(world));
  for (int p = 0; p < world; ++p)
    ptr_[static_cast<size_t>(p)] = reinterpret_cast<void*>(maps_[static_cast<size_t>(p)].va);
  return OVVS_STATUS_SUCCESS;
}

}  // namespace rt
}  // namespace ovvs
