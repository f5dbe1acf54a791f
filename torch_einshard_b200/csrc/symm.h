// Symmetric device heap for one process group on one node (one process per GPU).
//
// Every rank creates one physical allocation with cuMemCreate (exportable as a
// POSIX file descriptor).  The descriptors are passed between the ranks' processes
// over abstract-namespace Unix sockets (SCM_RIGHTS), each rank imports its
// peers' allocations and maps all of them into one reserved virtual range:
// rank p's memory is at uc_base + p * bytes on every rank, so a peer address
// is a base plus an offset and kernels can load from and store to any rank's
// heap over NVLink.  When every device supports multicast, rank 0 also creates
// an NVLS multicast object, every rank adds its device and binds its
// allocation, and the object is mapped at mc_base: a multimem.* access at
// mc_base + off touches offset off of every rank's heap through the NVSwitch
// (ld_reduce sums in the switch, st / red are replicated to every rank).
//
// Creation is collective and split in phases so that the host side can put a
// process-group barrier between them (peers' sockets must exist before they
// are connected to; every device must be added to the multicast object before
// any rank binds memory):
//   prepare  -> barrier -> exchange -> barrier -> bind -> barrier -> map_mc -> barrier
// A phase that fails returns a message; the caller then agrees with its peers
// (all-reduce of a status) and destroys the heap on every rank.
//
// Teardown (destroy) must follow a device synchronisation and a barrier: no
// kernel on any rank may still access the heap.
#pragma once

#include <cuda.h>
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace es {

struct SymmHeap {
  int rank = 0, size = 1, device = 0;
  size_t bytes = 0;            // per rank, multiple of the granularity
  size_t granularity = 0;      // allocation granularity (a power of two): alignment of the mappings
  std::string tag;             // unique name of this heap's sockets
  bool want_mc = false;
  // this rank's allocation
  CUmemGenericAllocationHandle local = 0;
  int local_fd = -1;
  int listen_fd = -1;
  // peers
  std::vector<CUmemGenericAllocationHandle> handles;  // imported (own handle at [rank])
  std::vector<bool> mapped;
  CUdeviceptr uc_base = 0;     // size * bytes of virtual range
  // multicast
  CUmemGenericAllocationHandle mc = 0;
  int mc_fd = -1;
  bool mc_added = false, mc_bound = false;
  CUdeviceptr mc_base = 0;
  bool mc_mapped = false;
};

// Whether the current device supports multicast objects (and so NVLS).
bool symm_multicast_supported(int device);
// Allocation granularity used for a heap of `size` ranks (memory and multicast).
size_t symm_granularity(int device, int size, bool want_mc);

// Phases (each returns "" on success or an error message).
std::string symm_prepare(SymmHeap& h, size_t bytes, int device, const std::string& tag, int rank, int size,
                         bool want_mc);
std::string symm_exchange(SymmHeap& h, double timeout_s);
std::string symm_bind(SymmHeap& h);
std::string symm_map_mc(SymmHeap& h);
void symm_destroy(SymmHeap& h);

}  // namespace es
