// Symmetric heap: cuMem allocations shared between the ranks' processes through
// POSIX file descriptors passed over Unix sockets, peer mappings in one virtual
// range, and an NVLS multicast object over every rank's allocation (symm.h).
//
// The driver API is reached through the runtime's driver entry points, so the
// extension needs no link against libcuda.
#include "symm.h"

#include <cuda_runtime.h>
#include <errno.h>
#include <poll.h>
#include <string.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <stdexcept>
#include <thread>

namespace es {
namespace {

// ------------------------------------------------------------------ driver entry points

template <typename Fn>
Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess ||
      p == nullptr)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

struct Driver {
  decltype(&cuDeviceGet) DeviceGet = nullptr;
  decltype(&cuDeviceGetAttribute) DeviceGetAttribute = nullptr;
  decltype(&cuMemCreate) MemCreate = nullptr;
  decltype(&cuMemRelease) MemRelease = nullptr;
  decltype(&cuMemExportToShareableHandle) MemExport = nullptr;
  decltype(&cuMemImportFromShareableHandle) MemImport = nullptr;
  decltype(&cuMemAddressReserve) AddressReserve = nullptr;
  decltype(&cuMemAddressFree) AddressFree = nullptr;
  decltype(&cuMemMap) MemMap = nullptr;
  decltype(&cuMemUnmap) MemUnmap = nullptr;
  decltype(&cuMemSetAccess) MemSetAccess = nullptr;
  decltype(&cuMemGetAllocationGranularity) MemGranularity = nullptr;
  decltype(&cuMulticastCreate) McCreate = nullptr;
  decltype(&cuMulticastAddDevice) McAddDevice = nullptr;
  decltype(&cuMulticastBindMem) McBindMem = nullptr;
  decltype(&cuMulticastUnbind) McUnbind = nullptr;
  decltype(&cuMulticastGetGranularity) McGranularity = nullptr;
  decltype(&cuGetErrorString) GetErrorString = nullptr;
  bool ok = false;
};

const Driver& drv() {
  static Driver d = [] {
    Driver x;
    x.DeviceGet = driver_fn<decltype(&cuDeviceGet)>("cuDeviceGet");
    x.DeviceGetAttribute = driver_fn<decltype(&cuDeviceGetAttribute)>("cuDeviceGetAttribute");
    x.MemCreate = driver_fn<decltype(&cuMemCreate)>("cuMemCreate");
    x.MemRelease = driver_fn<decltype(&cuMemRelease)>("cuMemRelease");
    x.MemExport = driver_fn<decltype(&cuMemExportToShareableHandle)>("cuMemExportToShareableHandle");
    x.MemImport = driver_fn<decltype(&cuMemImportFromShareableHandle)>("cuMemImportFromShareableHandle");
    x.AddressReserve = driver_fn<decltype(&cuMemAddressReserve)>("cuMemAddressReserve");
    x.AddressFree = driver_fn<decltype(&cuMemAddressFree)>("cuMemAddressFree");
    x.MemMap = driver_fn<decltype(&cuMemMap)>("cuMemMap");
    x.MemUnmap = driver_fn<decltype(&cuMemUnmap)>("cuMemUnmap");
    x.MemSetAccess = driver_fn<decltype(&cuMemSetAccess)>("cuMemSetAccess");
    x.MemGranularity = driver_fn<decltype(&cuMemGetAllocationGranularity)>("cuMemGetAllocationGranularity");
    x.McCreate = driver_fn<decltype(&cuMulticastCreate)>("cuMulticastCreate");
    x.McAddDevice = driver_fn<decltype(&cuMulticastAddDevice)>("cuMulticastAddDevice");
    x.McBindMem = driver_fn<decltype(&cuMulticastBindMem)>("cuMulticastBindMem");
    x.McUnbind = driver_fn<decltype(&cuMulticastUnbind)>("cuMulticastUnbind");
    x.McGranularity = driver_fn<decltype(&cuMulticastGetGranularity)>("cuMulticastGetGranularity");
    x.GetErrorString = driver_fn<decltype(&cuGetErrorString)>("cuGetErrorString");
    x.ok = x.DeviceGet && x.DeviceGetAttribute && x.MemCreate && x.MemRelease && x.MemExport && x.MemImport &&
           x.AddressReserve && x.AddressFree && x.MemMap && x.MemUnmap && x.MemSetAccess && x.MemGranularity;
    return x;
  }();
  return d;
}

bool mc_api() {
  const Driver& d = drv();
  return d.McCreate && d.McAddDevice && d.McBindMem && d.McUnbind && d.McGranularity;
}

std::string cu_err(const char* what, CUresult r) {
  const char* s = nullptr;
  if (drv().GetErrorString) drv().GetErrorString(r, &s);
  return std::string(what) + " failed: " + (s ? s : "CUDA driver error ") + " (" + std::to_string((int)r) + ")";
}

CUmemAllocationProp mem_prop(int device) {
  CUmemAllocationProp p;
  memset(&p, 0, sizeof(p));
  p.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  p.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  p.location.id = device;
  p.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

CUmulticastObjectProp mc_prop(int size, size_t bytes) {
  CUmulticastObjectProp p;
  memset(&p, 0, sizeof(p));
  p.numDevices = static_cast<unsigned>(size);
  p.size = bytes;
  p.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  return p;
}

// ------------------------------------------------------------------ sockets

// Abstract-namespace address "\0einshard-symm-<tag>-<rank>" (nothing on the file system).
socklen_t sock_addr(sockaddr_un* a, const std::string& tag, int rank) {
  memset(a, 0, sizeof(*a));
  a->sun_family = AF_UNIX;
  const std::string name = "einshard-symm-" + tag + "-" + std::to_string(rank);
  const size_t n = name.size() < sizeof(a->sun_path) - 1 ? name.size() : sizeof(a->sun_path) - 1;
  memcpy(a->sun_path + 1, name.data(), n);
  return static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + n);
}

// Send up to two descriptors (the memory, and the multicast object from rank 0;
// -1 = absent) in one message with a 4-byte payload holding how many were sent.
bool send_fds(int sock, int fd0, int fd1) {
  int fds[2] = {fd0, fd1};
  int n = fd1 >= 0 ? 2 : 1;
  char ctrl[CMSG_SPACE(sizeof(int) * 2)];
  memset(ctrl, 0, sizeof(ctrl));
  iovec iov;
  iov.iov_base = &n;
  iov.iov_len = sizeof(n);
  msghdr msg;
  memset(&msg, 0, sizeof(msg));
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = ctrl;
  msg.msg_controllen = CMSG_SPACE(sizeof(int) * n);
  cmsghdr* c = CMSG_FIRSTHDR(&msg);
  c->cmsg_level = SOL_SOCKET;
  c->cmsg_type = SCM_RIGHTS;
  c->cmsg_len = CMSG_LEN(sizeof(int) * n);
  memcpy(CMSG_DATA(c), fds, sizeof(int) * n);
  return sendmsg(sock, &msg, 0) == static_cast<ssize_t>(sizeof(n));
}

bool recv_fds(int sock, int* fd0, int* fd1) {
  int n = 0;
  char ctrl[CMSG_SPACE(sizeof(int) * 2)];
  iovec iov;
  iov.iov_base = &n;
  iov.iov_len = sizeof(n);
  msghdr msg;
  memset(&msg, 0, sizeof(msg));
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = ctrl;
  msg.msg_controllen = sizeof(ctrl);
  if (recvmsg(sock, &msg, 0) != static_cast<ssize_t>(sizeof(n))) return false;
  cmsghdr* c = CMSG_FIRSTHDR(&msg);
  if (!c || c->cmsg_level != SOL_SOCKET || c->cmsg_type != SCM_RIGHTS) return false;
  int fds[2] = {-1, -1};
  const size_t got = (c->cmsg_len - CMSG_LEN(0)) / sizeof(int);
  memcpy(fds, CMSG_DATA(c), sizeof(int) * (got < 2 ? got : 2));
  *fd0 = fds[0];
  *fd1 = got > 1 ? fds[1] : -1;
  return got >= 1;
}

}  // namespace

bool symm_multicast_supported(int device) {
  const Driver& d = drv();
  if (!d.ok || !mc_api()) return false;
  CUdevice dev;
  if (d.DeviceGet(&dev, device) != CUDA_SUCCESS) return false;
  int v = 0;
  if (d.DeviceGetAttribute(&v, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev) != CUDA_SUCCESS) return false;
  int fd_ok = 0;
  d.DeviceGetAttribute(&fd_ok, CU_DEVICE_ATTRIBUTE_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR_SUPPORTED, dev);
  return v != 0 && fd_ok != 0;
}

size_t symm_granularity(int device, int size, bool want_mc) {
  const Driver& d = drv();
  if (!d.ok) return 0;
  CUmemAllocationProp p = mem_prop(device);
  size_t g = 0;
  if (d.MemGranularity(&g, &p, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS || g == 0) return 0;
  if (want_mc && mc_api()) {
    CUmulticastObjectProp mp = mc_prop(size, g);
    size_t mg = 0;
    if (d.McGranularity(&mg, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED) == CUDA_SUCCESS && mg > g) g = mg;
  }
  return g;
}

std::string symm_prepare(SymmHeap& h, size_t bytes, int device, const std::string& tag, int rank, int size,
                         bool want_mc) {
  const Driver& d = drv();
  if (!d.ok) return "the CUDA virtual memory API is unavailable";
  h.rank = rank;
  h.size = size;
  h.device = device;
  h.tag = tag;
  h.want_mc = want_mc && mc_api();
  const size_t g = symm_granularity(device, size, h.want_mc);
  if (g == 0) return "cuMemGetAllocationGranularity failed";
  h.granularity = g;
  h.bytes = (bytes + g - 1) / g * g;
  CUmemAllocationProp p = mem_prop(device);
  CUresult r = d.MemCreate(&h.local, h.bytes, &p, 0);
  if (r != CUDA_SUCCESS) {
    h.local = 0;
    return cu_err("cuMemCreate", r);
  }
  r = d.MemExport(&h.local_fd, h.local, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (r != CUDA_SUCCESS) return cu_err("cuMemExportToShareableHandle", r);
  if (h.want_mc && rank == 0) {
    CUmulticastObjectProp mp = mc_prop(size, h.bytes);
    r = d.McCreate(&h.mc, &mp);
    if (r != CUDA_SUCCESS) {
      h.mc = 0;
      return cu_err("cuMulticastCreate", r);
    }
    r = d.MemExport(&h.mc_fd, h.mc, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
    if (r != CUDA_SUCCESS) return cu_err("cuMemExportToShareableHandle (multicast)", r);
  }
  h.listen_fd = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (h.listen_fd < 0) return std::string("socket: ") + strerror(errno);
  sockaddr_un a;
  const socklen_t len = sock_addr(&a, tag, rank);
  if (bind(h.listen_fd, reinterpret_cast<sockaddr*>(&a), len) != 0) return std::string("bind: ") + strerror(errno);
  if (listen(h.listen_fd, size) != 0) return std::string("listen: ") + strerror(errno);
  return "";
}

std::string symm_exchange(SymmHeap& h, double timeout_s) {
  const Driver& d = drv();
  const int peers = h.size - 1;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
  // serve: every peer connects once and receives our descriptors
  std::string serve_err;
  std::thread server([&] {
    for (int i = 0; i < peers; ++i) {
      pollfd pf{h.listen_fd, POLLIN, 0};
      int ready = 0;
      while ((ready = poll(&pf, 1, 100)) == 0)
        if (std::chrono::steady_clock::now() > deadline) break;
      if (ready <= 0) {
        serve_err = "timed out waiting for peers to connect";
        return;
      }
      const int c = accept4(h.listen_fd, nullptr, nullptr, SOCK_CLOEXEC);
      if (c < 0) {
        serve_err = std::string("accept: ") + strerror(errno);
        return;
      }
      const bool ok = send_fds(c, h.local_fd, h.rank == 0 ? h.mc_fd : -1);
      close(c);
      if (!ok) {
        serve_err = std::string("sendmsg: ") + strerror(errno);
        return;
      }
    }
  });
  // fetch every peer's descriptors
  std::string err;
  h.handles.assign(h.size, 0);
  h.handles[h.rank] = h.local;
  int mc_fd_in = -1;
  for (int p = 0; p < h.size && err.empty(); ++p) {
    if (p == h.rank) continue;
    int s = -1;
    for (;;) {
      s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
      sockaddr_un a;
      const socklen_t len = sock_addr(&a, h.tag, p);
      if (s >= 0 && connect(s, reinterpret_cast<sockaddr*>(&a), len) == 0) break;
      if (s >= 0) close(s);
      s = -1;
      if (std::chrono::steady_clock::now() > deadline) break;
      std::this_thread::sleep_for(std::chrono::milliseconds(2));
    }
    if (s < 0) {
      err = "could not connect to rank " + std::to_string(p);
      break;
    }
    int fd0 = -1, fd1 = -1;
    if (!recv_fds(s, &fd0, &fd1)) err = "did not receive the descriptors of rank " + std::to_string(p);
    close(s);
    if (!err.empty()) break;
    CUresult r = d.MemImport(&h.handles[p], reinterpret_cast<void*>(static_cast<uintptr_t>(fd0)),
                             CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
    close(fd0);
    if (r != CUDA_SUCCESS) {
      h.handles[p] = 0;
      err = cu_err("cuMemImportFromShareableHandle", r);
    }
    if (p == 0 && fd1 >= 0) mc_fd_in = fd1;
  }
  server.join();
  if (err.empty()) err = serve_err;
  close(h.listen_fd);
  h.listen_fd = -1;
  if (!err.empty()) {
    if (mc_fd_in >= 0) close(mc_fd_in);
    return err;
  }
  // map every rank's allocation: rank p at uc_base + p * bytes
  CUresult r = d.AddressReserve(&h.uc_base, h.bytes * h.size, h.granularity, 0, 0);
  if (r != CUDA_SUCCESS) {
    h.uc_base = 0;
    return cu_err("cuMemAddressReserve", r);
  }
  h.mapped.assign(h.size, false);
  for (int p = 0; p < h.size; ++p) {
    r = d.MemMap(h.uc_base + p * h.bytes, h.bytes, 0, h.handles[p], 0);
    if (r != CUDA_SUCCESS) return cu_err("cuMemMap", r);
    h.mapped[p] = true;
  }
  CUmemAccessDesc acc;
  memset(&acc, 0, sizeof(acc));
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = h.device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  r = d.MemSetAccess(h.uc_base, h.bytes * h.size, &acc, 1);
  if (r != CUDA_SUCCESS) return cu_err("cuMemSetAccess", r);
  // join the multicast team
  if (h.want_mc) {
    if (h.rank != 0) {
      if (mc_fd_in < 0) return "rank 0 sent no multicast object";
      r = d.MemImport(&h.mc, reinterpret_cast<void*>(static_cast<uintptr_t>(mc_fd_in)),
                      CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
      close(mc_fd_in);
      if (r != CUDA_SUCCESS) {
        h.mc = 0;
        return cu_err("cuMemImportFromShareableHandle (multicast)", r);
      }
    }
    CUdevice dev;
    r = d.DeviceGet(&dev, h.device);
    if (r == CUDA_SUCCESS) r = d.McAddDevice(h.mc, dev);
    if (r != CUDA_SUCCESS) return cu_err("cuMulticastAddDevice", r);
    h.mc_added = true;
  } else if (mc_fd_in >= 0) {
    close(mc_fd_in);
  }
  return "";
}

std::string symm_bind(SymmHeap& h) {
  if (!h.want_mc) return "";
  CUresult r = drv().McBindMem(h.mc, 0, h.local, 0, h.bytes, 0);
  if (r != CUDA_SUCCESS) return cu_err("cuMulticastBindMem", r);
  h.mc_bound = true;
  return "";
}

std::string symm_map_mc(SymmHeap& h) {
  const Driver& d = drv();
  if (!h.want_mc) return "";
  CUresult r = d.AddressReserve(&h.mc_base, h.bytes, h.granularity, 0, 0);
  if (r != CUDA_SUCCESS) {
    h.mc_base = 0;
    return cu_err("cuMemAddressReserve (multicast)", r);
  }
  r = d.MemMap(h.mc_base, h.bytes, 0, h.mc, 0);
  if (r != CUDA_SUCCESS) return cu_err("cuMemMap (multicast)", r);
  h.mc_mapped = true;
  CUmemAccessDesc acc;
  memset(&acc, 0, sizeof(acc));
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = h.device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  r = d.MemSetAccess(h.mc_base, h.bytes, &acc, 1);
  if (r != CUDA_SUCCESS) return cu_err("cuMemSetAccess (multicast)", r);
  return "";
}

void symm_destroy(SymmHeap& h) {
  const Driver& d = drv();
  if (!d.ok) return;
  if (h.mc_mapped) d.MemUnmap(h.mc_base, h.bytes);
  if (h.mc_base) d.AddressFree(h.mc_base, h.bytes);
  if (h.mc_bound) {
    CUdevice dev;
    if (d.DeviceGet(&dev, h.device) == CUDA_SUCCESS) d.McUnbind(h.mc, dev, 0, h.bytes);
  }
  if (h.mc) d.MemRelease(h.mc);
  for (size_t p = 0; p < h.mapped.size(); ++p)
    if (h.mapped[p]) d.MemUnmap(h.uc_base + p * h.bytes, h.bytes);
  if (h.uc_base) d.AddressFree(h.uc_base, h.bytes * h.size);
  for (size_t p = 0; p < h.handles.size(); ++p)
    if (h.handles[p] && static_cast<int>(p) != h.rank) d.MemRelease(h.handles[p]);
  if (h.local) d.MemRelease(h.local);
  if (h.local_fd >= 0) close(h.local_fd);
  if (h.mc_fd >= 0) close(h.mc_fd);
  if (h.listen_fd >= 0) close(h.listen_fd);
  h = SymmHeap();
}

}  // namespace es
