// Symmetric heap: one cuMem VMM allocation per rank, exported as a POSIX file
// descriptor, passed to every peer over a Unix-domain socket (SCM_RIGHTS) and
// mapped into each peer's address space with cuMemMap + cuMemSetAccess. When
// the node supports it, an NVLS multicast object is bound over the same
// allocation so kernels can use multimem.ld_reduce / multimem.st.
//
// Replaces the cudaIpcGetMemHandle/cudaIpcOpenMemHandle bootstrap of
// single_node_nccl_allreduce_benchmark/cuda_p2p_allreduce_kernel.cu:49-139
// (which also moved 64-byte IPC handles over an NCCL all_gather,
// single_node_nccl_allreduce_benchmark/p2p_twoshot_allreduce.py:49-59).
#include "lz_internal.h"

#include <errno.h>
#include <poll.h>
#include <string.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <string>
#include <thread>

// ----------------------------------------------------------------------------
// errors
// ----------------------------------------------------------------------------
static thread_local std::string g_last_error;

void lz_set_error(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

extern "C" const char* lz_last_error(void) { return g_last_error.c_str(); }
extern "C" int lz_version(void) { return 1; }

// ----------------------------------------------------------------------------
// driver table
// ----------------------------------------------------------------------------
LzDriver& lz_driver() {
  static LzDriver d;
  static std::atomic<bool> once{false};
  if (!once.exchange(true)) {
    bool all = true;
#define LZ_LOAD(name)                                                                     \
  {                                                                                       \
    cudaDriverEntryPointQueryResult q;                                                    \
    void* fn = nullptr;                                                                   \
    cudaError_t e = cudaGetDriverEntryPointByVersion(#name, &fn, 12080, cudaEnableDefault, \
                                                     &q);                                 \
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess && fn) {                    \
      d.name = reinterpret_cast<decltype(d.name)>(fn);                                    \
    } else {                                                                              \
      all = false;                                                                        \
      cudaGetLastError();                                                                 \
    }                                                                                     \
  }
    LZ_DRIVER_FNS(LZ_LOAD)
#undef LZ_LOAD
    d.loaded = true;
    d.ok = all || (d.cuMemCreate != nullptr && d.cuMemMap != nullptr);
  }
  return d;
}

const char* lz_cu_errstr(CUresult r) {
  static thread_local char buf[256];
  const char* s = nullptr;
  LzDriver& d = lz_driver();
  if (d.cuGetErrorString) d.cuGetErrorString(r, &s);
  snprintf(buf, sizeof(buf), "CUresult %d (%s)", (int)r, s ? s : "?");
  return buf;
}

// ----------------------------------------------------------------------------
// Unix-domain socket fd passing (abstract namespace, per job tag).
// ----------------------------------------------------------------------------
static void sock_name(const std::string& tag, int rank, sockaddr_un* addr, socklen_t* len) {
  memset(addr, 0, sizeof(*addr));
  addr->sun_family = AF_UNIX;
  std::string name = "lzcomm." + tag + "." + std::to_string(rank);
  if (name.size() > sizeof(addr->sun_path) - 2) name.resize(sizeof(addr->sun_path) - 2);
  addr->sun_path[0] = '\0';  // abstract
  memcpy(addr->sun_path + 1, name.data(), name.size());
  *len = (socklen_t)(offsetof(sockaddr_un, sun_path) + 1 + name.size());
}

static int send_fd(int sock, int fd, char tagbyte) {
  msghdr msg;
  memset(&msg, 0, sizeof(msg));
  char data = tagbyte;
  iovec iov{&data, 1};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  char cbuf[CMSG_SPACE(sizeof(int))];
  memset(cbuf, 0, sizeof(cbuf));
  if (fd >= 0) {
    msg.msg_control = cbuf;
    msg.msg_controllen = sizeof(cbuf);
    cmsghdr* cm = CMSG_FIRSTHDR(&msg);
    cm->cmsg_level = SOL_SOCKET;
    cm->cmsg_type = SCM_RIGHTS;
    cm->cmsg_len = CMSG_LEN(sizeof(int));
    memcpy(CMSG_DATA(cm), &fd, sizeof(int));
  }
  return sendmsg(sock, &msg, 0) == 1 ? 0 : -1;
}

static int recv_fd(int sock, int* fd_out) {
  msghdr msg;
  memset(&msg, 0, sizeof(msg));
  char data = 0;
  iovec iov{&data, 1};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  char cbuf[CMSG_SPACE(sizeof(int))];
  msg.msg_control = cbuf;
  msg.msg_controllen = sizeof(cbuf);
  if (recvmsg(sock, &msg, 0) != 1) return -1;
  *fd_out = -1;
  for (cmsghdr* cm = CMSG_FIRSTHDR(&msg); cm; cm = CMSG_NXTHDR(&msg, cm)) {
    if (cm->cmsg_level == SOL_SOCKET && cm->cmsg_type == SCM_RIGHTS) {
      memcpy(fd_out, CMSG_DATA(cm), sizeof(int));
    }
  }
  return *fd_out >= 0 ? 0 : -1;
}

// Asks `peer` for one of its fds ('H' heap, 'M' multicast). Retries while the
// peer's server is not up yet, for at most `timeout_s`.
static int fetch_fd(const std::string& tag, int peer, char what, double timeout_s, int* fd) {
  sockaddr_un addr;
  socklen_t len;
  sock_name(tag, peer, &addr, &len);
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
    if (s < 0) {
      lz_set_error("socket(): %s", strerror(errno));
      return LZE_SOCKET;
    }
    if (connect(s, (sockaddr*)&addr, len) == 0) {
      int rc = -1;
      if (write(s, &what, 1) == 1) rc = recv_fd(s, fd);
      close(s);
      if (rc == 0) return LZE_OK;
      lz_set_error("fd transfer from rank %d failed", peer);
      return LZE_SOCKET;
    }
    close(s);
    double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    if (el > timeout_s) {
      lz_set_error("connect to rank %d timed out: %s", peer, strerror(errno));
      return LZE_SOCKET;
    }
    std::this_thread::sleep_for(std::chrono::milliseconds(2));
  }
}

struct LzHeap {
  int device = -1, rank = 0, world = 1;
  size_t bytes = 0, gran = 0;
  std::string tag;
  bool want_mc = false;
  CUmemGenericAllocationHandle local{};
  int local_fd = -1;
  CUmemGenericAllocationHandle peer_handle[LZ_MAX_RANKS]{};
  bool peer_mapped[LZ_MAX_RANKS]{};
  CUdeviceptr va[LZ_MAX_RANKS]{};
  // multicast
  bool mc_created = false, mc_added = false, mc_bound = false, mc_mapped = false;
  CUmemGenericAllocationHandle mc{};
  int mc_fd = -1;
  CUdeviceptr mc_va = 0;
  size_t mc_gran = 0;
  // server
  int listen_fd = -1;
  std::thread server;
  std::atomic<bool> stop{false};
};

#define CU_TRY(call)                                                        \
  do {                                                                      \
    CUresult r__ = (call);                                                  \
    if (r__ != CUDA_SUCCESS) {                                              \
      lz_set_error("%s failed: %s (%s:%d)", #call, lz_cu_errstr(r__), __FILE__, __LINE__); \
      return LZE_DRIVER;                                                    \
    }                                                                       \
  } while (0)

static CUmemAccessDesc access_desc(int device) {
  CUmemAccessDesc d;
  memset(&d, 0, sizeof(d));
  d.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  d.location.id = device;
  d.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  return d;
}

extern "C" int lz_heap_create(int device, int rank, int world, size_t bytes, int want_mc,
                              const char* tag, LzHeap** out) {
  LzDriver& d = lz_driver();
  if (!d.ok) {
    lz_set_error("CUDA driver entry points unavailable (no GPU driver?)");
    return LZE_DRIVER;
  }
  if (world < 1 || world > LZ_MAX_RANKS || rank < 0 || rank >= world) {
    lz_set_error("bad rank/world %d/%d", rank, world);
    return LZE_ARG;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    lz_set_error("cudaSetDevice(%d) failed", device);
    return LZE_CUDA;
  }
  cudaFree(0);  // make sure the primary context exists
  LzHeap* h = new LzHeap();
  h->device = device;
  h->rank = rank;
  h->world = world;
  h->tag = tag ? tag : "default";
  h->want_mc = want_mc != 0 && world > 1;

  CUmemAllocationProp prop;
  memset(&prop, 0, sizeof(prop));
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  size_t gran = 0;
  {
    CUresult r = d.cuMemGetAllocationGranularity(&gran, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
    if (r != CUDA_SUCCESS) {
      lz_set_error("cuMemGetAllocationGranularity: %s", lz_cu_errstr(r));
      delete h;
      return LZE_DRIVER;
    }
  }
  if (h->want_mc) {
    int mc_ok = 0;
    CUdevice dev;
    d.cuDeviceGet(&dev, device);
    d.cuDeviceGetAttribute(&mc_ok, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev);
    if (!mc_ok || !d.cuMulticastCreate) {
      h->want_mc = false;
    } else {
      CUmulticastObjectProp mp;
      memset(&mp, 0, sizeof(mp));
      mp.numDevices = (unsigned)world;
      mp.size = bytes;
      mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
      size_t mg = 0;
      if (d.cuMulticastGetGranularity(&mg, &mp, CU_MULTICAST_GRANULARITY_MINIMUM) == CUDA_SUCCESS &&
          mg > 0) {
        h->mc_gran = mg;
        if (mg > gran) gran = mg;
      } else {
        h->want_mc = false;
      }
    }
  }
  h->gran = gran;
  h->bytes = (bytes + gran - 1) / gran * gran;

  CUresult r = d.cuMemCreate(&h->local, h->bytes, &prop, 0);
  if (r != CUDA_SUCCESS) {
    lz_set_error("cuMemCreate(%zu bytes) failed: %s", h->bytes, lz_cu_errstr(r));
    delete h;
    return LZE_DRIVER;
  }
  r = d.cuMemExportToShareableHandle(&h->local_fd, h->local,
                                     CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
  if (r != CUDA_SUCCESS) {
    lz_set_error("cuMemExportToShareableHandle failed: %s", lz_cu_errstr(r));
    d.cuMemRelease(h->local);
    delete h;
    return LZE_DRIVER;
  }
  CUmemAccessDesc ad = access_desc(device);
  if (d.cuMemAddressReserve(&h->va[rank], h->bytes, gran, 0, 0) != CUDA_SUCCESS ||
      d.cuMemMap(h->va[rank], h->bytes, 0, h->local, 0) != CUDA_SUCCESS ||
      d.cuMemSetAccess(h->va[rank], h->bytes, &ad, 1) != CUDA_SUCCESS) {
    lz_set_error("mapping the local heap failed");
    close(h->local_fd);
    d.cuMemRelease(h->local);
    delete h;
    return LZE_DRIVER;
  }
  h->peer_mapped[rank] = true;
  if (cudaMemset((void*)h->va[rank], 0, h->bytes) != cudaSuccess) {
    lz_set_error("cudaMemset of heap failed");
    return LZE_CUDA;
  }
  cudaDeviceSynchronize();
  *out = h;
  return LZE_OK;
}

extern "C" int lz_heap_serve(LzHeap* h) {
  if (h->world == 1) return LZE_OK;
  int s = socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
  if (s < 0) {
    lz_set_error("socket(): %s", strerror(errno));
    return LZE_SOCKET;
  }
  sockaddr_un addr;
  socklen_t len;
  sock_name(h->tag, h->rank, &addr, &len);
  if (bind(s, (sockaddr*)&addr, len) != 0 || listen(s, 64) != 0) {
    lz_set_error("bind/listen of fd server failed: %s", strerror(errno));
    close(s);
    return LZE_SOCKET;
  }
  h->listen_fd = s;
  h->stop = false;
  h->server = std::thread([h]() {
    while (!h->stop.load()) {
      pollfd p{h->listen_fd, POLLIN, 0};
      int pr = poll(&p, 1, 20);
      if (pr <= 0) continue;
      int c = accept(h->listen_fd, nullptr, nullptr);
      if (c < 0) continue;
      // serve GPU-memory handles only to processes of this user (the job's
      // other ranks); anyone else who finds the abstract socket name is refused
      ucred cred{};
      socklen_t cl = sizeof(cred);
      if (getsockopt(c, SOL_SOCKET, SO_PEERCRED, &cred, &cl) != 0 || cred.uid != getuid()) {
        close(c);
        continue;
      }
      char what = 0;
      if (read(c, &what, 1) == 1) {
        int fd = (what == 'M') ? h->mc_fd : h->local_fd;
        send_fd(c, fd, what);
      }
      close(c);
    }
  });
  return LZE_OK;
}

extern "C" int lz_heap_stop_serving(LzHeap* h) {
  if (h->listen_fd >= 0) {
    h->stop = true;
    if (h->server.joinable()) h->server.join();
    close(h->listen_fd);
    h->listen_fd = -1;
  }
  return LZE_OK;
}

extern "C" int lz_heap_connect(LzHeap* h) {
  LzDriver& d = lz_driver();
  cudaSetDevice(h->device);
  CUmemAccessDesc ad = access_desc(h->device);
  for (int i = 1; i < h->world; ++i) {
    int p = (h->rank + i) % h->world;
    int fd = -1;
    int rc = fetch_fd(h->tag, p, 'H', 120.0, &fd);
    if (rc) return rc;
    CUresult r = d.cuMemImportFromShareableHandle(&h->peer_handle[p], (void*)(uintptr_t)fd,
                                                  CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
    close(fd);
    if (r != CUDA_SUCCESS) {
      lz_set_error("import of rank %d heap failed: %s", p, lz_cu_errstr(r));
      return LZE_DRIVER;
    }
    CU_TRY(d.cuMemAddressReserve(&h->va[p], h->bytes, h->gran, 0, 0));
    CU_TRY(d.cuMemMap(h->va[p], h->bytes, 0, h->peer_handle[p], 0));
    CU_TRY(d.cuMemSetAccess(h->va[p], h->bytes, &ad, 1));
    h->peer_mapped[p] = true;
  }
  return LZE_OK;
}

extern "C" int lz_mc_create(LzHeap* h) {
  if (!h->want_mc) return LZE_OK;
  LzDriver& d = lz_driver();
  if (h->rank != 0) return LZE_OK;
  CUmulticastObjectProp mp;
  memset(&mp, 0, sizeof(mp));
  mp.numDevices = (unsigned)h->world;
  mp.size = h->bytes;
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  CU_TRY(d.cuMulticastCreate(&h->mc, &mp));
  h->mc_created = true;
  CU_TRY(d.cuMemExportToShareableHandle(&h->mc_fd, h->mc, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR,
                                        0));
  return LZE_OK;
}

extern "C" int lz_mc_attach(LzHeap* h) {
  if (!h->want_mc) return LZE_OK;
  LzDriver& d = lz_driver();
  if (h->rank != 0) {
    int fd = -1;
    int rc = fetch_fd(h->tag, 0, 'M', 120.0, &fd);
    if (rc) return rc;
    CUresult r = d.cuMemImportFromShareableHandle(&h->mc, (void*)(uintptr_t)fd,
                                                  CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
    close(fd);
    if (r != CUDA_SUCCESS) {
      lz_set_error("multicast import failed: %s", lz_cu_errstr(r));
      return LZE_DRIVER;
    }
    h->mc_created = true;
  }
  CUdevice dev;
  CU_TRY(d.cuDeviceGet(&dev, h->device));
  CU_TRY(d.cuMulticastAddDevice(h->mc, dev));
  h->mc_added = true;
  return LZE_OK;
}

extern "C" int lz_mc_bind(LzHeap* h) {
  if (!h->want_mc) return LZE_OK;
  LzDriver& d = lz_driver();
  CU_TRY(d.cuMulticastBindMem(h->mc, 0, h->local, 0, h->bytes, 0));
  h->mc_bound = true;
  return LZE_OK;
}

extern "C" int lz_mc_map(LzHeap* h) {
  if (!h->want_mc) return LZE_OK;
  LzDriver& d = lz_driver();
  CUmemAccessDesc ad = access_desc(h->device);
  CU_TRY(d.cuMemAddressReserve(&h->mc_va, h->bytes, h->mc_gran, 0, 0));
  CU_TRY(d.cuMemMap(h->mc_va, h->bytes, 0, h->mc, 0));
  CU_TRY(d.cuMemSetAccess(h->mc_va, h->bytes, &ad, 1));
  h->mc_mapped = true;
  return LZE_OK;
}

extern "C" int lz_heap_destroy(LzHeap* h) {
  if (!h) return LZE_OK;
  LzDriver& d = lz_driver();
  cudaSetDevice(h->device);
  cudaDeviceSynchronize();
  lz_heap_stop_serving(h);
  if (h->mc_mapped) {
    d.cuMemUnmap(h->mc_va, h->bytes);
    d.cuMemAddressFree(h->mc_va, h->bytes);
  }
  if (h->mc_bound) {
    CUdevice dev;
    d.cuDeviceGet(&dev, h->device);
    d.cuMulticastUnbind(h->mc, dev, 0, h->bytes);
  }
  if (h->mc_created) d.cuMemRelease(h->mc);
  if (h->mc_fd >= 0) close(h->mc_fd);
  for (int p = 0; p < h->world; ++p) {
    if (h->peer_mapped[p]) {
      d.cuMemUnmap(h->va[p], h->bytes);
      d.cuMemAddressFree(h->va[p], h->bytes);
    }
    if (p != h->rank && h->peer_mapped[p]) d.cuMemRelease(h->peer_handle[p]);
  }
  d.cuMemRelease(h->local);
  if (h->local_fd >= 0) close(h->local_fd);
  delete h;
  return LZE_OK;
}

extern "C" size_t lz_heap_size(LzHeap* h) { return h->bytes; }
extern "C" void* lz_heap_ptr(LzHeap* h, int rank) {
  if (rank < 0 || rank >= h->world) return nullptr;
  return (void*)h->va[rank];
}
extern "C" void* lz_heap_mc_ptr(LzHeap* h) { return h->mc_mapped ? (void*)h->mc_va : nullptr; }
extern "C" int lz_heap_has_mc(LzHeap* h) { return h->mc_mapped ? 1 : 0; }
int lz_heap_device(LzHeap* h) { return h->device; }
int lz_heap_rank(LzHeap* h) { return h->rank; }
int lz_heap_world(LzHeap* h) { return h->world; }

// ----------------------------------------------------------------------------
// device probes (topology)
// ----------------------------------------------------------------------------
extern "C" int lz_device_info(int device, int* sm_count, int* mc, int* major, int* minor,
                              size_t* total_mem) {
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) {
    cudaGetLastError();
    lz_set_error("cudaGetDeviceProperties(%d) failed", device);
    return LZE_CUDA;
  }
  *sm_count = p.multiProcessorCount;
  *major = p.major;
  *minor = p.minor;
  *total_mem = p.totalGlobalMem;
  *mc = 0;
  LzDriver& d = lz_driver();
  if (d.ok && d.cuDeviceGetAttribute) {
    CUdevice dev;
    if (d.cuDeviceGet(&dev, device) == CUDA_SUCCESS)
      d.cuDeviceGetAttribute(mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, dev);
  }
  return LZE_OK;
}

extern "C" int lz_can_access_peer(int device, int peer, int* can) {
  if (cudaDeviceCanAccessPeer(can, device, peer) != cudaSuccess) {
    cudaGetLastError();
    lz_set_error("cudaDeviceCanAccessPeer failed");
    return LZE_CUDA;
  }
  return LZE_OK;
}

extern "C" int lz_nvlink_p2p_attr(int device, int peer, int* perf_rank, int* native_atomics) {
  if (cudaDeviceGetP2PAttribute(perf_rank, cudaDevP2PAttrPerformanceRank, device, peer) !=
          cudaSuccess ||
      cudaDeviceGetP2PAttribute(native_atomics, cudaDevP2PAttrNativeAtomicSupported, device,
                                peer) != cudaSuccess) {
    cudaGetLastError();
    lz_set_error("cudaDeviceGetP2PAttribute failed");
    return LZE_CUDA;
  }
  return LZE_OK;
}
