#include "nvls.hpp"

#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>

#include "engine/engine.hpp"

namespace commux {
namespace cuda {

namespace {

std::string cu_err(CUresult r, const char* what) {
  const char* s = nullptr;
  cuGetErrorString(r, &s);
  return std::string(what) + ": " + (s ? s : "unknown CUDA driver error");
}

void store_set(Engine* eng, const std::string& key, const std::string& v) {
  eng->store().set(eng->store_prefix() + key, std::vector<std::uint8_t>(v.begin(), v.end()));
}

std::string store_get(Engine* eng, const std::string& key) {
  const std::string k = eng->store_prefix() + key;
  eng->store().wait({k}, eng->timeout());
  auto v = eng->store().get(k);
  return std::string(v.begin(), v.end());
}

// Abstract Unix-domain socket address (no file on disk, gone with the socket).
socklen_t abstract_addr(const std::string& name, sockaddr_un* a) {
  std::memset(a, 0, sizeof(*a));
  a->sun_family = AF_UNIX;
  const std::size_t n = std::min(name.size(), sizeof(a->sun_path) - 2);
  std::memcpy(a->sun_path + 1, name.data(), n);
  return static_cast<socklen_t>(offsetof(sockaddr_un, sun_path) + 1 + n);
}

bool send_fd(int sock, int fd) {
  char byte = 'F';
  iovec io{&byte, 1};
  alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int))];
  std::memset(ctrl, 0, sizeof(ctrl));
  msghdr m{};
  m.msg_iov = &io;
  m.msg_iovlen = 1;
  m.msg_control = ctrl;
  m.msg_controllen = sizeof(ctrl);
  cmsghdr* c = CMSG_FIRSTHDR(&m);
  c->cmsg_level = SOL_SOCKET;
  c->cmsg_type = SCM_RIGHTS;
  c->cmsg_len = CMSG_LEN(sizeof(int));
  std::memcpy(CMSG_DATA(c), &fd, sizeof(int));
  return ::sendmsg(sock, &m, MSG_NOSIGNAL) == 1;
}

int recv_fd(int sock) {
  char byte = 0;
  iovec io{&byte, 1};
  alignas(cmsghdr) char ctrl[CMSG_SPACE(sizeof(int))];
  msghdr m{};
  m.msg_iov = &io;
  m.msg_iovlen = 1;
  m.msg_control = ctrl;
  m.msg_controllen = sizeof(ctrl);
  if (::recvmsg(sock, &m, 0) != 1) return -1;
  for (cmsghdr* c = CMSG_FIRSTHDR(&m); c != nullptr; c = CMSG_NXTHDR(&m, c)) {
    if (c->cmsg_level == SOL_SOCKET && c->cmsg_type == SCM_RIGHTS) {
      int fd = -1;
      std::memcpy(&fd, CMSG_DATA(c), sizeof(int));
      return fd;
    }
  }
  return -1;
}

bool wait_readable(int fd, std::chrono::steady_clock::time_point deadline) {
  for (;;) {
    auto left = std::chrono::duration_cast<std::chrono::milliseconds>(deadline - std::chrono::steady_clock::now());
    if (left.count() <= 0) return false;
    pollfd p{fd, POLLIN, 0};
    int r = ::poll(&p, 1, static_cast<int>(std::min<long long>(left.count(), 1000)));
    if (r > 0) return true;
    if (r < 0 && errno != EINTR) return false;
  }
}

std::atomic<int> g_nvls_seq{0};

}  // namespace

bool NvlsBuffer::device_supported(int dev) {
  CUdevice d;
  if (cuDeviceGet(&d, dev) != CUDA_SUCCESS) return false;
  int mc = 0;
  if (cuDeviceGetAttribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, d) != CUDA_SUCCESS) return false;
  return mc != 0;
}

std::unique_ptr<NvlsBuffer> NvlsBuffer::create(Engine* eng, int dev, std::size_t bytes, std::string* why) {
  const int P = eng->size(), me = eng->rank();
  const std::string base = "nvls/" + std::to_string(g_nvls_seq.fetch_add(1)) + "/";
  const auto deadline = std::chrono::steady_clock::now() + eng->timeout();
  std::unique_ptr<NvlsBuffer> b(new NvlsBuffer());
  b->dev_ = dev;
  std::string err;
  auto fail_here = [&](const std::string& e) {
    if (err.empty()) err = e;
  };

  // sizes: multiple of the multicast and allocation granularities
  CUresult r = cuDeviceGet(&b->cudev_, dev);
  if (r != CUDA_SUCCESS) fail_here(cu_err(r, "cuDeviceGet"));
  CUmulticastObjectProp mp{};
  mp.numDevices = static_cast<unsigned int>(P);
  mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  std::size_t mgran = 0, agran = 0;
  CUmemAllocationProp ap{};
  ap.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  ap.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  ap.location.id = dev;
  // a shareable (exported or imported) multicast object binds only memory
  // that is itself shareable
  ap.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  if (err.empty()) {
    mp.size = bytes;
    r = cuMulticastGetGranularity(&mgran, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED);
    if (r != CUDA_SUCCESS) fail_here(cu_err(r, "cuMulticastGetGranularity"));
    r = cuMemGetAllocationGranularity(&agran, &ap, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED);
    if (r != CUDA_SUCCESS) fail_here(cu_err(r, "cuMemGetAllocationGranularity"));
  }
  // every rank must use the same size: rank 0's choice wins
  std::size_t g = std::max<std::size_t>(std::max<std::size_t>(mgran, agran), 1);
  std::size_t size = (bytes + g - 1) / g * g;
  if (me == 0) store_set(eng, base + "size", err.empty() ? std::to_string(size) : "0");
  size = static_cast<std::size_t>(std::stoull(store_get(eng, base + "size")));
  if (size == 0) fail_here("rank 0 could not size the multicast object");
  b->size_ = size;
  mp.size = size;

  // 1. rank 0 creates the multicast object and passes its descriptor on
  int fd = -1;
  if (me == 0) {
    int lsock = -1;
    if (err.empty()) {
      r = cuMulticastCreate(&b->mc_, &mp);
      if (r != CUDA_SUCCESS) {
        fail_here(cu_err(r, "cuMulticastCreate"));
      } else {
        r = cuMemExportToShareableHandle(&fd, b->mc_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0);
        if (r != CUDA_SUCCESS) fail_here(cu_err(r, "cuMemExportToShareableHandle"));
      }
    }
    std::string name = "commux-nvls-" + std::to_string(::getpid()) + "-" + base;
    if (err.empty() && P > 1) {
      lsock = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
      sockaddr_un a;
      socklen_t len = abstract_addr(name, &a);
      if (lsock < 0 || ::bind(lsock, reinterpret_cast<sockaddr*>(&a), len) != 0 || ::listen(lsock, P) != 0)
        fail_here(std::string("nvls socket: ") + std::strerror(errno));
    }
    store_set(eng, base + "sock", err.empty() ? name : "");
    if (err.empty()) {
      for (int k = 1; k < P; ++k) {
        if (!wait_readable(lsock, deadline)) {
          fail_here("nvls: a peer did not connect for the multicast handle");
          break;
        }
        int c = ::accept4(lsock, nullptr, nullptr, SOCK_CLOEXEC);
        if (c < 0 || !send_fd(c, fd))
          fail_here(std::string("nvls: sending the handle: ") + std::strerror(errno));
        if (c >= 0) ::close(c);
        if (!err.empty()) break;
      }
    }
    if (lsock >= 0) ::close(lsock);
  } else {
    std::string name = store_get(eng, base + "sock");
    if (name.empty()) fail_here("rank 0 could not create the multicast object");
    // connect even after a local failure, so rank 0 never waits for us
    if (!name.empty()) {
      int s = -1;
      sockaddr_un a;
      socklen_t len = abstract_addr(name, &a);
      for (;;) {
        s = ::socket(AF_UNIX, SOCK_STREAM | SOCK_CLOEXEC, 0);
        if (s >= 0 && ::connect(s, reinterpret_cast<sockaddr*>(&a), len) == 0) break;
        if (s >= 0) ::close(s);
        s = -1;
        if (std::chrono::steady_clock::now() > deadline) {
          fail_here("nvls: cannot reach rank 0's socket");
          break;
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(2));
      }
      if (s >= 0) {
        if (wait_readable(s, deadline)) fd = recv_fd(s);
        ::close(s);
      }
      if (err.empty() && fd < 0) fail_here("nvls: no multicast handle received");
      if (err.empty()) {
        r = cuMemImportFromShareableHandle(&b->mc_, reinterpret_cast<void*>(static_cast<std::uintptr_t>(fd)),
                                           CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
        if (r != CUDA_SUCCESS) fail_here(cu_err(r, "cuMemImportFromShareableHandle"));
      }
    }
  }
  if (fd >= 0) ::close(fd);

  // 2. every device joins before anyone binds memory
  if (err.empty()) {
    r = cuMulticastAddDevice(b->mc_, b->cudev_);
    if (r != CUDA_SUCCESS)
      fail_here(cu_err(r, "cuMulticastAddDevice"));
    else
      b->added_ = true;
  }
  store_set(eng, base + "added/" + std::to_string(me), err.empty() ? "1" : "0");
  for (int p = 0; p < P; ++p)
    if (store_get(eng, base + "added/" + std::to_string(p)) != "1")
      fail_here("a peer could not join the multicast object");

  // 3. bind this rank's memory and map it twice (unicast and multicast)
  if (err.empty()) {
    r = cuMemCreate(&b->phys_, size, &ap, 0);
    if (r != CUDA_SUCCESS) fail_here(cu_err(r, "cuMemCreate"));
  }
  if (err.empty()) {
    r = cuMulticastBindMem(b->mc_, 0, b->phys_, 0, size, 0);
    if (r != CUDA_SUCCESS)
      fail_here(cu_err(r, "cuMulticastBindMem") + " (size " + std::to_string(size) + ", granularity " +
                std::to_string(g) + ")");
    else
      b->bound_ = true;
  }
  CUmemAccessDesc acc{};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = dev;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  if (err.empty()) {
    r = cuMemAddressReserve(&b->uc_va_, size, g, 0, 0);
    if (r == CUDA_SUCCESS) r = cuMemMap(b->uc_va_, size, 0, b->phys_, 0);
    if (r == CUDA_SUCCESS) {
      b->uc_mapped_ = true;
      r = cuMemSetAccess(b->uc_va_, size, &acc, 1);
    }
    if (r != CUDA_SUCCESS) fail_here(cu_err(r, "mapping the NVLS buffer"));
  }
  if (err.empty()) {
    r = cuMemAddressReserve(&b->mc_va_, size, g, 0, 0);
    if (r == CUDA_SUCCESS) r = cuMemMap(b->mc_va_, size, 0, b->mc_, 0);
    if (r == CUDA_SUCCESS) {
      b->mc_mapped_ = true;
      r = cuMemSetAccess(b->mc_va_, size, &acc, 1);
    }
    if (r != CUDA_SUCCESS) fail_here(cu_err(r, "mapping the multicast object"));
  }
  if (err.empty()) {
    r = cuMemsetD8(b->uc_va_, 0, size);
    if (r == CUDA_SUCCESS) r = cuCtxSynchronize();
    if (r != CUDA_SUCCESS) fail_here(cu_err(r, "clearing the NVLS buffer"));
  }

  // 4. agree: every rank bound and mapped, or nobody uses NVLS
  store_set(eng, base + "bound/" + std::to_string(me), err.empty() ? "1" : "0");
  bool all = err.empty();
  for (int p = 0; p < P; ++p)
    if (store_get(eng, base + "bound/" + std::to_string(p)) != "1") all = false;
  if (!all) {
    if (why) *why = err.empty() ? "a peer could not set up its NVLS buffer" : err;
    b->release();
    return nullptr;
  }
  return b;
}

void NvlsBuffer::release() {
  if (mc_mapped_) cuMemUnmap(mc_va_, size_);
  if (mc_va_) cuMemAddressFree(mc_va_, size_);
  if (uc_mapped_) cuMemUnmap(uc_va_, size_);
  if (uc_va_) cuMemAddressFree(uc_va_, size_);
  if (bound_) cuMulticastUnbind(mc_, cudev_, 0, size_);
  if (phys_) cuMemRelease(phys_);
  if (mc_) cuMemRelease(mc_);
  mc_mapped_ = uc_mapped_ = bound_ = added_ = false;
  mc_va_ = uc_va_ = 0;
  phys_ = mc_ = 0;
}

NvlsBuffer::~NvlsBuffer() { release(); }

}  // namespace cuda
}  // namespace commux
