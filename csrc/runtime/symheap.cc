// Symmetric heap implementation (CUDA driver VMM + NVLS multicast).
#include "vb/symheap.h"

#include <cuda_runtime.h>
#include <errno.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/un.h>
#include <unistd.h>

#include <chrono>
#include <cstring>
#include <stdexcept>

namespace vb {
namespace {

void check(CUresult r, const char* what) {
  if (r != CUDA_SUCCESS) {
    const char* msg = nullptr;
    cuGetErrorString(r, &msg);
    throw std::runtime_error(std::string(what) + ": " + (msg ? msg : "unknown CUDA driver error"));
  }
}

size_t round_up(size_t x, size_t g) { return (x + g - 1) / g * g; }

size_t gcd(size_t a, size_t b) { return b ? gcd(b, a % b) : a; }

void send_fd(int sock, int fd) {
  char byte = 'F';
  struct iovec iov = {&byte, 1};
  char ctrl[CMSG_SPACE(sizeof(int))];
  std::memset(ctrl, 0, sizeof(ctrl));
  struct msghdr msg = {};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = ctrl;
  msg.msg_controllen = sizeof(ctrl);
  struct cmsghdr* c = CMSG_FIRSTHDR(&msg);
  c->cmsg_level = SOL_SOCKET;
  c->cmsg_type = SCM_RIGHTS;
  c->cmsg_len = CMSG_LEN(sizeof(int));
  std::memcpy(CMSG_DATA(c), &fd, sizeof(int));
  if (sendmsg(sock, &msg, 0) != 1) throw std::runtime_error("sendmsg of a memory handle failed");
}

int recv_fd(int sock) {
  char byte = 0;
  struct iovec iov = {&byte, 1};
  char ctrl[CMSG_SPACE(sizeof(int))];
  struct msghdr msg = {};
  msg.msg_iov = &iov;
  msg.msg_iovlen = 1;
  msg.msg_control = ctrl;
  msg.msg_controllen = sizeof(ctrl);
  if (recvmsg(sock, &msg, 0) != 1) throw std::runtime_error("recvmsg of a memory handle failed");
  struct cmsghdr* c = CMSG_FIRSTHDR(&msg);
  if (!c || c->cmsg_type != SCM_RIGHTS) throw std::runtime_error("peer did not send a file descriptor");
  int fd;
  std::memcpy(&fd, CMSG_DATA(c), sizeof(int));
  return fd;
}

sockaddr_un abstract_addr(const std::string& name, socklen_t* len) {
  sockaddr_un a = {};
  a.sun_family = AF_UNIX;
  a.sun_path[0] = '\0';
  size_t n = std::min(name.size(), sizeof(a.sun_path) - 2);
  std::memcpy(a.sun_path + 1, name.data(), n);
  *len = (socklen_t)(offsetof(sockaddr_un, sun_path) + 1 + n);
  return a;
}

}  // namespace

std::string SymHeap::socket_name(int r) const { return "vericcl_b200." + session_ + "." + std::to_string(r); }

SymHeap::SymHeap(int rank, int nranks, int device, size_t bytes, const std::string& session, bool want_multicast)
    : rank_(rank), nranks_(nranks), device_(device), session_(session), want_mc_(want_multicast && nranks > 1) {
  if (nranks < 1 || nranks > kMaxRanks || rank < 0 || rank >= nranks) throw std::runtime_error("invalid rank layout");
  if (cudaSetDevice(device) != cudaSuccess || cudaFree(0) != cudaSuccess) throw std::runtime_error("cannot activate the CUDA device");
  check(cuInit(0), "cuInit");
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
  check(cuMemGetAllocationGranularity(&granularity_, &prop, CU_MEM_ALLOC_GRANULARITY_RECOMMENDED), "allocation granularity");
  size_t gran = granularity_;
  size_t want = bytes + kReservedBytes;
  if (want_mc_) {
    CUmulticastObjectProp mp = {};
    mp.numDevices = (unsigned)nranks;
    mp.size = round_up(want, gran);
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t mg = 0;
    if (cuMulticastGetGranularity(&mg, &mp, CU_MULTICAST_GRANULARITY_MINIMUM) == CUDA_SUCCESS && mg)
      gran = gran / gcd(gran, mg) * mg;
    else
      want_mc_ = false;
  }
  size_ = round_up(want, gran);
  check(cuMemCreate(&local_, size_, &prop, 0), "cuMemCreate");
  check(cuMemExportToShareableHandle(&local_fd_, local_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0), "export handle");
  check(cuMemAddressReserve(&reserve_, size_ * nranks, gran, 0, 0), "reserve address range");
  for (int r = 0; r < nranks; ++r) va_[r] = reserve_ + (CUdeviceptr)r * size_;
  check(cuMemMap(va_[rank], size_, 0, local_, 0), "map local heap");
  mapped_[rank] = true;
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  check(cuMemSetAccess(va_[rank], size_, &acc, 1), "set local access");
  check(cuMemsetD8(va_[rank], 0, kReservedBytes), "clear control and flags");
  // control block: epoch starts at 1
  unsigned long long one = 1;
  check(cuMemcpyHtoD(va_[rank], &one, sizeof(one)), "init epoch");
  if (want_mc_ && rank == 0) {
    CUmulticastObjectProp mp = {};
    mp.numDevices = (unsigned)nranks;
    mp.size = size_;
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    if (cuMulticastCreate(&mc_, &mp) != CUDA_SUCCESS) {
      want_mc_ = false;
    } else {
      check(cuMemExportToShareableHandle(&mc_fd_, mc_, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0), "export multicast");
    }
  }
  used_[0] = kReservedBytes;
  if (nranks > 1) {
    listen_fd_ = socket(AF_UNIX, SOCK_STREAM, 0);
    socklen_t len;
    sockaddr_un addr = abstract_addr(socket_name(rank), &len);
    if (listen_fd_ < 0 || bind(listen_fd_, (sockaddr*)&addr, len) != 0 || listen(listen_fd_, 64) != 0)
      throw std::runtime_error("cannot open the handle socket " + socket_name(rank) + ": " + std::strerror(errno));
    server_ = std::thread([this] { serve(); });
  }
}

void SymHeap::serve() {
  while (!stop_.load()) {
    struct pollfd p = {listen_fd_, POLLIN, 0};
    int r = poll(&p, 1, 50);
    if (r <= 0) continue;
    int c = accept(listen_fd_, nullptr, nullptr);
    if (c < 0) continue;
    char what = 0;
    if (read(c, &what, 1) == 1) {
      try {
        if (what == 'H') send_fd(c, local_fd_);
        else if (what == 'M' && mc_fd_ >= 0) send_fd(c, mc_fd_);
      } catch (...) {
      }
    }
    close(c);
  }
}

int SymHeap::request_fd(int peer, char what, double timeout_s) {
  auto deadline = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
  socklen_t len;
  sockaddr_un addr = abstract_addr(socket_name(peer), &len);
  while (true) {
    int s = socket(AF_UNIX, SOCK_STREAM, 0);
    if (s >= 0 && connect(s, (sockaddr*)&addr, len) == 0) {
      if (write(s, &what, 1) != 1) { close(s); throw std::runtime_error("handle request failed"); }
      int fd = recv_fd(s);
      close(s);
      return fd;
    }
    if (s >= 0) close(s);
    if (std::chrono::steady_clock::now() > deadline)
      throw std::runtime_error("timed out connecting to rank " + std::to_string(peer) + " for its memory handle");
    std::this_thread::sleep_for(std::chrono::milliseconds(20));
  }
}

void SymHeap::exchange(double timeout_s) {
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device_;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  for (int p = 0; p < nranks_; ++p) {
    if (p == rank_) continue;
    int fd = request_fd(p, 'H', timeout_s);
    check(cuMemImportFromShareableHandle(&peers_[p], (void*)(uintptr_t)fd, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR), "import peer handle");
    close(fd);
    check(cuMemMap(va_[p], size_, 0, peers_[p], 0), "map peer heap");
    mapped_[p] = true;
    check(cuMemSetAccess(va_[p], size_, &acc, 1), "set peer access");
  }
  if (want_mc_) {
    if (rank_ != 0) {
      int fd = request_fd(0, 'M', timeout_s);
      CUresult r = cuMemImportFromShareableHandle(&mc_, (void*)(uintptr_t)fd, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR);
      close(fd);
      check(r, "import multicast handle");
    }
    CUdevice dev;
    check(cuDeviceGet(&dev, device_), "cuDeviceGet");
    check(cuMulticastAddDevice(mc_, dev), "cuMulticastAddDevice");
    mc_added_ = true;
  }
}

void SymHeap::bind_multicast() {
  if (!want_mc_ || !mc_added_) return;
  check(cuMulticastBindMem(mc_, 0, local_, 0, size_, 0), "cuMulticastBindMem");
  check(cuMemAddressReserve(&mc_va_, size_, granularity_, 0, 0), "reserve multicast range");
  check(cuMemMap(mc_va_, size_, 0, mc_, 0), "map multicast range");
  CUmemAccessDesc acc = {};
  acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  acc.location.id = device_;
  acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  check(cuMemSetAccess(mc_va_, size_, &acc, 1), "set multicast access");
  mc_mapped_ = true;
}

void SymHeap::finish() {
  stop_.store(true);
  if (server_.joinable()) server_.join();
  if (listen_fd_ >= 0) { close(listen_fd_); listen_fd_ = -1; }
}

void SymHeap::destroy() {
  if (destroyed_) return;
  destroyed_ = true;
  finish();
  cudaDeviceSynchronize();
  if (mc_mapped_) {
    cuMemUnmap(mc_va_, size_);
    cuMemAddressFree(mc_va_, size_);
    CUdevice dev;
    cuDeviceGet(&dev, device_);
    cuMulticastUnbind(mc_, dev, 0, size_);
    mc_mapped_ = false;
  }
  if (mc_) { cuMemRelease(mc_); mc_ = 0; }
  for (int p = 0; p < nranks_; ++p) {
    if (mapped_[p]) cuMemUnmap(va_[p], size_);
    mapped_[p] = false;
    if (p != rank_ && peers_[p]) { cuMemRelease(peers_[p]); peers_[p] = 0; }
  }
  if (local_) { cuMemRelease(local_); local_ = 0; }
  if (reserve_) { cuMemAddressFree(reserve_, size_ * nranks_); reserve_ = 0; }
  if (local_fd_ >= 0) { close(local_fd_); local_fd_ = -1; }
  if (mc_fd_ >= 0) { close(mc_fd_); mc_fd_ = -1; }
}

SymHeap::~SymHeap() {
  try {
    destroy();
  } catch (...) {
  }
}

size_t SymHeap::alloc(size_t bytes) {
  std::lock_guard<std::mutex> g(mu_);
  bytes = round_up(bytes ? bytes : 1, kHeapAlign);
  size_t cursor = 0;
  for (auto& kv : used_) {
    if (kv.first >= cursor + bytes) break;
    cursor = round_up(kv.first + kv.second, kHeapAlign);
  }
  if (cursor + bytes > size_) throw std::runtime_error("symmetric heap exhausted: " + std::to_string(bytes) + " bytes requested");
  used_[cursor] = bytes;
  return cursor;
}

void SymHeap::free(size_t offset) {
  std::lock_guard<std::mutex> g(mu_);
  if (offset == 0) return;
  used_.erase(offset);
}

size_t SymHeap::used() const {
  std::lock_guard<std::mutex> g(mu_);
  size_t n = 0;
  for (auto& kv : used_) n += kv.second;
  return n;
}

}  // namespace vb
