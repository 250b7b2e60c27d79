// Symmetric device heap: one physical allocation per GPU, mapped into every
// rank's address space through CUDA VMM (POSIX file-descriptor handles passed
// over a Unix-domain socket), optionally bound to an NVLS multicast object so
// kernels can use multimem.* on it.  Collective phases (create, exchange,
// bind, finish, destroy) are separated by host barriers run by the caller.
#pragma once
#include <cuda.h>

#include <atomic>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "vb/devprog.h"

namespace vb {

constexpr size_t kControlBytes = 4096;
constexpr int kMaxFlagBlocks = 512;
constexpr size_t kFlagBytes = (size_t)kMaxFlagBlocks * kMaxFlagLanes * 8 + 4096;
constexpr size_t kReservedBytes = kControlBytes + kFlagBytes;
constexpr size_t kHeapAlign = 256;

class SymHeap {
 public:
  SymHeap(int rank, int nranks, int device, size_t bytes, const std::string& session, bool want_multicast);
  ~SymHeap();
  SymHeap(const SymHeap&) = delete;
  SymHeap& operator=(const SymHeap&) = delete;

  void exchange(double timeout_s);      // import and map every peer (and the multicast handle)
  void bind_multicast();                // bind local memory to the multicast object and map it
  void finish();                        // stop serving handles
  void destroy();                       // unmap and release everything (collective: after a barrier)

  size_t alloc(size_t bytes);           // byte offset of a new block (deterministic first fit)
  void free(size_t offset);
  size_t used() const;

  int rank() const { return rank_; }
  int nranks() const { return nranks_; }
  int device() const { return device_; }
  size_t size() const { return size_; }
  bool multicast() const { return mc_mapped_; }
  char* base(int r) const { return reinterpret_cast<char*>(va_[r]); }
  char* mc_base() const { return mc_mapped_ ? reinterpret_cast<char*>(mc_va_) : nullptr; }
  size_t flag_offset() const { return kControlBytes; }
  long long start_slot() const { return (long long)kMaxFlagBlocks * kMaxFlagLanes; }

 private:
  void serve();
  int request_fd(int peer, char what, double timeout_s);
  std::string socket_name(int r) const;

  int rank_, nranks_, device_;
  size_t size_ = 0, granularity_ = 0;
  std::string session_;
  bool want_mc_ = false, mc_mapped_ = false, mc_added_ = false, destroyed_ = false;
  CUmemGenericAllocationHandle local_ = 0, mc_ = 0;
  CUmemGenericAllocationHandle peers_[kMaxRanks] = {};
  bool mapped_[kMaxRanks] = {};
  CUdeviceptr reserve_ = 0, va_[kMaxRanks] = {}, mc_va_ = 0;
  int local_fd_ = -1, mc_fd_ = -1, listen_fd_ = -1;
  std::thread server_;
  std::atomic<bool> stop_{false};
  mutable std::mutex mu_;
  std::map<size_t, size_t> used_;   // offset -> bytes
};

}  // namespace vb
