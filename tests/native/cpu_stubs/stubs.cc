// Host implementations behind the CPU stand-in headers: the CUDA runtime calls
// of the C API, a symmetric heap whose ranks are threads of one process (each
// rank's heap is a host buffer, peers see it through a process-wide table),
// and an interpreter launch that completes at once.  Allocation offsets are
// logged per rank so a test can check that every rank laid out its heap alike.
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <stdexcept>
#include <thread>
#include <vector>

#include "vb/launch.h"
#include "vb/symheap.h"

namespace {
std::atomic<bool> g_hung{false};
std::atomic<int> g_launches{0};
std::mutex g_mu;
std::map<std::string, std::vector<char*>> g_bases;                       // session -> heap of every rank
std::map<std::pair<std::string, int>, std::vector<std::pair<size_t, size_t>>> g_allocs;   // (session, rank)
}

struct CUstream_st { int unused; };
struct CUevent_st { bool recorded; };

cudaError_t cudaMalloc(void** p, size_t bytes) {
  *p = std::calloc(1, bytes ? bytes : 1);
  return *p ? cudaSuccess : cudaErrorInvalidValue;
}
cudaError_t cudaFree(void* p) { std::free(p); return cudaSuccess; }
cudaError_t cudaMemcpy(void* dst, const void* src, size_t bytes, cudaMemcpyKind) {
  std::memmove(dst, src, bytes);
  return cudaSuccess;
}
cudaError_t cudaMemcpyAsync(void* dst, const void* src, size_t bytes, cudaMemcpyKind k, cudaStream_t) {
  return cudaMemcpy(dst, src, bytes, k);
}
cudaError_t cudaMemsetAsync(void* dst, int value, size_t bytes, cudaStream_t) {
  std::memset(dst, value, bytes);
  return cudaSuccess;
}
cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned int) { *e = new CUevent_st{false}; return cudaSuccess; }
cudaError_t cudaEventRecord(cudaEvent_t e, cudaStream_t) { e->recorded = true; return cudaSuccess; }
cudaError_t cudaEventQuery(cudaEvent_t) { return g_hung ? cudaErrorNotReady : cudaSuccess; }
cudaError_t cudaEventDestroy(cudaEvent_t e) { delete e; return cudaSuccess; }
cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned int) { *s = new CUstream_st{0}; return cudaSuccess; }
cudaError_t cudaStreamDestroy(cudaStream_t s) { delete s; return cudaSuccess; }
cudaError_t cudaStreamSynchronize(cudaStream_t) { return cudaSuccess; }
cudaError_t cudaDeviceSynchronize() { return cudaSuccess; }
const char* cudaGetErrorString(cudaError_t e) { return e == cudaSuccess ? "no error" : "stub error"; }

namespace vb_stub {
void set_streams_hung(bool hung) { g_hung = hung; }
int interp_launches() { return g_launches; }
std::vector<std::pair<size_t, size_t>> alloc_log(const std::string& session, int rank) {
  std::lock_guard<std::mutex> l(g_mu);
  return g_allocs[{session, rank}];
}
int abort_request(const std::string& session, int rank) {
  std::lock_guard<std::mutex> l(g_mu);
  return reinterpret_cast<const vb::Control*>(g_bases[session].at(rank))->abort_request;
}
}  // namespace vb_stub

namespace vb {

SymHeap::SymHeap(int rank, int nranks, int device, size_t bytes, const std::string& session, bool)
    : rank_(rank), nranks_(nranks), device_(device), size_(bytes), session_(session) {
  char* mem = static_cast<char*>(std::calloc(1, bytes));
  std::lock_guard<std::mutex> l(g_mu);
  auto& v = g_bases[session];
  if ((int)v.size() < nranks) v.resize(nranks, nullptr);
  v[rank] = mem;
  va_[rank] = reinterpret_cast<CUdeviceptr>(mem);
  used_[0] = kReservedBytes;
}

SymHeap::~SymHeap() {}

void SymHeap::exchange(double timeout_s) {
  auto until = std::chrono::steady_clock::now() + std::chrono::duration<double>(timeout_s);
  for (;;) {
    {
      std::lock_guard<std::mutex> l(g_mu);
      auto& v = g_bases[session_];
      bool all = (int)v.size() >= nranks_;
      for (int r = 0; all && r < nranks_; ++r) all = v[r] != nullptr;
      if (all) {
        for (int r = 0; r < nranks_; ++r) va_[r] = reinterpret_cast<CUdeviceptr>(v[r]);
        return;
      }
    }
    if (std::chrono::steady_clock::now() > until) throw std::runtime_error("stub heap exchange timed out");
    std::this_thread::sleep_for(std::chrono::milliseconds(1));
  }
}
void SymHeap::bind_multicast() {}
void SymHeap::finish() {}
void SymHeap::destroy() { destroyed_ = true; }

size_t SymHeap::alloc(size_t bytes) {
  std::lock_guard<std::mutex> l(mu_);
  size_t want = (bytes + kHeapAlign - 1) / kHeapAlign * kHeapAlign;
  size_t at = 0;
  for (auto& [off, len] : used_) {
    if (off >= at + want) break;
    at = (off + len + kHeapAlign - 1) / kHeapAlign * kHeapAlign;
  }
  if (at + want > size_) throw std::runtime_error("stub heap exhausted");
  used_[at] = want;
  std::lock_guard<std::mutex> g(g_mu);
  g_allocs[{session_, rank_}].push_back({at, bytes});
  return at;
}
void SymHeap::free(size_t offset) {
  std::lock_guard<std::mutex> l(mu_);
  used_.erase(offset);
}
size_t SymHeap::used() const {
  std::lock_guard<std::mutex> l(mu_);
  size_t n = 0;
  for (auto& kv : used_) n += kv.second;
  return n;
}

cudaError_t launch_interp(const InterpArgs& a, cudaStream_t, int) {
  ++g_launches;
  a.control->epoch += 1;
  a.control->status = ST_OK;
  return cudaSuccess;
}
int interp_max_ctas(int) { return 1 << 20; }
void apply_emulation_env(InterpArgs*) {}

}  // namespace vb
