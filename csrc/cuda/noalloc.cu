// Allocation-free single-GPU AllReduce entry point (see vericcl_b200_noalloc.h).
//
// This entry point has no counterpart in the reference implementation.  It
// runs the single-rank AllReduce program - one interpreter step, "copy the
// staged chunk onto itself with the fused scale", exactly what the schedule
// compiler emits for a one-rank in-place AllReduce - with every piece of the
// interpreter's working memory taken from the static array below.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <string>

#include "vb/launch.h"
#include "vericcl_b200_noalloc.h"

namespace {

// The interpreter's working memory on every GPU that loads this library.
// Layout: [0, 256) control block | [256, 256 + (kMaxFlagLanes + 1) * 8) flag table |
// [8192, 8192 + 256) program tables | [VB_NOALLOC_RESERVED_BYTES, end) staging buffer.
static __device__ __align__(256) unsigned char g_noalloc_scratch[VB_NOALLOC_SCRATCH_BYTES];

constexpr size_t kFlagOff = 256;
constexpr size_t kTableOff = 8192;
constexpr size_t kStageOff = VB_NOALLOC_RESERVED_BYTES;
constexpr int kMaxDevices = 64;
constexpr int kMaxLanes = 148;

static_assert(kFlagOff + (vb::kMaxFlagLanes + 1) * 8 <= kTableOff, "flag table overlaps the program");
static_assert(kTableOff + 256 <= kStageOff, "program overlaps the staging buffer");
static_assert(sizeof(vb::Control) <= kFlagOff, "control block overlaps the flag table");

std::mutex g_setup_mutex;
unsigned char* g_base[kMaxDevices] = {};    // device address of the array, per device
CUcontext g_ctx[kMaxDevices] = {};          // the context that address belongs to
thread_local std::string g_last_error;

int fail(int code, const std::string& why) {
  g_last_error = why;
  return code;
}

// Once per device, with that device current: look the array up, clear the
// control block and flag table, write the epoch and the one-step program.
//
// The set-up is keyed by (device, current context): after cudaDeviceReset the
// runtime creates a new primary context whose copy of the array holds no
// control block or program, so a changed context redoes the set-up.
int setup_device(int device, unsigned char** base) {
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  CUcontext ctx = nullptr;
  if (cuCtxGetCurrent(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  if (g_base[device] && g_ctx[device] == ctx) {
    *base = g_base[device];
    return VB_NOALLOC_OK;
  }
  g_base[device] = nullptr;
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess) return fail(VB_NOALLOC_CUDA_ERROR, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  unsigned char* p = static_cast<unsigned char*>(ptr);
  e = cudaMemset(p, 0, kStageOff);
  if (e != cudaSuccess) return fail(VB_NOALLOC_CUDA_ERROR, std::string("clear control block: ") + cudaGetErrorString(e));
  const unsigned long long epoch = 1;   // flags are relative to epoch << 32; epoch 0 would alias cleared flags
  e = cudaMemcpy(p + offsetof(vb::Control, epoch), &epoch, sizeof epoch, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(VB_NOALLOC_CUDA_ERROR, std::string("write epoch: ") + cudaGetErrorString(e));
  struct Tables {
    vb::DevBlock block;
    vb::DevStep step;
    vb::DevSrc src;
  } t;
  std::memset(&t, 0, sizeof t);
  t.block = vb::DevBlock{0, 1, -1, 0, 0};
  t.step.dst_rank = -1;
  t.step.op = vb::OP_COPY;
  t.step.dst_buf = vb::BUF_OUT;
  t.step.flags = vb::F_SCALE;
  t.step.dst_chunk = 0;
  t.step.cnt = 1;
  t.step.src_begin = 0;
  t.step.nsrc = 1;
  t.src = vb::DevSrc{0, vb::BUF_OUT, 0, 0};
  e = cudaMemcpy(p + kTableOff, &t, sizeof t, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return fail(VB_NOALLOC_CUDA_ERROR, std::string("write program: ") + cudaGetErrorString(e));
  g_base[device] = p;
  g_ctx[device] = ctx;
  *base = p;
  return VB_NOALLOC_OK;
}

int current_base(unsigned char** base) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess || device < 0 || device >= kMaxDevices) return fail(VB_NOALLOC_CUDA_ERROR, "no current device");
  return setup_device(device, base);
}

}  // namespace

extern "C" const char* vb_noalloc_last_error(void) { return g_last_error.c_str(); }

extern "C" int vb_allreduce_local_noalloc(const void* in, void* out, size_t count, int dtype, float scale,
                                          void* cuda_stream) {
  if (!in || !out || count == 0) return fail(VB_NOALLOC_INVALID, "null buffer or zero count");
  if (dtype < vb::DT_F32 || dtype > vb::DT_F16) return fail(VB_NOALLOC_INVALID, "dtype must be 0, 1 or 2");
  const size_t esize = dtype == vb::DT_F32 ? 4 : 2;
  const size_t vec = 16 / esize;
  const size_t padded = (count + vec - 1) / vec * vec;
  if (count > VB_NOALLOC_MAX_BYTES / esize || padded * esize > VB_NOALLOC_MAX_BYTES)
    return fail(VB_NOALLOC_TOO_LARGE, "count * element size = " + std::to_string(count * esize) +
                                          " bytes exceeds the " + std::to_string(VB_NOALLOC_MAX_BYTES) +
                                          "-byte static staging buffer");
  unsigned char* base = nullptr;
  int rc = current_base(&base);
  if (rc != VB_NOALLOC_OK) return rc;
  cudaError_t e = cudaSuccess;
  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  vb::Control* ctl = reinterpret_cast<vb::Control*>(base);
  // status words that must start at zero for every call
  e = cudaMemsetAsync(&ctl->status, 0, sizeof(int) * 5, stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(&ctl->abort_request, 0, sizeof(int), stream);
  if (e == cudaSuccess && padded != count)
    e = cudaMemsetAsync(base + kStageOff + count * esize, 0, (padded - count) * esize, stream);
  if (e == cudaSuccess) e = cudaMemcpyAsync(base + kStageOff, in, count * esize, cudaMemcpyDeviceToDevice, stream);
  if (e != cudaSuccess) return fail(VB_NOALLOC_CUDA_ERROR, std::string("stage input: ") + cudaGetErrorString(e));
  vb::InterpArgs a = {};
  a.blocks = reinterpret_cast<const vb::DevBlock*>(base + kTableOff);
  a.steps = reinterpret_cast<const vb::DevStep*>(base + kTableOff + sizeof(vb::DevBlock));
  a.srcs = reinterpret_cast<const vb::DevSrc*>(base + kTableOff + sizeof(vb::DevBlock) + sizeof(vb::DevStep));
  a.waits = nullptr;
  a.nblocks = 1;
  size_t bytes = padded * esize;
  size_t lanes = bytes / (64u << 10);
  // at most one CTA per co-resident slot of the cooperative launch (fewer SMs under MPS or a partitioned GPU)
  size_t max_lanes = (size_t)vb::interp_max_ctas(512);
  if (max_lanes > (size_t)kMaxLanes) max_lanes = kMaxLanes;
  if (max_lanes < 1) return fail(VB_NOALLOC_CUDA_ERROR, "the interpreter kernel cannot be resident on this device");
  a.nlanes = (int)(lanes < 1 ? 1 : lanes > max_lanes ? max_lanes : lanes);
  a.niters = 1;
  a.nbatch = 1;
  a.rank = 0;
  a.nranks = 1;
  a.dtype = dtype;
  a.redop = vb::RED_SUM;
  a.scale = scale;
  a.chunk_elems = (long long)padded;
  long long piece = ((long long)padded + a.nlanes - 1) / a.nlanes;
  a.piece_elems = (piece + (long long)vec - 1) / (long long)vec * (long long)vec;
  a.buf_off[vb::BUF_IN] = (long long)kStageOff;
  a.buf_off[vb::BUF_OUT] = (long long)kStageOff;
  a.buf_off[vb::BUF_SCR] = (long long)kStageOff;
  a.flag_off = (long long)kFlagOff;
  a.start_slot = vb::kMaxFlagLanes;
  a.base[0] = reinterpret_cast<char*>(base);
  a.control = ctl;
  a.timeout_ns = 10ull * 1000000000ull;
  e = vb::launch_interp(a, stream, 512);
  if (e != cudaSuccess) return fail(VB_NOALLOC_CUDA_ERROR, std::string("launch: ") + cudaGetErrorString(e));
  e = cudaMemcpyAsync(out, base + kStageOff, count * esize, cudaMemcpyDeviceToDevice, stream);
  if (e != cudaSuccess) return fail(VB_NOALLOC_CUDA_ERROR, std::string("copy result: ") + cudaGetErrorString(e));
  return VB_NOALLOC_OK;
}

extern "C" int vb_noalloc_status(int* status, int detail[4]) {
  if (!status) return fail(VB_NOALLOC_INVALID, "null status pointer");
  unsigned char* base = nullptr;
  int rc = current_base(&base);
  if (rc != VB_NOALLOC_OK) return rc;
  const vb::Control* ctl = reinterpret_cast<const vb::Control*>(base);
  int words[5] = {};
  // a synchronous copy: it waits for the work already enqueued on the legacy default stream, but the
  // caller must synchronise its own stream first (the header says so)
  cudaError_t e = cudaMemcpy(words, &ctl->status, sizeof words, cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(VB_NOALLOC_CUDA_ERROR, std::string("read status: ") + cudaGetErrorString(e));
  *status = words[0];
  if (detail)
    for (int i = 0; i < 4; ++i) detail[i] = words[1 + i];
  return VB_NOALLOC_OK;
}
