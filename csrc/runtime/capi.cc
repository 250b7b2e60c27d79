// C API implementation on top of the symmetric heap, the schedule compiler,
// the interpreter and the TCP control plane (no Python, no torch).
#include "vericcl_b200.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <memory>
#include <mutex>
#include <string>
#include <thread>

#include "vb/contract.h"
#include "vb/control.h"
#include "vb/launch.h"
#include "vb/plan.h"
#include "vb/symheap.h"
#include "vb/trace_io.h"

using namespace vb;

struct vb_context {
  int rank = 0, nranks = 1, device = 0;
  std::unique_ptr<ControlTransport> control;
  std::unique_ptr<SymHeap> heap;
  CompiledPlan plan;
  bool prepared = false, closed = false;
  DevBlock* blocks = nullptr;
  DevStep* steps = nullptr;
  DevSrc* srcs = nullptr;
  DevWait* waits = nullptr;
  size_t stage_in = 0, stage_out = 0, stage_scr = 0;               // heap offsets of the staging buffers
  size_t cap_in = 0, cap_out = 0, cap_scr = 0;                      // their sizes
  bool staged = false;
  std::atomic<bool> busy{false};
  bool unresolved = false;
  std::string error;
  cudaStream_t abort_stream = nullptr;
  unsigned long long* trace_dev = nullptr;   // per-step trace of the next (armed) or last traced execution
  bool trace_armed = false, trace_ready = false;
};

namespace {

struct Guard {
  vb_context* c;
  bool ok;
  explicit Guard(vb_context* ctx) : c(ctx), ok(!ctx->busy.exchange(true)) {}
  ~Guard() { if (ok) c->busy.store(false); }
};

vb_result fail(vb_context* c, vb_result r, const std::string& m) {
  if (c) c->error = m;
  return r;
}

template <typename T>
T* upload(const std::vector<T>& v) {
  if (v.empty()) return nullptr;
  T* p = nullptr;
  if (cudaMalloc(&p, v.size() * sizeof(T)) != cudaSuccess) throw std::runtime_error("cudaMalloc plan table");
  cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice);
  return p;
}

void free_plan(vb_context* c) {
  cudaFree(c->blocks); cudaFree(c->steps); cudaFree(c->srcs); cudaFree(c->waits);
  c->blocks = nullptr; c->steps = nullptr; c->srcs = nullptr; c->waits = nullptr;
  cudaFree(c->trace_dev);
  c->trace_dev = nullptr;
  c->trace_armed = c->trace_ready = false;
  c->prepared = false;
}

TraceLayout trace_layout(const vb_context* c) {
  TraceLayout l;
  const RankProgram& rp = c->plan.ranks[c->rank];
  l.rank = c->rank;
  l.nlanes = c->plan.options.nlanes;
  l.niters = c->plan.options.niters;
  for (const DevBlock& b : rp.blocks) {
    std::vector<int> ops;
    for (int s = 0; s < b.nsteps; ++s) ops.push_back(rp.steps[b.step_begin + s].op);
    l.max_steps = std::max(l.max_steps, b.nsteps);
    l.block_ops.push_back(std::move(ops));
  }
  return l;
}

size_t esize(int dtype) { return dtype == VB_FLOAT32 ? 4 : 2; }

}  // namespace

extern "C" int vb_abi_version(void) { return VERICCL_B200_ABI_VERSION; }

extern "C" vb_result vb_init(const vb_init_params* p, vb_context** out) {
  if (!p || !out || p->abi_version != VERICCL_B200_ABI_VERSION || p->nranks < 1 || p->nranks > kMaxRanks ||
      p->rank < 0 || p->rank >= p->nranks || p->timeout_s <= 0 || !p->session)
    return VB_INVALID;
  auto c = std::make_unique<vb_context>();
  c->rank = p->rank;
  c->nranks = p->nranks;
  c->device = p->device;
  try {
    Deadline d = Deadline::after(p->timeout_s);
    c->control = std::make_unique<ControlTransport>(p->rank, p->nranks,
                                                    p->control_address ? p->control_address : "127.0.0.1",
                                                    p->control_port, p->session);
    c->control->barrier("INIT", d);
    c->heap = std::make_unique<SymHeap>(p->rank, p->nranks, p->device, p->heap_bytes, p->session, p->multicast != 0);
    c->control->barrier("HEAP_CREATED", d);
    c->heap->exchange(d.remaining());
    c->control->barrier("HEAP_MAPPED", d);
    c->heap->bind_multicast();
    c->control->barrier("HEAP_BOUND", d);
    c->heap->finish();
    cudaStreamCreateWithFlags(&c->abort_stream, cudaStreamNonBlocking);
  } catch (const ControlError& e) {
    return VB_TIMEOUT;
  } catch (const std::exception& e) {
    return VB_FAILED;
  }
  *out = c.release();
  return VB_OK;
}

extern "C" vb_result vb_prepare(vb_context* c, const char* xml, int nlanes, int niters, double timeout_s) {
  if (!c) return VB_INVALID;
  if (c->closed) return VB_CLOSED;
  Guard g(c);
  if (!g.ok) return VB_BUSY;
  if (!xml || nlanes < 1 || niters < 1) return fail(c, VB_INVALID, "invalid prepare arguments");
  try {
    Deadline d = Deadline::after(timeout_s);
    std::string text(xml);
    std::string digest = sha256_hex(text);
    auto all = c->control->gather("PREPARE_VALIDATE", digest, d);
    for (auto& h : all)
      if (h != digest) return fail(c, VB_INVALID, "ranks prepared different schedules");
    CompileOptions o;
    o.nlanes = nlanes;
    o.niters = niters;
    o.reducing = text.find("coll=\"allreduce\"") != std::string::npos ||
                 text.find("coll=\"reduce_scatter\"") != std::string::npos ||
                 text.find("coll=\"reduce\"") != std::string::npos;
    o.multicast = c->heap->multicast();
    CompiledPlan plan = compile_plan(parse_xml(text), o);
    if ((int)plan.ranks.size() != c->nranks) return fail(c, VB_INVALID, "schedule rank count differs");
    if (c->prepared) free_plan(c);
    c->plan = std::move(plan);
    const RankProgram& rp = c->plan.ranks[c->rank];
    c->blocks = upload(rp.blocks);
    c->steps = upload(rp.steps);
    c->srcs = upload(rp.srcs);
    c->waits = upload(rp.waits);
    c->prepared = true;
    c->control->barrier("READY", d);
  } catch (const CompileError& e) {
    return fail(c, VB_INVALID, e.what());
  } catch (const ControlError& e) {
    return fail(c, VB_TIMEOUT, e.what());
  } catch (const std::exception& e) {
    return fail(c, VB_FAILED, e.what());
  }
  return VB_OK;
}

extern "C" vb_result vb_execute(vb_context* c, const void* in, void* out, size_t count, int dtype, int redop,
                                float scale, void* stream_ptr, double timeout_s) {
  if (!c) return VB_INVALID;
  if (c->closed) return VB_CLOSED;
  Guard g(c);
  if (!g.ok) return VB_BUSY;
  if (!c->prepared) return fail(c, VB_INVALID, "no prepared schedule");
  if (c->unresolved) return fail(c, VB_FAILED, "an earlier execution is unresolved");
  if (!in || !out || count == 0 || dtype < 0 || dtype > 2 || redop < 0 || redop > 3)
    return fail(c, VB_INVALID, "invalid execute arguments");
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_ptr);
  const std::string& coll = c->plan.algo.coll;
  size_t runtime = count * ((coll == "allgather") ? c->nranks : 1);
  size_t nch = c->plan.algo.nchunksperloop;
  size_t vec = 16 / esize(dtype);
  if (runtime % nch || (runtime / nch) % vec) return fail(c, VB_INVALID, "count does not split into 16-byte chunks");
  long long chunk = (long long)(runtime / nch);
  const RankProgram& rp = c->plan.ranks[c->rank];
  size_t in_bytes = (size_t)rp.i_chunks * chunk * esize(dtype);
  size_t out_bytes = (size_t)rp.o_chunks * chunk * esize(dtype);
  size_t scr_bytes = (size_t)c->plan.max_scratch_used() * chunk * esize(dtype) + 16;
  // peers address each other's buffers by heap offset, so every rank allocates the largest input and output
  // buffer of any rank (a reduce, for one, has an output buffer on its root only)
  int max_i = 0, max_o = 0;
  for (const RankProgram& r : c->plan.ranks) {
    max_i = r.i_chunks > max_i ? r.i_chunks : max_i;
    max_o = r.o_chunks > max_o ? r.o_chunks : max_o;
  }
  size_t in_alloc = (size_t)max_i * chunk * esize(dtype), out_alloc = (size_t)max_o * chunk * esize(dtype);
  try {
    // staging buffers in the heap, sized identically on every rank; each grows on its own
    if (!c->staged || in_alloc > c->cap_in || out_alloc > c->cap_out || scr_bytes > c->cap_scr) {
      if (c->staged) { c->heap->free(c->stage_in); c->heap->free(c->stage_out); c->heap->free(c->stage_scr); }
      c->cap_in = in_alloc > c->cap_in ? in_alloc : c->cap_in;
      c->cap_out = out_alloc > c->cap_out ? out_alloc : c->cap_out;
      c->cap_scr = scr_bytes > c->cap_scr ? scr_bytes : c->cap_scr;
      c->stage_in = c->heap->alloc(c->cap_in);
      c->stage_out = c->heap->alloc(c->cap_out);
      c->stage_scr = c->heap->alloc(c->cap_scr);
      c->staged = true;
    }
    size_t user_in = count * esize(dtype);
    size_t user_out = (coll == "allgather" ? count * c->nranks : coll == "reduce_scatter" ? count / c->nranks : count) * esize(dtype);
    if (c->plan.algo.inplace) return fail(c, VB_INVALID, "the C API runs out-of-place schedules");
    // the staged copies must stay inside this rank's input and output buffers of the schedule; a reduce
    // defines an output on its root only (the other ranks' schedules have no output buffer), so a rank
    // without one leaves the user's output untouched
    if (coll == "reduce" && out_bytes == 0) user_out = 0;
    if (user_in > in_bytes || user_out > out_bytes)
      return fail(c, VB_INVALID, "schedule buffers are smaller than the user buffers for this count");
    cudaMemcpyAsync(c->heap->base(c->rank) + c->stage_in, in, user_in, cudaMemcpyDeviceToDevice, stream);
    InterpArgs a = {};
    a.blocks = c->blocks; a.steps = c->steps; a.srcs = c->srcs; a.waits = c->waits;
    a.nblocks = (int)rp.blocks.size();
    a.nlanes = c->plan.options.nlanes;
    a.niters = c->plan.options.niters;
    a.nbatch = 1;
    a.rank = c->rank;
    a.nranks = c->nranks;
    a.dtype = dtype;
    a.redop = redop;
    a.scale = scale;
    a.chunk_elems = chunk;
    long long pieces = (long long)a.nlanes * a.niters;
    long long piece = (chunk + pieces - 1) / pieces;
    a.piece_elems = (piece + vec - 1) / vec * vec;
    a.buf_off[BUF_IN] = (long long)c->stage_in;
    a.buf_off[BUF_OUT] = (long long)c->stage_out;
    a.buf_off[BUF_SCR] = (long long)c->stage_scr;
    a.flag_off = (long long)c->heap->flag_offset();
    a.start_slot = c->heap->start_slot();
    for (int r = 0; r < c->nranks; ++r) a.base[r] = c->heap->base(r);
    a.mc_base = c->heap->mc_base();
    a.control = reinterpret_cast<Control*>(c->heap->base(c->rank));
    a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
    apply_emulation_env(&a);
    if (c->trace_armed) {
      TraceLayout l = trace_layout(c);
      cudaMemsetAsync(c->trace_dev, 0, trace_words(l) * sizeof(unsigned long long), stream);
      a.trace_buf = c->trace_dev;
      a.trace_stride = l.niters * l.max_steps;
    }
    if (a.nblocks * a.nlanes > interp_max_ctas(512)) return fail(c, VB_INVALID, "too many CTAs for the device");
    cudaError_t e = launch_interp(a, stream, 512);
    if (c->trace_armed) {
      c->trace_armed = false;
      c->trace_ready = (e == cudaSuccess);
    }
    if (e != cudaSuccess) return fail(c, VB_FAILED, cudaGetErrorString(e));
    if (user_out) cudaMemcpyAsync(out, c->heap->base(c->rank) + c->stage_out, user_out, cudaMemcpyDeviceToDevice, stream);
    cudaEvent_t done;
    cudaEventCreateWithFlags(&done, cudaEventDisableTiming);
    cudaEventRecord(done, stream);
    Deadline d = Deadline::after(timeout_s + 1.0);
    while (cudaEventQuery(done) == cudaErrorNotReady) {
      if (d.expired()) {
        int one = 1;
        cudaMemcpyAsync(&a.control->abort_request, &one, sizeof one, cudaMemcpyHostToDevice, c->abort_stream);
        c->unresolved = true;
        return fail(c, VB_UNRESOLVED, "execution did not finish before its deadline");
      }
      std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
    cudaEventDestroy(done);
    Control ctl;
    cudaMemcpy(&ctl, a.control, sizeof ctl, cudaMemcpyDeviceToHost);
    if (ctl.status != ST_OK) return fail(c, VB_FAILED, "device status " + std::to_string(ctl.status));
  } catch (const std::exception& e) {
    return fail(c, VB_FAILED, e.what());
  }
  return VB_OK;
}

extern "C" vb_result vb_trace_arm(vb_context* c) {
  if (!c) return VB_INVALID;
  if (c->closed) return VB_CLOSED;
  Guard g(c);
  if (!g.ok) return VB_BUSY;
  if (!c->prepared) return fail(c, VB_INVALID, "no prepared schedule");
  TraceLayout l = trace_layout(c);
  size_t words = std::max<size_t>(trace_words(l), 3);
  cudaFree(c->trace_dev);
  c->trace_dev = nullptr;
  if (cudaMalloc(&c->trace_dev, words * sizeof(unsigned long long)) != cudaSuccess)
    return fail(c, VB_FAILED, "cannot allocate the trace buffer");
  c->trace_armed = true;
  c->trace_ready = false;
  return VB_OK;
}

extern "C" vb_result vb_trace_write(vb_context* c, const char* path) {
  if (!c || !path) return VB_INVALID;
  if (c->closed) return VB_CLOSED;
  Guard g(c);
  if (!g.ok) return VB_BUSY;
  if (!c->trace_ready) return fail(c, VB_INVALID, "no traced execution to write");
  try {
    TraceLayout l = trace_layout(c);
    std::vector<uint64_t> raw(trace_words(l));
    if (!raw.empty() &&
        cudaMemcpy(raw.data(), c->trace_dev, raw.size() * sizeof(uint64_t), cudaMemcpyDeviceToHost) != cudaSuccess)
      return fail(c, VB_FAILED, "cannot read the trace buffer");
    write_trace_file(path, l, raw);
  } catch (const std::exception& e) {
    return fail(c, VB_FAILED, e.what());
  }
  return VB_OK;
}

extern "C" vb_result vb_status(vb_context* c, int* device_status, unsigned long long* epoch) {
  if (!c) return VB_INVALID;
  if (c->closed) return VB_CLOSED;
  Control ctl;
  cudaStream_t s = c->abort_stream;
  if (cudaMemcpyAsync(&ctl, c->heap->base(c->rank), sizeof ctl, cudaMemcpyDeviceToHost, s) != cudaSuccess)
    return VB_FAILED;
  cudaStreamSynchronize(s);
  if (device_status) *device_status = ctl.status;
  if (epoch) *epoch = ctl.epoch;
  return VB_OK;
}

extern "C" vb_result vb_release(vb_context* c) {
  if (!c) return VB_INVALID;
  Guard g(c);
  if (!g.ok) return VB_BUSY;
  if (c->unresolved) return fail(c, VB_UNRESOLVED, "buffers of an unresolved execution stay owned");
  free_plan(c);
  return VB_OK;
}

extern "C" vb_result vb_close(vb_context* c, double timeout_s) {
  if (!c) return VB_INVALID;
  if (c->closed) return VB_CLOSED;
  Guard g(c);
  if (!g.ok) return VB_BUSY;
  if (c->unresolved) return fail(c, VB_UNRESOLVED, "close refused: an execution is unresolved");
  try {
    Deadline d = Deadline::after(timeout_s);
    cudaDeviceSynchronize();
    c->control->barrier("CLOSE", d);
    free_plan(c);
    c->heap->destroy();
    c->control->barrier("CLOSED", d);
  } catch (const ControlError& e) {
    return fail(c, VB_TIMEOUT, e.what());
  }
  c->closed = true;
  return VB_OK;
}

extern "C" vb_result vb_destroy(vb_context* c) {
  if (!c) return VB_INVALID;
  if (c->unresolved) return VB_UNRESOLVED;
  if (c->abort_stream) cudaStreamDestroy(c->abort_stream);
  cudaFree(c->trace_dev);
  delete c;
  return VB_OK;
}

extern "C" const char* vb_last_error(vb_context* c) { return c ? c->error.c_str() : "null context"; }
