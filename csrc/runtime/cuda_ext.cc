// PyTorch CUDA extension: symmetric heap, compiled device plans and launches.
#include <cuda_runtime.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>

#include "vb/launch.h"
#include "vb/plan.h"
#include "vb/symheap.h"

namespace py = pybind11;
using namespace vb;

namespace {

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

int elem_bytes(int dtype) { return dtype == DT_F32 ? 4 : 2; }

at::ScalarType scalar_type(int dtype) {
  switch (dtype) {
    case DT_F32: return at::kFloat;
    case DT_BF16: return at::kBFloat16;
    case DT_F16: return at::kHalf;
    default: throw std::runtime_error("unsupported dtype code");
  }
}

int dtype_code(at::ScalarType t) {
  if (t == at::kFloat) return DT_F32;
  if (t == at::kBFloat16) return DT_BF16;
  if (t == at::kHalf) return DT_F16;
  throw std::runtime_error("unsupported tensor dtype (float32, bfloat16, float16)");
}

template <typename T>
T* upload(const std::vector<T>& v) {
  if (v.empty()) return nullptr;
  T* p = nullptr;
  cuda_check(cudaMalloc(&p, v.size() * sizeof(T)), "cudaMalloc plan table");
  cuda_check(cudaMemcpy(p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice), "upload plan table");
  return p;
}

class Heap {
 public:
  Heap(int rank, int nranks, int device, size_t bytes, const std::string& session, bool multicast)
      : h_(std::make_unique<SymHeap>(rank, nranks, device, bytes, session, multicast)) {}
  SymHeap& get() { return *h_; }
  Control* control() { return reinterpret_cast<Control*>(h_->base(h_->rank())); }

  py::dict status() {
    Control c;
    cuda_check(cudaMemcpy(&c, control(), sizeof(Control), cudaMemcpyDeviceToHost), "read control block");
    py::dict d;
    d["epoch"] = c.epoch;
    d["status"] = c.status;
    d["detail"] = py::make_tuple(c.detail[0], c.detail[1], c.detail[2], c.detail[3]);
    d["arrive"] = c.arrive;
    d["ll_seq"] = c.ll_seq;
    return d;
  }

  void clear_status() {
    cuda_check(cudaMemset(&control()->status, 0, sizeof(int) * 5), "clear status");
    cuda_check(cudaMemset(&control()->abort_request, 0, sizeof(int)), "clear abort");
  }

  torch::Tensor tensor(size_t offset, int64_t numel, int dtype) {
    if (offset + (size_t)numel * elem_bytes(dtype) > h_->size()) throw std::runtime_error("tensor exceeds the heap");
    auto opts = torch::TensorOptions().dtype(scalar_type(dtype)).device(torch::kCUDA, h_->device());
    return torch::from_blob(h_->base(h_->rank()) + offset, {numel}, opts);
  }

  size_t offset_of(const torch::Tensor& t) {
    auto p = reinterpret_cast<char*>(t.data_ptr());
    char* b = h_->base(h_->rank());
    if (p < b || p >= b + h_->size()) throw std::runtime_error("tensor is not inside the symmetric heap");
    return (size_t)(p - b);
  }

 private:
  std::unique_ptr<SymHeap> h_;
};

struct BoundLaunch {
  InterpArgs args;
  int threads;
  void launch(uint64_t stream) {
    cuda_check(launch_interp(args, reinterpret_cast<cudaStream_t>(stream), threads), "launch interpreter");
  }
};

struct BoundOneShot {
  OneShotArgs args;
  void launch(uint64_t stream) {
    cuda_check(launch_oneshot(args, reinterpret_cast<cudaStream_t>(stream)), "launch one-shot collective");
  }
};

// Validated arguments of a one-shot launch: offsets inside the heap, 8-byte payload units, 16-byte lines.
BoundOneShot bind_oneshot(Heap& heap, size_t in_off, size_t out_off, size_t ll_off, int64_t ll_src_bytes,
                          int64_t bytes, int dtype, int redop, int coll, float scale, bool do_scale,
                          double timeout_s, bool multicast) {
  SymHeap& h = heap.get();
  if (coll != OS_ALLREDUCE && coll != OS_ALLGATHER && coll != OS_ALLREDUCE_TWOSHOT)
    throw std::runtime_error("one-shot: unknown collective");
  if (dtype != DT_F32 && dtype != DT_BF16 && dtype != DT_F16) throw std::runtime_error("one-shot: unsupported dtype");
  if (bytes <= 0 || bytes % 8) throw std::runtime_error("one-shot: payload must be a positive multiple of 8 bytes");
  if (in_off % 8 || out_off % 8) throw std::runtime_error("one-shot: buffers must be 8-byte aligned");
  if (ll_off % 16 || ll_src_bytes % 16) throw std::runtime_error("one-shot: LL region misaligned");
  if (coll == OS_ALLREDUCE_TWOSHOT) {
    if (bytes % (8ll * h.nranks())) throw std::runtime_error("two-shot: payload must split into 8-byte units per rank");
    if (4 * bytes > (int64_t)h.nranks() * ll_src_bytes) throw std::runtime_error("two-shot: LL region too small");
  } else if (ll_src_bytes < 2 * bytes) {
    throw std::runtime_error("one-shot: LL region too small for this payload");
  }
  const size_t out_bytes = (size_t)bytes * (coll == OS_ALLGATHER ? h.nranks() : 1);
  if (in_off + (size_t)bytes > h.size() || out_off + out_bytes > h.size() ||
      ll_off + 2 * (size_t)h.nranks() * (size_t)ll_src_bytes > h.size())
    throw std::runtime_error("one-shot: buffer exceeds the heap");
  if (in_off < kReservedBytes || out_off < kReservedBytes || ll_off < kReservedBytes)
    throw std::runtime_error("one-shot: buffer overlaps the control block or flag table");
  BoundOneShot b;
  OneShotArgs& a = b.args;
  a = OneShotArgs{};
  for (int r = 0; r < h.nranks(); ++r) a.base[r] = h.base(r);
  a.in_off = (long long)in_off;
  a.out_off = (long long)out_off;
  a.ll_off = (long long)ll_off;
  a.ll_src_bytes = ll_src_bytes;
  a.bytes = bytes;
  a.rank = h.rank();
  a.nranks = h.nranks();
  a.dtype = dtype;
  a.redop = redop;
  a.coll = coll;
  a.scale = scale;
  a.do_scale = do_scale ? 1 : 0;
  a.control = heap.control();
  a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  if (multicast && h.mc_base() == nullptr) throw std::runtime_error("one-shot: the heap has no multicast mapping");
  a.mc_base = multicast ? h.mc_base() : nullptr;
  return b;
}

class DevicePlan {
 public:
  DevicePlan(const std::string& xml, int rank, int nlanes, int niters, bool elide, bool fuse, bool multicast,
             bool reducing, int mc_keep, int mc_period, bool merge, bool push)
      : rank_(rank) {
    CompileOptions o;
    o.merge_blocks = merge;
    o.push = push;
    o.nlanes = nlanes;
    o.niters = niters;
    o.elide_sends = elide;
    o.fuse_chains = fuse;
    o.multicast = multicast;
    o.reducing = reducing;
    o.mc_keep = mc_keep;
    o.mc_period = mc_period;
    plan_ = compile_plan(parse_xml(xml), o);
    if (rank < 0 || rank >= (int)plan_.ranks.size()) throw std::runtime_error("rank outside the plan");
    const RankProgram& rp = plan_.ranks[rank];
    if (plan_.max_blocks() > kMaxFlagBlocks) throw std::runtime_error("plan has more blocks than the flag table holds");
    blocks_ = upload(rp.blocks);
    steps_ = upload(rp.steps);
    srcs_ = upload(rp.srcs);
    waits_ = upload(rp.waits);
    nblocks_ = (int)rp.blocks.size();
  }
  ~DevicePlan() {
    cudaFree(blocks_);
    cudaFree(steps_);
    cudaFree(srcs_);
    cudaFree(waits_);
  }

  py::tuple geometry(int64_t count_per_rank, int dtype) const {
    long long runtime = count_per_rank * ((plan_.algo.coll == "allgather" || plan_.algo.coll == "gather") ? plan_.ranks.size() : 1);
    long long nch = plan_.algo.nchunksperloop;
    if (runtime % nch) throw std::runtime_error("element count does not split into nchunksperloop chunks");
    long long chunk = runtime / nch;
    int vec = 16 / elem_bytes(dtype);
    if (chunk % vec) throw std::runtime_error("chunk is not a whole number of 16-byte vectors");
    long long pieces = (long long)plan_.options.nlanes * plan_.options.niters;
    long long piece = (chunk + pieces - 1) / pieces;
    piece = (piece + vec - 1) / vec * vec;
    return py::make_tuple(chunk, piece);
  }

  void run(Heap& heap, size_t in_off, size_t out_off, size_t scr_off, int64_t count_per_rank, int dtype, int redop,
           float scale, uint64_t stream, double timeout_s, int threads, int nbatch,
           std::vector<long long> batch_stride, uint64_t trace_ptr, int64_t trace_stride) {
    InterpArgs a = bind(heap, in_off, out_off, scr_off, count_per_rank, dtype, redop, scale, timeout_s, threads, nbatch,
                        batch_stride, trace_ptr, trace_stride);
    cuda_check(launch_interp(a, reinterpret_cast<cudaStream_t>(stream), threads), "launch interpreter");
  }

  // Validated launch arguments for repeated launches of the same buffers (no per-launch checks).
  InterpArgs bind(Heap& heap, size_t in_off, size_t out_off, size_t scr_off, int64_t count_per_rank, int dtype,
                  int redop, float scale, double timeout_s, int threads, int nbatch,
                  std::vector<long long> batch_stride, uint64_t trace_ptr, int64_t trace_stride) {
    SymHeap& h = heap.get();
    if (h.nranks() != (int)plan_.ranks.size()) throw std::runtime_error("heap and plan rank counts differ");
    py::tuple g = geometry(count_per_rank, dtype);
    InterpArgs a = {};
    a.blocks = blocks_;
    a.steps = steps_;
    a.srcs = srcs_;
    a.waits = waits_;
    a.nblocks = nblocks_;
    a.nlanes = plan_.options.nlanes;
    a.niters = plan_.options.niters;
    a.rank = rank_;
    a.nranks = h.nranks();
    a.dtype = dtype;
    a.redop = redop;
    a.scale = scale;
    a.chunk_elems = g[0].cast<long long>();
    a.piece_elems = g[1].cast<long long>();
    a.buf_off[BUF_IN] = (long long)in_off;
    a.buf_off[BUF_OUT] = (long long)out_off;
    a.buf_off[BUF_SCR] = (long long)scr_off;
    if (nbatch < 1 || batch_stride.size() != 3) throw std::runtime_error("invalid batch description");
    a.nbatch = nbatch;
    for (int b = 0; b < 3; ++b) a.batch_stride[b] = batch_stride[b];
    const RankProgram& rp = plan_.ranks[rank_];
    size_t esz = elem_bytes(dtype);
    auto need = [&](size_t off, int chunks, long long stride, const char* name) {
      size_t last = off + (size_t)(nbatch - 1) * (size_t)stride;
      if (chunks && last + (size_t)chunks * a.chunk_elems * esz > h.size())
        throw std::runtime_error(std::string(name) + " buffer exceeds the heap");
      if (off % 16 || stride % 16 || stride < 0) throw std::runtime_error(std::string(name) + " buffer is not 16-byte aligned");
    };
    need(in_off, rp.i_chunks, a.batch_stride[BUF_IN], "input");
    need(out_off, rp.o_chunks, a.batch_stride[BUF_OUT], "output");
    need(scr_off, plan_.max_scratch_used(), a.batch_stride[BUF_SCR], "scratch");
    a.flag_off = (long long)h.flag_offset();
    a.start_slot = h.start_slot();
    for (int r = 0; r < h.nranks(); ++r) a.base[r] = h.base(r);
    a.mc_base = h.mc_base();
    if (plan_.stats.multicast_ops > 0 && a.mc_base == nullptr)
      throw std::runtime_error("the plan uses NVLS multicast but the heap has no multicast mapping");
    a.control = heap.control();
    a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
    a.trace_buf = reinterpret_cast<unsigned long long*>(trace_ptr);
    apply_emulation_env(&a);
    a.trace_stride = (int)trace_stride;
    int max_ctas = interp_max_ctas(threads);
    if (a.nblocks * a.nlanes > max_ctas)
      throw std::runtime_error("plan needs " + std::to_string(a.nblocks * a.nlanes) + " co-resident CTAs; the device holds " +
                               std::to_string(max_ctas));
    return a;
  }

  int nblocks() const { return nblocks_; }
  int nlanes() const { return plan_.options.nlanes; }
  int niters() const { return plan_.options.niters; }
  py::tuple slots() const {
    const RankProgram& rp = plan_.ranks[rank_];
    // scratch: chunks every rank reserves (symmetric), only those device steps use
    return py::make_tuple(rp.i_chunks, rp.o_chunks, plan_.max_scratch_used());
  }
  std::string describe() const { return describe_rank(plan_, rank_); }
  int max_steps() const {
    int m = 0;
    for (auto& b : plan_.ranks[rank_].blocks) m = b.nsteps > m ? b.nsteps : m;
    return m;
  }
  std::vector<int> step_ops() const {
    std::vector<int> out;
    const RankProgram& rp = plan_.ranks[rank_];
    if (!rp.blocks.empty())
      for (int s = 0; s < rp.blocks[0].nsteps; ++s) out.push_back(rp.steps[rp.blocks[0].step_begin + s].op);
    return out;
  }
  // (XML thread block id, XML step index) of every device step, per block ({-1, -1}: compiler-made step).
  std::vector<std::vector<std::array<int, 2>>> step_origins() const {
    std::vector<std::vector<std::array<int, 2>>> out;
    const RankProgram& rp = plan_.ranks[rank_];
    for (const auto& b : rp.blocks)
      out.emplace_back(rp.step_origins.begin() + b.step_begin, rp.step_origins.begin() + b.step_begin + b.nsteps);
    return out;
  }
  // Opcode of every step, per block (the trace buffer indexes a CTA's records by its block's step count).
  std::vector<std::vector<int>> block_ops() const {
    std::vector<std::vector<int>> out;
    const RankProgram& rp = plan_.ranks[rank_];
    for (const auto& b : rp.blocks) {
      std::vector<int> ops;
      for (int s = 0; s < b.nsteps; ++s) ops.push_back(rp.steps[b.step_begin + s].op);
      out.push_back(std::move(ops));
    }
    return out;
  }
  py::dict stats() const {
    py::dict d;
    d["device_steps"] = plan_.stats.device_steps;
    d["elided_blocks"] = plan_.stats.elided_blocks;
    d["fused_reduces"] = plan_.stats.fused_reduces;
    d["waits"] = plan_.stats.waits;
    d["remote_waits"] = plan_.stats.remote_waits;
    d["fused"] = plan_.options.fuse_chains;
    d["multicast_ops"] = plan_.stats.multicast_ops;
    d["deferred_waits"] = plan_.stats.deferred_waits;
    d["dropped_nops"] = plan_.stats.dropped_nops;
    d["staged_forwards"] = plan_.stats.staged_forwards;
    d["pushes"] = plan_.stats.pushes;
    return d;
  }

 private:
  CompiledPlan plan_;
  int rank_, nblocks_ = 0;
  DevBlock* blocks_ = nullptr;
  DevStep* steps_ = nullptr;
  DevSrc* srcs_ = nullptr;
  DevWait* waits_ = nullptr;
};

}  // namespace

PYBIND11_MODULE(_vbcuda, m) {
  m.doc() = "vericcl_b200 CUDA runtime: symmetric heap, schedule interpreter, helper kernels";
  py::class_<Heap>(m, "Heap")
      .def(py::init<int, int, int, size_t, const std::string&, bool>())
      .def("exchange", [](Heap& h, double t) { py::gil_scoped_release r; h.get().exchange(t); })
      .def("bind_multicast", [](Heap& h) { h.get().bind_multicast(); })
      .def("finish", [](Heap& h) { h.get().finish(); })
      .def("destroy", [](Heap& h) { h.get().destroy(); })
      .def("alloc", [](Heap& h, size_t b) { return h.get().alloc(b); })
      .def("free", [](Heap& h, size_t o) { h.get().free(o); })
      .def("used", [](Heap& h) { return h.get().used(); })
      .def("tensor", &Heap::tensor)
      .def("offset_of", &Heap::offset_of)
      .def("status", &Heap::status)
      .def("clear_status", &Heap::clear_status)
      .def_property_readonly("size", [](Heap& h) { return h.get().size(); })
      .def_property_readonly("multicast", [](Heap& h) { return h.get().multicast(); })
      .def("base", [](Heap& h, int r) { return (uint64_t)h.get().base(r); });
  py::class_<BoundLaunch>(m, "BoundLaunch").def("launch", &BoundLaunch::launch);
  py::class_<BoundOneShot>(m, "BoundOneShot").def("launch", &BoundOneShot::launch);
  m.def("bind_oneshot", &bind_oneshot, py::arg("heap"), py::arg("in_off"), py::arg("out_off"), py::arg("ll_off"),
        py::arg("ll_src_bytes"), py::arg("bytes"), py::arg("dtype"), py::arg("redop"), py::arg("coll"),
        py::arg("scale"), py::arg("do_scale"), py::arg("timeout_s"), py::arg("multicast") = false);
  m.def("oneshot_region_bytes", [](int nranks, int64_t max_bytes) { return oneshot_region_bytes(nranks, max_bytes); });
  m.def("push_allgather_max_ctas", []() { return push_allgather_max_ctas(); });
  // Push AllGather: `inp` (bytes per rank, local device memory) into the heap output at out_off on every rank.
  m.def("push_allgather", [](Heap& heap, uint64_t in_ptr, size_t out_off, int64_t bytes, size_t flag_off, int ctas,
                             double timeout_s, bool fanout) {
    SymHeap& h = heap.get();
    TORCH_CHECK(bytes > 0 && bytes % 16 == 0, "push AllGather needs a positive multiple of 16 bytes per rank");
    TORCH_CHECK(out_off >= kReservedBytes && flag_off >= kReservedBytes, "region overlaps the control block");
    TORCH_CHECK(out_off + (size_t)bytes * h.nranks() <= h.size() && flag_off + 8 * (size_t)(ctas + 1) <= h.size(),
                "push AllGather output or flags exceed the heap");
    PushAgArgs a{};
    for (int r = 0; r < h.nranks(); ++r) a.base[r] = h.base(r);
    a.in = reinterpret_cast<const void*>(in_ptr);
    a.out_off = (long long)out_off;
    a.bytes = bytes;
    a.flag_off = (long long)flag_off;
    a.rank = h.rank();
    a.nranks = h.nranks();
    a.ctas = ctas;
    a.fanout = fanout ? 1 : 0;
    a.control = heap.control();
    a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
    cuda_check(launch_push_allgather(a, at::cuda::getCurrentCUDAStream().stream()), "push AllGather launch");
  }, py::arg("heap"), py::arg("in_ptr"), py::arg("out_off"), py::arg("bytes"), py::arg("flag_off"), py::arg("ctas"),
     py::arg("timeout_s") = 10.0, py::arg("fanout") = false);
  m.def("fp8_stage_bytes", [](int64_t n) { return fp8_stage_bytes(n); });
  m.def("fp8_allgather_max_ctas", []() { return fp8_allgather_max_ctas(); });
  // Fused block-scaled FP8 AllGather over the heap's peer mappings: `in` (n elements) and `out`
  // (nranks * n) may be any device tensors; the staging parities and the per-CTA flags are heap regions
  // reserved at the same offsets on every rank.
  m.def("fp8_allgather", [](Heap& heap, torch::Tensor in, torch::Tensor out, size_t stage_off, size_t flag_off,
                            int ctas, double timeout_s) {
    SymHeap& h = heap.get();
    TORCH_CHECK(in.is_cuda() && out.is_cuda() && in.is_contiguous() && out.is_contiguous(), "contiguous CUDA tensors");
    TORCH_CHECK(in.scalar_type() == out.scalar_type(), "input and output dtypes differ");
    TORCH_CHECK(out.numel() == in.numel() * h.nranks(), "output must hold nranks x input elements");
    const int64_t n = in.numel();
    TORCH_CHECK(n > 0 && n % 16 == 0, "fp8 AllGather needs a positive multiple of 16 elements per rank");
    TORCH_CHECK(stage_off >= kReservedBytes && flag_off >= kReservedBytes, "region overlaps the control block");
    TORCH_CHECK(stage_off + 2 * (size_t)fp8_stage_bytes(n) <= h.size() && flag_off + 8 * (size_t)ctas <= h.size(),
                "fp8 staging or flags exceed the heap");
    Fp8AgArgs a{};
    for (int r = 0; r < h.nranks(); ++r) a.base[r] = h.base(r);
    a.in = in.data_ptr();
    a.out = out.data_ptr();
    a.n = n;
    a.stage_off = (long long)stage_off;
    a.flag_off = (long long)flag_off;
    a.rank = h.rank();
    a.nranks = h.nranks();
    a.dtype = dtype_code(in.scalar_type());
    a.ctas = ctas;
    a.control = heap.control();
    a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
    cuda_check(launch_fp8_allgather(a, at::cuda::getCurrentCUDAStream().stream()), "fp8 AllGather launch");
  }, py::arg("heap"), py::arg("inp"), py::arg("out"), py::arg("stage_off"), py::arg("flag_off"), py::arg("ctas"),
     py::arg("timeout_s") = 10.0);
  py::class_<DevicePlan>(m, "DevicePlan")
      .def(py::init<const std::string&, int, int, int, bool, bool, bool, bool, int, int, bool, bool>(), py::arg("xml"),
           py::arg("rank"), py::arg("nlanes"), py::arg("niters"), py::arg("elide"), py::arg("fuse"),
           py::arg("multicast"), py::arg("reducing"), py::arg("mc_keep") = 1, py::arg("mc_period") = 1,
           py::arg("merge") = true, py::arg("push") = false)
      .def("run", &DevicePlan::run, py::arg("heap"), py::arg("in_off"), py::arg("out_off"), py::arg("scr_off"),
           py::arg("count_per_rank"), py::arg("dtype"), py::arg("redop"), py::arg("scale"), py::arg("stream"),
           py::arg("timeout_s") = 10.0, py::arg("threads") = 512, py::arg("nbatch") = 1,
           py::arg("batch_stride") = std::vector<long long>{0, 0, 0}, py::arg("trace_ptr") = 0,
           py::arg("trace_stride") = 0)
      .def("bind", [](DevicePlan& p, Heap& heap, size_t in_off, size_t out_off, size_t scr_off, int64_t count, int dtype,
                      int redop, float scale, double timeout_s, int threads, int nbatch,
                      std::vector<long long> strides, uint64_t timeline_ptr, bool lean, int bulk) {
        InterpArgs a = p.bind(heap, in_off, out_off, scr_off, count, dtype, redop, scale, timeout_s, threads, nbatch,
                              strides, 0, 0);
        if ((timeline_ptr || lean) && redop != RED_SUM)
          throw std::runtime_error("the launch timeline and the lean kernel cover sum/avg reductions and copies");
        a.timeline = reinterpret_cast<unsigned long long*>(timeline_ptr);
        a.lean = lean ? 1 : 0;
        a.bulk = bulk & 3;
        if (bulk && timeline_ptr) throw std::runtime_error("the launch timeline has no TMA-staged kernel instance");
        return BoundLaunch{a, threads};
      }, py::arg("heap"), py::arg("in_off"), py::arg("out_off"), py::arg("scr_off"), py::arg("count"),
         py::arg("dtype"), py::arg("redop"), py::arg("scale"), py::arg("timeout_s"), py::arg("threads"),
         py::arg("nbatch"), py::arg("strides"), py::arg("timeline_ptr") = 0, py::arg("lean") = false,
         py::arg("bulk") = 0)
      .def("geometry", &DevicePlan::geometry)
      .def("slots", &DevicePlan::slots)
      .def("describe", &DevicePlan::describe)
      .def("stats", &DevicePlan::stats)
      .def("max_steps", &DevicePlan::max_steps)
      .def("step_ops", &DevicePlan::step_ops)
      .def("block_ops", &DevicePlan::block_ops)
      .def("step_origins", &DevicePlan::step_origins)
      .def_property_readonly("nblocks", &DevicePlan::nblocks)
      .def_property_readonly("nlanes", &DevicePlan::nlanes)
      .def_property_readonly("niters", &DevicePlan::niters);
  m.def("max_ctas", [](int threads) { return interp_max_ctas(threads); }, py::arg("threads") = 512);
  // Launches a one-step program whose only wait targets an event this CTA would publish later:
  // nothing ever sets it, so the bounded wait must expire and report ST_TIMEOUT.  Every address is
  // local and valid; used by the failure-detection test.
  m.def("wait_probe", [](Heap& heap, double timeout_s) {
    SymHeap& h = heap.get();
    std::vector<DevBlock> blocks(1);
    blocks[0] = DevBlock{0, 1, -1, 0, 0};
    std::vector<DevStep> steps(1);
    steps[0] = DevStep{};
    steps[0].dst_rank = -1;
    steps[0].op = OP_NOP;
    steps[0].cnt = 1;
    steps[0].wait_begin = 0;
    steps[0].wait_count = 1;
    std::vector<DevWait> waits(1);
    waits[0] = DevWait{(int16_t)h.rank(), 0, 2, 2, 0};   // this block's own completion event: never ahead of itself
    DevBlock* b = upload(blocks);
    DevStep* st = upload(steps);
    DevWait* w = upload(waits);
    InterpArgs a = {};
    a.blocks = b; a.steps = st; a.waits = w; a.srcs = nullptr;
    a.nblocks = 1; a.nlanes = 1; a.niters = 1; a.nbatch = 1; a.rank = h.rank(); a.nranks = h.nranks();
    a.dtype = DT_F32; a.redop = RED_SUM; a.scale = 1.f; a.chunk_elems = 4; a.piece_elems = 4;
    a.flag_off = (long long)h.flag_offset();
    a.start_slot = h.start_slot();
    for (int r = 0; r < h.nranks(); ++r) a.base[r] = h.base(r);
    a.control = heap.control();
    a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
    cuda_check(launch_interp(a, at::cuda::getCurrentCUDAStream().stream(), 64), "wait probe");
    cuda_check(cudaStreamSynchronize(at::cuda::getCurrentCUDAStream().stream()), "wait probe sync");
    cudaFree(b); cudaFree(st); cudaFree(w);
    return heap.status();
  });
  m.def("fill", [](torch::Tensor t, int pattern, int rank, uint64_t seed) {
    cuda_check(launch_fill(t.data_ptr(), t.numel(), dtype_code(t.scalar_type()), pattern, rank, seed,
                           at::cuda::getCurrentCUDAStream().stream()), "fill");
  });
  m.def("scale", [](torch::Tensor dst, torch::Tensor src, float s) {
    cuda_check(launch_scale(dst.data_ptr(), src.data_ptr(), dst.numel(), dtype_code(dst.scalar_type()), s,
                            at::cuda::getCurrentCUDAStream().stream()), "scale");
  });
  m.def("strided_copy", [](torch::Tensor dst, torch::Tensor src) {
    // 2D tensors of one dtype and shape whose rows are contiguous (stride(1) == 1)
    if (dst.dim() != 2 || src.dim() != 2 || dst.sizes() != src.sizes() || dst.scalar_type() != src.scalar_type())
      throw std::runtime_error("strided_copy needs 2D tensors of the same shape and dtype");
    if (!dst.is_cuda() || !src.is_cuda() || (dst.size(1) > 1 && (dst.stride(1) != 1 || src.stride(1) != 1)))
      throw std::runtime_error("strided_copy needs CUDA tensors with contiguous rows");
    int64_t es = dst.element_size();
    cuda_check(launch_strided_copy(dst.data_ptr(), dst.stride(0) * es, src.data_ptr(), src.stride(0) * es,
                                   dst.size(1) * es, dst.size(0), at::cuda::getCurrentCUDAStream().stream()),
               "strided_copy");
  }, py::arg("dst"), py::arg("src"));
  m.def("check", [](torch::Tensor out, int coll, int redop, int nranks, int rank, int64_t count, double atol, double rtol) {
    auto bad = torch::zeros({1}, torch::TensorOptions().dtype(torch::kInt64).device(out.device()));
    cuda_check(launch_check(out.data_ptr(), out.numel(), dtype_code(out.scalar_type()), coll, redop, nranks, rank, count,
                            atol, rtol, reinterpret_cast<unsigned long long*>(bad.data_ptr()),
                            at::cuda::getCurrentCUDAStream().stream()), "check");
    return bad;
  });
  m.def("copy_probe", [](uint64_t dst, uint64_t src, int64_t bytes, int ctas, int threads, int unroll) {
    cuda_check(launch_copy_probe(reinterpret_cast<void*>(dst), reinterpret_cast<const void*>(src), bytes, ctas, threads,
                                 unroll, at::cuda::getCurrentCUDAStream().stream()), "copy probe");
  });
  // dst = scale? * op(srcs[0], ..., srcs[K-1]) on this GPU through the interpreter kernel: a one-rank,
  // one-step program whose step reads K chunks of `srcs` ([K, n], contiguous).  This is the n-ary local reduce
  // of a single-rank schedule (the reference's onerank reduce, third_party/msccl/src/collectives/device/
  // onerank_reduce.cu:13-41, generalised to K sources); it runs the same move paths as a K-source pull reduce.
  m.def("local_reduce", [](torch::Tensor dst, torch::Tensor srcs, int redop, double scale, bool do_scale, int lanes,
                           int iters, bool lean, int bulk) {
    TORCH_CHECK(srcs.is_cuda() && dst.is_cuda() && srcs.is_contiguous() && dst.is_contiguous(), "contiguous CUDA tensors");
    TORCH_CHECK(srcs.dim() == 2 && srcs.size(1) == dst.numel() && srcs.scalar_type() == dst.scalar_type(),
                "srcs must be [K, dst.numel()] of dst's dtype");
    const int dtype = dtype_code(dst.scalar_type());
    const int64_t k = srcs.size(0), n = dst.numel(), vec = 16 / elem_bytes(dtype);
    TORCH_CHECK(k >= 1 && k <= 16 && n > 0 && n % vec == 0, "1..16 sources of a multiple of 16 bytes each");
    TORCH_CHECK(lanes >= 1 && iters >= 1 && redop >= RED_SUM && redop <= RED_MAX, "bad geometry or reduction");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(srcs.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(dst.data_ptr()) % 16 == 0,
                "16-byte aligned buffers");
    TORCH_CHECK(lanes <= interp_max_ctas(512) && lanes <= kMaxFlagLanes, "more lanes than co-resident CTAs");
    // workspace: [0, 256) control | [256, ...) flags of one block | [8192, ...) program tables
    const int64_t table_off = 8192;
    const int64_t bytes = table_off + sizeof(DevBlock) + sizeof(DevStep) + k * sizeof(DevSrc);
    auto ws = torch::zeros({(bytes + 255) / 256 * 256}, torch::TensorOptions().dtype(torch::kUInt8).device(dst.device()));
    char* w = reinterpret_cast<char*>(ws.data_ptr());
    std::vector<char> host(bytes - table_off);
    DevBlock blk{0, 1, -1, 0, 0};
    DevStep st{};
    st.dst_rank = -1;
    st.op = k == 1 ? OP_COPY : OP_REDUCE;
    st.dst_buf = BUF_OUT;
    st.flags = do_scale ? F_SCALE : 0;
    st.cnt = 1;
    st.nsrc = (int32_t)k;
    std::vector<DevSrc> src(k);
    for (int64_t i = 0; i < k; ++i) src[i] = DevSrc{0, BUF_IN, 0, (int32_t)i};
    std::memcpy(host.data(), &blk, sizeof blk);
    std::memcpy(host.data() + sizeof blk, &st, sizeof st);
    std::memcpy(host.data() + sizeof blk + sizeof st, src.data(), k * sizeof(DevSrc));
    auto stream = at::cuda::getCurrentCUDAStream().stream();
    const unsigned long long epoch = 1;
    cuda_check(cudaMemcpyAsync(w + offsetof(Control, epoch), &epoch, sizeof epoch, cudaMemcpyHostToDevice, stream), "epoch");
    cuda_check(cudaMemcpyAsync(w + table_off, host.data(), host.size(), cudaMemcpyHostToDevice, stream), "tables");
    InterpArgs a{};
    a.blocks = reinterpret_cast<const DevBlock*>(w + table_off);
    a.steps = reinterpret_cast<const DevStep*>(w + table_off + sizeof(DevBlock));
    a.srcs = reinterpret_cast<const DevSrc*>(w + table_off + sizeof(DevBlock) + sizeof(DevStep));
    a.nblocks = 1;
    a.nlanes = lanes;
    a.niters = iters;
    a.nbatch = 1;
    a.rank = 0;
    a.nranks = 1;
    a.dtype = dtype;
    a.redop = redop;
    a.scale = (float)scale;
    a.chunk_elems = n;
    const int64_t pieces = (int64_t)lanes * iters;
    a.piece_elems = ((n + pieces - 1) / pieces + vec - 1) / vec * vec;
    // offsets are relative to the workspace, which stands in for this rank's heap base
    a.buf_off[BUF_IN] = (long long)(reinterpret_cast<char*>(srcs.data_ptr()) - w);
    a.buf_off[BUF_OUT] = (long long)(reinterpret_cast<char*>(dst.data_ptr()) - w);
    a.buf_off[BUF_SCR] = a.buf_off[BUF_OUT];
    a.flag_off = 256;
    a.start_slot = kMaxFlagLanes;
    a.base[0] = w;
    a.control = reinterpret_cast<Control*>(w);
    a.timeout_ns = 10ull * 1000000000ull;
    a.lean = lean ? 1 : 0;
    a.bulk = bulk & 3;
    cuda_check(launch_interp(a, stream, 512), "local reduce launch");
    return ws;   // keeps the workspace alive until the caller drops it; its first int words hold the status
  }, py::arg("dst"), py::arg("srcs"), py::arg("redop") = 0, py::arg("scale") = 1.0, py::arg("do_scale") = false,
     py::arg("lanes") = 1, py::arg("iters") = 1, py::arg("lean") = false, py::arg("bulk") = 0);
  m.def("reduce_probe", [](uint64_t dst, std::vector<uint64_t> srcs, int64_t bytes, int ctas, int threads) {
    std::vector<const void*> p;
    for (auto s : srcs) p.push_back(reinterpret_cast<const void*>(s));
    cuda_check(launch_reduce_probe(reinterpret_cast<void*>(dst), p.data(), (int)p.size(), bytes, ctas, threads,
                                   at::cuda::getCurrentCUDAStream().stream()), "reduce probe");
  });
  m.def("quantize_fp8", [](torch::Tensor in, torch::Tensor q, torch::Tensor scales, int block) {
    cuda_check(launch_quantize_fp8(in.data_ptr(), reinterpret_cast<unsigned char*>(q.data_ptr()),
                                   reinterpret_cast<float*>(scales.data_ptr()), in.numel(), block,
                                   dtype_code(in.scalar_type()), at::cuda::getCurrentCUDAStream().stream()),
               "quantize fp8");
  });
  m.def("dequantize_fp8", [](torch::Tensor q, torch::Tensor scales, torch::Tensor out, int block) {
    cuda_check(launch_dequantize_fp8(reinterpret_cast<const unsigned char*>(q.data_ptr()),
                                     reinterpret_cast<const float*>(scales.data_ptr()), out.data_ptr(), out.numel(),
                                     block, dtype_code(out.scalar_type()), at::cuda::getCurrentCUDAStream().stream()),
               "dequantize fp8");
  });
  m.def("enable_peer_access", [](int device, int peer) {
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) { cudaGetLastError(); e = cudaSuccess; }
    cudaSetDevice(cur);
    cuda_check(e, "enable peer access");
  });
  m.def("read_timer", [](torch::Tensor dst) {
    cuda_check(launch_read_timer(reinterpret_cast<unsigned long long*>(dst.data_ptr()),
                                 at::cuda::getCurrentCUDAStream().stream()), "timer");
  });
}
