// Python bindings of the schedule compiler and the CPU interpreter.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstring>

#include "vb/plan.h"

namespace py = pybind11;
using namespace vb;

namespace {

py::dict stats_dict(const CompileStats& s) {
  py::dict d;
  d["xml_steps"] = s.xml_steps;
  d["device_steps"] = s.device_steps;
  d["elided_blocks"] = s.elided_blocks;
  d["fused_reduces"] = s.fused_reduces;
  d["multicast_ops"] = s.multicast_ops;
  d["waits"] = s.waits;
  d["remote_waits"] = s.remote_waits;
  d["scale_steps"] = s.scale_steps;
  d["deferred_waits"] = s.deferred_waits;
  d["dropped_nops"] = s.dropped_nops;
  d["staged_forwards"] = s.staged_forwards;
  d["pushes"] = s.pushes;
  return d;
}

template <typename T>
py::bytes as_bytes(const std::vector<T>& v) {
  return py::bytes(reinterpret_cast<const char*>(v.data()), v.size() * sizeof(T));
}

void fill(std::vector<std::vector<unsigned char>>& dst, const py::list& src) {
  dst.clear();
  for (auto item : src) {
    py::buffer_info info = py::cast<py::buffer>(item).request();
    size_t n = (size_t)info.size * (size_t)info.itemsize;
    std::vector<unsigned char> v(n);
    if (n) std::memcpy(v.data(), info.ptr, n);
    dst.push_back(std::move(v));
  }
}

void drain(const std::vector<std::vector<unsigned char>>& src, const py::list& dst) {
  for (size_t i = 0; i < src.size(); ++i) {
    py::buffer_info info = py::cast<py::buffer>(dst[i]).request(true);
    size_t n = (size_t)info.size * (size_t)info.itemsize;
    if (n != src[i].size()) throw std::runtime_error("buffer size changed");
    if (n) std::memcpy(info.ptr, src[i].data(), n);
  }
}

}  // namespace

PYBIND11_MODULE(_vbplan, m) {
  m.doc() = "vericcl_b200 schedule compiler and CPU interpreter";
  py::register_exception<CompileError>(m, "CompileError");
  py::class_<CompiledPlan>(m, "CompiledPlan")
      .def_property_readonly("ranks", [](const CompiledPlan& p) { return (int)p.ranks.size(); })
      .def_property_readonly("nlanes", [](const CompiledPlan& p) { return p.options.nlanes; })
      .def_property_readonly("niters", [](const CompiledPlan& p) { return p.options.niters; })
      .def_property_readonly("nchunks", [](const CompiledPlan& p) { return p.algo.nchunksperloop; })
      .def_property_readonly("collective", [](const CompiledPlan& p) { return p.algo.coll; })
      .def_property_readonly("inplace", [](const CompiledPlan& p) { return (bool)p.algo.inplace; })
      .def_property_readonly("max_blocks", &CompiledPlan::max_blocks)
      .def_property_readonly("fused", [](const CompiledPlan& p) { return p.options.fuse_chains; })
      .def_property_readonly("stats", [](const CompiledPlan& p) { return stats_dict(p.stats); })
      .def("blocks", [](const CompiledPlan& p, int r) { return (int)p.ranks.at(r).blocks.size(); })
      .def("slots", [](const CompiledPlan& p, int r) {
        const RankProgram& rp = p.ranks.at(r);
        return py::make_tuple(rp.i_chunks, rp.o_chunks, rp.s_chunks);
      })
      .def_property_readonly("scratch_used", &CompiledPlan::max_scratch_used)
      .def("describe", [](const CompiledPlan& p, int r) { return describe_rank(p, r); })
      .def("origins", [](const CompiledPlan& p, int r) {
        // per device block: the (XML thread block id, XML step index) each device step came from
        const RankProgram& rp = p.ranks.at(r);
        py::list out;
        for (const DevBlock& b : rp.blocks) {
          py::list blk;
          for (int s = 0; s < b.nsteps; ++s) {
            const auto& o = rp.step_origins.at(b.step_begin + s);
            blk.append(py::make_tuple(o[0], o[1]));
          }
          out.append(blk);
        }
        return out;
      })
      .def("tables", [](const CompiledPlan& p, int r) {
        const RankProgram& rp = p.ranks.at(r);
        return py::make_tuple(as_bytes(rp.blocks), as_bytes(rp.steps), as_bytes(rp.srcs), as_bytes(rp.waits));
      });
  m.def("parse_and_compile",
        [](const std::string& xml, int nlanes, int niters, bool elide, bool fuse, bool multicast, bool reducing,
           bool merge, bool push) {
          CompileOptions o;
          o.push = push;
          o.nlanes = nlanes;
          o.niters = niters;
          o.elide_sends = elide;
          o.fuse_chains = fuse;
          o.multicast = multicast;
          o.reducing = reducing;
          o.merge_blocks = merge;
          return compile_plan(parse_xml(xml), o);
        },
        py::arg("xml"), py::arg("nlanes") = 1, py::arg("niters") = 1, py::arg("elide") = true,
        py::arg("fuse") = true, py::arg("multicast") = false, py::arg("reducing") = false, py::arg("merge") = true,
        py::arg("push") = false);
  m.def("cpu_interpret",
        [](const CompiledPlan& plan, py::list in, py::list out, py::list scr, int dtype, int redop, float scale,
           long long chunk_elems, long long piece_elems, unsigned seed, int launches) {
          HostBuffers b;
          fill(b.in, in);
          fill(b.out, out);
          fill(b.scr, scr);
          InterpResult r;
          {
            py::gil_scoped_release nogil;
            r = cpu_interpret(plan, b, dtype, redop, scale, chunk_elems, piece_elems, seed, launches);
          }
          drain(b.in, in);
          drain(b.out, out);
          drain(b.scr, scr);
          return py::make_tuple(r.ok, r.error, r.events);
        });
  m.attr("MAX_RANKS") = kMaxRanks;
  m.attr("MAX_FLAG_LANES") = kMaxFlagLanes;
  m.attr("SIZEOF_STEP") = (int)sizeof(DevStep);
  m.attr("SIZEOF_WAIT") = (int)sizeof(DevWait);
  m.attr("SIZEOF_SRC") = (int)sizeof(DevSrc);
  m.attr("SIZEOF_BLOCK") = (int)sizeof(DevBlock);
}
