// Host-side schedule compiler: MSCCL-style XML -> per-rank device programs.
#pragma once
#include <map>
#include <stdexcept>
#include <string>
#include <array>
#include <vector>

#include "vb/devprog.h"

namespace vb {

struct CompileError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

enum XKind { X_S, X_R, X_RRC, X_RCS, X_RRS, X_RRCS, X_CPY, X_RE, X_NOP };

struct XStep {
  XKind kind;
  int srcbuf, srcoff, dstbuf, dstoff, cnt, depid, deps, hasdep;
};

struct XTB {
  int id, send, recv, chan;
  std::vector<XStep> steps;
};

struct XGpu {
  int id, i_chunks, o_chunks, s_chunks;
  std::vector<XTB> tbs;
};

struct XAlgo {
  std::string name, proto, coll, redop;
  int nchannels = 1, nchunksperloop = 1, inplace = 0, ngpus = 0;
  long long min_bytes = 0, max_bytes = 0;
  std::vector<XGpu> gpus;
};

// Parse an MSCCL algorithm file (attributes-only elements, comments allowed).
XAlgo parse_xml(const std::string& text);

struct CompileOptions {
  int nlanes = 1;            // CTAs per block
  int niters = 1;            // pipeline iterations per chunk
  bool elide_sends = true;   // blocks made only of sends run no CTA
  bool fuse_chains = true;   // fold chains of receive-reduce steps into one n-ary reduce
  bool multicast = false;    // map whole-group reduce/broadcast patterns to NVLS multimem ops
  bool merge_blocks = true;  // run each rank's steps as one CTA group in a global topological order
  bool push = false;         // a plain send/receive pair becomes a store into the receiver's memory
  int mc_keep = 1, mc_period = 1;  // map a reduce chunk to NVLS when chunk % mc_period < mc_keep (rest stays P2P)
  bool reducing = false;     // the collective reduces (enables scale placement)
};

struct RankProgram {
  std::vector<DevBlock> blocks;
  std::vector<DevStep> steps;
  std::vector<DevSrc> srcs;
  std::vector<DevWait> waits;
  int i_chunks = 0, o_chunks = 0, s_chunks = 0;
  int s_used = 0;   // scratch chunks the device steps actually touch (fusion can drop them all)
  // XML origin of every device step (same order as `steps`): thread-block id and step index, or
  // {-1, -1} for steps the compiler added (in-place scaling)
  std::vector<std::array<int, 2>> step_origins;
};

struct CompileStats {
  int xml_steps = 0, device_steps = 0, elided_blocks = 0, fused_reduces = 0, multicast_ops = 0;
  int waits = 0, remote_waits = 0, scale_steps = 0, deferred_waits = 0, dropped_nops = 0;
  int staged_forwards = 0;   // 'rrs' steps given a scratch store so the next hop can pull the value
  int pushes = 0;            // send/receive pairs carried out as stores into the receiver's memory
};

struct CompiledPlan {
  XAlgo algo;
  CompileOptions options;
  std::vector<RankProgram> ranks;
  CompileStats stats;
  // The max number of blocks on any rank (flag table sizing).
  int max_blocks() const {
    size_t m = 0;
    for (auto& r : ranks) m = r.blocks.size() > m ? r.blocks.size() : m;
    return (int)m;
  }
  // Scratch chunks per rank that every rank must reserve (symmetric layout).
  int max_scratch_used() const {
    int m = 0;
    for (auto& r : ranks) m = r.s_used > m ? r.s_used : m;
    return m;
  }
};

CompiledPlan compile_plan(const XAlgo& algo, const CompileOptions& options);

// A readable dump of one rank's device program (tests and debugging).
std::string describe_rank(const CompiledPlan& plan, int rank);

// ---- CPU reference interpreter -------------------------------------------
// Runs every rank's device program in one process on host buffers, with
// virtual CTAs scheduled in a seeded random order, using exactly the piece
// geometry and flag protocol of the GPU kernel.  It is the oracle for the
// kernel and detects missing synchronisation (a pull that can observe a
// later overwrite yields wrong numbers under some order).
struct HostBuffers {
  std::vector<std::vector<unsigned char>> in, out, scr;   // per rank
};

struct InterpResult {
  bool ok = false;
  std::string error;
  long long events = 0;
};

InterpResult cpu_interpret(const CompiledPlan& plan, HostBuffers& bufs, int dtype, int redop, float scale,
                           long long chunk_elems, long long piece_elems, unsigned seed, int launches);

}  // namespace vb
