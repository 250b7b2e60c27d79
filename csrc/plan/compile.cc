// Schedule compiler: XML program -> pull-based device programs.
//
// Pipeline:
//   1. index steps, check peers/channels/dependencies, pair every send with
//      its receive (per connection (src, dst, channel) in TB order, as in
//      MSCCL's FIFO connections);
//   2. topological order of the global step graph (TB order, explicit deps,
//      send->receive); a cycle is a deadlock under MSCCL semantics;
//   3. symbolic replay (contributor masks) to place the fused scale on the
//      step that completes each reduction;
//   4. thread blocks made only of sends are elided (the receiver pulls; the
//      sender only needs its dependencies to be complete), every other block
//      becomes a device block;
//   5. waits: explicit dependencies, data readiness of pulled sends, and
//      write-after-read acknowledgements: a step that overwrites a region a
//      send reads waits for that send's receiver to finish; each rank finally
//      waits for all of its sends to be consumed before the kernel ends;
//   6. optional chain fusion (receive-reduce chains into one n-ary reduce);
//   7. a final deadlock check of the device event graph.
// Push mode (CompileOptions::push) turns every plain send/receive pair into a
// store by the sender into the receiver's buffer: the sender's step waits for
// everything the receive would have waited for on the receiving rank (its
// predecessor in its thread block, its explicit dependency, the readers of the
// destination it overwrites, the receiver's start flag), the receive becomes a
// NOP that waits for the push.  The data leaves the sender when the send runs,
// as with MSCCL's FIFO connections, so overwriting the send's source only
// waits for the push itself, and NVLink carries stores instead of the read
// requests of pulls.  Reductions keep pulling; push mode excludes NVLS mapping.
#include <algorithm>
#include <deque>
#include <functional>
#include <map>
#include <set>
#include <sstream>
#include <tuple>

#include "vb/plan.h"

namespace vb {
namespace {

bool has_send(XKind k) { return k == X_S || k == X_RCS || k == X_RRS || k == X_RRCS; }
bool has_recv(XKind k) { return k == X_R || k == X_RRC || k == X_RCS || k == X_RRS || k == X_RRCS; }
bool writes_dst(XKind k) { return k == X_R || k == X_RRC || k == X_RCS || k == X_RRCS || k == X_CPY || k == X_RE; }
bool reduces(XKind k) { return k == X_RRC || k == X_RRS || k == X_RRCS || k == X_RE; }
const char* kname(XKind k) {
  static const char* names[] = {"s", "r", "rrc", "rcs", "rrs", "rrcs", "cpy", "re", "nop"};
  return names[k];
}

struct SRef {
  int rank = -1, tb = -1, step = -1;
  bool valid() const { return rank >= 0; }
  bool operator<(const SRef& o) const { return std::tie(rank, tb, step) < std::tie(o.rank, o.tb, o.step); }
  bool operator==(const SRef& o) const { return rank == o.rank && tb == o.tb && step == o.step; }
};

struct Region {
  int rank, buf, chunk;
  bool operator<(const Region& o) const { return std::tie(rank, buf, chunk) < std::tie(o.rank, o.buf, o.chunk); }
};

// (rank, device block) -> max event.  Block -1 is the per-rank start flag.
using EventSet = std::map<std::pair<int, int>, int>;

void merge(EventSet& into, const EventSet& from) {
  for (auto& kv : from) {
    auto it = into.find(kv.first);
    if (it == into.end() || it->second < kv.second) into[kv.first] = kv.second;
  }
}

struct Value {
  int index = -1;
  uint32_t mask = 0;
  bool scaled = false;
  bool known = false;
};

class Compiler {
 public:
  Compiler(const XAlgo& a, const CompileOptions& o) : a_(a), o_(o), P_(a.ngpus) {}

  CompiledPlan run() {
    index_steps();
    pair_connections();
    topo_order();
    if (o_.reducing) place_scale();
    assign_blocks();
    build_waits_and_hazards();
    if (o_.merge_blocks) merge_blocks();
    if (o_.multicast && !o_.push && merged_ && P_ > 1) map_multicast();
    dedupe_start_waits();
    if (merged_) drop_idle_nops();
    emit();
    deadlock_check();
    CompiledPlan plan;
    plan.algo = a_;
    plan.options = o_;
    plan.ranks = std::move(out_);
    plan.stats = stats_;
    return plan;
  }

 private:
  [[noreturn]] void fail(const std::string& m) { throw CompileError(m); }

  const XStep& step(const SRef& r) const { return a_.gpus[r.rank].tbs[r.tb].steps[r.step]; }
  const XTB& tb(int rank, int t) const { return a_.gpus[rank].tbs[t]; }

  // In-place aliasing resolved to one canonical (buffer, chunk).
  Region canon(int rank, int buf, int chunk) const {
    if (!a_.inplace || buf == BUF_SCR) return Region{rank, buf, chunk};
    const XGpu& g = a_.gpus[rank];
    if (a_.coll == "allgather") return buf == BUF_IN ? Region{rank, BUF_OUT, rank * g.i_chunks + chunk} : Region{rank, BUF_OUT, chunk};
    if (a_.coll == "reduce_scatter") return buf == BUF_OUT ? Region{rank, BUF_IN, rank * g.o_chunks + chunk} : Region{rank, BUF_IN, chunk};
    return Region{rank, BUF_OUT, chunk};
  }

  int slots(int rank, int buf) const {
    const XGpu& g = a_.gpus[rank];
    return buf == BUF_IN ? g.i_chunks : buf == BUF_OUT ? g.o_chunks : g.s_chunks;
  }

  void check_region(int rank, int buf, int off, int cnt, const char* what) {
    if (off < 0) fail(std::string("step ") + what + " offset is missing");
    Region c = canon(rank, buf, off);
    int limit = slots(rank, c.buf);
    if (c.chunk + cnt > limit) {
      std::ostringstream m;
      m << "rank " << rank << " " << what << " region " << "ios"[buf] << "[" << off << "+" << cnt
        << "] exceeds its " << limit << " slots";
      fail(m.str());
    }
  }

  void index_steps() {
    for (int r = 0; r < P_; ++r) {
      const XGpu& g = a_.gpus[r];
      std::map<int, int> ids;
      for (int t = 0; t < (int)g.tbs.size(); ++t) {
        if (ids.count(g.tbs[t].id)) fail("rank " + std::to_string(r) + " has duplicate TB id");
        ids[g.tbs[t].id] = t;
      }
      tb_index_.push_back(ids);
      for (int t = 0; t < (int)g.tbs.size(); ++t) {
        const XTB& b = g.tbs[t];
        if (b.send >= P_ || b.recv >= P_ || b.send == r || b.recv == r) fail("TB peer outside the rank range");
        for (int s = 0; s < (int)b.steps.size(); ++s) {
          const XStep& st = b.steps[s];
          ++stats_.xml_steps;
          if (has_send(st.kind) && b.send < 0) fail(std::string("step '") + kname(st.kind) + "' in a TB without a send peer");
          if (has_recv(st.kind) && b.recv < 0) fail(std::string("step '") + kname(st.kind) + "' in a TB without a receive peer");
          if (st.kind == X_S || st.kind == X_CPY || st.kind == X_RRC || st.kind == X_RE) check_region(r, st.srcbuf, st.srcoff, st.cnt, "source");
          if (writes_dst(st.kind)) check_region(r, st.dstbuf, st.dstoff, st.cnt, "destination");
          if (st.depid >= 0) {
            auto it = ids.find(st.depid);
            if (it == ids.end()) fail("dependency names an unknown TB");
            if (st.deps < 0 || st.deps >= (int)g.tbs[it->second].steps.size()) fail("dependency names an unknown step");
            if (it->second == t && st.deps >= s) fail("dependency points at the same or a later step of its TB");
          } else if (st.deps >= 0) {
            fail("dependency step without a dependency TB");
          }
          all_.push_back(SRef{r, t, s});
        }
      }
    }
  }

  void pair_connections() {
    std::map<std::tuple<int, int, int>, std::vector<SRef>> sends, recvs;
    std::set<std::tuple<int, int, int, int>> owners;
    for (const SRef& x : all_) {
      const XTB& b = tb(x.rank, x.tb);
      const XStep& st = step(x);
      if (has_send(st.kind)) sends[{x.rank, b.send, b.chan}].push_back(x);
      if (has_recv(st.kind)) recvs[{b.recv, x.rank, b.chan}].push_back(x);
    }
    for (int r = 0; r < P_; ++r)
      for (auto& b : a_.gpus[r].tbs) {
        bool s = false, v = false;
        for (auto& st : b.steps) { s |= has_send(st.kind); v |= has_recv(st.kind); }
        if (s && !owners.insert({r, b.send, b.chan, 0}).second) fail("two TBs send to one peer on one channel");
        if (v && !owners.insert({r, b.recv, b.chan, 1}).second) fail("two TBs receive from one peer on one channel");
      }
    for (auto& kv : sends) {
      auto it = recvs.find(kv.first);
      size_t n = it == recvs.end() ? 0 : it->second.size();
      if (n != kv.second.size()) {
        std::ostringstream m;
        m << "connection " << std::get<0>(kv.first) << "->" << std::get<1>(kv.first) << " channel " << std::get<2>(kv.first)
          << " has " << kv.second.size() << " sends but " << n << " receives";
        fail(m.str());
      }
      for (size_t i = 0; i < n; ++i) {
        match_recv_[kv.second[i]] = it->second[i];
        match_send_[it->second[i]] = kv.second[i];
        if (step(kv.second[i]).cnt != step(it->second[i]).cnt) fail("matched send and receive disagree on cnt");
      }
    }
    for (auto& kv : recvs)
      if (!sends.count(kv.first)) fail("a receive has no matching send");
  }

  std::vector<SRef> preds(const SRef& x) const {
    std::vector<SRef> p;
    if (x.step > 0) p.push_back(SRef{x.rank, x.tb, x.step - 1});
    const XStep& st = step(x);
    if (st.depid >= 0) p.push_back(SRef{x.rank, tb_index_[x.rank].at(st.depid), st.deps});
    auto it = match_send_.find(x);
    if (it != match_send_.end()) p.push_back(it->second);
    return p;
  }

  void topo_order() {
    std::map<SRef, int> indeg;
    std::map<SRef, std::vector<SRef>> succ;
    for (const SRef& x : all_) indeg[x] = 0;
    for (const SRef& x : all_)
      for (const SRef& p : preds(x)) { indeg[x]++; succ[p].push_back(x); }
    std::deque<SRef> ready;
    for (const SRef& x : all_) if (indeg[x] == 0) ready.push_back(x);
    while (!ready.empty()) {
      SRef x = ready.front();
      ready.pop_front();
      topo_pos_[x] = (int)order_.size();
      order_.push_back(x);
      for (const SRef& y : succ[x]) if (--indeg[y] == 0) ready.push_back(y);
    }
    if (order_.size() != all_.size()) fail("schedule deadlocks: the step dependency graph has a cycle");
    for (const SRef& x : order_) {
      int lv = 0;
      for (const SRef& p : preds(x)) lv = std::max(lv, level_[p] + 1);
      level_[x] = lv;
    }
  }

  void place_scale() {
    const uint32_t full = P_ >= 32 ? 0xffffffffu : ((1u << P_) - 1u);
    std::map<Region, Value> state;
    for (int r = 0; r < P_; ++r)
      for (int k = 0; k < a_.gpus[r].i_chunks; ++k) {
        Value v;
        v.index = k; v.mask = 1u << r; v.known = true;
        state[canon(r, BUF_IN, k)] = v;
      }
    std::map<SRef, std::vector<Value>> carried;   // value captured at each send
    auto read = [&](int rank, int buf, int off, int cnt) {
      std::vector<Value> vs;
      for (int k = 0; k < cnt; ++k) vs.push_back(state[canon(rank, buf, off + k)]);
      return vs;
    };
    auto combine = [&](const Value& a, const Value& b, bool& scale) {
      Value v;
      if (!a.known || !b.known) return v;
      v.known = true;
      v.index = a.index;
      v.mask = a.mask | b.mask;
      v.scaled = a.scaled || b.scaled;
      if (v.mask == full && !v.scaled && !(a.mask & b.mask)) { v.scaled = true; scale = true; }
      return v;
    };
    for (const SRef& x : order_) {
      const XStep& st = step(x);
      bool scale = false;
      std::vector<Value> result;
      std::vector<Value> incoming;
      if (has_recv(st.kind)) incoming = carried[match_send_.at(x)];
      switch (st.kind) {
        case X_S: carried[x] = read(x.rank, st.srcbuf, st.srcoff, st.cnt); break;
        case X_R: case X_RCS: result = incoming; break;
        case X_CPY: result = read(x.rank, st.srcbuf, st.srcoff, st.cnt); break;
        case X_RRC: case X_RRCS: {
          auto local = read(x.rank, st.srcbuf, st.srcoff, st.cnt);
          for (int k = 0; k < st.cnt; ++k) result.push_back(combine(incoming[k], local[k], scale));
          break;
        }
        case X_RE: {
          auto src = read(x.rank, st.srcbuf, st.srcoff, st.cnt);
          auto dst = read(x.rank, st.dstbuf, st.dstoff, st.cnt);
          for (int k = 0; k < st.cnt; ++k) result.push_back(combine(src[k], dst[k], scale));
          break;
        }
        default: break;
      }
      if (st.kind == X_R || st.kind == X_RCS || st.kind == X_CPY) {
        // A complete value that was never scaled (single-rank programs) is scaled where it is copied.
        for (auto& v : result)
          if (v.known && v.mask == full && !v.scaled) { v.scaled = true; scale = true; }
      }
      if (writes_dst(st.kind))
        for (int k = 0; k < st.cnt; ++k) state[canon(x.rank, st.dstbuf, st.dstoff + k)] = result[k];
      if (st.kind == X_RCS || st.kind == X_RRCS) carried[x] = result;
      if (scale) { scale_steps_.insert(x); ++stats_.scale_steps; }
      if (writes_dst(st.kind))
        for (int k = 0; k < st.cnt; ++k) last_writer_[canon(x.rank, st.dstbuf, st.dstoff + k)] = x;
    }
    // Outputs that hold a complete value nobody scaled (single-rank programs, or an
    // in-place output that already aliases its complete input) get an in-place scale step.
    for (int r = 0; r < P_; ++r)
      for (int k = 0; k < a_.gpus[r].o_chunks; ++k) {
        Region reg = canon(r, BUF_OUT, k);
        auto it = state.find(reg);
        if (it != state.end() && it->second.known && it->second.mask == full && !it->second.scaled) {
          it->second.scaled = true;
          unscaled_outputs_.push_back(reg);
          ++stats_.scale_steps;
        }
      }
  }

  void assign_blocks() {
    dblock_.resize(P_);
    out_.resize(P_);
    for (int r = 0; r < P_; ++r) {
      const XGpu& g = a_.gpus[r];
      dblock_[r].assign(g.tbs.size(), -1);
      int next = 0;
      for (int t = 0; t < (int)g.tbs.size(); ++t) {
        bool only_sends = true, pushes = false;
        for (int s = 0; s < (int)g.tbs[t].steps.size(); ++s) {
          const XStep& st = g.tbs[t].steps[s];
          if (st.kind != X_S && st.kind != X_NOP) only_sends = false;
          if (pushed(SRef{r, t, s})) pushes = true;
        }
        if (o_.elide_sends && only_sends && !pushes) { ++stats_.elided_blocks; continue; }
        dblock_[r][t] = next++;
      }
      out_[r].i_chunks = g.i_chunks;
      out_[r].o_chunks = g.o_chunks;
      out_[r].s_chunks = g.s_chunks;
      nblocks_.push_back(next == 0 ? 1 : next);   // a rank always runs at least one (possibly empty) block
      synthetic_.push_back(next == 0);
    }
  }

  bool elided(const SRef& x) const { return dblock_[x.rank][x.tb] < 0; }

  // Push mode: a plain send whose receive is a plain receive is carried out by the sender.
  bool pushed(const SRef& x) const {
    if (!o_.push) return false;
    const XStep& st = step(x);
    if (st.kind != X_S) return false;
    auto it = match_recv_.find(x);
    return it != match_recv_.end() && step(it->second).kind == X_R;
  }
  bool pushed_recv(const SRef& y) const {
    auto it = match_send_.find(y);
    return it != match_send_.end() && pushed(it->second);
  }

  // Event set that is complete once step x is complete under pull semantics.
  EventSet completion(const SRef& x) {
    auto it = completion_memo_.find(x);
    if (it != completion_memo_.end()) return it->second;
    EventSet e;
    const XStep& st = step(x);
    if (pushed(x)) {
      e[{x.rank, dblock_[x.rank][x.tb]}] = 2 * x.step + 2;   // the push is done: the data left the source
    } else if (st.kind == X_S) {
      SRef rv = match_recv_.at(x);
      e[{rv.rank, redirect_block(rv)}] = 2 * redirect_step(rv) + 2;
    } else if (elided(x)) {
      e = arrival(x);
    } else {
      e[{x.rank, redirect_block(x)}] = 2 * redirect_step(x) + 2;
      if (st.kind == X_RCS || st.kind == X_RRCS) {
        SRef rv = match_recv_.at(x);
        merge(e, EventSet{{{rv.rank, redirect_block(rv)}, 2 * redirect_step(rv) + 2}});
      }
    }
    completion_memo_[x] = e;
    return e;
  }

  // Events implied once an elided TB reaches step x (all earlier dependencies complete).
  EventSet arrival(const SRef& x) {
    auto it = arrival_memo_.find(x);
    if (it != arrival_memo_.end()) return it->second;
    EventSet e;
    if (x.step > 0) e = arrival(SRef{x.rank, x.tb, x.step - 1});
    const XStep& st = step(x);
    if (st.depid >= 0) merge(e, completion(SRef{x.rank, tb_index_[x.rank].at(st.depid), st.deps}));
    arrival_memo_[x] = e;
    return e;
  }

  // Events after which the data a receive pulls from send x is ready.
  EventSet data_ready(const SRef& x) {
    const XStep& st = step(x);
    EventSet e;
    if (elided(x)) {
      e = arrival(x);
    } else if (st.kind == X_S) {
      e[{x.rank, dblock_[x.rank][x.tb]}] = 2 * x.step + 1;
      need_arrive_.insert(x);
    } else {
      e[{x.rank, dblock_[x.rank][x.tb]}] = 2 * x.step + 2;
    }
    bool local = false;
    for (auto& kv : e) if (kv.first.first == x.rank) local = true;
    if (!local) e[{x.rank, -1}] = 1;   // the sender's kernel must have started
    return e;
  }

  // Source region a receive of send x pulls from (sender's memory).
  Region pull_source(const SRef& x) const {
    const XStep& st = step(x);
    if (st.kind == X_S) return canon(x.rank, st.srcbuf, st.srcoff);
    return canon(x.rank, st.dstbuf, st.dstoff);   // rcs / rrcs forward what they stored
  }

  // Chain fusion bookkeeping: a fused-away step's events are served by its chain's final step.
  int redirect_block(const SRef& x) const {
    auto it = fused_into_.find(x);
    const SRef& y = it == fused_into_.end() ? x : it->second;
    return dblock_[y.rank][y.tb];
  }
  int redirect_step(const SRef& x) const {
    auto it = fused_into_.find(x);
    return it == fused_into_.end() ? x.step : it->second.step;
  }

  void find_chains() {
    if (!o_.fuse_chains) return;
    // readers of each canonical region, in topological order
    std::map<Region, std::vector<SRef>> readers, writers;
    for (const SRef& x : order_) {
      const XStep& st = step(x);
      auto add_read = [&](int buf, int off) { for (int k = 0; k < st.cnt; ++k) readers[canon(x.rank, buf, off + k)].push_back(x); };
      if (st.kind == X_S || st.kind == X_CPY || st.kind == X_RRC || st.kind == X_RE) add_read(st.srcbuf, st.srcoff);
      if (st.kind == X_RE || st.kind == X_RCS || st.kind == X_RRCS) add_read(st.dstbuf, st.dstoff);
      if (writes_dst(st.kind)) for (int k = 0; k < st.cnt; ++k) writers[canon(x.rank, st.dstbuf, st.dstoff + k)].push_back(x);
    }
    // an rrc y whose local source is exactly the destination written by rrc x, where y is the only
    // reader of that value and nothing else writes the region in between, extends x's chain.
    std::map<SRef, SRef> next;
    for (const SRef& x : order_) {
      const XStep& sx = step(x);
      if (sx.kind != X_RRC || sx.cnt != 1 || elided(x)) continue;
      Region d = canon(x.rank, sx.dstbuf, sx.dstoff);
      auto& rd = readers[d];
      auto& wr = writers[d];
      int px = topo_pos_[x];
      std::vector<SRef> later;
      for (auto& r : rd) if (topo_pos_[r] > px) later.push_back(r);
      if (later.empty()) continue;
      const SRef& y = later.front();
      const XStep& sy = step(y);
      if (sy.kind != X_RRC || sy.cnt != 1 || y.rank != x.rank) continue;
      if (!(canon(y.rank, sy.srcbuf, sy.srcoff).buf == d.buf && canon(y.rank, sy.srcbuf, sy.srcoff).chunk == d.chunk)) continue;
      // y must be the only reader of x's value before the region is written again
      int nw = 1 << 30;
      for (auto& w : wr) if (topo_pos_[w] > px) nw = std::min(nw, topo_pos_[w]);
      bool exclusive = true;
      for (auto& r : later)
        if (topo_pos_[r] <= nw && !(r == y)) exclusive = false;
      if (topo_pos_[y] > nw) exclusive = false;
      if (!exclusive) continue;
      if (scale_steps_.count(x)) continue;
      next[x] = y;
    }
    std::set<SRef> has_prev;
    for (auto& kv : next) has_prev.insert(kv.second);
    for (auto& kv : next) {
      if (has_prev.count(kv.first)) continue;   // not a chain head
      std::vector<SRef> chain{kv.first};
      SRef cur = kv.first;
      while (next.count(cur) && (int)chain.size() < 15) { cur = next[cur]; chain.push_back(cur); }
      if (chain.size() < 2) continue;
      SRef last = chain.back();
      for (size_t i = 0; i + 1 < chain.size(); ++i) fused_into_[chain[i]] = last;
      chains_[last] = chain;
      stats_.fused_reduces++;
    }
  }

  struct PendingStep {
    DevStep st{};
    std::vector<DevSrc> srcs;
    EventSet waits;
    int prio = 0;
    int level = 0;             // dependency depth of the XML step
    int xml_tb = -1;
    int xml_step = -1;         // index of the originating step in its XML thread block (-1: compiler-made)
    bool mc_peer = false;      // a copy replaced by the owner's multicast store
    int mc_buf = -1, mc_chunk = -1;
    PendingStep() { st.dst_rank = -1; }
  };

  void build_waits_and_hazards() {
    find_chains();
    dsteps_count_.resize(P_);
    for (int r = 0; r < P_; ++r) {
      dsteps_count_[r].assign(nblocks_[r], 0);
      for (int t = 0; t < (int)a_.gpus[r].tbs.size(); ++t)
        if (dblock_[r][t] >= 0) dsteps_count_[r][dblock_[r][t]] = (int)a_.gpus[r].tbs[t].steps.size();
    }
    // write-after-read acknowledgements: sends reading a region since its previous write
    std::map<Region, std::vector<SRef>> open_sends;
    std::map<SRef, std::vector<SRef>> acks;   // writer -> sends whose receivers it must wait for
    for (const SRef& x : order_) {
      const XStep& st = step(x);
      if (writes_dst(st.kind)) {
        for (int k = 0; k < st.cnt; ++k) {
          Region d = canon(x.rank, st.dstbuf, st.dstoff + k);
          auto it = open_sends.find(d);
          if (it != open_sends.end()) {
            for (auto& s : it->second) if (!(s == x)) acks[x].push_back(s);
            open_sends.erase(it);
          }
        }
      }
      if (has_send(st.kind)) {
        Region src = pull_source(x);
        for (int k = 0; k < st.cnt; ++k) open_sends[Region{src.rank, src.buf, src.chunk + k}].push_back(x);
      }
    }
    pending_.resize(P_);
    for (int r = 0; r < P_; ++r) pending_[r].resize(nblocks_[r]);
    for (const SRef& x : all_) {
      int db = dblock_[x.rank][x.tb];
      if (db < 0) continue;
      const XStep& st = step(x);
      PendingStep ps{};
      ps.prio = topo_pos_[x];
      ps.level = level_[x];
      ps.xml_tb = a_.gpus[x.rank].tbs[x.tb].id;
      ps.xml_step = x.step;
      ps.st.cnt = st.cnt;
      ps.st.flags = 0;
      if (st.depid >= 0) merge(ps.waits, completion(SRef{x.rank, tb_index_[x.rank].at(st.depid), st.deps}));
      for (auto& s : acks[x]) merge(ps.waits, completion(s));
      auto fused = fused_into_.find(x);
      if (pushed(x)) {
        // the sender stores into the receiver's destination once the receive could have run there: after
        // its predecessor in its thread block, its explicit dependency and the readers of what it overwrites
        const SRef y = match_recv_.at(x);
        const XStep& ry = step(y);
        Region src = pull_source(x);
        Region d = canon(y.rank, ry.dstbuf, ry.dstoff);
        ps.st.op = OP_COPY;
        ps.srcs.push_back(DevSrc{(int16_t)x.rank, (uint8_t)src.buf, 0, src.chunk});
        ps.st.dst_buf = (uint8_t)d.buf;
        ps.st.dst_chunk = d.chunk;
        ps.st.dst_rank = y.rank;
        if (y.step > 0) merge(ps.waits, completion(SRef{y.rank, y.tb, y.step - 1}));
        if (ry.depid >= 0) merge(ps.waits, completion(SRef{y.rank, tb_index_[y.rank].at(ry.depid), ry.deps}));
        for (auto& s : acks[y]) merge(ps.waits, completion(s));
        merge(ps.waits, EventSet{{{y.rank, -1}, 1}});   // the receiver's kernel has started
        if (scale_steps_.count(y)) ps.st.flags |= F_SCALE;
        ++stats_.pushes;
      } else if (pushed_recv(x)) {
        ps.st.op = OP_NOP;                                // the push into this rank does the work
        merge(ps.waits, completion(match_send_.at(x)));
      } else if (fused != fused_into_.end()) {
        ps.st.op = OP_NOP;   // work moves to the chain's final step
      } else if (chains_.count(x)) {
        const auto& chain = chains_[x];
        const XStep& head = step(chain.front());
        Region base = canon(x.rank, head.srcbuf, head.srcoff);
        ps.srcs.push_back(DevSrc{(int16_t)x.rank, (uint8_t)base.buf, 0, base.chunk});
        for (const SRef& c : chain) {
          const SRef& snd = match_send_.at(c);
          Region src = pull_source(snd);
          ps.srcs.push_back(DevSrc{(int16_t)src.rank, (uint8_t)src.buf, 0, src.chunk});
          merge(ps.waits, data_ready(snd));
          const XStep& cs = step(c);
          if (cs.depid >= 0) merge(ps.waits, completion(SRef{c.rank, tb_index_[c.rank].at(cs.depid), cs.deps}));
          for (auto& s : acks[c]) merge(ps.waits, completion(s));
        }
        Region d = canon(x.rank, st.dstbuf, st.dstoff);
        ps.st.op = OP_REDUCE;
        ps.st.dst_buf = (uint8_t)d.buf;
        ps.st.dst_chunk = d.chunk;
      } else {
        switch (st.kind) {
          case X_S: case X_NOP: ps.st.op = OP_NOP; break;
          case X_R: case X_RCS: {
            Region src = pull_source(match_send_.at(x));
            ps.srcs.push_back(DevSrc{(int16_t)src.rank, (uint8_t)src.buf, 0, src.chunk});
            merge(ps.waits, data_ready(match_send_.at(x)));
            ps.st.op = OP_COPY;
            break;
          }
          case X_RRC: case X_RRCS: {
            Region loc = canon(x.rank, st.srcbuf, st.srcoff);
            Region src = pull_source(match_send_.at(x));
            ps.srcs.push_back(DevSrc{(int16_t)x.rank, (uint8_t)loc.buf, 0, loc.chunk});
            ps.srcs.push_back(DevSrc{(int16_t)src.rank, (uint8_t)src.buf, 0, src.chunk});
            merge(ps.waits, data_ready(match_send_.at(x)));
            ps.st.op = OP_REDUCE;
            break;
          }
          case X_CPY: {
            Region loc = canon(x.rank, st.srcbuf, st.srcoff);
            ps.srcs.push_back(DevSrc{(int16_t)x.rank, (uint8_t)loc.buf, 0, loc.chunk});
            ps.st.op = OP_COPY;
            break;
          }
          case X_RE: {
            Region s1 = canon(x.rank, st.srcbuf, st.srcoff);
            Region s2 = canon(x.rank, st.dstbuf, st.dstoff);
            ps.srcs.push_back(DevSrc{(int16_t)x.rank, (uint8_t)s1.buf, 0, s1.chunk});
            ps.srcs.push_back(DevSrc{(int16_t)x.rank, (uint8_t)s2.buf, 0, s2.chunk});
            ps.st.op = OP_REDUCE;
            break;
          }
          default: fail("unsupported step kind");
        }
        if (writes_dst(st.kind)) {
          Region d = canon(x.rank, st.dstbuf, st.dstoff);
          ps.st.dst_buf = (uint8_t)d.buf;
          ps.st.dst_chunk = d.chunk;
        }
      }
      if (scale_steps_.count(x) && !pushed_recv(x)) ps.st.flags |= F_SCALE;
      // drop waits implied by this CTA's own sequential order
      auto own = ps.waits.find({x.rank, db});
      if (own != ps.waits.end()) {
        // earlier steps of this CTA are complete by program order; a fused chain member's completion
        // is redirected to this very step and needs no wait either
        if (own->second <= 2 * x.step || (chains_.count(x) && own->second == 2 * x.step + 2)) ps.waits.erase(own);
        else fail("a step waits on its own or a later step of its block");
      }
      pending_[x.rank][db].resize(std::max<size_t>(pending_[x.rank][db].size(), x.step + 1));
      pending_[x.rank][db][x.step] = ps;
    }
    // in-place scale steps for complete but unscaled outputs
    for (const Region& reg : unscaled_outputs_) {
      int r = reg.rank;
      int db = synthetic_[r] ? 0 : nblocks_[r];
      if (!synthetic_[r] && (int)pending_[r].size() <= db) {
        pending_[r].resize(db + 1);
        nblocks_[r] = db + 1;
        dsteps_count_[r].resize(db + 1, 0);
        synthetic_extra_.insert(r);
      }
      PendingStep ps{};
      ps.prio = (int)order_.size();
      ps.st.op = OP_COPY;
      ps.st.cnt = 1;
      ps.st.flags = F_SCALE;
      ps.st.dst_buf = (uint8_t)reg.buf;
      ps.st.dst_chunk = reg.chunk;
      ps.srcs.push_back(DevSrc{(int16_t)r, (uint8_t)reg.buf, 0, reg.chunk});
      auto lw = last_writer_.find(reg);
      if (lw != last_writer_.end()) merge(ps.waits, completion(lw->second));
      // every pull of this region by a send must finish before it is rescaled
      for (const SRef& x : all_) {
        const XStep& st = step(x);
        if (has_send(st.kind) && x.rank == r) {
          Region src = pull_source(x);
          if (src.buf == reg.buf && reg.chunk >= src.chunk && reg.chunk < src.chunk + st.cnt) merge(ps.waits, completion(x));
        }
      }
      pending_[r][db].push_back(ps);
      dsteps_count_[r][db] = (int)pending_[r][db].size();
    }
    // end-of-kernel acknowledgements: every send must be consumed
    end_waits_.resize(P_);
    for (const SRef& x : all_) {
      const XStep& st = step(x);
      if (!has_send(st.kind) || pushed(x)) continue;   // a push is over when its own step is
      SRef rv = match_recv_.at(x);
      merge(end_waits_[x.rank], EventSet{{{rv.rank, redirect_block(rv)}, 2 * redirect_step(rv) + 2}});
    }
  }


  // Merge every rank's device blocks into one block whose steps follow one global
  // topological order of the device event graph.  Every wait then refers to a
  // step that precedes it in that order, so the merged program cannot deadlock,
  // and every step is spread over all lanes of the rank.
  void merge_blocks() {
    using Node = std::tuple<int, int, int>;   // rank, block, step
    std::map<Node, std::vector<Node>> succ;
    std::map<Node, int> indeg;
    for (int r = 0; r < P_; ++r)
      for (int b = 0; b < nblocks_[r]; ++b)
        for (int s = 0; s < (int)pending_[r][b].size(); ++s) {
          Node n{r, b, s};
          indeg[n];
          if (s > 0) { succ[Node{r, b, s - 1}].push_back(n); indeg[n]++; }
          for (auto& kv : pending_[r][b][s].waits) {
            if (kv.first.second < 0) continue;
            Node src{kv.first.first, kv.first.second, (kv.second - 1) / 2};
            succ[src].push_back(n);
            indeg[n]++;
          }
        }
    // Order: dependency depth, then, among steps of one depth, the cyclic distance from the rank to the
    // peer it pulls from, so that at each depth rank r reads from r+1, r+2, ... instead of every rank
    // reading the same peer first; then the XML topological position.
    auto rotation = [&](const Node& n) {
      const PendingStep& ps = pending_[std::get<0>(n)][std::get<1>(n)][std::get<2>(n)];
      const int r = std::get<0>(n);
      if (ps.st.dst_rank >= 0 && ps.st.dst_rank != r) return (ps.st.dst_rank - r + P_) % P_;   // push target
      for (auto& sr : ps.srcs)
        if (sr.rank != r) return (sr.rank - r + P_) % P_;
      return 0;
    };
    auto prio = [&](const Node& n) {
      const PendingStep& ps = pending_[std::get<0>(n)][std::get<1>(n)][std::get<2>(n)];
      return std::make_tuple(ps.level, rotation(n), ps.prio, std::get<0>(n), std::get<1>(n), std::get<2>(n));
    };
    std::set<std::tuple<int, int, int, int, int, int>> ready;
    for (auto& kv : indeg) if (kv.second == 0) ready.insert(prio(kv.first));
    std::map<Node, int> newidx;
    std::vector<int> count(P_, 0);
    std::vector<std::vector<Node>> order(P_);
    while (!ready.empty()) {
      auto t = *ready.begin();
      ready.erase(ready.begin());
      Node n{std::get<3>(t), std::get<4>(t), std::get<5>(t)};
      int r = std::get<0>(n);
      newidx[n] = count[r]++;
      order[r].push_back(n);
      for (auto& m : succ[n]) if (--indeg[m] == 0) ready.insert(prio(m));
    }
    if (newidx.size() != indeg.size()) fail("device program has a cyclic wait graph");
    auto remap = [&](const EventSet& in) {
      EventSet out;
      for (auto& kv : in) {
        if (kv.first.second < 0) { merge(out, EventSet{{kv.first, kv.second}}); continue; }
        int idx = newidx.at(Node{kv.first.first, kv.first.second, (kv.second - 1) / 2});
        int ev = 2 * idx + ((kv.second % 2) ? 1 : 2);
        merge(out, EventSet{{{kv.first.first, 0}, ev}});
      }
      return out;
    };
    std::vector<std::vector<std::vector<PendingStep>>> merged(P_);
    for (int r = 0; r < P_; ++r) {
      merged[r].resize(1);
      for (size_t i = 0; i < order[r].size(); ++i) {
        const Node& n = order[r][i];
        PendingStep ps = pending_[r][std::get<1>(n)][std::get<2>(n)];
        ps.waits = remap(ps.waits);
        auto own = ps.waits.find({r, 0});
        if (own != ps.waits.end()) {
          if (own->second <= 2 * (int)i) ps.waits.erase(own);
          else fail("merged step waits on a later step of its own rank");
        }
        merged[r][0].push_back(ps);
      }
      end_waits_[r] = remap(end_waits_[r]);
      nblocks_[r] = 1;
      dsteps_count_[r].assign(1, (int)order[r].size());
    }
    pending_ = std::move(merged);
    merged_ = true;
  }

  // NVLS mapping on merged programs.  A reduce whose sources are the same
  // (buffer, chunk) on every rank, whose result every other rank only copies,
  // becomes one multimem.ld_reduce + multimem.st on the owner: the switch sums
  // the chunk and writes the result to every rank's destination; the other
  // ranks' copies become waits on the owner's completion.
  void map_multicast() {
    for (int r = 0; r < P_; ++r) {
      auto& steps = pending_[r][0];
      for (int i = 0; i < (int)steps.size(); ++i) {
        PendingStep& ps = steps[i];
        if (ps.st.op != OP_REDUCE || ps.st.cnt != 1 || (int)ps.srcs.size() != P_) continue;
        if (o_.mc_period > 1 && (ps.st.dst_chunk % o_.mc_period) >= o_.mc_keep) continue;
        std::set<int> ranks;
        bool same = true;
        for (auto& sr : ps.srcs) {
          ranks.insert(sr.rank);
          if (sr.buf != ps.srcs[0].buf || sr.chunk != ps.srcs[0].chunk) same = false;
        }
        if (!same || (int)ranks.size() != P_) continue;
        const int owner_done = 2 * i + 2;
        std::vector<std::pair<int, int>> peers;
        for (int p = 0; p < P_ && peers.size() + 1 < (size_t)P_ + 1; ++p) {
          if (p == r) continue;
          auto& ps2 = pending_[p][0];
          int found = -1;
          for (int j = 0; j < (int)ps2.size(); ++j) {
            const PendingStep& c = ps2[j];
            if (c.st.op != OP_COPY || c.st.cnt != 1 || c.srcs.size() != 1) continue;
            const DevSrc& sr = c.srcs[0];
            if (sr.rank != r || sr.buf != ps.st.dst_buf || sr.chunk != ps.st.dst_chunk) continue;
            if (c.st.dst_buf != ps.st.dst_buf || c.st.dst_chunk != ps.st.dst_chunk || (c.st.flags & F_SCALE)) continue;
            bool only_owner = true;
            for (auto& kv : c.waits)
              if (kv.first.second >= 0 && !(kv.first.first == r && kv.first.second == 0 && kv.second == owner_done))
                only_owner = false;
            if (only_owner) { found = j; break; }
          }
          if (found < 0) break;
          peers.emplace_back(p, found);
        }
        if ((int)peers.size() != P_ - 1) continue;
        ps.st.op = OP_MC_ALLREDUCE;
        DevSrc first = ps.srcs[0];
        first.rank = (int16_t)r;
        ps.srcs.assign(1, first);
        for (auto& pj : peers) {
          PendingStep& c = pending_[pj.first][0][pj.second];
          c.st.op = OP_NOP;
          c.srcs.clear();
          c.mc_peer = true;
          c.mc_buf = ps.st.dst_buf;
          c.mc_chunk = ps.st.dst_chunk;
        }
        stats_.multicast_ops++;
      }
    }
    map_multicast_broadcasts();
    defer_multicast_arrivals();
  }

  // A chunk the owner copies locally into (OUT, c) while every other rank pulls the
  // same source into its own (OUT, c) is a broadcast: the owner's copy becomes one
  // multimem.st that writes (OUT, c) on every rank, the pulls become waits.
  void map_multicast_broadcasts() {
    for (int r = 0; r < P_; ++r) {
      auto& steps = pending_[r][0];
      for (int i = 0; i < (int)steps.size(); ++i) {
        PendingStep& ps = steps[i];
        if (ps.st.op != OP_COPY || ps.st.cnt != 1 || ps.srcs.size() != 1 || ps.srcs[0].rank != r ||
            (ps.st.flags & F_SCALE))
          continue;
        const DevSrc src = ps.srcs[0];
        const int owner_done = 2 * i + 2;
        std::vector<std::pair<int, int>> peers;
        for (int p = 0; p < P_; ++p) {
          if (p == r) continue;
          auto& ps2 = pending_[p][0];
          int found = -1;
          for (int j = 0; j < (int)ps2.size(); ++j) {
            const PendingStep& c = ps2[j];
            if (c.st.op != OP_COPY || c.st.cnt != 1 || c.srcs.size() != 1 || (c.st.flags & F_SCALE)) continue;
            const DevSrc& sr = c.srcs[0];
            if (sr.rank != r || sr.buf != src.buf || sr.chunk != src.chunk) continue;
            if (c.st.dst_buf != ps.st.dst_buf || c.st.dst_chunk != ps.st.dst_chunk) continue;
            // the pull may only wait for the data to be ready (start flags / owner events)
            bool plain = true;
            for (auto& kv : c.waits)
              if (kv.first.second >= 0 && kv.first.first != r) plain = false;
            if (plain) { found = j; break; }
          }
          if (found < 0) break;
          peers.emplace_back(p, found);
        }
        if ((int)peers.size() != P_ - 1) continue;
        // the owner now writes the peers' destinations: it must wait for their kernels to have started
        for (int p = 0; p < P_; ++p)
          if (p != r) merge(ps.waits, EventSet{{{p, -1}, 1}});
        ps.st.op = OP_MC_STORE;
        for (auto& pj : peers) {
          PendingStep& c = pending_[pj.first][0][pj.second];
          c.st.op = OP_NOP;
          c.srcs.clear();
          c.waits.clear();
          c.waits[{r, 0}] = owner_done;
          c.mc_peer = true;
          c.mc_buf = ps.st.dst_buf;
          c.mc_chunk = ps.st.dst_chunk;
        }
        stats_.multicast_ops++;
      }
    }
  }

  // A rank learns that an owner's multicast store reached its memory by waiting
  // for the owner's completion.  When nothing later on this rank reads that
  // destination, the wait is only needed before the kernel returns: it moves to
  // the end-of-kernel waits (last pipeline iteration), so the ranks no longer
  // meet at every chunk and stream through all iterations independently.
  void defer_multicast_arrivals() {
    for (int r = 0; r < P_; ++r) {
      auto& steps = pending_[r][0];
      for (int i = 0; i < (int)steps.size(); ++i) {
        PendingStep& ps = steps[i];
        if (!ps.mc_peer || ps.waits.empty()) continue;
        bool read_later = false;
        for (int j = i + 1; j < (int)steps.size() && !read_later; ++j)
          for (auto& sr : steps[j].srcs)
            if (sr.rank == r && sr.buf == ps.mc_buf && sr.chunk == ps.mc_chunk) read_later = true;
        for (int q = 0; q < P_ && !read_later; ++q)
          if (q != r)
            for (auto& other : pending_[q][0])
              for (auto& sr : other.srcs)
                if (sr.rank == r && sr.buf == ps.mc_buf && sr.chunk == ps.mc_chunk) read_later = true;
        if (read_later) continue;
        for (auto& kv : ps.waits)
          if (kv.first.second >= 0) merge(end_waits_[r], EventSet{{kv.first, kv.second}});
        ps.waits.clear();
        stats_.deferred_waits++;
      }
    }
  }

  // A peer's start flag holds for the whole launch: once a block waited for it,
  // later steps of the block need not poll it again.
  void dedupe_start_waits() {
    for (int r = 0; r < P_; ++r)
      for (auto& blk : pending_[r]) {
        std::set<int> seen;
        for (auto& ps : blk) {
          for (auto it = ps.waits.begin(); it != ps.waits.end();) {
            if (it->first.second < 0 && seen.count(it->first.first)) it = ps.waits.erase(it);
            else ++it;
          }
          for (auto& kv : ps.waits)
            if (kv.first.second < 0) seen.insert(kv.first.first);
        }
      }
  }

  // A merged NOP step that waits for nothing and whose events no step waits
  // for does no work: it marks an elided send or a copy that a multicast
  // store replaced.  Such steps are removed (every rank keeps at least one
  // step) and the events of later steps are renumbered in every wait.  End
  // waits are unaffected: they target the block's final event, which emit
  // derives from the final step count.
  void drop_idle_nops() {
    std::vector<std::set<int>> named(P_);
    for (int r = 0; r < P_; ++r)
      for (auto& ps : pending_[r][0])
        for (auto& kv : ps.waits)
          if (kv.first.second >= 0) named[kv.first.first].insert((kv.second - 1) / 2);
    std::vector<std::vector<int>> newidx(P_);
    for (int r = 0; r < P_; ++r) {
      auto& steps = pending_[r][0];
      std::vector<bool> keep(steps.size(), true);
      int kept = 0;
      for (int i = 0; i < (int)steps.size(); ++i) {
        const PendingStep& ps = steps[i];
        if (ps.st.op == OP_NOP && ps.waits.empty() && !named[r].count(i)) keep[i] = false;
        kept += keep[i] ? 1 : 0;
      }
      if (kept == 0 && !steps.empty()) keep.back() = true;
      newidx[r].assign(steps.size(), -1);
      int n = 0;
      for (int i = 0; i < (int)steps.size(); ++i)
        if (keep[i]) newidx[r][i] = n++;
      stats_.dropped_nops += (int)steps.size() - n;
    }
    for (int r = 0; r < P_; ++r) {
      std::vector<PendingStep> out;
      auto& steps = pending_[r][0];
      for (int i = 0; i < (int)steps.size(); ++i) {
        if (newidx[r][i] < 0) continue;
        PendingStep ps = steps[i];
        EventSet waits;
        for (auto& kv : ps.waits) {
          if (kv.first.second < 0) {
            merge(waits, EventSet{{kv.first, kv.second}});
            continue;
          }
          int target = newidx[kv.first.first][(kv.second - 1) / 2];
          if (target < 0) fail("a wait names a removed step");
          merge(waits, EventSet{{kv.first, 2 * target + ((kv.second % 2) ? 1 : 2)}});
        }
        ps.waits = std::move(waits);
        out.push_back(std::move(ps));
      }
      steps = std::move(out);
      dsteps_count_[r].assign(1, (int)steps.size());
    }
  }

  void emit() {
    for (int r = 0; r < P_; ++r) {
      RankProgram& rp = out_[r];
      for (int db = 0; db < nblocks_[r]; ++db) {
        DevBlock blk{};
        blk.step_begin = (int)rp.steps.size();
        blk.xml_tb = -1;
        if (!merged_)
          for (int t = 0; t < (int)dblock_[r].size(); ++t) if (dblock_[r][t] == db) blk.xml_tb = a_.gpus[r].tbs[t].id;
        auto& steps = pending_[r][db];
        blk.nsteps = (int)steps.size();
        for (int s = 0; s < (int)steps.size(); ++s) {
          PendingStep& ps = steps[s];
          DevStep st = ps.st;
          st.src_begin = (int)rp.srcs.size();
          st.nsrc = (int)ps.srcs.size();
          for (auto& sr : ps.srcs) rp.srcs.push_back(sr);
          st.wait_begin = (int)rp.waits.size();
          st.wait_count = 0;
          for (auto& kv : ps.waits) {
            DevWait w{};
            w.rank = (int16_t)kv.first.first;
            w.block = (int16_t)kv.first.second;
            w.stride = w.block < 0 ? 0 : 2 * dsteps_count_[w.rank][w.block];
            w.event = kv.second;
            w.iter_delta = 0;
            rp.waits.push_back(w);
            st.wait_count++;
            stats_.waits++;
            if (w.rank != r) stats_.remote_waits++;
            if (w.block >= 0) published_.insert({w.rank, w.block, w.event});
          }
          rp.steps.push_back(st);
          rp.step_origins.push_back({ps.xml_step >= 0 ? ps.xml_tb : -1, ps.xml_step});
          ++stats_.device_steps;
        }
        blk.end_wait_begin = (int)rp.waits.size();
        blk.end_wait_count = 0;
        if (db == 0) {
          // End-of-kernel waits target the peer block's final event (every CTA publishes it once,
          // after its last step), which implies every earlier event of that block.
          for (auto& kv : end_waits_[r]) {
            DevWait w{};
            w.rank = (int16_t)kv.first.first;
            w.block = (int16_t)kv.first.second;
            w.stride = 2 * dsteps_count_[w.rank][w.block];
            w.event = 2 * dsteps_count_[w.rank][w.block];
            w.iter_delta = -1;
            rp.waits.push_back(w);
            blk.end_wait_count++;
          }
        }
        rp.blocks.push_back(blk);
      }
    }
    // scratch actually referenced by device steps
    for (int r = 0; r < P_; ++r) out_[r].s_used = 0;
    for (int r = 0; r < P_; ++r) {
      RankProgram& rp = out_[r];
      for (auto& st : rp.steps) {
        if (st.op == OP_NOP) continue;
        if (st.dst_buf == BUF_SCR) rp.s_used = std::max(rp.s_used, st.dst_chunk + st.cnt);
        for (int i = 0; i < st.nsrc; ++i) {
          const DevSrc& sr = rp.srcs[st.src_begin + i];
          if (sr.buf == BUF_SCR) {
            // a remote source lives in the source rank's scratch
            out_[sr.rank].s_used = std::max(out_[sr.rank].s_used, sr.chunk + st.cnt);
          }
        }
      }
    }
    // publication flags
    for (auto& e : published_) {
      int rank, block, event;
      std::tie(rank, block, event) = e;
      DevStep& st = out_[rank].steps[out_[rank].blocks[block].step_begin + (event - 1) / 2];
      st.flags |= (event % 2 == 1) ? F_PUB_ARRIVE : F_PUB_DONE;
    }
  }

  // Device-level deadlock check: arrive/done events of every step as graph nodes.
  void deadlock_check() {
    std::map<std::tuple<int, int, int>, std::vector<std::tuple<int, int, int>>> succ;
    std::map<std::tuple<int, int, int>, int> indeg;
    auto node = [&](int r, int b, int e) { return std::make_tuple(r, b, e); };
    for (int r = 0; r < P_; ++r)
      for (int b = 0; b < (int)out_[r].blocks.size(); ++b) {
        const DevBlock& blk = out_[r].blocks[b];
        for (int s = 0; s < blk.nsteps; ++s) {
          indeg[node(r, b, 2 * s + 1)];
          indeg[node(r, b, 2 * s + 2)];
          succ[node(r, b, 2 * s + 1)].push_back(node(r, b, 2 * s + 2));
          indeg[node(r, b, 2 * s + 2)]++;
          if (s > 0) { succ[node(r, b, 2 * s)].push_back(node(r, b, 2 * s + 1)); indeg[node(r, b, 2 * s + 1)]++; }
          const DevStep& st = out_[r].steps[blk.step_begin + s];
          for (int w = 0; w < st.wait_count; ++w) {
            const DevWait& dw = out_[r].waits[st.wait_begin + w];
            if (dw.block < 0) continue;
            if (dw.rank >= P_ || dw.block >= (int)out_[dw.rank].blocks.size() || dw.event < 1 ||
                dw.event > 2 * out_[dw.rank].blocks[dw.block].nsteps)
              fail("compiled wait names an unknown event");
            succ[node(dw.rank, dw.block, dw.event)].push_back(node(r, b, 2 * s + 1));
            indeg[node(r, b, 2 * s + 1)]++;
          }
        }
      }
    std::deque<std::tuple<int, int, int>> q;
    for (auto& kv : indeg) if (kv.second == 0) q.push_back(kv.first);
    size_t seen = 0;
    while (!q.empty()) {
      auto n = q.front();
      q.pop_front();
      ++seen;
      for (auto& m : succ[n]) if (--indeg[m] == 0) q.push_back(m);
    }
    if (seen != indeg.size())
      fail("compiled device program deadlocks under pull semantics (the schedule relies on FIFO buffering)");
  }

  const XAlgo& a_;
  CompileOptions o_;
  int P_;
  std::vector<std::map<int, int>> tb_index_;
  std::vector<SRef> all_, order_;
  std::map<SRef, int> topo_pos_, level_;
  std::map<SRef, SRef> match_recv_, match_send_;
  std::set<SRef> scale_steps_, need_arrive_;
  std::vector<std::vector<int>> dblock_;
  std::vector<int> nblocks_;
  std::vector<bool> synthetic_;
  std::vector<std::vector<int>> dsteps_count_;
  std::map<SRef, EventSet> completion_memo_, arrival_memo_;
  std::map<SRef, SRef> fused_into_;
  std::map<SRef, std::vector<SRef>> chains_;
  std::vector<std::vector<std::vector<PendingStep>>> pending_;
  std::vector<EventSet> end_waits_;
  std::set<std::tuple<int, int, int>> published_;
  std::vector<RankProgram> out_;
  CompileStats stats_;
  bool merged_ = false;
  std::map<Region, SRef> last_writer_;
  std::vector<Region> unscaled_outputs_;
  std::set<int> synthetic_extra_;
};

}  // namespace

namespace {

// Under pull semantics the next hop reads a forwarded value out of the forwarding rank's memory, so an
// 'rrs' (receive, reduce with a local operand, send on, without a local store) becomes an 'rrcs' whose
// store goes to a scratch region of its own, appended to that rank's scratch buffer.
XAlgo stage_forwarded_reductions(const XAlgo& algo, int* staged) {
  XAlgo out = algo;
  *staged = 0;
  for (XGpu& g : out.gpus)
    for (XTB& b : g.tbs)
      for (XStep& st : b.steps) {
        if (st.kind != X_RRS) continue;
        if (st.cnt < 1) throw CompileError("an 'rrs' step needs a positive count");
        st.kind = X_RRCS;
        st.dstbuf = BUF_SCR;
        st.dstoff = g.s_chunks;
        g.s_chunks += st.cnt;
        ++*staged;
      }
  return out;
}

CompiledPlan compile_staged(const XAlgo& algo, const CompileOptions& options) {
  if (options.fuse_chains) {
    try {
      Compiler c(algo, options);
      return c.run();
    } catch (const CompileError& e) {
      // Fusion can order a chain's reads later than a dependent overwrite; retry without it.
      if (std::string(e.what()).find("deadlocks under pull") == std::string::npos) throw;
      CompileOptions plain = options;
      plain.fuse_chains = false;
      Compiler c(algo, plain);
      return c.run();
    }
  }
  Compiler c(algo, options);
  return c.run();
}

}  // namespace

CompiledPlan compile_plan(const XAlgo& algo, const CompileOptions& options) {
  if (options.nlanes < 1 || options.nlanes > kMaxFlagLanes) throw CompileError("nlanes must be in [1, 256]");
  if (options.niters < 1) throw CompileError("niters must be positive");
  int staged = 0;
  XAlgo prepared = stage_forwarded_reductions(algo, &staged);
  CompiledPlan plan = compile_staged(prepared, options);
  plan.stats.staged_forwards = staged;
  return plan;
}

std::string describe_rank(const CompiledPlan& plan, int rank) {
  static const char* ops[] = {"nop", "copy", "reduce", "mc_reduce", "mc_store", "mc_allreduce"};
  std::ostringstream o;
  const RankProgram& rp = plan.ranks.at(rank);
  for (size_t b = 0; b < rp.blocks.size(); ++b) {
    const DevBlock& blk = rp.blocks[b];
    o << "block " << b << " (xml tb " << blk.xml_tb << ")\n";
    for (int s = 0; s < blk.nsteps; ++s) {
      const DevStep& st = rp.steps[blk.step_begin + s];
      o << "  " << s << ": " << ops[st.op];
      if (st.op != OP_NOP) {
        o << " -> ";
        if (st.dst_rank >= 0 && st.dst_rank != rank) o << "r" << st.dst_rank << ":";
        o << "ios"[st.dst_buf] << "[" << st.dst_chunk << "]";
      }
      for (int i = 0; i < st.nsrc; ++i) {
        const DevSrc& sr = rp.srcs[st.src_begin + i];
        o << (i ? ", " : " <- ") << "r" << sr.rank << ":" << "ios"[sr.buf] << "[" << sr.chunk << "]";
      }
      if (st.flags & F_SCALE) o << " scale";
      if (st.flags & F_PUB_ARRIVE) o << " pubA";
      if (st.flags & F_PUB_DONE) o << " pubD";
      for (int w = 0; w < st.wait_count; ++w) {
        const DevWait& dw = rp.waits[st.wait_begin + w];
        o << " wait(r" << dw.rank << ",b" << dw.block << ",e" << dw.event << ")";
      }
      o << "\n";
    }
    for (int w = 0; w < blk.end_wait_count; ++w) {
      const DevWait& dw = rp.waits[blk.end_wait_begin + w];
      o << "  end wait(r" << dw.rank << ",b" << dw.block << ",e" << dw.event << ")\n";
    }
  }
  return o.str();
}

}  // namespace vb
