// The C API's execute path on the CPU stand-ins (tests/native/cpu_stubs): two
// ranks as threads over the loopback control plane.  Checks that staging
// buffers get the same heap offsets on every rank (also for a reduce, whose
// output buffer exists on its root only), that each staging buffer grows on
// its own, and that an execution whose stream never completes is left
// unresolved: the abort flag is raised, later calls are refused and the
// context keeps its buffers (release, close and destroy all refuse).
// Usage: test_capi_cpu <allreduce.xml> <reduce-root1.xml>
#include <cuda_runtime.h>

#include <cstdio>
#include <fstream>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

#include "vb/launch.h"
#include "vericcl_b200.h"

#include <unistd.h>

namespace vb_stub {
std::vector<std::pair<size_t, size_t>> alloc_log(const std::string& session, int rank);
int abort_request(const std::string& session, int rank);
}

#define CHECK(x) do { if (!(x)) { fprintf(stderr, "FAILED %s:%d %s\n", __FILE__, __LINE__, #x); failures++; } } while (0)

static int failures = 0;

static std::string slurp(const char* path) {
  std::ifstream f(path);
  std::stringstream ss;
  ss << f.rdbuf();
  return ss.str();
}

struct Rank {
  vb_context* ctx = nullptr;
  vb_result init = VB_FAILED, prepare = VB_FAILED;
};

// vb_init + vb_prepare on two threads (they rendezvous over the control plane)
static std::vector<Rank> start(const std::string& session, int port, const std::string& xml) {
  std::vector<Rank> ranks(2);
  std::vector<std::thread> ts;
  for (int r = 0; r < 2; ++r) {
    ts.emplace_back([&, r] {
      vb_init_params p = {};
      p.abi_version = VERICCL_B200_ABI_VERSION;
      p.rank = r;
      p.nranks = 2;
      p.device = r;
      p.control_address = "127.0.0.1";
      p.control_port = port;
      p.session = session.c_str();
      p.timeout_s = 10;
      p.heap_bytes = 8 << 20;
      ranks[r].init = vb_init(&p, &ranks[r].ctx);
      if (ranks[r].init == VB_OK) ranks[r].prepare = vb_prepare(ranks[r].ctx, xml.c_str(), 2, 1, 10);
    });
  }
  for (auto& t : ts) t.join();
  return ranks;
}

static void execute_both(std::vector<Rank>& ranks, size_t count, std::vector<vb_result>& res, double timeout = 5) {
  std::vector<std::vector<float>> in(2, std::vector<float>(count, 1.0f)), out(2, std::vector<float>(count * 2));
  std::vector<std::thread> ts;
  for (int r = 0; r < 2; ++r)
    ts.emplace_back([&, r] { res[r] = vb_execute(ranks[r].ctx, in[r].data(), out[r].data(), count, VB_FLOAT32, 0,
                                                 1.0f, nullptr, timeout); });
  for (auto& t : ts) t.join();
}

int main(int argc, char** argv) {
  if (argc != 3) {
    fprintf(stderr, "usage: %s <allreduce.xml> <reduce-root1.xml>\n", argv[0]);
    return 2;
  }
  const int port = 20000 + (int)(getpid() % 20000);
  {
    // a reduce has an output buffer on its root only: the staging layout must still agree
    auto ranks = start("reduce", port, slurp(argv[2]));
    CHECK(ranks[0].init == VB_OK && ranks[1].init == VB_OK);
    CHECK(ranks[0].prepare == VB_OK && ranks[1].prepare == VB_OK);
    std::vector<vb_result> res(2, VB_FAILED);
    execute_both(ranks, 1024, res);
    CHECK(res[0] == VB_OK && res[1] == VB_OK);
    auto a = vb_stub::alloc_log("reduce", 0), b = vb_stub::alloc_log("reduce", 1);
    CHECK(!a.empty() && a == b);
    std::vector<vb_result> closed(2, VB_FAILED);
    std::vector<std::thread> ts;
    for (int r = 0; r < 2; ++r) ts.emplace_back([&, r] { closed[r] = vb_close(ranks[r].ctx, 5); });
    for (auto& t : ts) t.join();
    CHECK(closed[0] == VB_OK && closed[1] == VB_OK);
    for (auto& r : ranks) CHECK(vb_destroy(r.ctx) == VB_OK);
  }
  {
    auto ranks = start("allreduce", port + 1, slurp(argv[1]));
    CHECK(ranks[0].prepare == VB_OK && ranks[1].prepare == VB_OK);
    std::vector<vb_result> res(2, VB_FAILED);
    execute_both(ranks, 1024, res);
    CHECK(res[0] == VB_OK && res[1] == VB_OK);
    size_t first = vb_stub::alloc_log("allreduce", 0).size();
    execute_both(ranks, 512, res);                      // smaller: the staging buffers are reused
    CHECK(res[0] == VB_OK && res[1] == VB_OK);
    CHECK(vb_stub::alloc_log("allreduce", 0).size() == first);
    execute_both(ranks, 4096, res);                     // larger: they grow, alike on both ranks
    CHECK(res[0] == VB_OK && res[1] == VB_OK);
    CHECK(vb_stub::alloc_log("allreduce", 0).size() > first);
    CHECK(vb_stub::alloc_log("allreduce", 0) == vb_stub::alloc_log("allreduce", 1));
    int status = -1;
    unsigned long long epoch = 0;
    CHECK(vb_status(ranks[0].ctx, &status, &epoch) == VB_OK && status == 0 && epoch == 3);

    // a stream that never completes: the execution is unresolved and ownership is kept
    vb_stub::set_streams_hung(true);
    execute_both(ranks, 1024, res, 0.05);
    vb_stub::set_streams_hung(false);
    CHECK(res[0] == VB_UNRESOLVED && res[1] == VB_UNRESOLVED);
    for (int rank = 0; rank < 2; ++rank) {
      vb_context* ctx = ranks[rank].ctx;
      // the abort request reached the rank's control block, where the device's bounded waits read it
      CHECK(vb_stub::abort_request("allreduce", rank) == 1);
      std::vector<float> in(1024), out(1024);
      CHECK(vb_execute(ctx, in.data(), out.data(), 1024, VB_FLOAT32, 0, 1.0f, nullptr, 1) == VB_FAILED);
      CHECK(vb_release(ctx) == VB_UNRESOLVED);
      CHECK(vb_close(ctx, 1) == VB_UNRESOLVED);
      CHECK(vb_destroy(ctx) == VB_UNRESOLVED);
    }
  }
  if (failures) {
    fprintf(stderr, "%d check(s) failed\n", failures);
    return 1;
  }
  printf("capi cpu tests passed\n");
  return 0;
}
