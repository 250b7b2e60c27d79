// vericcl-native: run one rank of a synthesized schedule and write a receipt.
//
// Usage: vericcl-native <config.json>
// config: {"xml": path, "rank": r, "nranks": p, "device": d, "control_address": "127.0.0.1",
//          "control_port": port, "session": id, "count": elements per rank, "dtype": 0|1|2,
//          "redop": 0..3, "scale": f, "nlanes": L, "niters": I, "warmup": W, "iters": K,
//          "timeout_s": t, "receipt": path[, "trace": path of a per-step trace of the last invocation]
//          [, "root": r for broadcast / reduce]}
// Inputs follow the analytic pattern value = 1 + ((3*rank + i) mod 5); outputs
// are checked on the device in fp64 against the analytic result of the
// schedule's collective (scale applied to reductions), and the input buffer is
// re-checked afterwards (it is read-only).  The receipt reports both counts.
#include <cuda_runtime.h>

#include <cstdio>
#include <fstream>
#include <sstream>
#include <vector>

#include "vb/contract.h"
#include "vb/launch.h"
#include "vericcl_b200.h"

using namespace vb;

int main(int argc, char** argv) {
  if (argc != 2) {
    fprintf(stderr, "usage: %s <config.json>\n", argv[0]);
    return 2;
  }
  std::ifstream f(argv[1]);
  std::stringstream ss;
  ss << f.rdbuf();
  Json cfg = parse_json(ss.str());
  std::ifstream xf(cfg.at("xml").as_string());
  std::stringstream xs;
  xs << xf.rdbuf();
  int rank = (int)cfg.at("rank").as_int(), nranks = (int)cfg.at("nranks").as_int();
  int dtype = (int)cfg.at("dtype").as_int(), redop = (int)cfg.at("redop").as_int();
  size_t count = (size_t)cfg.at("count").as_int();
  double timeout = cfg.at("timeout_s").as_double();
  cudaSetDevice((int)cfg.at("device").as_int());
  vb_init_params p = {};
  p.abi_version = VERICCL_B200_ABI_VERSION;
  p.rank = rank;
  p.nranks = nranks;
  p.device = (int)cfg.at("device").as_int();
  std::string addr = cfg.at("control_address").as_string(), session = cfg.at("session").as_string();
  p.control_address = addr.c_str();
  p.control_port = (int)cfg.at("control_port").as_int();
  p.session = session.c_str();
  p.timeout_s = timeout;
  p.heap_bytes = (size_t)64 << 20;
  p.heap_bytes += count * 4 * (size_t)nranks * 3;
  vb_context* ctx = nullptr;
  vb_result r = vb_init(&p, &ctx);
  if (r != VB_OK) { fprintf(stderr, "vb_init failed: %d\n", r); return 8; }
  r = vb_prepare(ctx, xs.str().c_str(), (int)cfg.at("nlanes").as_int(), (int)cfg.at("niters").as_int(), timeout);
  if (r != VB_OK) { fprintf(stderr, "vb_prepare failed: %d %s\n", r, vb_last_error(ctx)); return 8; }
  // the collective named by the <algo coll="..."> attribute
  std::string coll = "allreduce";
  {
    const std::string& text = xs.str();
    size_t at = text.find("coll=\"");
    if (at != std::string::npos) {
      size_t end = text.find('"', at + 6);
      if (end != std::string::npos) coll = text.substr(at + 6, end - at - 6);
    }
  }
  int check_code = coll == "allgather" ? 1 : coll == "reduce_scatter" ? 2 : coll == "broadcast" ? 3
                   : coll == "reduce" ? 4 : coll == "alltoall" ? 5 : 0;
  const Json* root_cfg = cfg.get("root");
  int root = root_cfg ? (int)root_cfg->as_int() : 0;
  size_t esz = dtype == 0 ? 4 : 2;
  size_t out_count = coll == "allgather" ? count * nranks : coll == "reduce_scatter" ? count / nranks : count;
  void *in = nullptr, *out = nullptr;
  unsigned long long* bad = nullptr;
  cudaMalloc(&in, count * esz);
  cudaMalloc(&out, out_count * esz);
  cudaMalloc(&bad, 2 * sizeof(unsigned long long));
  cudaStream_t s;
  cudaStreamCreate(&s);
  launch_fill(in, (long long)count, dtype, 0, rank, 0, s);
  float scale = (float)cfg.at("scale").as_double();
  int warmup = (int)cfg.at("warmup").as_int(), iters = (int)cfg.at("iters").as_int();
  std::vector<double> times;
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  const Json* trace_path = cfg.get("trace");
  for (int i = 0; i < warmup + iters; ++i) {
    if (trace_path && i == warmup + iters - 1 && vb_trace_arm(ctx) != VB_OK) {
      fprintf(stderr, "vb_trace_arm failed: %s\n", vb_last_error(ctx));
      return 8;
    }
    cudaEventRecord(e0, s);
    r = vb_execute(ctx, in, out, count, dtype, redop, scale, s, timeout);
    cudaEventRecord(e1, s);
    cudaEventSynchronize(e1);
    if (r != VB_OK) { fprintf(stderr, "vb_execute failed: %d %s\n", r, vb_last_error(ctx)); return 8; }
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    if (i >= warmup) times.push_back(ms * 1e3);
  }
  if (trace_path && vb_trace_write(ctx, trace_path->as_string().c_str()) != VB_OK) {
    fprintf(stderr, "vb_trace_write failed: %s\n", vb_last_error(ctx));
    return 8;
  }
  cudaMemsetAsync(bad, 0, 2 * sizeof(unsigned long long), s);
  // a reduce defines the output on its root only
  long long checked = (check_code == 4 && rank != root) ? 0 : (long long)out_count;
  launch_check(out, checked, dtype, check_code, redop, nranks, rank, (long long)count, 1e-2, 1e-2, bad, s, root,
               (double)scale);
  // the input is read-only: it must still hold this rank's pattern
  launch_check(in, (long long)count, dtype, 6, redop, nranks, rank, (long long)count, 0.0, 0.0, bad + 1, s);
  unsigned long long nbad[2] = {0, 0};
  cudaMemcpyAsync(nbad, bad, sizeof nbad, cudaMemcpyDeviceToHost, s);
  cudaStreamSynchronize(s);
  std::ofstream receipt(cfg.at("receipt").as_string());
  receipt << "{\"rank\":" << rank << ",\"nranks\":" << nranks << ",\"count\":" << count << ",\"coll\":\"" << coll
          << "\",\"bad\":" << nbad[0] << ",\"bad_input\":" << nbad[1] << ",\"device_times_us\":[";
  for (size_t i = 0; i < times.size(); ++i) receipt << (i ? "," : "") << times[i];
  receipt << "],\"abi\":" << vb_abi_version() << "}\n";
  receipt.close();
  vb_close(ctx, timeout);
  vb_destroy(ctx);
  return (nbad[0] || nbad[1]) ? 5 : 0;
}
