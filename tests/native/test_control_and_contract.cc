// CPU-only tests of the native contract utilities and the control transport.
#include <cassert>
#include <cstdio>
#include <stdexcept>
#include <thread>
#include <vector>

#include "vb/contract.h"
#include "vb/control.h"
#include "vb/trace_io.h"

using namespace vb;

#define CHECK(x) do { if (!(x)) { fprintf(stderr, "FAILED %s:%d %s\n", __FILE__, __LINE__, #x); return 1; } } while (0)

template <typename F>
bool throws(F f) {
  try { f(); } catch (const std::exception&) { return true; }
  return false;
}

int main(int argc, char** argv) {
  // FIPS 180-2 example vectors
  CHECK(sha256_hex("abc") == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad");
  CHECK(sha256_hex("") == "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855");
  CHECK(sha256_hex("abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq") ==
        "248d6a61d20638b8e5c026930c3e6039a33ce45964ff2167f6ecedd419db06c1");
  Json j = parse_json("{\"a\": [1, 2.5, \"x\"], \"b\": {\"c\": null}}");
  CHECK(j.at("a").arr[1].as_double() == 2.5);
  CHECK(throws([] { parse_json("{\"a\":1,\"a\":2}"); }));
  CHECK(throws([] { parse_json("[1e999]"); }));
  CHECK(throws([] { parse_json("[1] x"); }));
  std::string deep(70, '[');
  CHECK(throws([&] { parse_json(deep); }));
  CHECK(throws([] { require_exact_keys(parse_json("{\"a\":1,\"z\":2}"), {"a"}, "doc"); }));
  CHECK(throws([] { checked_mul(SIZE_MAX, 2); }));

  // three ranks as threads over loopback, with lost replies
  ControlTransport r0(0, 3, "127.0.0.1", 0, "s1");
  int port = r0.coordinator()->port();
  r0.coordinator()->inject_lost_replies_for_test(2);
  std::vector<std::vector<std::string>> got(3);
  std::thread t1([&] { ControlTransport t(1, 3, "127.0.0.1", port, "s1"); got[1] = t.gather("PREPARE", "b", Deadline::after(10)); got[1].push_back(t.gather("READY", "y", Deadline::after(10))[2]); });
  std::thread t2([&] { ControlTransport t(2, 3, "127.0.0.1", port, "s1"); got[2] = t.gather("PREPARE", "c", Deadline::after(10)); got[2].push_back(t.gather("READY", "z", Deadline::after(10))[2]); });
  got[0] = r0.gather("PREPARE", "a", Deadline::after(10));
  got[0].push_back(r0.gather("READY", "x", Deadline::after(10))[2]);
  t1.join();
  t2.join();
  for (int r = 0; r < 3; ++r) {
    CHECK(got[r].size() == 4 && got[r][0] == "a" && got[r][1] == "b" && got[r][2] == "c" && got[r][3] == "z");
  }
  // a member that never arrives: the phase times out instead of hanging
  ControlTransport lonely(0, 2, "127.0.0.1", 0, "s2");
  CHECK(throws([&] { lonely.gather("INIT", "", Deadline::after(0.5)); }));
  // a phase mismatch breaks the session
  ControlTransport m0(0, 2, "127.0.0.1", 0, "s3");
  int p3 = m0.coordinator()->port();
  std::thread bad([&] { ControlTransport t(1, 2, "127.0.0.1", p3, "s3"); try { t.gather("OTHER", "", Deadline::after(3)); } catch (...) {} });
  bool broke = throws([&] { m0.gather("INIT", "", Deadline::after(3)); });
  bad.join();
  CHECK(broke || m0.coordinator()->broken());
  // wrong session id is rejected
  ControlTransport w0(0, 2, "127.0.0.1", 0, "s4");
  int p4 = w0.coordinator()->port();
  bool rejected = throws([&] { ControlTransport t(1, 2, "127.0.0.1", p4, "other"); t.gather("INIT", "", Deadline::after(2)); });
  CHECK(rejected);
  // trace file: block 0 has 3 steps, block 1 has 1 step; 2 lanes, 2 iterations
  if (argc > 1) {
    TraceLayout l;
    l.rank = 3;
    l.nlanes = 2;
    l.niters = 2;
    l.max_steps = 3;
    l.block_ops = {{1, 2, 0}, {4}};
    std::vector<uint64_t> raw(trace_words(l), 0);
    CHECK(raw.size() == (size_t)2 * 2 * 2 * 3 * 3);
    for (int cta = 0; cta < 4; ++cta) {
      int nsteps = (int)l.block_ops[cta / 2].size();
      for (int it = 0; it < 2; ++it)
        for (int s = 0; s < nsteps; ++s) {
          size_t slot = (size_t)cta * 6 + (size_t)it * nsteps + s;
          raw[slot * 3] = 1000 * cta + 100 * it + 10 * s + 1;
          raw[slot * 3 + 1] = 1000 * cta + 100 * it + 10 * s + 5;
          raw[slot * 3 + 2] = 2;
        }
    }
    CHECK(write_trace_file(argv[1], l, raw) == 2 * 2 * 3 + 2 * 2 * 1);
    CHECK(throws([&] { write_trace_file(argv[1], l, std::vector<uint64_t>(3)); }));
  }
  printf("native cpu tests passed\n");
  return 0;
}
