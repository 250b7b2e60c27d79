// TCP control plane for native collective set-up and launch agreement.
//
// Rank 0 runs a coordinator (a non-blocking poll loop on its own thread).
// ``gather(phase, payload)`` sends a length-prefixed strict-JSON frame
// {session, rank, phase, sequence, payload} and waits for the decision: every
// rank's payload for that sequence, in rank order.  The coordinator keeps the
// decisions of the last two sequences, so a retransmitted request gets the
// same reply (idempotent retries after a lost reply).  A session, phase or
// sequence mismatch breaks the session: every later request fails.  Frames
// are limited to 4 MiB.  ``inject_lost_replies_for_test`` makes the
// coordinator drop replies to exercise the retry path.
#pragma once
#include <atomic>
#include <condition_variable>
#include <deque>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "vb/contract.h"

namespace vb {

struct ControlError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

class Coordinator {
 public:
  Coordinator(const std::string& address, int port, int nranks, const std::string& session);
  ~Coordinator();
  int port() const { return port_; }
  void stop();
  void inject_lost_replies_for_test(int n) { lose_replies_.store(n); }
  bool broken() const { return broken_.load(); }

 private:
  struct Pending {
    int fd;
    int rank;
    std::string inbuf;
  };
  void loop();
  std::string handle(const Json& req, bool* drop);
  int listen_fd_ = -1, port_ = 0, nranks_;
  std::string session_;
  std::thread thread_;
  std::atomic<bool> stop_{false}, broken_{false};
  std::atomic<int> lose_replies_{0};
  std::string break_reason_;
  // sequence -> (phase, payload per rank)
  std::map<long long, std::pair<std::string, std::map<int, std::string>>> open_;
  std::map<long long, std::string> decided_;   // last two decisions
  std::map<long long, std::vector<int>> waiters_;
};

class ControlTransport {
 public:
  ControlTransport(int rank, int nranks, const std::string& address, int port, const std::string& session);
  ~ControlTransport();
  // All ranks' payloads for this phase (collective; same call order on every rank).
  std::vector<std::string> gather(const std::string& phase, const std::string& payload, const Deadline& deadline);
  void barrier(const std::string& phase, const Deadline& deadline) { gather(phase, "", deadline); }
  Coordinator* coordinator() { return coord_.get(); }
  int rank() const { return rank_; }
  int nranks() const { return nranks_; }

 private:
  int rank_, nranks_, port_;
  std::string address_, session_;
  long long sequence_ = 0;
  std::unique_ptr<Coordinator> coord_;
};

// Frame helpers (length-prefixed JSON) with a deadline; return false on timeout/close.
bool send_frame(int fd, const std::string& body, const Deadline& deadline);
bool recv_frame(int fd, std::string* body, const Deadline& deadline);

}  // namespace vb
