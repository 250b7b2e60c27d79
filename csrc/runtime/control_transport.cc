// TCP control plane implementation.
#include "vb/control.h"

#include <arpa/inet.h>
#include <errno.h>
#include <fcntl.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <cstring>

namespace vb {
namespace {

constexpr size_t kMaxFrame = 4u << 20;

int wait_fd(int fd, short events, const Deadline& d) {
  double rem = d.remaining();
  if (rem <= 0) return 0;
  struct pollfd p = {fd, events, 0};
  int ms = (int)(rem * 1000) + 1;
  return poll(&p, 1, ms > 200 ? 200 : ms);
}

}  // namespace

bool send_frame(int fd, const std::string& body, const Deadline& deadline) {
  if (body.size() > kMaxFrame) throw ControlError("control frame exceeds 4 MiB");
  uint32_t n = htonl((uint32_t)body.size());
  std::string buf(reinterpret_cast<const char*>(&n), 4);
  buf += body;
  size_t off = 0;
  while (off < buf.size()) {
    if (deadline.expired()) return false;
    if (wait_fd(fd, POLLOUT, deadline) <= 0) continue;
    ssize_t k = ::send(fd, buf.data() + off, buf.size() - off, MSG_NOSIGNAL);
    if (k <= 0) {
      if (errno == EAGAIN || errno == EINTR) continue;
      return false;
    }
    off += (size_t)k;
  }
  return true;
}

bool recv_frame(int fd, std::string* body, const Deadline& deadline) {
  std::string buf;
  size_t need = 4;
  bool have_len = false;
  while (buf.size() < need) {
    if (deadline.expired()) return false;
    if (wait_fd(fd, POLLIN, deadline) <= 0) continue;
    char tmp[65536];
    size_t want = need - buf.size();
    ssize_t k = ::recv(fd, tmp, want < sizeof tmp ? want : sizeof tmp, 0);
    if (k == 0) return false;
    if (k < 0) {
      if (errno == EAGAIN || errno == EINTR) continue;
      return false;
    }
    buf.append(tmp, (size_t)k);
    if (!have_len && buf.size() >= 4) {
      uint32_t n;
      memcpy(&n, buf.data(), 4);
      n = ntohl(n);
      if (n > kMaxFrame) return false;
      need = 4 + n;
      have_len = true;
    }
  }
  *body = buf.substr(4);
  return true;
}

Coordinator::Coordinator(const std::string& address, int port, int nranks, const std::string& session)
    : nranks_(nranks), session_(session) {
  listen_fd_ = socket(AF_INET, SOCK_STREAM, 0);
  int one = 1;
  setsockopt(listen_fd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof one);
  sockaddr_in a = {};
  a.sin_family = AF_INET;
  a.sin_port = htons((uint16_t)port);
  if (inet_pton(AF_INET, address.c_str(), &a.sin_addr) != 1) throw ControlError("invalid control address " + address);
  if (bind(listen_fd_, (sockaddr*)&a, sizeof a) != 0 || listen(listen_fd_, 128) != 0)
    throw ControlError(std::string("cannot listen on the control port: ") + strerror(errno));
  socklen_t len = sizeof a;
  getsockname(listen_fd_, (sockaddr*)&a, &len);
  port_ = ntohs(a.sin_port);
  fcntl(listen_fd_, F_SETFL, O_NONBLOCK);
  thread_ = std::thread([this] { loop(); });
}

Coordinator::~Coordinator() { stop(); }

void Coordinator::stop() {
  stop_.store(true);
  if (thread_.joinable()) thread_.join();
  if (listen_fd_ >= 0) { close(listen_fd_); listen_fd_ = -1; }
}

std::string Coordinator::handle(const Json& req, bool* drop) {
  *drop = false;
  if (broken_.load()) return "{\"error\":\"session broken: " + break_reason_ + "\"}";
  auto fail = [&](const std::string& why) {
    broken_.store(true);
    break_reason_ = why;
    return "{\"error\":\"session broken: " + why + "\"}";
  };
  if (req.at("session").as_string() != session_) return fail("session mismatch");
  int rank = (int)req.at("rank").as_int();
  long long seq = req.at("sequence").as_int();
  const std::string& phase = req.at("phase").as_string();
  if (rank < 0 || rank >= nranks_) return fail("rank out of range");
  auto done = decided_.find(seq);
  if (done != decided_.end()) return done->second;   // idempotent retransmit
  if (!decided_.empty() && seq <= decided_.rbegin()->first - 2) return fail("stale sequence");
  auto& slot = open_[seq];
  if (slot.first.empty()) slot.first = phase;
  else if (slot.first != phase) return fail("phase mismatch at sequence " + std::to_string(seq));
  auto prev = slot.second.find(rank);
  std::string payload = req.at("payload").as_string();
  if (prev != slot.second.end() && prev->second != payload) return fail("payload changed on retransmit");
  slot.second[rank] = payload;
  if ((int)slot.second.size() < nranks_) return "";   // wait for everyone
  Json d;
  d.kind = Json::Object;
  Json s; s.kind = Json::Number; s.num = (double)seq;
  Json p; p.kind = Json::String; p.str = phase;
  Json arr; arr.kind = Json::Array;
  for (auto& kv : slot.second) { Json v; v.kind = Json::String; v.str = kv.second; arr.arr.push_back(v); }
  d.obj.emplace_back("sequence", s);
  d.obj.emplace_back("phase", p);
  d.obj.emplace_back("payloads", arr);
  std::string decision = d.dump();
  decided_[seq] = decision;
  while (decided_.size() > 2) decided_.erase(decided_.begin());
  open_.erase(seq);
  return decision;
}

void Coordinator::loop() {
  std::vector<Pending> conns;
  std::map<long long, std::vector<size_t>> parked;   // sequence -> conns waiting for a decision
  while (!stop_.load()) {
    std::vector<struct pollfd> fds;
    fds.push_back({listen_fd_, POLLIN, 0});
    for (auto& c : conns) fds.push_back({c.fd, POLLIN, 0});
    int r = poll(fds.data(), fds.size(), 50);
    if (r <= 0) continue;
    if (fds[0].revents & POLLIN) {
      int c = accept(listen_fd_, nullptr, nullptr);
      if (c >= 0) conns.push_back(Pending{c, -1, ""});
    }
    std::vector<size_t> closed;
    for (size_t i = 1; i < fds.size(); ++i) {
      if (!(fds[i].revents & (POLLIN | POLLHUP | POLLERR))) continue;
      Pending& c = conns[i - 1];
      std::string body;
      if (!recv_frame(c.fd, &body, Deadline::after(1.0))) { closed.push_back(i - 1); continue; }
      try {
        Json req = parse_json(body);
        bool drop = false;
        long long seq = req.at("sequence").as_int();
        std::string reply = handle(req, &drop);
        if (reply.empty()) {
          parked[seq].push_back(i - 1);
          continue;
        }
        auto reply_to = [&](size_t idx) {
          if (lose_replies_.load() > 0) {
            lose_replies_.fetch_sub(1);
            closed.push_back(idx);   // the reply is "lost": close without answering
            return;
          }
          send_frame(conns[idx].fd, reply, Deadline::after(2.0));
          closed.push_back(idx);
        };
        reply_to(i - 1);
        for (size_t idx : parked[seq]) reply_to(idx);
        parked.erase(seq);
      } catch (const std::exception& e) {
        send_frame(c.fd, std::string("{\"error\":\"bad request: ") + "malformed" + "\"}", Deadline::after(1.0));
        closed.push_back(i - 1);
      }
    }
    if (!closed.empty()) {
      std::sort(closed.begin(), closed.end());
      closed.erase(std::unique(closed.begin(), closed.end()), closed.end());
      std::vector<Pending> keep;
      std::map<size_t, size_t> remap;
      size_t ci = 0;
      for (size_t k = 0; k < conns.size(); ++k) {
        if (ci < closed.size() && closed[ci] == k) { close(conns[k].fd); ++ci; continue; }
        remap[k] = keep.size();
        keep.push_back(conns[k]);
      }
      conns.swap(keep);
      for (auto& kv : parked) {
        std::vector<size_t> moved;
        for (size_t idx : kv.second) if (remap.count(idx)) moved.push_back(remap[idx]);
        kv.second.swap(moved);
      }
    }
  }
  for (auto& c : conns) close(c.fd);
}

ControlTransport::ControlTransport(int rank, int nranks, const std::string& address, int port,
                                   const std::string& session)
    : rank_(rank), nranks_(nranks), port_(port), address_(address), session_(session) {
  if (rank == 0) {
    coord_ = std::make_unique<Coordinator>(address, port, nranks, session);
    port_ = coord_->port();
  }
}

ControlTransport::~ControlTransport() {
  if (coord_) coord_->stop();
}

std::vector<std::string> ControlTransport::gather(const std::string& phase, const std::string& payload,
                                                  const Deadline& deadline) {
  long long seq = ++sequence_;
  Json req;
  req.kind = Json::Object;
  auto str = [](const std::string& s) { Json j; j.kind = Json::String; j.str = s; return j; };
  auto num = [](double v) { Json j; j.kind = Json::Number; j.num = v; return j; };
  req.obj.emplace_back("session", str(session_));
  req.obj.emplace_back("rank", num(rank_));
  req.obj.emplace_back("phase", str(phase));
  req.obj.emplace_back("sequence", num((double)seq));
  req.obj.emplace_back("payload", str(payload));
  std::string body = req.dump();
  while (!deadline.expired()) {
    int fd = socket(AF_INET, SOCK_STREAM, 0);
    sockaddr_in a = {};
    a.sin_family = AF_INET;
    a.sin_port = htons((uint16_t)port_);
    inet_pton(AF_INET, address_.c_str(), &a.sin_addr);
    if (connect(fd, (sockaddr*)&a, sizeof a) != 0) {
      close(fd);
      usleep(20000);
      continue;
    }
    std::string reply;
    bool ok = send_frame(fd, body, deadline) && recv_frame(fd, &reply, deadline);
    close(fd);
    if (!ok) continue;   // lost reply or dropped connection: retransmit (idempotent)
    Json d = parse_json(reply);
    if (const Json* err = d.get("error")) throw ControlError(err->as_string());
    if (d.at("sequence").as_int() != seq || d.at("phase").as_string() != phase)
      throw ControlError("control decision does not match the request");
    std::vector<std::string> out;
    for (auto& v : d.at("payloads").arr) out.push_back(v.as_string());
    return out;
  }
  throw ControlError("control phase '" + phase + "' timed out");
}

}  // namespace vb
