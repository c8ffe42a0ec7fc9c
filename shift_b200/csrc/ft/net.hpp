// Minimal epoll line server and blocking line client used by the
// fault-tolerance control plane (lighthouse and replica manager server).
//
// Wire format: one request or reply per line ('\n'), tokens separated by a
// single space.  Token values never contain spaces or newlines (addresses,
// ids and percent-encoded strings).
#pragma once

#include <arpa/inet.h>
#include <errno.h>
#include <fcntl.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <sys/epoll.h>
#include <sys/eventfd.h>
#include <sys/socket.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <cstring>
#include <functional>
#include <map>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

namespace sbft {

inline int64_t now_ms() {
  return std::chrono::duration_cast<std::chrono::milliseconds>(
             std::chrono::steady_clock::now().time_since_epoch())
      .count();
}

inline std::vector<std::string> split(const std::string& s) {
  std::vector<std::string> out;
  std::istringstream is(s);
  std::string t;
  while (is >> t) out.push_back(t);
  return out;
}

// Event-driven TCP line server on its own thread.  Handlers run on the server
// thread; a handler may defer its reply (return false) and answer later with
// reply(fd, line).  on_tick runs at least every tick_ms.
class LineServer {
 public:
  using Handler = std::function<bool(int fd, const std::vector<std::string>& req, std::string& reply)>;
  using Tick = std::function<void()>;
  using Close = std::function<void(int fd)>;

  LineServer() = default;
  ~LineServer() { stop(); }

  // Bind host:port (port 0 = ephemeral).  Returns the bound port or -1.
  int start(const std::string& host, int port, int tick_ms, Handler h, Tick t, Close c) {
    handler_ = std::move(h);
    tick_ = std::move(t);
    close_ = std::move(c);
    tick_ms_ = tick_ms > 0 ? tick_ms : 100;
    listen_fd_ = ::socket(AF_INET, SOCK_STREAM, 0);
    if (listen_fd_ < 0) return -1;
    int one = 1;
    setsockopt(listen_fd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in addr{};
    addr.sin_family = AF_INET;
    addr.sin_port = htons(static_cast<uint16_t>(port));
    if (host.empty() || host == "0.0.0.0" || host == "::" || host == "[::]") addr.sin_addr.s_addr = INADDR_ANY;
    else if (inet_pton(AF_INET, host.c_str(), &addr.sin_addr) != 1) addr.sin_addr.s_addr = INADDR_ANY;
    if (::bind(listen_fd_, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) != 0) {
      ::close(listen_fd_);
      listen_fd_ = -1;
      return -1;
    }
    ::listen(listen_fd_, 256);
    socklen_t len = sizeof(addr);
    getsockname(listen_fd_, reinterpret_cast<sockaddr*>(&addr), &len);
    port_ = ntohs(addr.sin_port);
    set_nonblock(listen_fd_);
    ep_ = epoll_create1(0);
    wake_fd_ = eventfd(0, EFD_NONBLOCK);
    add_fd(listen_fd_);
    add_fd(wake_fd_);
    running_ = true;
    thread_ = std::thread([this] { loop(); });
    return port_;
  }

  void stop() {
    if (!running_.exchange(false)) return;
    uint64_t v = 1;
    (void)!::write(wake_fd_, &v, sizeof(v));
    if (thread_.joinable()) thread_.join();
    for (auto& kv : bufs_) ::close(kv.first);
    bufs_.clear();
    if (listen_fd_ >= 0) ::close(listen_fd_);
    if (ep_ >= 0) ::close(ep_);
    if (wake_fd_ >= 0) ::close(wake_fd_);
    listen_fd_ = ep_ = wake_fd_ = -1;
  }

  int port() const { return port_; }

  // Send a line to a client (server thread only).
  void reply(int fd, const std::string& line) {
    std::string s = line;
    s.push_back('\n');
    size_t off = 0;
    while (off < s.size()) {
      ssize_t n = ::send(fd, s.data() + off, s.size() - off, MSG_NOSIGNAL);
      if (n > 0) {
        off += static_cast<size_t>(n);
      } else if (n < 0 && (errno == EAGAIN || errno == EWOULDBLOCK)) {
        std::this_thread::sleep_for(std::chrono::microseconds(50));
      } else {
        break;
      }
    }
  }

  // Run fn on the server thread soon (thread safe).
  void wake() {
    uint64_t v = 1;
    (void)!::write(wake_fd_, &v, sizeof(v));
  }

 private:
  static void set_nonblock(int fd) { fcntl(fd, F_SETFL, fcntl(fd, F_GETFL, 0) | O_NONBLOCK); }
  void add_fd(int fd) {
    epoll_event ev{};
    ev.events = EPOLLIN;
    ev.data.fd = fd;
    epoll_ctl(ep_, EPOLL_CTL_ADD, fd, &ev);
  }
  void drop(int fd) {
    epoll_ctl(ep_, EPOLL_CTL_DEL, fd, nullptr);
    ::close(fd);
    bufs_.erase(fd);
    if (close_) close_(fd);
  }

  void loop() {
    std::vector<epoll_event> evs(64);
    int64_t last_tick = now_ms();
    while (running_) {
      int n = epoll_wait(ep_, evs.data(), static_cast<int>(evs.size()), tick_ms_);
      for (int i = 0; i < n; ++i) {
        int fd = evs[i].data.fd;
        if (fd == listen_fd_) {
          while (true) {
            int c = ::accept(listen_fd_, nullptr, nullptr);
            if (c < 0) break;
            int one = 1;
            setsockopt(c, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
            set_nonblock(c);
            add_fd(c);
            bufs_[c] = std::string();
          }
        } else if (fd == wake_fd_) {
          uint64_t v;
          (void)!::read(wake_fd_, &v, sizeof(v));
        } else {
          char buf[4096];
          bool closed = false;
          while (true) {
            ssize_t r = ::recv(fd, buf, sizeof(buf), 0);
            if (r > 0) {
              bufs_[fd].append(buf, static_cast<size_t>(r));
            } else if (r == 0) {
              closed = true;
              break;
            } else {
              if (errno != EAGAIN && errno != EWOULDBLOCK) closed = true;
              break;
            }
          }
          std::string& b = bufs_[fd];
          size_t pos;
          while ((pos = b.find('\n')) != std::string::npos) {
            std::string line = b.substr(0, pos);
            b.erase(0, pos + 1);
            std::string rep;
            if (handler_(fd, split(line), rep)) reply(fd, rep);
          }
          if (closed) drop(fd);
        }
      }
      int64_t t = now_ms();
      if (t - last_tick >= tick_ms_ || n == 0) {
        last_tick = t;
        if (tick_) tick_();
      } else if (tick_) {
        tick_();  // event driven: re-evaluate state after every batch of events
      }
    }
  }

  Handler handler_;
  Tick tick_;
  Close close_;
  int tick_ms_ = 100;
  int listen_fd_ = -1, ep_ = -1, wake_fd_ = -1, port_ = 0;
  std::atomic<bool> running_{false};
  std::thread thread_;
  std::map<int, std::string> bufs_;
};

// Blocking client: connect, send one line, read one line.
class LineClient {
 public:
  ~LineClient() { close(); }
  bool connect(const std::string& host, int port, int timeout_ms) {
    close();
    addrinfo hints{}, *res = nullptr;
    hints.ai_family = AF_INET;
    hints.ai_socktype = SOCK_STREAM;
    if (getaddrinfo(host.c_str(), std::to_string(port).c_str(), &hints, &res) != 0 || !res) return false;
    int64_t deadline = now_ms() + timeout_ms;
    while (true) {
      fd_ = ::socket(AF_INET, SOCK_STREAM, 0);
      if (::connect(fd_, res->ai_addr, res->ai_addrlen) == 0) break;
      ::close(fd_);
      fd_ = -1;
      if (now_ms() > deadline) {
        freeaddrinfo(res);
        return false;
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(20));
    }
    freeaddrinfo(res);
    int one = 1;
    setsockopt(fd_, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
    return true;
  }
  // Returns false on error or timeout.
  bool request(const std::string& line, std::string& out, int timeout_ms) {
    if (fd_ < 0) return false;
    std::string s = line + "\n";
    if (::send(fd_, s.data(), s.size(), MSG_NOSIGNAL) != static_cast<ssize_t>(s.size())) return false;
    int64_t deadline = now_ms() + timeout_ms;
    while (true) {
      size_t pos = buf_.find('\n');
      if (pos != std::string::npos) {
        out = buf_.substr(0, pos);
        buf_.erase(0, pos + 1);
        return true;
      }
      int64_t left = deadline - now_ms();
      if (left <= 0) return false;
      timeval tv{static_cast<time_t>(left / 1000), static_cast<suseconds_t>((left % 1000) * 1000)};
      setsockopt(fd_, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
      char b[4096];
      ssize_t r = ::recv(fd_, b, sizeof(b), 0);
      if (r <= 0) return false;
      buf_.append(b, static_cast<size_t>(r));
    }
  }
  void close() {
    if (fd_ >= 0) ::close(fd_);
    fd_ = -1;
    buf_.clear();
  }

 private:
  int fd_ = -1;
  std::string buf_;
};

inline bool parse_hostport(const std::string& addr, std::string& host, int& port) {
  std::string a = addr;
  auto p = a.find("://");
  if (p != std::string::npos) a = a.substr(p + 3);
  auto slash = a.find('/');
  if (slash != std::string::npos) a = a.substr(0, slash);
  auto c = a.rfind(':');
  if (c == std::string::npos) return false;
  host = a.substr(0, c);
  if (host.size() >= 2 && host.front() == '[' && host.back() == ']') host = host.substr(1, host.size() - 2);
  if (host.empty() || host == "::") host = "127.0.0.1";
  port = std::atoi(a.c_str() + c + 1);
  return port > 0;
}

}  // namespace sbft
