// Quorum lighthouse and per-replica manager server (C++ control plane).
//
// Lighthouse
//   Replicas heartbeat (HB) and request a quorum (Q).  A quorum forms as soon
//   as at least min_replicas replicas are waiting AND every replica that is
//   still heartbeating is among them (event driven: no tick is waited for in
//   the common case), or when join_timeout_ms has passed since the first
//   request of the round -- unless a live replica outside the waiting set is
//   ahead of every waiting one (then the round waits for it, up to a bounded
//   cap), so that a relaunched replica heals instead of training alone.
//   Replicas whose heartbeat is older than heartbeat_timeout_ms do not hold a
//   quorum back.  The quorum id increases
//   whenever membership changes.  Members are ordered by replica id.
//   Behaviour mirrors the torchft lighthouse that the reference launches with
//   --min_replicas / --join_timeout_ms / --heartbeat_timeout_ms /
//   --quorum_tick_ms (shift_full/supervisor.py:182-201).
//
//   HB <replica_id>                                         -> OK
//   Q <replica_id> <step> <world_size> <shrink_only> <manager_addr> <store_addr>
//                                                           -> QR <quorum_id> <n> (<rid> <step> <ws> <maddr> <saddr>)*
//   STATUS                                                  -> ST <quorum_id> <n_alive> <n_waiting> <formed>
//
// Manager server (one per replica, hosted by the replica's rank 0)
//   Aggregates the quorum requests of the replica's world_size local ranks,
//   asks the lighthouse once, and answers every rank with its replica rank,
//   the max step and the heal source / destinations; aggregates the commit
//   vote (all local ranks must vote yes); serves per-rank checkpoint metadata
//   to healing peers.  Mirrors torchft's ManagerServer as used through
//   Manager(...) at shift_full/planned_train.py:418-424.
//
//   Q <rank> <step> <shrink_only> <ckpt_meta> <timeout_ms>
//        -> MR <quorum_id> <replica_rank> <replica_world_size> <src_maddr|-> <src_replica_rank>
//              <dst_ranks_csv|-> <store_addr> <max_step> <max_replica_rank> <max_world_size> <heal>
//              <n> (<rid> <step>)*
//   C <rank> <step> <vote>                                  -> CR <decision>
//   M <rank>                                                -> MD <ckpt_meta|->
//   KILL                                                    -> OK   (test hook: stop serving)
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <mutex>
#include <set>

#include "net.hpp"

namespace sbft {

struct Member {
  std::string rid;
  int64_t step = 0;
  int world_size = 1;
  std::string maddr, saddr;
};

class Lighthouse {
 public:
  Lighthouse(int min_replicas, int join_timeout_ms, int heartbeat_timeout_ms, int tick_ms)
      : min_replicas_(min_replicas), join_timeout_ms_(join_timeout_ms), hb_timeout_ms_(heartbeat_timeout_ms),
        tick_ms_(tick_ms) {}

  int start(const std::string& host, int port) {
    return srv_.start(
        host, port, tick_ms_,
        [this](int fd, const std::vector<std::string>& r, std::string& rep) { return handle(fd, r, rep); },
        [this] { maybe_form(); }, [this](int fd) { on_close(fd); });
  }
  void stop() { srv_.stop(); }
  int port() const { return srv_.port(); }

 private:
  bool handle(int fd, const std::vector<std::string>& r, std::string& rep) {
    if (r.empty()) {
      rep = "ERR empty";
      return true;
    }
    const int64_t t = now_ms();
    if (r[0] == "HB" && r.size() >= 2) {
      last_hb_[r[1]] = t;
      rep = "OK";
      return true;
    }
    if (r[0] == "Q" && r.size() >= 7) {
      Member m;
      m.rid = r[1];
      m.step = std::atoll(r[2].c_str());
      m.world_size = std::atoi(r[3].c_str());
      m.maddr = r[5];
      m.saddr = r[6];
      last_hb_[m.rid] = t;
      last_step_[m.rid] = m.step;
      if (waiting_.empty()) first_wait_ms_ = t;
      // a replica re-requesting replaces its previous pending request
      for (auto it = waiting_.begin(); it != waiting_.end();) {
        if (it->second.rid == m.rid) {
          srv_.reply(it->first, "ERR superseded");
          it = waiting_.erase(it);
        } else {
          ++it;
        }
      }
      waiting_.emplace_back(fd, m);
      maybe_form();
      return false;  // deferred
    }
    if (r[0] == "STATUS") {
      int alive = 0;
      for (auto& kv : last_hb_)
        if (t - kv.second <= hb_timeout_ms_) ++alive;
      rep = "ST " + std::to_string(quorum_id_) + " " + std::to_string(alive) + " " +
            std::to_string(waiting_.size()) + " " + std::to_string(formed_);
      return true;
    }
    rep = "ERR unknown";
    return true;
  }

  void on_close(int fd) {
    for (auto it = waiting_.begin(); it != waiting_.end();) {
      if (it->first == fd) it = waiting_.erase(it);
      else ++it;
    }
  }

  void maybe_form() {
    if (waiting_.empty()) return;
    const int64_t t = now_ms();
    std::set<std::string> waiting_ids;
    for (auto& w : waiting_) waiting_ids.insert(w.second.rid);
    if (static_cast<int>(waiting_ids.size()) < min_replicas_) return;
    bool all_alive_waiting = true;
    for (auto& kv : last_hb_) {
      if (t - kv.second > hb_timeout_ms_) continue;  // considered dead
      if (!waiting_ids.count(kv.first)) {
        all_alive_waiting = false;
        break;
      }
    }
    if (!all_alive_waiting && t - first_wait_ms_ < join_timeout_ms_) return;
    if (!all_alive_waiting) {
      // Joining on the timeout must not leave behind a live replica that is
      // AHEAD of every waiting one: a relaunched replica (step 0) would
      // otherwise form a quorum of its own and train from scratch instead of
      // healing from the live state.  Bounded: after stale_cap the live
      // replica is presumed stuck and the quorum forms without it.
      int64_t max_waiting = 0;
      for (auto& w : waiting_) max_waiting = std::max(max_waiting, w.second.step);
      bool ahead_alive = false;
      for (auto& kv : last_hb_) {
        if (t - kv.second > hb_timeout_ms_ || waiting_ids.count(kv.first)) continue;
        auto st = last_step_.find(kv.first);
        if (st != last_step_.end() && st->second > max_waiting) ahead_alive = true;
      }
      const int64_t stale_cap = std::max<int64_t>(5LL * hb_timeout_ms_, 20LL * join_timeout_ms_);
      if (ahead_alive && t - first_wait_ms_ < stale_cap) return;
    }
    // form
    std::vector<Member> members;
    for (auto& w : waiting_) members.push_back(w.second);
    std::sort(members.begin(), members.end(), [](const Member& a, const Member& b) { return a.rid < b.rid; });
    std::vector<std::string> ids;
    for (auto& m : members) ids.push_back(m.rid);
    if (ids != prev_ids_) {
      ++quorum_id_;
      prev_ids_ = ids;
    }
    std::string line = "QR " + std::to_string(quorum_id_) + " " + std::to_string(members.size());
    for (auto& m : members)
      line += " " + m.rid + " " + std::to_string(m.step) + " " + std::to_string(m.world_size) + " " + m.maddr + " " +
              m.saddr;
    for (auto& w : waiting_) srv_.reply(w.first, line);
    waiting_.clear();
    ++formed_;
  }

  int min_replicas_, join_timeout_ms_, hb_timeout_ms_, tick_ms_;
  LineServer srv_;
  std::map<std::string, int64_t> last_hb_;
  std::map<std::string, int64_t> last_step_;   // step of each replica's latest quorum request
  std::vector<std::pair<int, Member>> waiting_;
  int64_t first_wait_ms_ = 0;
  int64_t quorum_id_ = 0;
  int64_t formed_ = 0;
  std::vector<std::string> prev_ids_;
};

// ---------------------------------------------------------------------------
class ManagerServer {
 public:
  ManagerServer(const std::string& replica_id, const std::string& lighthouse, int world_size,
                const std::string& store_addr, int hb_interval_ms, int quorum_timeout_ms)
      : rid_(replica_id), lighthouse_(lighthouse), world_(world_size), store_addr_(store_addr),
        hb_ms_(hb_interval_ms), qtimeout_ms_(quorum_timeout_ms) {}

  int start(const std::string& host, int port, const std::string& advertise_host) {
    int p = srv_.start(
        host, port, 50, [this](int fd, const std::vector<std::string>& r, std::string& rep) { return handle(fd, r, rep); },
        nullptr, [this](int fd) { on_close(fd); });
    if (p < 0) return p;
    maddr_ = advertise_host + ":" + std::to_string(p);
    running_ = true;
    // First heartbeat is synchronous: once start() returns, the lighthouse
    // counts this replica as alive, so a peer's quorum cannot form without it.
    {
      std::string host;
      int port;
      if (parse_hostport(lighthouse_, host, port)) {
        LineClient c;
        std::string out;
        if (c.connect(host, port, 5000)) c.request("HB " + rid_, out, 2000);
      }
    }
    hb_thread_ = std::thread([this] { heartbeat_loop(); });
    return p;
  }
  void stop() {
    running_ = false;
    if (hb_thread_.joinable()) hb_thread_.join();
    if (q_thread_.joinable()) q_thread_.join();
    srv_.stop();
  }
  int port() const { return srv_.port(); }

 private:
  void heartbeat_loop() {
    LineClient c;
    std::string host;
    int port;
    if (!parse_hostport(lighthouse_, host, port)) return;
    c.connect(host, port, 1000);
    while (running_) {
      if (!killed_) {
        std::string out;
        if (!c.request("HB " + rid_, out, 1000)) {
          if (c.connect(host, port, 200)) c.request("HB " + rid_, out, 1000);
        }
      }
      for (int i = 0; i < hb_ms_ / 10 && running_; ++i) std::this_thread::sleep_for(std::chrono::milliseconds(10));
    }
  }

  bool handle(int fd, const std::vector<std::string>& r, std::string& rep) {
    if (r.empty() || killed_) {
      rep = "ERR";
      return !killed_;
    }
    if (r[0] == "Q" && r.size() >= 6) {
      const int rank = std::atoi(r[1].c_str());
      const int64_t step = std::atoll(r[2].c_str());
      if (q_round_.count(rank)) srv_.reply(q_round_[rank].fd, "ERR superseded");
      q_round_[rank] = Pending{fd, step, r[3] == "1"};
      meta_[rank] = r[4];
      if (static_cast<int>(q_round_.size()) == world_) launch_quorum();
      return false;
    }
    if (r[0] == "C" && r.size() >= 4) {
      const int rank = std::atoi(r[1].c_str());
      votes_[rank] = std::make_pair(fd, r[3] == "1");
      if (static_cast<int>(votes_.size()) == world_) {
        bool all = true;
        for (auto& kv : votes_) all = all && kv.second.second;
        for (auto& kv : votes_) srv_.reply(kv.second.first, std::string("CR ") + (all ? "1" : "0"));
        votes_.clear();
      }
      return false;
    }
    if (r[0] == "M" && r.size() >= 2) {
      const int rank = std::atoi(r[1].c_str());
      auto it = meta_.find(rank);
      rep = "MD " + (it == meta_.end() ? std::string("-") : it->second);
      return true;
    }
    if (r[0] == "KILL") {
      killed_ = true;
      rep = "OK";
      return true;
    }
    rep = "ERR unknown";
    return true;
  }

  void on_close(int fd) {
    for (auto it = votes_.begin(); it != votes_.end();) {
      if (it->second.first == fd) it = votes_.erase(it);
      else ++it;
    }
  }

  struct Pending {
    int fd;
    int64_t step;
    bool shrink;
  };

  // All local ranks asked: one lighthouse request on a helper thread, then
  // answer every rank from the server thread's perspective (reply is thread
  // safe enough for distinct fds; we serialise with a mutex).
  void launch_quorum() {
    std::map<int, Pending> round = q_round_;
    q_round_.clear();
    int64_t step = 0;
    bool shrink = false;
    for (auto& kv : round) {
      step = std::max(step, kv.second.step);
      shrink = shrink || kv.second.shrink;
    }
    if (q_thread_.joinable()) q_thread_.join();
    q_thread_ = std::thread([this, round, step, shrink] {
      std::string host;
      int port;
      std::string out;
      bool ok = parse_hostport(lighthouse_, host, port);
      LineClient c;
      ok = ok && c.connect(host, port, qtimeout_ms_);
      ok = ok && c.request("Q " + rid_ + " " + std::to_string(step) + " " + std::to_string(world_) + " " +
                               (shrink ? "1" : "0") + " " + maddr_ + " " + store_addr_,
                           out, qtimeout_ms_);
      std::lock_guard<std::mutex> g(reply_mu_);
      if (!ok || out.rfind("QR ", 0) != 0) {
        for (auto& kv : round) srv_.reply(kv.second.fd, "ERR quorum " + (ok ? out : std::string("timeout")));
        return;
      }
      auto t = split(out);
      const std::string qid = t[1];
      const int n = std::atoi(t[2].c_str());
      std::vector<Member> mem(n);
      for (int i = 0; i < n; ++i) {
        mem[i].rid = t[3 + 5 * i];
        mem[i].step = std::atoll(t[4 + 5 * i].c_str());
        mem[i].world_size = std::atoi(t[5 + 5 * i].c_str());
        mem[i].maddr = t[6 + 5 * i];
        mem[i].saddr = t[7 + 5 * i];
      }
      int my = -1;
      int64_t max_step = 0;
      for (int i = 0; i < n; ++i) {
        if (mem[i].rid == rid_) my = i;
        max_step = std::max(max_step, mem[i].step);
      }
      std::vector<int> up;  // replica ranks at max step
      for (int i = 0; i < n; ++i)
        if (mem[i].step == max_step) up.push_back(i);
      const bool heal = my >= 0 && mem[my].step < max_step;
      std::string src_addr = "-";
      int src_rank = -1;
      if (heal) {
        src_rank = up[my % up.size()];
        src_addr = mem[src_rank].maddr;
      }
      std::string dst;
      if (!heal && my >= 0) {
        for (int i = 0; i < n; ++i) {
          if (mem[i].step < max_step && up[i % up.size()] == my) dst += (dst.empty() ? "" : ",") + std::to_string(i);
        }
      }
      if (dst.empty()) dst = "-";
      const int max_rank = up.empty() ? -1 : up[0];
      const std::string store = n > 0 ? mem[0].saddr : store_addr_;
      std::string line = "MR " + qid + " " + std::to_string(my) + " " + std::to_string(n) + " " + src_addr + " " +
                         std::to_string(src_rank) + " " + dst + " " + store + " " + std::to_string(max_step) + " " +
                         std::to_string(max_rank) + " " + std::to_string(up.size()) + " " + (heal ? "1" : "0") + " " +
                         std::to_string(n);
      for (auto& m : mem) line += " " + m.rid + " " + std::to_string(m.step);
      for (auto& kv : round) srv_.reply(kv.second.fd, line);
    });
  }

  std::string rid_, lighthouse_;
  int world_;
  std::string store_addr_, maddr_;
  int hb_ms_, qtimeout_ms_;
  LineServer srv_;
  std::map<int, Pending> q_round_;
  std::map<int, std::pair<int, bool>> votes_;
  std::map<int, std::string> meta_;
  std::atomic<bool> running_{false}, killed_{false};
  std::thread hb_thread_, q_thread_;
  std::mutex reply_mu_;
};

}  // namespace sbft

// ---------------------------------------------------------------------------
// C API (loaded with ctypes by shift_b200.ft.native)
// ---------------------------------------------------------------------------
extern "C" {

void* sbft_lighthouse_start(const char* host, int port, int min_replicas, int join_timeout_ms,
                            int heartbeat_timeout_ms, int tick_ms, int* bound_port) {
  auto* lh = new sbft::Lighthouse(min_replicas, join_timeout_ms, heartbeat_timeout_ms, tick_ms);
  int p = lh->start(host ? host : "", port);
  if (p < 0) {
    delete lh;
    return nullptr;
  }
  if (bound_port) *bound_port = p;
  return lh;
}

void sbft_lighthouse_stop(void* h) {
  auto* lh = static_cast<sbft::Lighthouse*>(h);
  if (!lh) return;
  lh->stop();
  delete lh;
}

void* sbft_manager_start(const char* replica_id, const char* lighthouse, int world_size, const char* store_addr,
                         const char* bind_host, int port, const char* advertise_host, int hb_interval_ms,
                         int quorum_timeout_ms, int* bound_port) {
  auto* m = new sbft::ManagerServer(replica_id, lighthouse, world_size, store_addr, hb_interval_ms, quorum_timeout_ms);
  int p = m->start(bind_host ? bind_host : "", port, advertise_host ? advertise_host : "127.0.0.1");
  if (p < 0) {
    delete m;
    return nullptr;
  }
  if (bound_port) *bound_port = p;
  return m;
}

void sbft_manager_stop(void* h) {
  auto* m = static_cast<sbft::ManagerServer*>(h);
  if (!m) return;
  m->stop();
  delete m;
}

}  // extern "C"
