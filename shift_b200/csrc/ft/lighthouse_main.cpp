// Standalone lighthouse daemon:
//   shift_lighthouse --bind 0.0.0.0:29510 --min_replicas 1 --join_timeout_ms 200
//                    --heartbeat_timeout_ms 500 --quorum_tick_ms 50
// (same flags as the torchft lighthouse the reference launches,
//  shift_full/supervisor.py:182-201).  Prints "LISTENING <port>" once bound.
#include <csignal>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>

extern "C" {
void* sbft_lighthouse_start(const char* host, int port, int min_replicas, int join_timeout_ms,
                            int heartbeat_timeout_ms, int tick_ms, int* bound_port);
void sbft_lighthouse_stop(void* h);
}

static volatile std::sig_atomic_t g_stop = 0;
static void on_signal(int) { g_stop = 1; }

int main(int argc, char** argv) {
  std::string bind = "0.0.0.0:29510";
  int min_replicas = 1, join = 200, hb = 500, tick = 50;
  for (int i = 1; i + 1 < argc; i += 2) {
    std::string k = argv[i];
    std::string v = argv[i + 1];
    if (k == "--bind") bind = v;
    else if (k == "--min_replicas") min_replicas = std::atoi(v.c_str());
    else if (k == "--join_timeout_ms") join = std::atoi(v.c_str());
    else if (k == "--heartbeat_timeout_ms") hb = std::atoi(v.c_str());
    else if (k == "--quorum_tick_ms") tick = std::atoi(v.c_str());
  }
  auto c = bind.rfind(':');
  std::string host = c == std::string::npos ? "0.0.0.0" : bind.substr(0, c);
  int port = c == std::string::npos ? 29510 : std::atoi(bind.c_str() + c + 1);
  if (host == "[::]" || host == "::") host = "0.0.0.0";
  int bound = 0;
  void* h = sbft_lighthouse_start(host.c_str(), port, min_replicas, join, hb, tick, &bound);
  if (!h) {
    std::fprintf(stderr, "lighthouse: cannot bind %s\n", bind.c_str());
    return 1;
  }
  std::printf("LISTENING %d\n", bound);
  std::fflush(stdout);
  std::signal(SIGTERM, on_signal);
  std::signal(SIGINT, on_signal);
  while (!g_stop) std::this_thread::sleep_for(std::chrono::milliseconds(50));
  sbft_lighthouse_stop(h);
  return 0;
}
