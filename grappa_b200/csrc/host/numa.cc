// NUMA placement and bandwidth probing (see numa.h).
#include "numa.h"

#include <linux/mempolicy.h>
#include <sched.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cmath>
#include <condition_variable>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <mutex>
#include <sstream>
#include <stdexcept>
#include <string>
#include <thread>

namespace grappa {
namespace host {

namespace {

constexpr unsigned long kMaskBits = 1024;  // nodes the policy masks can name
constexpr size_t kMaskWords = kMaskBits / (8 * sizeof(unsigned long));

std::string read_line(const std::string& path) {
  std::ifstream f(path);
  std::string s;
  if (f) std::getline(f, s);
  return s;
}

std::vector<int> allowed_cpus() {
  cpu_set_t set;
  CPU_ZERO(&set);
  std::vector<int> out;
  if (sched_getaffinity(0, sizeof(set), &set) != 0) return out;
  for (int c = 0; c < CPU_SETSIZE; ++c)
    if (CPU_ISSET(c, &set)) out.push_back(c);
  return out;
}

// Runs fn(t) on `threads` threads, thread t pinned to cpus[t % cpus.size()]; returns the
// seconds from their common release to the last one's end.
double run_team(int threads, const std::vector<int>& cpus, const std::function<void(int)>& fn) {
  std::mutex mu;
  std::condition_variable cv;
  bool go = false;
  int ready = 0;
  std::vector<std::chrono::steady_clock::time_point> end(static_cast<size_t>(threads));
  std::vector<std::thread> team;
  team.reserve(static_cast<size_t>(threads));
  for (int t = 0; t < threads; ++t) {
    team.emplace_back([&, t] {
      cpu_set_t set;
      CPU_ZERO(&set);
      CPU_SET(cpus[static_cast<size_t>(t) % cpus.size()], &set);
      sched_setaffinity(0, sizeof(set), &set);  // best effort: a refused pin still measures
      {
        std::unique_lock<std::mutex> lk(mu);
        ++ready;
        cv.notify_all();
        cv.wait(lk, [&] { return go; });
      }
      fn(t);
      end[static_cast<size_t>(t)] = std::chrono::steady_clock::now();
    });
  }
  std::chrono::steady_clock::time_point t0;
  {
    std::unique_lock<std::mutex> lk(mu);
    cv.wait(lk, [&] { return ready == threads; });
    t0 = std::chrono::steady_clock::now();
    go = true;
  }
  cv.notify_all();
  for (auto& th : team) th.join();
  const auto last = *std::max_element(end.begin(), end.end());
  return std::chrono::duration<double>(last - t0).count();
}

}  // namespace

std::vector<int> parse_cpulist(const char* s) {
  std::vector<int> out;
  if (!s) return out;
  std::stringstream ss(s);
  std::string part;
  while (std::getline(ss, part, ',')) {
    part.erase(std::remove_if(part.begin(), part.end(), [](char c) { return c == ' ' || c == '\n'; }),
               part.end());
    if (part.empty()) continue;
    const size_t dash = part.find('-');
    try {
      if (dash == std::string::npos) {
        out.push_back(std::stoi(part));
      } else {
        const int a = std::stoi(part.substr(0, dash)), b = std::stoi(part.substr(dash + 1));
        for (int c = a; c <= b; ++c) out.push_back(c);
      }
    } catch (const std::exception&) {
      return {};  // not a cpulist
    }
  }
  return out;
}

std::vector<int> numa_nodes() {
  std::vector<int> nodes = parse_cpulist(read_line("/sys/devices/system/node/online").c_str());
  if (nodes.empty()) nodes.push_back(0);
  return nodes;
}

std::vector<int> numa_node_cpus(int node) {
  if (node < 0) return {};
  std::vector<int> cpus =
      parse_cpulist(read_line("/sys/devices/system/node/node" + std::to_string(node) + "/cpulist").c_str());
  if (cpus.empty()) {
    const std::vector<int> nodes = numa_nodes();
    if (nodes.size() == 1 && nodes[0] == node) cpus = allowed_cpus();  // no sysfs: one node, every CPU
    return cpus;
  }
  const std::vector<int> ok = allowed_cpus();  // a cpuset may hide some of the node's CPUs
  std::vector<int> both;
  for (int c : cpus)
    if (std::find(ok.begin(), ok.end(), c) != ok.end()) both.push_back(c);
  return both;
}

int numa_node_of(const void* p) {
  int node = -1;
  if (syscall(SYS_get_mempolicy, &node, nullptr, 0UL, const_cast<void*>(p), MPOL_F_NODE | MPOL_F_ADDR) != 0)
    return -1;
  return node;
}

MemPolicyScope::MemPolicyScope(int node) {
  const std::vector<int> nodes = numa_nodes();
  if (node < 0 || node >= static_cast<int>(kMaskBits) || std::find(nodes.begin(), nodes.end(), node) == nodes.end())
    return;
  old_mask_.assign(kMaskWords, 0UL);
  if (syscall(SYS_get_mempolicy, &old_mode_, old_mask_.data(), kMaskBits, nullptr, 0UL) != 0) return;
  std::vector<unsigned long> mask(kMaskWords, 0UL);
  mask[static_cast<size_t>(node) / (8 * sizeof(unsigned long))] |= 1UL << (node % (8 * sizeof(unsigned long)));
  active_ = syscall(SYS_set_mempolicy, MPOL_PREFERRED, mask.data(), kMaskBits) == 0;
}

MemPolicyScope::~MemPolicyScope() {
  if (!active_) return;
  if ((old_mode_ & ~MPOL_MODE_FLAGS) == MPOL_DEFAULT)
    syscall(SYS_set_mempolicy, MPOL_DEFAULT, nullptr, 0UL);
  else
    syscall(SYS_set_mempolicy, old_mode_, old_mask_.data(), kMaskBits);
}

bool pin_thread_to_node(int node) {
  const std::vector<int> cpus = numa_node_cpus(node);
  if (cpus.empty()) return false;
  cpu_set_t set;
  CPU_ZERO(&set);
  for (int c : cpus)
    if (c < CPU_SETSIZE) CPU_SET(c, &set);
  return sched_setaffinity(0, sizeof(set), &set) == 0;
}

Bandwidth memory_bandwidth(int cpu_node, int mem_node, size_t bytes, int threads, int reps) {
  const std::vector<int> cpus = numa_node_cpus(cpu_node);
  if (cpus.empty()) throw std::invalid_argument("node " + std::to_string(cpu_node) + " has no usable CPU");
  const std::vector<int> nodes = numa_nodes();
  if (std::find(nodes.begin(), nodes.end(), mem_node) == nodes.end())
    throw std::invalid_argument("node " + std::to_string(mem_node) + " is not online");
  if (threads <= 0) threads = static_cast<int>(cpus.size());
  if (reps < 1) reps = 1;
  const size_t n = bytes / sizeof(double);
  if (n < static_cast<size_t>(threads) * 512) throw std::invalid_argument("buffer too small for the thread count");
  const size_t alloc = (n * sizeof(double) + 63) / 64 * 64;
  double* buf = static_cast<double*>(std::aligned_alloc(64, alloc));
  if (!buf) throw std::bad_alloc();
  auto range = [&](int t, size_t* b, size_t* e) {
    const size_t per = (n + static_cast<size_t>(threads) - 1) / static_cast<size_t>(threads);
    *b = std::min(n, per * static_cast<size_t>(t));
    *e = std::min(n, *b + per);
  };
  // first touch of every page under the memory node's policy places the buffer there
  run_team(threads, cpus, [&](int t) {
    MemPolicyScope scope(mem_node);
    size_t b, e;
    range(t, &b, &e);
    for (size_t i = b; i < e; i += 512) buf[i] = 0.0;
  });
  Bandwidth r;
  r.mem_node_seen = numa_node_of(buf);
  std::vector<double> sums(static_cast<size_t>(threads) * 8, 0.0);  // one cache line per thread
  double best_w = 1e30, best_r = 1e30;
  for (int rep = 0; rep < reps; ++rep) {
    best_w = std::min(best_w, run_team(threads, cpus, [&](int t) {
      size_t b, e;
      range(t, &b, &e);
      for (size_t i = b; i < e; ++i) buf[i] = static_cast<double>(i);
    }));
    best_r = std::min(best_r, run_team(threads, cpus, [&](int t) {
      size_t b, e;
      range(t, &b, &e);
      double s0 = 0, s1 = 0, s2 = 0, s3 = 0;
      size_t i = b;
      for (; i + 4 <= e; i += 4) {
        s0 += buf[i];
        s1 += buf[i + 1];
        s2 += buf[i + 2];
        s3 += buf[i + 3];
      }
      for (; i < e; ++i) s0 += buf[i];
      sums[static_cast<size_t>(t) * 8] = s0 + s1 + s2 + s3;
    }));
  }
  // the sums are checked so that the read pass stays in the program
  double total = 0;
  for (int t = 0; t < threads; ++t) total += sums[static_cast<size_t>(t) * 8];
  const double want = static_cast<double>(n) * static_cast<double>(n - 1) / 2.0;
  std::free(buf);
  if (std::abs(total - want) > 1e-6 * want + 1.0) throw std::runtime_error("bandwidth probe read back wrong data");
  r.write_gbs = static_cast<double>(n * sizeof(double)) / best_w / 1e9;
  r.read_gbs = static_cast<double>(n * sizeof(double)) / best_r / 1e9;
  return r;
}

}  // namespace host
}  // namespace grappa
