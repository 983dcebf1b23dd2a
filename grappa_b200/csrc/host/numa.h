// NUMA placement and bandwidth probing without libnuma: the node lists under
// /sys/devices/system/node and the set_mempolicy / get_mempolicy system calls.
//
// Reference: csrc/python/py_graph.cc:23-34 binds the host CSC to the GPU's NUMA node
// with numa_set_membind (and leaves the binding on for the thread afterwards);
// test/numa_bench.c measures read/write bandwidth of memory on node 0 and node 1
// from unpinned OpenMP threads.  Here the placement is a scope that restores the
// thread's policy, and the probe fills a matrix over (CPU node, memory node) pairs
// with threads pinned to the CPU node.
#pragma once
#include <cstddef>
#include <cstdint>
#include <vector>

namespace grappa {
namespace host {

// Online NUMA node ids (sysfs); {0} when the system exposes none.
std::vector<int> numa_nodes();

// CPUs of a node (its sysfs cpulist), empty for an unknown node.
std::vector<int> numa_node_cpus(int node);

// Parses a sysfs cpulist such as "0-3,8,10-11".
std::vector<int> parse_cpulist(const char* s);

// Node that holds the page at `p` (faulted in), -1 when the kernel does not say.
int numa_node_of(const void* p);

// While alive, pages that this thread faults in are taken from `node` first
// (MPOL_PREFERRED: other nodes when it is full).  The thread's previous policy is
// put back at the end.  active() is false when the node is unknown or the system
// call is refused (for example by a container's seccomp profile); nothing changes then.
class MemPolicyScope {
 public:
  explicit MemPolicyScope(int node);
  ~MemPolicyScope();
  MemPolicyScope(const MemPolicyScope&) = delete;
  MemPolicyScope& operator=(const MemPolicyScope&) = delete;
  bool active() const { return active_; }

 private:
  bool active_ = false;
  int old_mode_ = 0;
  std::vector<unsigned long> old_mask_;
};

// Pins the calling thread to the CPUs of `node`; false (and unchanged) when it has none.
bool pin_thread_to_node(int node);

struct Bandwidth {
  double write_gbs = 0, read_gbs = 0;
  int mem_node_seen = -1;  // node of the buffer's first page, as the kernel reports it
};

// Write and read bandwidth of `bytes` of memory placed on `mem_node`, streamed by
// `threads` threads pinned to `cpu_node` (threads <= 0: the node's CPU count).
// Best of `reps` passes of each.
Bandwidth memory_bandwidth(int cpu_node, int mem_node, size_t bytes, int threads, int reps = 3);

}  // namespace host
}  // namespace grappa
