// Native tests of the C++ host engine (CSC build, sampling rule, coverage ratio,
// compaction order, random walks, cross-partition ids, chunk writer, multilevel
// partitioner, batch prefetch pipeline, NUMA placement), built and run without Python:
//   g++ -O2 -std=c++17 -fopenmp -Igrappa_b200/csrc/include -Igrappa_b200/csrc/host \
//       grappa_b200/csrc/host/tests/test_host.cc \
//       grappa_b200/csrc/host/{graph_host,xborder,chunking,mlpart,numa}.cc -lpthread
// The test suite also builds it with -fsanitize=address,undefined and, without
// OpenMP (whose runtime the thread sanitizer cannot see into), -fsanitize=thread.
// The reference ships smoke executables on a toy graph u = {1,2,3,4,5,100,101,101},
// v = {10,12,200,24,200,120,200,300} (csrc/test/test_build_graph.cc:11-20,
// test_sampling_h.cc:12-61); the same graph is used here, with assertions.
#include <linux/mempolicy.h>
#include <sys/syscall.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <set>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "chunking.h"
#include "graph_host.h"
#include "grappa/rng.h"
#include "mlpart.h"
#include "numa.h"
#include "pipeline.h"
#include "xborder.h"

using namespace grappa::host;

static int g_failed = 0;
#define CHECK(cond)                                                         \
  do {                                                                      \
    if (!(cond)) {                                                          \
      std::fprintf(stderr, "%s:%d: CHECK failed: %s\n", __FILE__, __LINE__, #cond); \
      ++g_failed;                                                           \
    }                                                                       \
  } while (0)

static CSC toy() {
  const std::vector<int64_t> u = {1, 2, 3, 4, 5, 100, 101, 101, 101};  // (101, 300) twice: dedup
  const std::vector<int64_t> v = {10, 12, 200, 24, 200, 120, 200, 300, 300};
  return build_csc(u.data(), v.data(), static_cast<int64_t>(u.size()), -1);
}

static void test_build() {
  CSC g = toy();
  CHECK(g.n_nodes == 301);
  CHECK(g.n_edges == 8);
  CHECK(g.degree(200) == 3);
  CHECK(g.indices[g.indptr[200]] == 3 && g.indices[g.indptr[200] + 1] == 5 && g.indices[g.indptr[200] + 2] == 101);
  CHECK(g.degree(300) == 1);
  CHECK(g.degree(0) == 0);
}

static void test_pick_offsets() {
  for (uint32_t d : {5u, 17u, 100u, 1000u}) {
    for (uint32_t k : {1u, 4u, d - 1}) {
      std::vector<int64_t> out(k);
      pick_offsets(grappa::hop_key(1, 2, 3, 0), 77, d, k, out.data());
      std::set<int64_t> s(out.begin(), out.end());
      CHECK(s.size() == k);
      for (int64_t o : out) CHECK(o >= 0 && o < d);
      std::vector<int64_t> again(k);
      pick_offsets(grappa::hop_key(1, 2, 3, 0), 77, d, k, again.data());
      CHECK(again == out);  // deterministic
    }
  }
}

static void test_sample_hop() {
  CSC g = toy();
  const std::vector<int64_t> dst = {200, 300, 10, 0};
  std::vector<int64_t> gideg = {3, 2, 1, 0};
  double cs = 0, cn = 0;
  Block b = sample_hop(g, dst.data(), nullptr, 4, 2, grappa::hop_key(0, 0, 0, 0), gideg.data(), &cs, &cn);
  CHECK(b.n_dst == 4);
  CHECK(b.indptr[1] == 2 && b.indptr[2] == 3 && b.indptr[3] == 4 && b.indptr[4] == 4);  // min(deg, fanout)
  for (int i = 0; i < 4; ++i) CHECK(b.src_nid[i] == dst[i]);                          // dst first
  CHECK(b.n_src == static_cast<int64_t>(b.src_nid.size()));
  // coverage: min(1, (max(deg-1,0)+1) / (max(gdeg,0)+1)): 3/4, 1/3, 1/2, 1/1
  CHECK(cn == 4.0);
  const double want = 3.0 / 4 + 1.0 / 3 + 1.0 / 2 + 1.0;
  CHECK(cs > want - 1e-5 && cs < want + 1e-5);
  Block all = sample_hop(g, dst.data(), nullptr, 4, -1, 0, nullptr, nullptr, nullptr);
  CHECK(all.indptr[4] == 5);
}

static void test_random_walk() {
  CSC g = toy();
  const std::vector<int64_t> seeds = {200, 300};
  std::vector<float> w1, w2;
  Block a = random_walk_topk(g, seeds.data(), 2, 3, 0.5, 4, 2, 99, &w1);
  Block b = random_walk_topk(g, seeds.data(), 2, 3, 0.5, 4, 2, 99, &w2);
  CHECK(a.indices == b.indices && w1 == w2);
  for (int64_t i = 0; i < 2; ++i) {
    CHECK(a.indptr[i + 1] - a.indptr[i] <= 2);
    for (int64_t e = a.indptr[i] + 1; e < a.indptr[i + 1]; ++e) CHECK(w1[e - 1] >= w1[e]);  // most visited first
  }
}

static void test_xborder() {
  XBorder xb(0, 3, {0, 10, 20, 30});
  CHECK(xb.owner(0) == 0 && xb.owner(19) == 1 && xb.owner(29) == 2 && xb.owner(30) == -1);
  const std::vector<int64_t> ids = {25, 3, 11, 29, 0};
  auto groups = xb.group_by_partition(ids.data(), 5, nullptr);
  CHECK(groups[0] == (std::vector<int64_t>{3, 0}));
  CHECK(groups[1] == (std::vector<int64_t>{11}));
  CHECK(groups[2] == (std::vector<int64_t>{25, 29}));
  const std::vector<int64_t> halo = {25, 29};
  xb.ad_hoc_build_id_mapping(2, halo.data(), 2);
  int64_t pid = -1, row = -1;
  CHECK(xb.resolve(29, &pid, &row) && pid == 2 && row == 1);
  CHECK(xb.resolve(5, &pid, &row) && pid == 0 && row == 5);
}

static void test_group_by_partition_large() {
  // many slices (one per thread), ids outside every partition, input order kept per owner
  const std::vector<int64_t> prefix = {0, 1000, 1001, 50000, 50000, 70000};  // an empty partition too
  XBorder xb(0, 5, prefix);
  const int64_t n = 200003;
  std::vector<int64_t> ids(n);
  uint64_t x = 12345;
  for (int64_t i = 0; i < n; ++i) {
    x = x * 6364136223846793005ull + 1442695040888963407ull;
    ids[i] = static_cast<int64_t>((x >> 33) % 71000) - 500;  // some below 0, some past the last node
  }
  std::vector<int8_t> mask(static_cast<size_t>(5 * n), 7);
  auto g = xb.group_by_partition(ids.data(), n, mask.data());
  std::vector<std::vector<int64_t>> want(5);
  bool mask_ok = true;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t p = xb.owner(ids[i]);
    if (p >= 0) want[p].push_back(ids[i]);
    for (int64_t q = 0; q < 5; ++q) mask_ok &= mask[static_cast<size_t>(q * n + i)] == (q == p ? 1 : 0);
  }
  CHECK(g == want);
  CHECK(mask_ok);
  CHECK(g[3].empty());
  std::vector<int8_t> mask2(static_cast<size_t>(5 * n), 7);
  xb.mask_by_partition(ids.data(), n, mask2.data());
  CHECK(mask2 == mask);
  CHECK(xb.group_by_partition(ids.data(), n, nullptr) == want);
}

static void test_owner_lookup() {
  // the bucket table, the linear count (table too large) and the binary search (more than
  // 64 partitions, table too large) against std::upper_bound
  auto oracle = [](const std::vector<int64_t>& ps, int64_t gid) -> int64_t {
    if (gid < ps.front() || gid >= ps.back()) return -1;
    return static_cast<int64_t>(std::upper_bound(ps.begin(), ps.end(), gid) - ps.begin()) - 1;
  };
  std::vector<std::vector<int64_t>> cases;
  cases.push_back({5, 1005, 1005, 1006, 70000, 70000, 90000});   // empty partitions, one of size 1
  cases.push_back({0, 1, 1000000000, 1000000001, 3000000000});   // size-1 partitions: no table
  std::vector<int64_t> many = {0};
  for (int p = 0; p < 100; ++p) many.push_back(many.back() + (p == 50 ? 1 : 40000000));  // > 64 parts
  cases.push_back(many);
  uint64_t x = 99;
  for (const auto& ps : cases) {
    XBorder xb(0, static_cast<int64_t>(ps.size()) - 1, ps);
    bool ok = true;
    for (int i = 0; i < 200000; ++i) {
      x = x * 6364136223846793005ull + 1442695040888963407ull;
      const int64_t span = ps.back() - ps.front() + 20;
      const int64_t gid = ps.front() - 10 + static_cast<int64_t>((x >> 11) % static_cast<uint64_t>(span));
      ok &= xb.owner(gid) == oracle(ps, gid);
    }
    for (int64_t b : ps)
      for (int64_t d = -1; d <= 1; ++d) ok &= xb.owner(b + d) == oracle(ps, b + d);
    CHECK(ok);
  }
}

static void test_chunks() {
  char tmpl[] = "/tmp/grappa_chunk_XXXXXX";
  const char* dir = mkdtemp(tmpl);
  CHECK(dir != nullptr);
  if (!dir) return;
  const std::vector<int64_t> u = {0, 1, 2, 3, 4, 5};
  const std::vector<int64_t> v = {1, 2, 3, 4, 5, 0};
  const std::vector<int64_t> pid = {0, 0, 0, 1, 1, 1};
  ChunkStats st = chunk_build(dir, 6, 6, 2, u.data(), v.data(), pid.data());
  CHECK(st.part_nodes[0] == 3 && st.part_nodes[1] == 3);
  CHECK(st.part_edges[0] == 2 + 3 && st.part_edges[1] == 2 + 3);  // intra + one self-loop per node
  CHECK(st.bridge_edges[0 * 2 + 1] == 1 && st.bridge_edges[1 * 2 + 0] == 1);
}

// Grid graph rows x cols (4-neighbour), both directions listed.
static void grid(int64_t rows, int64_t cols, std::vector<int64_t>* u, std::vector<int64_t>* v) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      const int64_t a = r * cols + c;
      if (c + 1 < cols) {
        u->push_back(a); v->push_back(a + 1);
        u->push_back(a + 1); v->push_back(a);
      }
      if (r + 1 < rows) {
        u->push_back(a); v->push_back(a + cols);
        u->push_back(a + cols); v->push_back(a);
      }
    }
}

static void test_multilevel_partition() {
  const int64_t rows = 40, cols = 50, n = rows * cols;
  std::vector<int64_t> u, v;
  grid(rows, cols, &u, &v);
  std::vector<int8_t> train(n, 0);
  for (int64_t i = 0; i < n; i += 3) train[i] = 1;  // a third of the nodes train
  const int64_t m = static_cast<int64_t>(u.size());
  for (int64_t k : {2, 4, 7}) {
    MlPartOptions opt;
    opt.n_parts = k;
    opt.imbalance = 0.05;
    opt.seed = 11;
    const std::vector<int64_t> p = multilevel_partition(n, u.data(), v.data(), m, train.data(), opt);
    CHECK(static_cast<int64_t>(p.size()) == n);
    std::vector<int64_t> nodes(k, 0), seeds(k, 0);
    bool in_range = true;
    for (int64_t i = 0; i < n; ++i) {
      if (p[i] < 0 || p[i] >= k) { in_range = false; continue; }
      ++nodes[p[i]];
      seeds[p[i]] += train[i];
    }
    CHECK(in_range);
    const int64_t n_train = (n + 2) / 3;
    for (int64_t q = 0; q < k; ++q) {
      // both weights within the allowed excess over the even share (plus one vertex of slack)
      CHECK(nodes[q] <= static_cast<int64_t>(1.05 * n / k) + 1);
      CHECK(seeds[q] <= static_cast<int64_t>(1.05 * n_train / k) + 1);
      CHECK(nodes[q] > 0);
    }
    // a grid cut into k blocks cuts O(sqrt(n)) edges per part; hashing cuts ~(k-1)/k of them
    const int64_t cut = edge_cut(n, u.data(), v.data(), m, p.data());
    std::vector<int64_t> hashed(n);
    for (int64_t i = 0; i < n; ++i) hashed[i] = static_cast<int64_t>(grappa::mix64(static_cast<uint64_t>(i)) % k);
    const int64_t cut_hash = edge_cut(n, u.data(), v.data(), m, hashed.data());
    CHECK(cut * 5 < cut_hash);
    CHECK(multilevel_partition(n, u.data(), v.data(), m, train.data(), opt) == p);  // deterministic
  }
  // one part: everything in part 0, no cut
  MlPartOptions one;
  one.n_parts = 1;
  const std::vector<int64_t> p1 = multilevel_partition(n, u.data(), v.data(), m, nullptr, one);
  CHECK(edge_cut(n, u.data(), v.data(), m, p1.data()) == 0);
  bool threw = false;
  try {
    const std::vector<int64_t> bu = {0}, bv = {n};  // endpoint out of range
    MlPartOptions two;
    multilevel_partition(n, bu.data(), bv.data(), 1, nullptr, two);
  } catch (const std::invalid_argument&) {
    threw = true;
  }
  CHECK(threw);
}

struct Item {
  int64_t step;
  std::vector<int64_t> payload;
};

static void test_pipeline_order_and_depth() {
  BatchPipeline<Item> pipe(2);
  std::atomic<int64_t> calls{0};
  pipe.start(50, [&](int64_t s) {
    calls++;
    auto it = std::make_unique<Item>();
    it->step = s;
    it->payload.assign(static_cast<size_t>(s % 7 + 1), s);
    return it;
  });
  for (int64_t s = 0; s < 50; ++s) {
    if (s == 10) {
      // give the producer time to run ahead: it must stop at the depth
      std::this_thread::sleep_for(std::chrono::milliseconds(20));
      CHECK(pipe.ready() <= pipe.depth());
      CHECK(pipe.produced() - pipe.consumed() <= static_cast<int64_t>(pipe.depth()));
    }
    auto it = pipe.next();
    CHECK(it && it->step == s && it->payload.size() == static_cast<size_t>(s % 7 + 1));
  }
  CHECK(pipe.next() == nullptr);  // exhausted
  CHECK(calls.load() == 50 && pipe.consumed() == 50);
}

static void test_pipeline_restart_and_stop() {
  BatchPipeline<Item> pipe(2);
  auto make = [](int64_t base) {
    return [base](int64_t s) {
      auto it = std::make_unique<Item>();
      it->step = base + s;
      return it;
    };
  };
  pipe.start(1000, make(0));
  auto a = pipe.next();
  CHECK(a && a->step == 0);
  std::this_thread::sleep_for(std::chrono::milliseconds(5));  // producer now blocks on a full queue
  pipe.start(3, make(100));                                    // restart drops the old epoch
  for (int64_t s = 0; s < 3; ++s) {
    auto it = pipe.next();
    CHECK(it && it->step == 100 + s);
  }
  CHECK(pipe.next() == nullptr);
  pipe.start(1000, make(0));
  pipe.stop();
  CHECK(pipe.next() == nullptr);  // stopped: no item, no wait
  for (int r = 0; r < 20; ++r) pipe.start(5, make(r));  // rapid restarts join cleanly
  CHECK(pipe.next()->step == 19);
  // a consumer blocked in next() is woken by stop() from another thread
  pipe.start(1000, [](int64_t s) -> std::unique_ptr<Item> {
    if (s > 0) std::this_thread::sleep_for(std::chrono::milliseconds(200));
    auto it = std::make_unique<Item>();
    it->step = s;
    return it;
  });
  CHECK(pipe.next()->step == 0);
  std::thread stopper([&] {
    std::this_thread::sleep_for(std::chrono::milliseconds(10));
    pipe.stop();
  });
  auto none = pipe.next();  // waits for item 1 until stop() wakes it (or item 1 arrives)
  stopper.join();
  CHECK(none == nullptr || none->step == 1);
}

static void test_pipeline_failure() {
  BatchPipeline<Item> pipe(2);
  pipe.start(10, [](int64_t s) -> std::unique_ptr<Item> {
    if (s == 3) throw std::runtime_error("bad seed block");
    auto it = std::make_unique<Item>();
    it->step = s;
    return it;
  });
  for (int64_t s = 0; s < 3; ++s) {
    auto it = pipe.next();
    CHECK(it && it->step == s);  // items made before the failure still arrive
  }
  bool threw = false;
  try {
    pipe.next();
  } catch (const std::runtime_error& e) {
    threw = std::string(e.what()).find("bad seed block") != std::string::npos;
  }
  CHECK(threw);
  pipe.start(2, [](int64_t s) {  // a new start clears the failure
    auto it = std::make_unique<Item>();
    it->step = s;
    return it;
  });
  CHECK(pipe.next()->step == 0 && pipe.next()->step == 1);
}

static int thread_policy_mode() {
  int mode = -1;
  unsigned long mask[16] = {0};
  if (syscall(SYS_get_mempolicy, &mode, mask, 1024UL, nullptr, 0UL) != 0) return -1;
  return mode & ~MPOL_MODE_FLAGS;
}

static void test_numa() {
  CHECK(parse_cpulist("0-3,8,10-11\n") == (std::vector<int>{0, 1, 2, 3, 8, 10, 11}));
  CHECK(parse_cpulist("5") == (std::vector<int>{5}));
  CHECK(parse_cpulist("").empty());
  CHECK(parse_cpulist("x-y").empty());
  const std::vector<int> nodes = numa_nodes();
  CHECK(!nodes.empty());
  const int node = nodes.front();
  CHECK(!numa_node_cpus(node).empty());
  CHECK(numa_node_cpus(-1).empty());
  {
    MemPolicyScope bad(100000);  // not a node: nothing changes
    CHECK(!bad.active());
  }
  const int mode0 = thread_policy_mode();
  {
    MemPolicyScope scope(node);
    if (scope.active()) {
      CHECK(thread_policy_mode() == MPOL_PREFERRED);
      std::vector<int64_t> v(1 << 20, 1);  // faulted in by this thread under the policy
      const int seen = numa_node_of(v.data());
      CHECK(seen == -1 || seen == node);
    }
  }
  CHECK(thread_policy_mode() == mode0);  // the thread's policy is back
  // a CSC built under the policy is the same graph
  CSC a = toy();
  CSC b;
  {
    MemPolicyScope scope(node);
    b = toy();
  }
  CHECK(a.indptr == b.indptr && a.indices == b.indices);
  Bandwidth bw = memory_bandwidth(node, node, 16u << 20, 2, 1);
  CHECK(bw.write_gbs > 0.1 && bw.read_gbs > 0.1);
  CHECK(bw.mem_node_seen == -1 || bw.mem_node_seen == node);
  bool threw = false;
  try {
    memory_bandwidth(node, 100000, 16u << 20, 2, 1);
  } catch (const std::invalid_argument&) {
    threw = true;
  }
  CHECK(threw);
}

int main() {
  test_build();
  test_pick_offsets();
  test_sample_hop();
  test_random_walk();
  test_xborder();
  test_group_by_partition_large();
  test_owner_lookup();
  test_chunks();
  test_multilevel_partition();
  test_pipeline_order_and_depth();
  test_pipeline_restart_and_stop();
  test_pipeline_failure();
  test_numa();
  if (g_failed) {
    std::fprintf(stderr, "%d check(s) failed\n", g_failed);
    return 1;
  }
  std::printf("host engine tests passed\n");
  return 0;
}
