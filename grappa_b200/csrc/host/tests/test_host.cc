// Native tests of the C++ host engine (CSC build, sampling rule, coverage ratio,
// compaction order, random walks, cross-partition ids, chunk writer), built and run
// without Python:
//   g++ -O2 -std=c++17 -fopenmp -Igrappa_b200/csrc/include -Igrappa_b200/csrc/host \
//       grappa_b200/csrc/host/tests/test_host.cc grappa_b200/csrc/host/{graph_host,xborder,chunking}.cc
// The reference ships smoke executables on a toy graph u = {1,2,3,4,5,100,101,101},
// v = {10,12,200,24,200,120,200,300} (csrc/test/test_build_graph.cc:11-20,
// test_sampling_h.cc:12-61); the same graph is used here, with assertions.
#include <cstdio>
#include <cstdlib>
#include <set>
#include <string>
#include <vector>

#include "chunking.h"
#include "graph_host.h"
#include "grappa/rng.h"
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

int main() {
  test_build();
  test_pick_offsets();
  test_sample_hop();
  test_random_walk();
  test_xborder();
  test_chunks();
  if (g_failed) {
    std::fprintf(stderr, "%d check(s) failed\n", g_failed);
    return 1;
  }
  std::printf("host engine tests passed\n");
  return 0;
}
