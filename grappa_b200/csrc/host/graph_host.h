// Host (CPU) graph engine: CSC construction, neighbour sampling without
// replacement with the coverage counter, and block compaction.
//
// This is the CPU path of the framework (the gloo/CPU training config runs on it)
// and the oracle of the GPU kernels: it draws the same Philox streams and applies
// the same selection rule as grappa_b200/csrc/cuda/sample.cu, so a GPU batch can be
// compared with a CPU batch element by element.
//
// Reference behaviour reproduced (file:line in mpi-dsg/grappa):
//   CSC build with parallel-edge de-duplication   csrc/graph/build.h:20-70
//   pick_n = deg < fanout ? deg : fanout            csrc/graph/sampling_h.h:20-38
//   coverage ratio min(1,(max(deg-1,0)+1)/(max(gdeg,0)+1)), first hop only
//                                                   csrc/graph/sampling_h.h:67-140,
//                                                   csrc/python/py_graph.cc:258-292
//   next-hop sources = unique sampled neighbours    csrc/python/py_graph.cc:140-190
//   block: dst nodes first, then new sources        t10n/dgl_dsg/compliant.py:32-49
#pragma once
#include <cstdint>
#include <vector>

namespace grappa {
namespace host {

struct CSC {
  int64_t n_nodes = 0;
  int64_t n_edges = 0;
  std::vector<int64_t> indptr;   // n_nodes + 1, by destination
  std::vector<int64_t> indices;  // sources, ascending within each destination
  int64_t degree(int64_t v) const { return indptr[v + 1] - indptr[v]; }
};

// Build a CSC (in-edges by destination) from directed edges u->v.  Parallel
// edges are removed; neighbours are sorted ascending.  n_nodes < 0 means
// max id + 1.
CSC build_csc(const int64_t* u, const int64_t* v, int64_t n_e, int64_t n_nodes);

// One sampled hop laid out as a block (message-flow graph) in CSR-by-dst form.
struct Block {
  int64_t n_dst = 0;
  int64_t n_src = 0;
  std::vector<int64_t> indptr;         // n_dst + 1
  std::vector<int64_t> indices;        // local src index per edge
  std::vector<int64_t> src_nid;        // graph ids of the src nodes, dst nodes first
  std::vector<uint8_t> src_sampled;    // 1 if the src node was sampled as a neighbour
};

// Select k distinct offsets of [0, d) for node `nid` (d > k) with the shared rule
// of grappa/rng.h.  Writes k offsets to out in acceptance order.
void pick_offsets(uint64_t key, uint64_t nid, uint32_t d, uint32_t k, int64_t* out);

// Sample one hop.  dst_nid[i] are the block's destination nodes; only those with
// frontier[i] != 0 (or all, when frontier is null) draw neighbours.  fanout < 0
// takes every neighbour.  If gideg is given, the coverage ratios of the frontier
// nodes are summed into *cov_sum and their count into *cov_n.
Block sample_hop(const CSC& g, const int64_t* dst_nid, const uint8_t* frontier, int64_t n_dst,
                 int64_t fanout, uint64_t key, const int64_t* gideg, double* cov_sum,
                 double* cov_n);

// PinSAGE neighbourhood (the random-walk neighbour sampler DGL provides to the
// reference, t10n/dgl_dsg/sampler.py:323-366): every seed starts num_walks walks
// over in-edges; before each of at most `length` steps a walk stops with
// probability restart_prob (and at a node without in-edges).  Every node a walk
// visits after its start is counted for the seed; the num_neighbors most visited
// (ties: smaller id first) become the seed's neighbours, their counts the edge
// weights.  Walker w = i * num_walks + j, step t draws index_draw4(key, w, t):
// word x decides the stop (x < restart_prob * 2^32), word y the in-neighbour
// (draw_below(y, deg)).  Same rule on the GPU.
Block random_walk_topk(const CSC& g, const int64_t* seeds, int64_t n_seeds, int length,
                       double restart_prob, int num_walks, int num_neighbors, uint64_t key,
                       std::vector<float>* weights);

// Coverage ratio of one seed (shared definition with the GPU sampler).
inline float coverage_ratio(int64_t local_deg, int64_t global_deg) {
  const int64_t up = local_deg - 1 < 0 ? 0 : local_deg - 1;
  const int64_t sup = global_deg < 0 ? 0 : global_deg;
  float t = (static_cast<float>(up) + 1.0f) / (static_cast<float>(sup) + 1.0f);
  if (!(t <= 1.0f)) t = 1.0f;  // also catches NaN
  return t;
}

// RMAT candidate edges [e_begin, e_end): key = u * n + v for valid candidates
// (u, v < n, u != v, stored with u < v), -1 otherwise.
void rmat_candidates(int64_t n, int scale, double a, double b, double c, uint64_t seed,
                     int64_t e_begin, int64_t e_end, int64_t* keys);

// Keys used to shuffle node ids: mix64(ids ^ f(seed, epoch)).  Sorting by these
// keys gives the same permutation on the CPU and on the GPU.
void shuffle_keys(const int64_t* ids, int64_t n, uint64_t seed, uint64_t epoch, int64_t* keys);

}  // namespace host
}  // namespace grappa
