// Multilevel k-way edge-cut graph partitioner (the role METIS plays in the reference's
// chunker, t10n/dataset/chunk_seq.py:47-50: dgl.metis_partition_assignment with the
// training mask as a balance type).
//
// Coarsening by heavy-edge matching until the graph is small, a greedy graph-growing
// k-way partition of the coarsest graph, then projection level by level with greedy
// boundary refinement.  Every vertex carries two weights (1, and 1 if it is a
// training node), and both are kept within (1 + imbalance) of their even share per
// part, which balances the partitions' node counts and their training seeds.
#pragma once
#include <cstdint>
#include <vector>

namespace grappa {
namespace host {

struct MlPartOptions {
  int64_t n_parts = 2;
  double imbalance = 0.03;       // allowed excess over the even share, per weight type
  uint64_t seed = 0;
  int refine_passes = 8;         // boundary refinement passes per level
  int64_t coarsest = 0;          // stop coarsening at this many vertices (0: 40 per part, >= 2000)
};

// u, v: directed edges (any order; self-loops and duplicates allowed, the graph is
// symmetrised); train: per-vertex 0/1 (may be null).  Returns the part of every vertex.
std::vector<int64_t> multilevel_partition(int64_t n, const int64_t* u, const int64_t* v, int64_t m,
                                          const int8_t* train, const MlPartOptions& opt);

// Number of undirected edges whose endpoints lie in different parts.
int64_t edge_cut(int64_t n, const int64_t* u, const int64_t* v, int64_t m, const int64_t* part);

}  // namespace host
}  // namespace grappa
