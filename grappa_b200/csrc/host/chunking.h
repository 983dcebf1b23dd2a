// Partition-chunk writer (CPU): splits a global graph into the on-disk layout
// the reference's loaders read, file for file:
//   p{i}.u.bin / p{i}.v.bin   int64 local ids of intra-partition edges u->v, with one
//                             self-loop per node of the partition appended
//   p{i}.oid.bin              int64 original id of each local id
//   p{i}.ideg.bin             int64 global in-degree of each local node
//   p{i}.nfeat.bin            float32 [n_i, dim]
//   p{i}.label.bin            float32 labels
//   p{i}.train/.valid/.test.bin  int8 masks
//   b{i}_{j}.u.bin / .v.bin   bridge edges from partition i into j (u local to i,
//                             v local to j); absent when there are none
// Reference: csrc/python/py_seq_chunking.cc:16-328, t10n/dataset/io_dist.py:234-245.
//
// Local ids are assigned in increasing original-id order and every node assigned
// to a partition is kept, also those without intra-partition edges.  (The
// reference numbers nodes by first appearance in the intra edge list and drops
// nodes without such an edge, then maps their bridge endpoints to 0:
// csrc/python/py_seq_chunking.cc:63-97,170,182.)
#pragma once
#include <cstdint>
#include <string>
#include <vector>

namespace grappa {
namespace host {

struct ChunkStats {
  std::vector<int64_t> part_nodes;
  std::vector<int64_t> part_edges;      // intra edges incl. self-loops
  std::vector<int64_t> bridge_edges;    // [n_part * n_part]
};

ChunkStats chunk_build(const std::string& path, int64_t n_n, int64_t n_e, int64_t n_part,
                       const int64_t* src, const int64_t* dst, const int64_t* nid2pid);

void chunk_split_node_feat(const std::string& path, int64_t n_n, int64_t dim, int64_t n_part,
                           const float* feat);

void chunk_split_node_data(const std::string& path, int64_t n_n, int64_t n_part,
                           const float* label, const int8_t* train, const int8_t* valid,
                           const int8_t* test);

}  // namespace host
}  // namespace grappa
