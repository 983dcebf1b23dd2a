// S2: block compaction (the GPU equivalent of DGL's to_block as used by
// t10n/dgl_dsg/compliant.py:32-49): the block's src nodes are its dst nodes, in
// order, followed by the sampled neighbours that are not dst nodes, in order of
// first appearance in the edge list; every edge gets the local index of its
// source; src_sampled marks the src nodes that were sampled as a neighbour (the
// frontier of the next hop, csrc/python/py_graph.cc:140-190).
//
// Instead of a hash table the kernels use a dense map over the graph's node ids
// (8 bytes per node, resident in HBM and mostly in the 126 MB L2): entry =
// (tag << 32) | position.  Tags decrease from call to call, so an atomicMin with
// the current tag always wins over anything left by an earlier call and the map
// is never cleared.
//   K1  map[dst[i]] = min(., tag|i);  map[nbr[e]] = min(., tag|(n_dst+e))
//   K2  edge e is a first appearance iff map[nbr[e]] == tag|(n_dst+e); decoupled
//       look-back scan of those flags gives new local ids n_dst + rank;
//       map[nbr[e]] = tag|lid, src_nid[lid] = nbr[e]
//   K3  indices[e] = low32(map[nbr[e]]); src_sampled[indices[e]] = 1
// The neighbour sampler can do K1's work as it writes the block (SampleHopArgs.map):
// the compaction then starts at K2 (k1_done).
// A first-appearance test in K2 can never see a rewritten entry as its own value:
// a rewritten entry holds a local id <= n_dst + e0 < n_dst + e for any later e.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace grappa {
namespace dev {

namespace {

constexpr int kThreads = 256;
constexpr int kItems = 4;  // edges per thread in K2
constexpr int kTile = kThreads * kItems;

__device__ __forceinline__ unsigned long long tag_word(const int64_t* gen, int slot) {
  return compact_tag_word(gen, slot);
}

__global__ void __launch_bounds__(kThreads) compact_k1(CompactArgs a, const int64_t* gen, int slot) {
  GB_PDL_ENTRY();
  const int n_dst = *a.n_dst_ptr;
  const int n_e = *a.n_edges_ptr;
  const unsigned long long tw = tag_word(gen, slot);
  const long long total = static_cast<long long>(n_dst) + n_e;
  for (long long j = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; j < total;
       j += static_cast<long long>(gridDim.x) * blockDim.x) {
    int32_t id;
    if (j < n_dst) {
      id = a.dst_nid[j];
      a.src_nid[j] = id;
      a.src_sampled[j] = 0;
    } else {
      id = a.nbr[j - n_dst];
    }
    if (id < 0 || id >= a.n_graph_nodes) {
      set_error(a.err, kErrBadIndex);
      continue;
    }
    atomicMin(a.map + id, tw | static_cast<unsigned long long>(j));
  }
}

__global__ void __launch_bounds__(kThreads) compact_k2(CompactArgs a, const int64_t* gen, int slot) {
  GB_PDL_ENTRY();
  __shared__ long long s_scan[kThreads / 32];
  __shared__ int s_tile[2];
  __shared__ long long s_prefix;
  const LookBack::Ticket tk = LookBack::ticket(a.scan_scratch, s_tile);
  const int tile = tk.tile;
  const int n_dst = *a.n_dst_ptr;
  const int n_e = *a.n_edges_ptr;
  // capacity-sized grid: tiles past the last live one leave before the scan
  const int last_tile = n_e > 0 ? (n_e - 1) / kTile : 0;
  if (tile > last_tile) return;
  const unsigned long long tw = tag_word(gen, slot);
  const int e0 = tile * kTile + threadIdx.x * kItems;
  int32_t ids[kItems];
  bool fresh[kItems];
  int cnt = 0;
#pragma unroll
  for (int q = 0; q < kItems; ++q) {
    const int e = e0 + q;
    fresh[q] = false;
    ids[q] = -1;
    if (e < n_e) {
      ids[q] = a.nbr[e];
      if (ids[q] >= 0 && ids[q] < a.n_graph_nodes) {
        const unsigned long long m = a.map[ids[q]];
        fresh[q] = m == (tw | static_cast<unsigned long long>(n_dst + e));
        // a destination node sampled as a neighbour: part of the next hop's frontier
        // (marked here so that the edge rewrite K3 can run after the later hops)
        const unsigned long long pos = m & 0xffffffffull;
        if (!fresh[q] && (m >> 32) == (tw >> 32) && pos < static_cast<unsigned long long>(n_dst))
          a.src_sampled[pos] = 1;
      }
      cnt += fresh[q];
    }
  }
  long long total;
  const long long excl = block_exclusive_scan<kThreads, long long>(cnt, s_scan, &total);
  if ((threadIdx.x >> 5) == 0) {
    const long long p = LookBack::exclusive_prefix(a.scan_scratch, tk, total, a.err);
    if (lane_id() == 0) s_prefix = p;
  }
  __syncthreads();
  long long lid = static_cast<long long>(n_dst) + s_prefix + excl;
#pragma unroll
  for (int q = 0; q < kItems; ++q) {
    if (!fresh[q]) continue;
    if (lid < a.cap_src) {
      a.map[ids[q]] = tw | static_cast<unsigned long long>(lid);
      a.src_nid[lid] = ids[q];
      a.src_sampled[lid] = 1;  // first appearance as a neighbour
    } else {
      set_error(a.err, kErrCapacity);
    }
    ++lid;
  }
  if (tile == last_tile && threadIdx.x == 0) {
    long long ns = static_cast<long long>(n_dst) + s_prefix + total;
    if (ns > a.cap_src) ns = a.cap_src;
    *a.n_src_out = static_cast<int32_t>(ns);
  }
}

__global__ void __launch_bounds__(kThreads) compact_k3(CompactArgs a) {
  GB_PDL_ENTRY();
  const int n_e = *a.n_edges_ptr;
  for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n_e;
       e += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int32_t id = a.nbr[e];
    int32_t lid = 0;
    if (id >= 0 && id < a.n_graph_nodes) lid = static_cast<int32_t>(a.map[id] & 0xffffffffull);
    if (lid >= a.cap_src || lid < 0) lid = 0;
    a.indices[e] = lid;
    a.src_sampled[lid] = 1;
    if (a.t_cnt) a.t_rank[e] = atomicAdd(a.t_cnt + lid, 1);
  }
}

// K3 of several hops in one launch, after the last hop's K2.  A node's local position
// survives the later hops' passes: the next hop's destinations are this hop's sources
// in order, so its K1 writes the same position under a new tag, and its K2 rewrites only
// nodes that are not among them; so low32(map[id]) still is the local source index of
// every neighbour id of every earlier hop.
__global__ void __launch_bounds__(kThreads) compact_k3_multi(CompactEdgesArgs a) {
  GB_PDL_ENTRY();
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (int h = 0; h < a.n_hops; ++h) {
    const CompactEdgesArgs::Hop hp = a.hops[h];
    const int n_e = *hp.n_edges_ptr;
    for (long long e = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; e < n_e; e += stride) {
      const int32_t id = hp.nbr[e];
      int32_t lid = 0;
      if (id >= 0 && id < a.n_graph_nodes) lid = static_cast<int32_t>(a.map[id] & 0xffffffffull);
      if (lid >= hp.cap_src || lid < 0) lid = 0;
      hp.indices[e] = lid;
    }
  }
}

constexpr int kTpThreads = 1024;

// Exclusive scan of the per-source edge counts into tptr (one CTA, coalesced: 1024
// counts per iteration, each iteration's block scan plus a running carry); the counts
// are cleared for the next block.
__global__ void __launch_bounds__(kTpThreads) block_transpose_scan_kernel(const int32_t* n_src_ptr, int32_t* t_cnt,
                                                                           int32_t* tptr, int cap_src) {
  GB_PDL_ENTRY();
  __shared__ int s_scan[kTpThreads / 32];
  const int n_src = min(*n_src_ptr, cap_src);
  int carry = 0;
  for (int base = 0; base < n_src; base += kTpThreads) {
    const int i = base + static_cast<int>(threadIdx.x);
    const int c = i < n_src ? t_cnt[i] : 0;
    int total;
    const int excl = block_exclusive_scan<kTpThreads, int>(c, s_scan, &total);
    if (i < n_src) {
      tptr[i] = carry + excl;
      t_cnt[i] = 0;
    }
    carry += total;
  }
  if (threadIdx.x == 0) tptr[n_src] = carry;
}

// tdst[tptr[s] + rank_e] = v for every edge e = (s -> v): one warp per destination.
__global__ void __launch_bounds__(kThreads) block_transpose_fill_kernel(const int32_t* indptr, const int32_t* indices,
                                                                         const int32_t* n_dst_ptr,
                                                                         const int32_t* n_src_ptr, const int32_t* t_rank,
                                                                         const int32_t* tptr, int32_t* tdst,
                                                                         int cap_edges, int32_t* err) {
  GB_PDL_ENTRY();
  const int n_dst = *n_dst_ptr;
  const int n_src = *n_src_ptr;
  const int warps = (gridDim.x * kThreads) >> 5;
  for (int v = (blockIdx.x * kThreads + threadIdx.x) >> 5; v < n_dst; v += warps) {
    const int beg = indptr[v], end = indptr[v + 1];
    for (int e = beg + static_cast<int>(lane_id()); e < end; e += 32) {
      const int s = indices[e];
      const int k = (s >= 0 && s < n_src) ? tptr[s] + t_rank[e] : -1;
      if (k >= 0 && k < cap_edges) tdst[k] = v;
      else set_error(err, kErrBadIndex);
    }
  }
}

}  // namespace

void launch_block_transpose(const int32_t* indptr, const int32_t* indices, const int32_t* n_dst_ptr,
                            const int32_t* n_src_ptr, int32_t* t_cnt, const int32_t* t_rank, int32_t* tptr,
                            int32_t* tdst, int cap_src, int cap_edges, int32_t* err, cudaStream_t stream) {
  launch_k(block_transpose_scan_kernel, 1, kTpThreads, 0, stream, n_src_ptr, t_cnt, tptr, cap_src);
  GB_LAUNCH_CHECK();
  const int cap_dst = cap_src;  // destinations are the first sources
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = static_cast<int>(std::min<long long>(ceil_div(cap_dst > 0 ? cap_dst : 1, kThreads / 32),
                                                        static_cast<long long>(sms) * 8));
  launch_k(block_transpose_fill_kernel, grid, kThreads, 0, stream, indptr, indices, n_dst_ptr, n_src_ptr, t_rank, tptr, tdst,
                                                            cap_edges, err);
  GB_LAUNCH_CHECK();
}

int compact_scan_scratch_words(int cap_edges) {
  return static_cast<int>(ceil_div(cap_edges > 0 ? cap_edges : 1, kTile)) + 1;
}

void launch_compact_edges(const CompactEdgesArgs& a, int64_t cap_edges_total, int num_sms, cudaStream_t stream) {
  if (a.n_hops < 1 || a.n_hops > CompactEdgesArgs::kMaxHops) throw std::invalid_argument("compact_edges: 1..8 hops");
  const int g = static_cast<int>(std::min<long long>(static_cast<long long>(num_sms) * 8,
                                                     ceil_div(cap_edges_total > 0 ? cap_edges_total : 1, kThreads)));
  launch_k(compact_k3_multi, g, kThreads, 0, stream, a);
  GB_LAUNCH_CHECK();
}

void launch_compact(const CompactArgs& a, int cap_dst, int cap_edges, const int64_t* gen, int slot, int num_sms,
                    cudaStream_t stream, bool k1_done, bool run_k3) {
  const int grid_stride = num_sms * 8;
  if (!k1_done) {
    const long long work1 = static_cast<long long>(cap_dst) + cap_edges;
    const int g1 = static_cast<int>(std::min<long long>(grid_stride, ceil_div(work1 > 0 ? work1 : 1, kThreads)));
    launch_k(compact_k1, g1, kThreads, 0, stream, a, gen, slot);
    GB_LAUNCH_CHECK();
  }
  const int tiles = static_cast<int>(ceil_div(cap_edges > 0 ? cap_edges : 1, kTile));
  // no clearing of the scan scratch: its look-back words carry the launch number
  launch_k(compact_k2, tiles, kThreads, 0, stream, a, gen, slot);
  GB_LAUNCH_CHECK();
  if (!run_k3) return;
  const int g3 = static_cast<int>(std::min<long long>(grid_stride, ceil_div(cap_edges > 0 ? cap_edges : 1, kThreads)));
  launch_k(compact_k3, g3, kThreads, 0, stream, a);
  GB_LAUNCH_CHECK();
}

}  // namespace dev
}  // namespace grappa
