// PinSAGE neighbourhood on the GPU: random walks with restart over in-edges and the
// top-k most visited nodes of every destination, fused with the exclusive scan of
// the per-node neighbour counts (decoupled look-back), producing a block in the
// same CSR form as the neighbour sampler (then relabelled by the S2 compaction).
//
// Rule (shared with the CPU oracle grappa_b200/csrc/host/graph_host.cc,
// random_walk_topk): for dst i, walk j (walker w = i * num_walks + j) and step t,
// r = index_draw4(key, w, t); the walk stops when r.x < restart_prob * 2^32 or the
// node has no in-edge, else moves to in-neighbour draw_below(r.y, deg).  Every
// node visited after the start counts once per visit; the num_neighbors most
// visited (ties: smaller id) become the neighbours, the counts their weights.
// (reference: DGL RandomWalkNeighborSampler behind t10n/dgl_dsg/sampler.py:323-366)
//
// One warp per destination: lane j < num_walks runs walk j and records its visits
// in shared memory; then lane l holds visit l (num_walks * length <= 32), equal
// ids are grouped with __match_any_sync, and every group leader computes its rank
// against the other leaders with shuffles.
#include "common.cuh"
#include "grappa/rng.h"
#include "kernels.h"

namespace grappa {
namespace dev {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTileNodes = 64;
constexpr int kMaxK = 32;

__global__ void __launch_bounds__(kThreads) walk_hop_kernel(WalkHopArgs a) {
  GB_PDL_ENTRY();
  __shared__ long long s_scan[kWarps];
  __shared__ int32_t s_cnt[kTileNodes];
  __shared__ int32_t s_nbr[kTileNodes][kMaxK];
  __shared__ float s_w[kTileNodes][kMaxK];
  __shared__ int32_t s_visit[kWarps][32];
  __shared__ int s_tile[2];
  __shared__ long long s_prefix;

  const LookBack::Ticket tk = LookBack::ticket(a.scan_scratch, s_tile);
  const int tile = tk.tile;
  const int n_dst = a.n_dst_ptr ? *a.n_dst_ptr : a.n_dst;
  // capacity-sized grid: tiles past the last live one leave before the scan
  const int last_tile = n_dst > 0 ? (n_dst - 1) / kTileNodes : 0;
  if (tile > last_tile) return;
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint64_t key = hop_key(static_cast<uint64_t>(a.counters[0]), static_cast<uint64_t>(a.counters[1]),
                               static_cast<uint64_t>(a.counters[2]), static_cast<uint64_t>(a.hop));
  const int nv = a.num_walks * a.length;
  for (int r = w; r < kTileNodes; r += kWarps) {
    const int i = tile * kTileNodes + r;
    int kept = 0;
    if (i < n_dst) {
      s_visit[w][lane] = -1;
      __syncwarp();
      const int32_t s0 = a.dst_nid[i];
      if (lane < a.num_walks) {
        int64_t cur = s0;
        const uint64_t walker = static_cast<uint64_t>(i) * static_cast<uint64_t>(a.num_walks) + lane;
        for (int t = 0; t < a.length; ++t) {
          if (cur < 0 || cur >= a.n_graph_nodes) break;
          const U4 rr = index_draw4(key, walker, static_cast<uint32_t>(t));
          if (rr.x < a.restart_thr) break;
          const int64_t beg = a.indptr[cur];
          const int64_t d = a.indptr[cur + 1] - beg;
          if (d == 0) break;
          cur = a.indices[beg + draw_below(rr.y, static_cast<uint32_t>(d))];
          s_visit[w][lane * a.length + t] = static_cast<int32_t>(cur);
        }
      }
      __syncwarp();
      const int32_t v = lane < nv ? s_visit[w][lane] : -1;
      const uint32_t grp = __match_any_sync(0xffffffffu, v);
      const int cnt = __popc(grp);
      const bool leader = v >= 0 && lane == __ffs(grp) - 1;
      // rank among the leaders: more visits first, then smaller id
      int rank = 0;
      for (int s = 0; s < 32; ++s) {
        const int32_t vs = __shfl_sync(0xffffffffu, v, s);
        const int cs = __shfl_sync(0xffffffffu, cnt, s);
        const bool ls = __shfl_sync(0xffffffffu, leader ? 1 : 0, s) != 0;
        if (ls && s != lane && (cs > cnt || (cs == cnt && vs < v))) ++rank;
      }
      const uint32_t leaders = __ballot_sync(0xffffffffu, leader);
      kept = min(__popc(leaders), a.num_neighbors);
      if (leader && rank < a.num_neighbors) {
        s_nbr[r][rank] = v;
        s_w[r][rank] = static_cast<float>(cnt);
      }
    }
    if (lane == 0) s_cnt[r] = kept;
    __syncwarp();
  }
  __syncthreads();
  const int32_t my_cnt = threadIdx.x < kTileNodes ? s_cnt[threadIdx.x] : 0;
  long long total;
  const long long excl = block_exclusive_scan<kThreads, long long>(my_cnt, s_scan, &total);
  if (w == 0) {
    const long long p = LookBack::exclusive_prefix(a.scan_scratch, tk, total, a.err);
    if (lane == 0) s_prefix = p;
  }
  __syncthreads();
  const int i = tile * kTileNodes + threadIdx.x;
  if (threadIdx.x < kTileNodes && i < n_dst) {
    const long long off = s_prefix + excl;
    a.out_indptr[i] = static_cast<int32_t>(off < a.cap_edges ? off : a.cap_edges);
    if (off + my_cnt > a.cap_edges) {
      set_error(a.err, kErrCapacity);
    } else {
      for (int k = 0; k < my_cnt; ++k) {
        a.out_nbr[off + k] = s_nbr[threadIdx.x][k];
        a.out_w[off + k] = s_w[threadIdx.x][k];
      }
    }
  }
  if (tile == last_tile && threadIdx.x == 0) {
    const long long tile_end = s_prefix + total;
    if (tile_end > a.cap_edges) set_error(a.err, kErrCapacity);
    const int32_t tot = static_cast<int32_t>(tile_end > a.cap_edges ? a.cap_edges : tile_end);
    a.out_indptr[n_dst] = tot;
    *a.n_edges_out = tot;
  }
}

}  // namespace

void launch_walk_hop(const WalkHopArgs& a, int cap_dst, cudaStream_t stream) {
  if (a.num_walks <= 0 || a.length <= 0 || a.num_walks * a.length > 32)
    throw std::invalid_argument("walk_hop: num_walks * length must be in [1, 32]");
  if (a.num_neighbors <= 0 || a.num_neighbors > kMaxK) throw std::invalid_argument("walk_hop: 1..32 neighbours");
  const int tiles = static_cast<int>(ceil_div(cap_dst > 0 ? cap_dst : 1, kTileNodes));
  // no clearing of the scan scratch: its look-back words carry the launch number
  launch_k(walk_hop_kernel, tiles, kThreads, 0, stream, a);
  GB_LAUNCH_CHECK();
}

int walk_scan_scratch_words(int cap_dst) {
  return static_cast<int>(ceil_div(cap_dst > 0 ? cap_dst : 1, kTileNodes)) + 1;
}

}  // namespace dev
}  // namespace grappa
