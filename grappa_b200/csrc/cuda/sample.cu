// S1: one hop of neighbour sampling without (or with) replacement, fused with the
// exclusive scan of the per-node pick counts (decoupled look-back) and with the
// coverage-ratio reduction of the seed hop.
//
// Per destination node i of the block (dst_nid[i], i < *n_dst):
//   pick_i = !frontier[i] ? 0 : (fanout < 0 || deg <= fanout ? deg : fanout)
// (reference: csrc/graph/sampling_h.h:20-38, "unique sampled neighbours only"
// frontier of csrc/python/py_graph.cc:140-190), then k = pick_i distinct offsets
// with the rule of grappa/rng.h: the first k distinct values of the node's
// Philox sequence, found 32 draws at a time by one warp (duplicates found with
// register shuffles against the other lanes and against the accepted list in
// shared memory).  The CPU oracle grappa_b200/csrc/host/graph_host.cc
// (pick_offsets, sample_hop) produces the same picks.
//
// Outputs: out_indptr[0..n_dst] (CSR by dst of the block), out_nbr[e] (graph id of
// the sampled neighbour), *n_edges.  Sizes beyond the buffers set kErrCapacity.
#include "common.cuh"
#include "grappa/rng.h"
#include "kernels.h"

namespace grappa {
namespace dev {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
// destination nodes per CTA: 16 warps share 64 nodes (four each), so that enough
// warps are in flight to hide the dependent index gathers of every node
constexpr int kTileNodes = 64;
constexpr int kSmemAcc = 64;  // accepted offsets kept in shared memory up to this fanout

__device__ __forceinline__ uint64_t step_key(const int64_t* counters, int hop) {
  // counters = [seed, epoch, step, ...]
  return hop_key(static_cast<uint64_t>(counters[0]), static_cast<uint64_t>(counters[1]),
                 static_cast<uint64_t>(counters[2]), static_cast<uint64_t>(hop));
}

// The warp draws k distinct offsets of [0, d) for node nid into acc[0..k).
__device__ void warp_pick_distinct(uint64_t key, uint64_t nid, uint32_t d, uint32_t k, int32_t* acc) {
  const uint32_t lane = lane_id();
  uint32_t n_acc = 0;
  for (uint32_t base = 0; base < kMaxDraws && n_acc < k; base += 32) {
    const uint32_t t = base + lane;
    const int32_t o = static_cast<int32_t>(draw_below(node_draw(key, nid, t), d));
    bool dup = false;
#pragma unroll 8
    for (int s = 0; s < 32; ++s) {
      const int32_t os = __shfl_sync(0xffffffffu, o, s);
      dup |= (static_cast<uint32_t>(s) < lane) && (os == o);
    }
    for (uint32_t j = 0; j < n_acc; ++j) dup |= (acc[j] == o);
    const uint32_t first = __ballot_sync(0xffffffffu, !dup);
    const uint32_t rank = n_acc + __popc(first & lanemask_lt());
    if (!dup && rank < k) acc[rank] = o;
    n_acc = min(k, n_acc + __popc(first));
    __syncwarp();
  }
  if (n_acc < k && lane == 0) {
    // deterministic completion with the smallest unused offsets (same as the oracle)
    for (uint32_t o = 0; o < d && n_acc < k; ++o) {
      bool seen = false;
      for (uint32_t j = 0; j < n_acc; ++j) seen |= (acc[j] == static_cast<int32_t>(o));
      if (!seen) acc[n_acc++] = static_cast<int32_t>(o);
    }
  }
  __syncwarp();
}

__global__ void __launch_bounds__(kThreads) sample_hop_kernel(SampleHopArgs a) {
  GB_PDL_ENTRY();
  __shared__ long long s_scan[kWarps];
  __shared__ long long s_off[kTileNodes];
  __shared__ int32_t s_pick[kTileNodes];
  __shared__ int32_t s_nid[kTileNodes];
  __shared__ long long s_beg[kTileNodes];
  __shared__ long long s_deg[kTileNodes];
  __shared__ int32_t s_acc[kWarps][kSmemAcc];
  __shared__ int s_tile[2];
  __shared__ long long s_prefix;
  __shared__ float s_cov[2][kWarps];

  const LookBack::Ticket tk = LookBack::ticket(a.scan_scratch, s_tile);
  const int tile = tk.tile;
  const int n_dst = a.n_dst_ptr ? *a.n_dst_ptr : a.n_dst;
  // the grid is sized by the capacity; tiles past the last live one take no part in
  // the scan (no live tile waits on them), so they leave at once
  const int last_tile = n_dst > 0 ? (n_dst - 1) / kTileNodes : 0;
  if (tile > last_tile) return;
  const int i = tile * kTileNodes + threadIdx.x;
  const bool valid = threadIdx.x < kTileNodes && i < n_dst;
  int32_t nid = -1;
  int64_t deg = 0, beg = 0;
  int32_t pick = 0;
  float cov = 0.f, covn = 0.f;
  const unsigned long long tw = a.map ? compact_tag_word(a.counters + 4, a.hop) : 0ull;
  if (valid) {
    nid = a.dst_nid[i];
    if (a.map) {  // compaction K1 for the destinations
      a.src_nid[i] = nid;
      a.src_sampled[i] = 0;
      if (nid >= 0 && nid < a.map_nodes) atomicMin(a.map + nid, tw | static_cast<unsigned long long>(i));
    }
    const bool f = a.frontier ? a.frontier[i] != 0 : true;
    if (nid >= 0 && nid < a.n_graph_nodes) {
      beg = a.indptr[nid];
      deg = a.indptr[nid + 1] - beg;
      if (f) {
        if (a.replace)
          pick = deg == 0 ? 0 : (a.fanout < 0 ? static_cast<int32_t>(deg) : a.fanout);
        else
          pick = (a.fanout < 0 || deg <= a.fanout) ? static_cast<int32_t>(deg) : a.fanout;
        if (a.gideg) {
          const int64_t up = deg - 1 < 0 ? 0 : deg - 1;
          const int64_t g = a.gideg[i] < 0 ? 0 : a.gideg[i];
          float r = (static_cast<float>(up) + 1.0f) / (static_cast<float>(g) + 1.0f);
          if (!(r <= 1.0f)) r = 1.0f;
          cov = r;
          covn = 1.f;
        }
      }
    } else if (nid >= a.n_graph_nodes) {
      set_error(a.err, kErrBadIndex);
    }
  }
  if (a.gideg) {
    cov = warp_sum(cov);
    covn = warp_sum(covn);
    if (lane_id() == 0) {
      s_cov[0][threadIdx.x >> 5] = cov;
      s_cov[1][threadIdx.x >> 5] = covn;
    }
  }
  long long total;
  const long long excl = block_exclusive_scan<kThreads, long long>(pick, s_scan, &total);
  if ((threadIdx.x >> 5) == 0) {
    const long long p = LookBack::exclusive_prefix(a.scan_scratch, tk, total, a.err);
    if (lane_id() == 0) s_prefix = p;
    if (a.gideg && a.cov_accum && lane_id() < 2) {
      float s = 0.f;
      for (int w = 0; w < kWarps; ++w) s += s_cov[lane_id()][w];
      if (s != 0.f) atomicAdd(a.cov_accum + lane_id(), s);
    }
  }
  __syncthreads();
  const long long off = s_prefix + excl;
  if (threadIdx.x < kTileNodes) {
    s_off[threadIdx.x] = off;
    s_pick[threadIdx.x] = pick;
    s_nid[threadIdx.x] = nid;
    s_beg[threadIdx.x] = beg;
    s_deg[threadIdx.x] = deg;
  }
  if (valid) a.out_indptr[i] = static_cast<int32_t>(off < a.cap_edges ? off : a.cap_edges);
  const long long tile_end = s_prefix + total;
  // the tile holding the last destination (or tile 0 when there is none) writes the total
  if (tile == last_tile && threadIdx.x == 0) {
    if (tile_end > a.cap_edges) set_error(a.err, kErrCapacity);
    const int32_t tot = static_cast<int32_t>(tile_end > a.cap_edges ? a.cap_edges : tile_end);
    a.out_indptr[n_dst] = tot;
    *a.n_edges_out = tot;
  }
  __syncthreads();
  if (tile_end == s_prefix) return;  // nothing sampled in this tile

  const uint64_t key = step_key(a.counters, a.hop);
  const int w = threadIdx.x >> 5;
  const uint32_t lane = lane_id();
  for (int r = w; r < kTileNodes; r += kWarps) {
    const int32_t k = s_pick[r];
    if (k == 0) continue;
    const long long o = s_off[r];
    if (o + k > a.cap_edges) {
      if (lane == 0) set_error(a.err, kErrCapacity);
      continue;
    }
    const int32_t v = s_nid[r];
    const int64_t beg = s_beg[r];  // the node's CSR range, read once in the count phase
    const int64_t d = s_deg[r];
    int32_t* out = a.out_nbr + o;
    // edge o + j gets neighbour u (and, fused compaction K1, map[u] its position)
    auto emit = [&](int j, int32_t u) {
      out[j] = u;
      if (a.map && u >= 0 && u < a.map_nodes)
        atomicMin(a.map + u, tw | static_cast<unsigned long long>(static_cast<long long>(n_dst) + o + j));
    };
    if (!a.replace && k == d) {
      for (int j = lane; j < k; j += 32) emit(j, a.indices[beg + j]);
    } else if (a.replace) {
      for (int j = lane; j < k; j += 32) {
        const uint32_t off_j = a.fanout < 0 ? static_cast<uint32_t>(j)
                                            : draw_below(node_draw(key, static_cast<uint64_t>(v), j),
                                                         static_cast<uint32_t>(d));
        emit(j, a.indices[beg + off_j]);
      }
    } else {
      int32_t* acc = k <= kSmemAcc ? s_acc[w] : out;
      warp_pick_distinct(key, static_cast<uint64_t>(v), static_cast<uint32_t>(d), static_cast<uint32_t>(k), acc);
      for (int j = lane; j < k; j += 32) emit(j, a.indices[beg + acc[j]]);
      __syncwarp();
    }
  }
}

}  // namespace

void launch_sample_hop(const SampleHopArgs& a, int cap_dst, cudaStream_t stream) {
  const int tiles = static_cast<int>(ceil_div(cap_dst > 0 ? cap_dst : 1, kTileNodes));
  // no clearing of the scan scratch: its look-back words carry the launch number
  launch_k(sample_hop_kernel, tiles, kThreads, 0, stream, a);
  GB_LAUNCH_CHECK();
}

int sample_scan_scratch_words(int cap_dst) {
  return static_cast<int>(ceil_div(cap_dst > 0 ? cap_dst : 1, kTileNodes)) + 1;
}

}  // namespace dev
}  // namespace grappa

// ---------------------------------------------------------------------------------------
// Allocation-free entry point (declared and documented in sample_noalloc.h; it has no
// counterpart in the reference).  Same kernel as launch_sample_hop; the look-back scan
// scratch is the file-scope device array below instead of a caller-allocated buffer.
#include <mutex>

#include "sample_noalloc.h"

namespace {
constexpr int kNoAllocScratchWords = kGrappaNoAllocMaxDst / grappa::dev::kTileNodes + 1;  // tile statuses + ticket
constexpr int kNoAllocMaxDevices = 128;
std::mutex g_noalloc_mu;
unsigned long long* g_noalloc_dev_ptr[kNoAllocMaxDevices] = {};
}  // namespace

// The scratch: every GPU that loads this library holds these 128 KiB until exit.  In host
// code the name is only a stand-in; its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned long long g_noalloc_scan_scratch[kNoAllocScratchWords];

extern "C" __attribute__((visibility("default"))) int grappa_sample_hop_noalloc_max_dst(void) {
  return kGrappaNoAllocMaxDst;
}

extern "C" __attribute__((visibility("default"))) int grappa_sample_hop_noalloc(
    const int64_t* indptr, const int32_t* indices, int64_t n_graph_nodes, const int32_t* dst_nid, int32_t n_dst,
    const uint8_t* frontier, int32_t fanout, int32_t replace, const int64_t* counters, int32_t hop,
    const int64_t* gideg, float* cov_accum, int32_t* out_indptr, int32_t* out_nbr, int32_t cap_edges,
    int32_t* n_edges_out, int32_t* err, void* stream) {
  if (n_dst < 0 || n_dst > kGrappaNoAllocMaxDst) return GRAPPA_NOALLOC_TOO_MANY_DST;
  if (!indptr || !indices || (!dst_nid && n_dst > 0) || !counters || !out_indptr || !n_edges_out || n_graph_nodes < 0 ||
      cap_edges < 0 || (cap_edges > 0 && !out_nbr))
    return GRAPPA_NOALLOC_BAD_ARGUMENT;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return GRAPPA_NOALLOC_SETUP_FAILED;
  unsigned long long* scratch = nullptr;
  {
    // once per device, with that device current: the device address of the array
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_dev_ptr[dev]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scan_scratch) != cudaSuccess || p == nullptr)
        return GRAPPA_NOALLOC_SETUP_FAILED;
      g_noalloc_dev_ptr[dev] = static_cast<unsigned long long*>(p);
    }
    scratch = g_noalloc_dev_ptr[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int tiles = static_cast<int>(grappa::dev::ceil_div(n_dst > 0 ? n_dst : 1, grappa::dev::kTileNodes));
  // the array keeps the previous call's contents: the scan needs it zeroed
  if (cudaMemsetAsync(scratch, 0, sizeof(unsigned long long) * (tiles + 1), s) != cudaSuccess)
    return GRAPPA_NOALLOC_LAUNCH_FAILED;
  grappa::dev::SampleHopArgs a;
  a.indptr = indptr;
  a.indices = indices;
  a.n_graph_nodes = n_graph_nodes;
  a.dst_nid = dst_nid;
  a.n_dst_ptr = nullptr;
  a.n_dst = n_dst;
  a.frontier = frontier;
  a.fanout = fanout;
  a.replace = replace != 0;
  a.counters = counters;
  a.hop = hop;
  a.gideg = gideg;
  a.cov_accum = cov_accum;
  a.out_indptr = out_indptr;
  a.out_nbr = out_nbr;
  a.cap_edges = cap_edges;
  a.n_edges_out = n_edges_out;
  a.scan_scratch = scratch;
  a.err = err;
  grappa::dev::sample_hop_kernel<<<tiles, grappa::dev::kThreads, 0, s>>>(a);
  if (cudaGetLastError() != cudaSuccess) return GRAPPA_NOALLOC_LAUNCH_FAILED;
  return GRAPPA_NOALLOC_OK;
}
