// Peer-memory kernels (see peer.h): repartition pulls (pull_rows, csr_merge,
// mark / mark_compact), the pull all-to-all and the device barrier.  Every remote
// access is an ordinary 16-byte ld/st.global through an IPC mapping; waits are
// bounded by a %globaltimer deadline and report kErrPeerTimeout.
#include "common.cuh"
#include "peer.h"

#include <algorithm>

namespace grappa {
namespace peer {

using dev::ceil_div;

void* alloc(int64_t bytes) {
  void* p = nullptr;
  GB_CUDA_CHECK(cudaMalloc(&p, static_cast<size_t>(bytes > 0 ? bytes : 16)));
  GB_CUDA_CHECK(cudaMemset(p, 0, static_cast<size_t>(bytes > 0 ? bytes : 16)));
  return p;
}
void release(void* p) {
  if (p) GB_CUDA_CHECK(cudaFree(p));
}
std::string ipc_handle(void* p) {
  cudaIpcMemHandle_t h;
  GB_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}
void* ipc_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::invalid_argument("bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::copy(handle.begin(), handle.end(), reinterpret_cast<char*>(&h));
  void* p = nullptr;
  GB_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}
void ipc_close(void* p) {
  if (p) GB_CUDA_CHECK(cudaIpcCloseMemHandle(p));
}

namespace {

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// ---------------------------------------------------------------- repartition
// Rows of up to 2 KB: a row takes 8, 16 or 32 lanes (each up to four 16-byte chunks),
// a warp moves 32 / lanes rows per step and four steps' rows are loaded before the
// first store, so that many peer reads are in flight per warp (a halo pull is a few
// hundred thousand random rows, bound by the round trip of each).
constexpr int kPullUnroll = 4;
__global__ void pull_rows_kernel(PullRowsArgs a) {
  int64_t n = a.n_ptr ? *a.n_ptr : a.n;
  if (n > a.cap) {
    if (blockIdx.x == 0 && threadIdx.x == 0) dev::set_error(a.err, dev::kErrCapacity);
    n = a.cap;
  }
  const int lane = threadIdx.x & 31;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int chunks = a.row_bytes >> 4;
  const int lpr = chunks <= 8 ? 8 : (chunks <= 16 ? 16 : 32);
  const int rpw = 32 / lpr;
  const int sub = lane % lpr, slot = lane / lpr;
  const int64_t g_lo = a.prefix[0], g_hi = a.prefix[a.world];
  const int64_t per_step = static_cast<int64_t>(rpw) * kPullUnroll;
  for (int64_t r0 = wid * per_step; r0 < n; r0 += warps * per_step) {
    const uint4* src[kPullUnroll];
    uint4* dst[kPullUnroll];
#pragma unroll
    for (int u = 0; u < kPullUnroll; ++u) {
      const int64_t r = r0 + u * rpw + slot;
      src[u] = nullptr;
      dst[u] = nullptr;
      if (r >= n) continue;
      const int64_t g = a.gids[r];
      if (g < g_lo || g >= g_hi) {
        if (sub == 0) dev::set_error(a.err, dev::kErrBadIndex);
        continue;
      }
      int p = 0;
      while (p + 1 < a.world && g >= a.prefix[p + 1]) ++p;
      src[u] = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(a.tables[p]) +
                                              (g - a.prefix[p]) * a.table_stride * a.elem_bytes);
      dst[u] = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(a.out) + (a.out_row0 + r) * a.out_stride * a.elem_bytes);
    }
    uint4 v[kPullUnroll][4];
#pragma unroll
    for (int u = 0; u < kPullUnroll; ++u)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = sub + k * lpr;
        if (src[u] && c < chunks) v[u][k] = src[u][c];
      }
#pragma unroll
    for (int u = 0; u < kPullUnroll; ++u)
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = sub + k * lpr;
        if (dst[u] && c < chunks) dst[u][c] = v[u][k];
      }
  }
}

// rows wider than 2 KB: one warp per row
__global__ void pull_rows_wide_kernel(PullRowsArgs a) {
  int64_t n = a.n_ptr ? *a.n_ptr : a.n;
  if (n > a.cap) {
    if (blockIdx.x == 0 && threadIdx.x == 0) dev::set_error(a.err, dev::kErrCapacity);
    n = a.cap;
  }
  const int lane = threadIdx.x & 31;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int chunks = a.row_bytes >> 4;
  const int64_t g_lo = a.prefix[0], g_hi = a.prefix[a.world];
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; r < n; r += warps) {
    const int64_t g = a.gids[r];
    if (g < g_lo || g >= g_hi) {
      if (lane == 0) dev::set_error(a.err, dev::kErrBadIndex);
      continue;
    }
    int p = 0;
    while (p + 1 < a.world && g >= a.prefix[p + 1]) ++p;
    const int64_t row = g - a.prefix[p];
    const uint8_t* src = reinterpret_cast<const uint8_t*>(a.tables[p]) + row * a.table_stride * a.elem_bytes;
    uint8_t* dst = reinterpret_cast<uint8_t*>(a.out) + (a.out_row0 + r) * a.out_stride * a.elem_bytes;
    for (int c = lane; c < chunks; c += 32)
      reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
  }
}

// four independent 16-byte loads in flight per thread (peer sources: the NVLink round
// trip is hidden by the loads in flight, not by the grid size)
__global__ void copy_kernel(uint4* dst, const uint4* src, int64_t n16) {
  constexpr int kU = 4;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n16; i += kU * stride) {
    uint4 v[kU];
#pragma unroll
    for (int k = 0; k < kU; ++k)
      if (i + k * stride < n16) v[k] = src[i + k * stride];
#pragma unroll
    for (int k = 0; k < kU; ++k)
      if (i + k * stride < n16) dst[i + k * stride] = v[k];
  }
}

// Each thread moves 8 independent 16-byte words per iteration (8 P2P loads in flight)
// so that the NVLink round trips are hidden without a large grid.
__global__ void a2a_pull_kernel(A2aArgs a) {
  constexpr int kUnroll = 8;
  // segments in pull order: peer (first + j) % world is the j-th
  int64_t pre[kMaxRanks + 1];
  int seg[kMaxRanks];
  pre[0] = 0;
  for (int j = 0; j < a.world; ++j) {
    seg[j] = (a.first + j) % a.world;
    pre[j + 1] = pre[j] + (a.len[seg[j]] >> 4);
  }
  const int64_t total = pre[a.world];
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; base < total;
       base += stride * kUnroll) {
    uint4 v[kUnroll];
    uint4* d[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      d[u] = nullptr;
      if (i < total) {
        int j = 0;
        while (i >= pre[j + 1]) ++j;
        const int64_t k = i - pre[j];
        const int p = seg[j];
        v[u] = reinterpret_cast<const uint4*>(a.src[p] + a.src_off[p])[k];
        d[u] = reinterpret_cast<uint4*>(a.dst + a.dst_off[p]) + k;
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u)
      if (d[u]) *d[u] = v[u];
  }
}

struct BarrierArgs {
  uint32_t* flags_local;
  uint32_t* flags_peer[kMaxRanks];
  int64_t* epoch;
  int64_t timeout_ns;
  int32_t* err;
  int32_t rank, world;
};

__global__ void peer_barrier_kernel(BarrierArgs a) {
  const uint32_t tag = static_cast<uint32_t>(*a.epoch + 1);
  const int p = threadIdx.x;
  if (p < a.world) st_release_sys(a.flags_peer[p] + a.rank, tag);
  __syncthreads();
  if (p < a.world) {
    const uint32_t* f = a.flags_local + p;
    const uint64_t t0 = dev::globaltimer_ns();
    uint32_t polls = 0;
    while (static_cast<int32_t>(ld_acquire_sys(f) - tag) < 0) {
      if ((++polls & 63u) == 0) {
        if (dev::globaltimer_ns() - t0 > static_cast<uint64_t>(a.timeout_ns)) {
          dev::set_error(a.err, dev::kErrPeerTimeout);
          break;
        }
        __nanosleep(64);
      }
    }
  }
  __syncthreads();
  if (p == 0) *a.epoch = tag;
}

__global__ void mark_kernel(const int32_t* ids, const int32_t* n_ptr, int64_t n_static, uint8_t* mark) {
  const int64_t n = n_ptr ? *n_ptr : n_static;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    mark[ids[i]] = 1;
}

__global__ void iota_map_kernel(int32_t* map, int64_t g0, int64_t count, int32_t base, uint8_t* clear_mark) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    map[g0 + i] = base + static_cast<int32_t>(i);
    if (clear_mark) clear_mark[g0 + i] = 0;
  }
}

constexpr int kMcThreads = 256;
constexpr int kMcItems = 16;
constexpr int kMcTile = kMcThreads * kMcItems;

__global__ void __launch_bounds__(kMcThreads) mark_compact_kernel(uint8_t* mark, int64_t n_global, int64_t* out_ids,
                                                                   int32_t* map, int32_t base, int32_t* n_out,
                                                                   unsigned long long* scratch, int64_t cap_out,
                                                                   int32_t* err) {
  __shared__ long long s_scan[kMcThreads / 32];
  __shared__ int s_tile[2];
  __shared__ long long s_prefix;
  const dev::LookBack::Ticket tk = dev::LookBack::ticket(scratch, s_tile);
  const int tile = tk.tile;
  const int64_t g0 = static_cast<int64_t>(tile) * kMcTile + threadIdx.x * kMcItems;
  // the thread's 16 mark bytes as one 16-byte load (byte loads for the ragged tail)
  uint32_t bits = 0;
  if (g0 + kMcItems <= n_global) {
    const uint4 w = *reinterpret_cast<const uint4*>(mark + g0);
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int q = 0; q < kMcItems; ++q)
      if ((words[q >> 2] >> (8 * (q & 3))) & 0xFFu) bits |= 1u << q;
  } else {
    for (int q = 0; q < kMcItems; ++q)
      if (g0 + q < n_global && mark[g0 + q]) bits |= 1u << q;
  }
  const int cnt = __popc(bits);
  long long total;
  const long long excl = dev::block_exclusive_scan<kMcThreads, long long>(cnt, s_scan, &total);
  if ((threadIdx.x >> 5) == 0) {
    const long long p = dev::LookBack::exclusive_prefix(scratch, tk, total, err);
    if (dev::lane_id() == 0) s_prefix = p;
  }
  __syncthreads();
  long long k = s_prefix + excl;
  if (bits) {  // clear the marks for the next repartition
    if (g0 + kMcItems <= n_global) *reinterpret_cast<uint4*>(mark + g0) = make_uint4(0, 0, 0, 0);
    else
      for (int q = 0; q < kMcItems; ++q)
        if (g0 + q < n_global) mark[g0 + q] = 0;
  }
#pragma unroll
  for (int q = 0; q < kMcItems; ++q) {
    if (!(bits & (1u << q))) continue;
    const int64_t g = g0 + q;
    if (k < cap_out) {
      out_ids[k] = g;
      map[g] = base + static_cast<int32_t>(k);
    } else {
      dev::set_error(err, dev::kErrCapacity);
    }
    ++k;
  }
  const int64_t last = n_global > 0 ? (n_global - 1) / kMcTile : 0;
  if (tile == last && threadIdx.x == 0) {
    const long long tot = s_prefix + total;
    *n_out = static_cast<int32_t>(tot < cap_out ? tot : cap_out);
  }
}

// out[e] = map[src[e]] for e < n: the source (peer memory) read as 16-byte words, two
// in flight per thread, after a scalar head up to the first 16-byte boundary; the
// translated values are stored as single words (local memory, any alignment)
// working id of global id g: the two partitions' ranges arithmetically, the rest
// (halo sources) through the map
struct Translate {
  const int32_t* map;
  int64_t g0_a, n_a, g0_b, n_b;
  __device__ __forceinline__ int32_t operator[](int32_t g) const {
    const int64_t da = static_cast<int64_t>(g) - g0_a, db = static_cast<int64_t>(g) - g0_b;
    if (g0_a >= 0 && da >= 0 && da < n_a) return static_cast<int32_t>(da);
    if (g0_b >= 0 && db >= 0 && db < n_b) return static_cast<int32_t>(n_a + db);
    return map[g];
  }
};

__device__ __forceinline__ void merge_segment(const int32_t* src, int64_t n, int32_t* out, const Translate map,
                                              int64_t tid, int64_t stride) {
  if (n <= 0) return;
  const int64_t mis = static_cast<int64_t>((reinterpret_cast<uintptr_t>(src) >> 2) & 3);
  const int64_t head = mis ? (4 - mis < n ? 4 - mis : n) : 0;
  if (tid < head) out[tid] = map[src[tid]];
  const int4* s4 = reinterpret_cast<const int4*>(src + head);
  int32_t* o = out + head;
  const int64_t n4 = (n - head) >> 2;
  for (int64_t i = tid; i < n4; i += 2 * stride) {
    const bool two = i + stride < n4;
    const int4 x = s4[i];
    int4 y = make_int4(0, 0, 0, 0);
    if (two) y = s4[i + stride];
    int32_t* p = o + 4 * i;
    p[0] = map[x.x]; p[1] = map[x.y]; p[2] = map[x.z]; p[3] = map[x.w];
    if (two) {
      int32_t* q = o + 4 * (i + stride);
      q[0] = map[y.x]; q[1] = map[y.y]; q[2] = map[y.z]; q[3] = map[y.w];
    }
  }
  const int64_t t0 = head + 4 * n4;
  if (tid < n - t0) out[t0 + tid] = map[src[t0 + tid]];
}

__global__ void csr_merge_kernel(CsrMergeArgs a) {
  const int64_t ea0 = a.indptr_a[0], ea = a.indptr_a[a.n_a] - ea0;
  const int64_t eb0 = a.n_b > 0 ? a.indptr_b[0] : 0;
  const int64_t eb = a.n_b > 0 ? a.indptr_b[a.n_b] - eb0 : 0;
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (tid == 0 && ea + eb > a.cap_edges) dev::set_error(a.err, dev::kErrCapacity);
  for (int64_t v = tid; v <= a.n_rows_total; v += stride) {
    int64_t o;
    if (v <= a.n_a) o = a.indptr_a[v] - ea0;
    else if (v <= a.n_a + a.n_b) o = ea + (a.indptr_b[v - a.n_a] - eb0);
    else o = ea + eb;
    a.indptr_out[v] = o < a.cap_edges ? o : a.cap_edges;
  }
  const int64_t na = ea < a.cap_edges ? ea : a.cap_edges;
  const int64_t nb = ea + eb < a.cap_edges ? eb : a.cap_edges - na;
  const Translate tr{a.map, a.g0_a, a.n_a, a.g0_b, a.n_b};
  merge_segment(a.indices_a + ea0, na, a.indices_out, tr, tid, stride);
  merge_segment(a.indices_b + eb0, nb, a.indices_out + na, tr, tid, stride);
}

int sm_count() {
  static int s = 0;
  if (!s) {
    int d = 0;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&s, cudaDevAttrMultiProcessorCount, d);
    if (s <= 0) s = 148;
  }
  return s;
}

int grid_for(int64_t n, int threads, int per_sm = 8) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n > 0 ? n : 1, threads), int64_t(sm_count()) * per_sm)));
}

}  // namespace

void launch_pull_rows(const PullRowsArgs& a_in, int64_t cap, cudaStream_t stream) {
  if (a_in.world < 1 || a_in.world > kMaxRanks) throw std::invalid_argument("pull_rows: world out of range");
  if (a_in.row_bytes % 16 != 0) throw std::invalid_argument("pull_rows: row bytes must be a multiple of 16");
  if (cap < 0) throw std::invalid_argument("pull_rows: negative capacity");
  if (!a_in.n_ptr && a_in.n > cap) throw std::invalid_argument("pull_rows: more rows than the output holds");
  PullRowsArgs a = a_in;
  a.cap = cap;
  if (cap == 0) return;
  if (a.row_bytes <= 2048) {
    const int chunks = a.row_bytes / 16;
    const int rows_per_warp = 32 / (chunks <= 8 ? 8 : (chunks <= 16 ? 16 : 32));
    pull_rows_kernel<<<grid_for(ceil_div(cap, static_cast<int64_t>(rows_per_warp) * kPullUnroll) * 32, 256, 16), 256, 0,
                       stream>>>(a);
  } else {
    pull_rows_wide_kernel<<<grid_for(cap * 32, 256, 16), 256, 0, stream>>>(a);
  }
  GB_LAUNCH_CHECK();
}

void launch_copy(void* dst, const void* src, int64_t bytes, cudaStream_t stream) {
  if (bytes % 16 != 0) throw std::invalid_argument("copy: bytes must be a multiple of 16");
  const int64_t n16 = bytes / 16;
  if (n16 == 0) return;
  copy_kernel<<<grid_for(n16, 256, 16), 256, 0, stream>>>(reinterpret_cast<uint4*>(dst), reinterpret_cast<const uint4*>(src), n16);
  GB_LAUNCH_CHECK();
}

void launch_a2a_pull(const A2aArgs& a, cudaStream_t stream) {
  if (a.world < 1 || a.world > kMaxRanks) throw std::invalid_argument("a2a: world out of range");
  int64_t total = 0;
  for (int p = 0; p < a.world; ++p) {
    if ((a.len[p] | a.src_off[p] | a.dst_off[p]) & 15) throw std::invalid_argument("a2a: 16-byte alignment");
    total += a.len[p] >> 4;
  }
  if (total == 0) return;
  a2a_pull_kernel<<<grid_for(ceil_div(total, 8), 256, 8), 256, 0, stream>>>(a);
  GB_LAUNCH_CHECK();
}

void launch_peer_barrier(int32_t rank, int32_t world, uint32_t* flags_local, uint32_t* const* flags_peer,
                         int64_t* epoch, int64_t timeout_ns, int32_t* err, cudaStream_t stream) {
  if (world < 1 || world > kMaxRanks) throw std::invalid_argument("barrier: world out of range");
  BarrierArgs a;
  a.flags_local = flags_local;
  for (int p = 0; p < world; ++p) a.flags_peer[p] = flags_peer[p];
  a.epoch = epoch;
  a.timeout_ns = timeout_ns;
  a.err = err;
  a.rank = rank;
  a.world = world;
  peer_barrier_kernel<<<1, 32, 0, stream>>>(a);
  GB_LAUNCH_CHECK();
}

void launch_mark(const int32_t* ids, const int32_t* n_ptr, int64_t n, uint8_t* mark, cudaStream_t stream) {
  if (n <= 0 && !n_ptr) return;
  mark_kernel<<<grid_for(n, 256), 256, 0, stream>>>(ids, n_ptr, n, mark);
  GB_LAUNCH_CHECK();
}

void launch_iota_map(int32_t* map, int64_t g0, int64_t count, int32_t base, uint8_t* clear_mark, cudaStream_t stream) {
  if (count <= 0) return;
  iota_map_kernel<<<grid_for(count, 256), 256, 0, stream>>>(map, g0, count, base, clear_mark);
  GB_LAUNCH_CHECK();
}

int64_t mark_compact_scratch_words(int64_t n_global) { return ceil_div(n_global > 0 ? n_global : 1, kMcTile) + 1; }

void launch_mark_compact(uint8_t* mark, int64_t n_global, int64_t* out_ids, int32_t* map, int32_t base, int32_t* n_out,
                         unsigned long long* scan_scratch, int64_t cap_out, int32_t* err, cudaStream_t stream) {
  const int64_t tiles = ceil_div(n_global > 0 ? n_global : 1, kMcTile);
  GB_CUDA_CHECK(cudaMemsetAsync(scan_scratch, 0, sizeof(unsigned long long) * (tiles + 1), stream));
  mark_compact_kernel<<<static_cast<unsigned>(tiles), kMcThreads, 0, stream>>>(mark, n_global, out_ids, map, base, n_out,
                                                                             scan_scratch, cap_out, err);
  GB_LAUNCH_CHECK();
}

void launch_csr_merge(const CsrMergeArgs& a, cudaStream_t stream) {
  csr_merge_kernel<<<grid_for(std::max<int64_t>(a.cap_edges, a.n_rows_total + 1), 256, 16), 256, 0, stream>>>(a);
  GB_LAUNCH_CHECK();
}

}  // namespace peer
}  // namespace grappa
