// Shared device helpers for the sm_100a kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <utility>
#include <stdexcept>
#include <string>

#include "cuda_check.h"

namespace grappa {
namespace dev {

// Error bits a kernel sets in the device error word instead of trapping.
enum : int32_t {
  kErrScanTimeout = 1 << 0,    // a look-back wait ran out of iterations
  kErrCapacity = 1 << 1,       // an output did not fit its buffer; writes were dropped
  kErrBadIndex = 1 << 2,       // an index was outside its table
  kErrPeerTimeout = 1 << 3,    // a wait on a peer GPU's flag ran out of time
  kErrMmaTimeout = 1 << 4,     // a wait on a tensor-core/TMA barrier ran out of time
};

// Programmatic dependent launch (PDL).  A kernel launched by launch_k with PDL on may
// be scheduled while the previous kernel of its stream is finishing; GB_PDL_ENTRY(),
// the first statement of every kernel here, waits (griddepcontrol.wait) until the
// grids it depends on have completed and their writes are visible.  No kernel triggers
// its dependents early (griddepcontrol.launch_dependents at kernel entry measured
// slower: the waiting blocks took SM slots from the concurrent sampling stream), so
// the overlap is the launch latency at each grid's tail.  Without the launch
// attribute the wait is a no-op.
#define GB_PDL_ENTRY() asm volatile("griddepcontrol.wait;" ::: "memory")

// PDL launches unless GRAPPA_PDL=0 (read once per process).  Wait-only PDL measured
// 0.0399 against 0.0410 s/epoch on the GraphSAGE workload and 0.904 against 0.928 on
// GAT; triggering at kernel entry was slower than no PDL.
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("GRAPPA_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

// kernel<<<grid, block, smem, stream>>>(args...) with the programmatic-serialisation
// attribute (the kernel must start with GB_PDL_ENTRY()).
template <typename... KArgs, typename... Args>
inline void launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                     Args&&... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  GB_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

__device__ __forceinline__ void set_error(int32_t* err, int32_t bit) {
  if (err) atomicOr(err, bit);
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }
__device__ __forceinline__ uint32_t lanemask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

__device__ __forceinline__ void st_release_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

template <typename T>
__device__ __forceinline__ T warp_inclusive_scan(T v) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane_id() >= static_cast<uint32_t>(o)) v += n;
  }
  return v;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Block-wide exclusive scan of one value per thread; returns the exclusive
// prefix and writes the block total to *total.  smem needs kThreads/32 entries.
template <int kThreads, typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* smem, T* total) {
  constexpr int kWarps = kThreads / 32;
  const int w = threadIdx.x >> 5;
  T inc = warp_inclusive_scan(v);
  if (lane_id() == 31) smem[w] = inc;
  __syncthreads();
  if (w == 0) {
    T s = lane_id() < kWarps ? smem[lane_id()] : T(0);
    s = warp_inclusive_scan(s);
    if (lane_id() < kWarps) smem[lane_id()] = s;
  }
  __syncthreads();
  const T warp_prefix = w > 0 ? smem[w - 1] : T(0);
  *total = smem[kWarps - 1];
  __syncthreads();
  return warp_prefix + inc - v;
}

// Decoupled look-back (D. Merrill, M. Garland, "Single-pass Parallel Prefix Scan
// with Decoupled Look-back", NVIDIA TR NVR-2016-002).  scratch[0] is the tile
// ticket; scratch[1 + t] the status word of tile t: bits 63..62 = flag
// (1 aggregate, 2 inclusive prefix), bits 61..0 = value.  The caller zeroes the
// scratch before the launch.  Waits are bounded: after kSpinLimit polls the tile
// records kErrScanTimeout and proceeds with what it has.
// Decoupled look-back scan over the tiles of one launch.  scratch[0] is a ticket
// counter that is never reset: the CTAs of a launch take consecutive tickets (every CTA
// takes exactly one, and a launch starts after the previous one on its stream has
// finished), so ticket / gridDim.x numbers the launch and ticket % gridDim.x is the
// tile.  Tile t's status word scratch[1 + t] = flag (2 bits) | launch tag (30 bits) |
// value (32 bits); a word whose tag is not this launch's is not ready.  So the scratch
// needs no clearing between launches (no memset node in a captured step); clearing it
// (tag 0, flag 0) is also valid.  The same grid size must be used with one scratch.
struct LookBack {
  static constexpr unsigned long long kAgg = 1ull << 62;
  static constexpr unsigned long long kPre = 2ull << 62;
  static constexpr unsigned long long kTagMask = (1ull << 30) - 1;
  static constexpr unsigned long long kValMask = 0xFFFFFFFFull;
  static constexpr int kSpinLimit = 1 << 20;

  struct Ticket {
    int tile;
    unsigned long long tag;
  };

  // smem_slot: two ints of shared memory
  __device__ static Ticket ticket(unsigned long long* scratch, int* smem_slot) {
    if (threadIdx.x == 0) {
      const unsigned long long t = atomicAdd(scratch, 1ull);
      smem_slot[0] = static_cast<int>(t % gridDim.x);
      smem_slot[1] = static_cast<int>((t / gridDim.x) & kTagMask);
    }
    __syncthreads();
    return {smem_slot[0], static_cast<unsigned long long>(smem_slot[1])};
  }

  __device__ static unsigned long long word(unsigned long long flag, unsigned long long tag, long long v) {
    return flag | (tag << 32) | (static_cast<unsigned long long>(v) & kValMask);
  }

  // Called by all lanes of warp 0.  Returns the exclusive prefix of tile tk.tile (values
  // below 2^32).
  __device__ static long long exclusive_prefix(unsigned long long* scratch, Ticket tk, long long agg,
                                               int32_t* err) {
    unsigned long long* status = scratch + 1;
    const int t = tk.tile;
    if (t == 0) {
      if (lane_id() == 0) st_release_u64(status, word(kPre, tk.tag, agg));
      return 0;
    }
    if (lane_id() == 0) st_release_u64(status + t, word(kAgg, tk.tag, agg));
    long long prefix = 0;
    int j = t - 1;
    while (j >= 0) {
      const int idx = j - static_cast<int>(lane_id());
      unsigned long long s = kPre | (tk.tag << 32);  // lanes past tile 0 act as a zero prefix
      if (idx >= 0) {
        int spins = 0;
        s = ld_acquire_u64(status + idx);
        while ((s >> 62) == 0 || ((s >> 32) & kTagMask) != tk.tag) {
          if (++spins > kSpinLimit) {
            set_error(err, kErrScanTimeout);
            s = kPre | (tk.tag << 32);
            break;
          }
          if (spins > 64) __nanosleep(32);
          s = ld_acquire_u64(status + idx);
        }
      }
      const uint32_t pre_mask = __ballot_sync(0xffffffffu, (s >> 62) == 2);
      const int first_pre = pre_mask ? __ffs(pre_mask) - 1 : 32;  // nearest prefix lane
      long long v = (static_cast<int>(lane_id()) <= first_pre && idx >= 0) ? static_cast<long long>(s & kValMask) : 0;
      prefix += warp_sum(v);
      if (pre_mask) break;
      j -= 32;
    }
    if (lane_id() == 0) st_release_u64(status + t, word(kPre, tk.tag, prefix + agg));
    return prefix;
  }
};

// Tag word of one block compaction (compact.cu): derived on the device from the
// generation counter *gen and the hop slot, decreasing from call to call, so that a
// captured CUDA graph draws fresh tags on every replay.
__device__ __forceinline__ unsigned long long compact_tag_word(const int64_t* gen, int slot) {
  const uint32_t tag = 0xFFFFFFFFu - static_cast<uint32_t>(static_cast<uint64_t>(*gen) * 16u + static_cast<uint32_t>(slot));
  return static_cast<unsigned long long>(tag) << 32;
}

// bf16x8 <-> float helpers for 16-byte vector access.
__device__ __forceinline__ void bf16x8_to_f32(const uint4& u, float* f) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ uint4 f32_to_bf16x8(const float* f) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

__host__ __device__ __forceinline__ int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace dev
}  // namespace grappa
