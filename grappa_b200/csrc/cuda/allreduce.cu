// K-AR kernels: coverage-weighted gradient all-reduce fused with Adam (see allreduce.h).
//
// Memory ordering.  A rank signals "my data is ready" with a release pattern: after
// __syncthreads(), thread 0 runs fence.acq_rel.sys and stores the tag into every
// reader's flag word with st.relaxed.sys; the reader polls with ld.acquire.sys (one
// thread per flag), then __syncthreads() orders the CTA's loads after the acquire.  Gradients written by earlier kernels of the stream are
// complete when the kernel starts.
//
// Buffer reuse.  kShard: rank r clears piece j of shard s of its gradient only after
// it has seen owner s's "done" flag for piece j (s read it before raising the flag);
// its master weights of shard r are rewritten at step t+1 only after every peer's
// "ready" flag of step t+1, which a peer raises only after its step-t kernel (whose
// all-gather read shard r) has finished.  kOneShot: the send slots alternate with the
// step parity; a rank publishes step t+2 only after every peer published step t+1,
// which each peer does only after it finished reading step t.  The published scales
// c_r/W alternate the same way.
#include "allreduce.h"
#include "common.cuh"

#include <algorithm>

namespace grappa {
namespace ar {
namespace {

using dev::ceil_div;

constexpr int kThreads = 512;
constexpr int kU = 4;  // 16-byte vectors per thread in flight per peer

// A release pattern: one fence.acq_rel.sys, then a relaxed system-scope store per
// reader.  (A st.release per reader would fence once per store; each fence waits for
// the previous remote store to be acknowledged over NVLink.)
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ld_relaxed_sys_f32(const float* p) {
  float v;
  asm volatile("ld.relaxed.sys.global.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until *f reaches tag (wrap-safe); false (and kErrPeerTimeout) on expiry.
__device__ bool wait_tag(const uint32_t* f, uint32_t tag, int64_t timeout_ns, int32_t* err) {
  if (static_cast<int32_t>(ld_acquire_sys(f) - tag) >= 0) return true;
  const uint64_t t0 = dev::globaltimer_ns();
  uint32_t polls = 0;
  while (static_cast<int32_t>(ld_acquire_sys(f) - tag) < 0) {
    if ((++polls & 63u) == 0) {
      if (dev::globaltimer_ns() - t0 > static_cast<uint64_t>(timeout_ns)) {
        dev::set_error(err, dev::kErrPeerTimeout);
        return false;
      }
      __nanosleep(32);
    }
  }
  return true;
}

__device__ __forceinline__ uint32_t* ready_flag(uint32_t* page, int rank, int cta) {
  return page + rank * kMaxCtas + cta;
}
__device__ __forceinline__ uint32_t* done_flag(uint32_t* page, int rank, int cta) {
  return page + kMaxRanks * kMaxCtas + rank * kMaxCtas + cta;
}

struct AdamK {
  float b1, b2, eps, wd, step_size, inv_sqrt_bc2;
};

__device__ __forceinline__ AdamK adam_constants(const Args& a) {
  const float t = static_cast<float>(a.counters[5] + 1);
  AdamK k;
  k.b1 = a.beta1;
  k.b2 = a.beta2;
  k.eps = a.eps;
  k.wd = a.weight_decay;
  k.step_size = a.lr / (1.f - powf(a.beta1, t));
  k.inv_sqrt_bc2 = rsqrtf(1.f - powf(a.beta2, t));
  return k;
}

__device__ __forceinline__ float adam1(const AdamK& k, float g, float& p, float& m, float& v) {
  if (k.wd != 0.f) g += k.wd * p;
  m = k.b1 * m + (1.f - k.b1) * g;
  v = k.b2 * v + (1.f - k.b2) * g * g;
  p -= k.step_size * m / (sqrtf(v) * k.inv_sqrt_bc2 + k.eps);
  return p;
}

// Adam over 4 consecutive elements at i (16-byte aligned): fp32 master, moments, bf16 copy.
__device__ __forceinline__ void adam4(const Args& a, const AdamK& k, int64_t i, const float* g) {
  float4 p = *reinterpret_cast<const float4*>(a.param + i);
  float4 m = *reinterpret_cast<const float4*>(a.m + i);
  float4 v = *reinterpret_cast<const float4*>(a.v + i);
  adam1(k, g[0], p.x, m.x, v.x);
  adam1(k, g[1], p.y, m.y, v.y);
  adam1(k, g[2], p.z, m.z, v.z);
  adam1(k, g[3], p.w, m.w, v.w);
  *reinterpret_cast<float4*>(a.param + i) = p;
  *reinterpret_cast<float4*>(a.m + i) = m;
  *reinterpret_cast<float4*>(a.v + i) = v;
  if (a.wbf) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(p.x, p.y), hi = __floats2bfloat162_rn(p.z, p.w);
    uint2 w;
    w.x = *reinterpret_cast<uint32_t*>(&lo);
    w.y = *reinterpret_cast<uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(a.wbf + i) = w;
  }
}

__device__ __forceinline__ void finish_scalar(const Args& a, const AdamK& k, int64_t i, float g) {
  if (!a.do_adam) {
    a.grad_out[i] = g;
    return;
  }
  float p = a.param[i], m = a.m[i], v = a.v[i];
  adam1(k, g, p, m, v);
  a.param[i] = p;
  a.m[i] = m;
  a.v[i] = v;
  if (a.wbf) a.wbf[i] = __float2bfloat16_rn(p);
}

// VE gradient elements (one 16-byte vector) at element i of a gradient buffer.
template <bool kBf16>
struct GradVec {
  static constexpr int VE = kBf16 ? 8 : 4;
  __device__ __forceinline__ static void load(const void* base, int64_t i, float* x) {
    if constexpr (kBf16) {
      const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(base) + i);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(h[q]);
        x[2 * q] = f.x;
        x[2 * q + 1] = f.y;
      }
    } else {
      const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + i);
      x[0] = f.x;
      x[1] = f.y;
      x[2] = f.z;
      x[3] = f.w;
    }
  }
  __device__ __forceinline__ static float load1(const void* base, int64_t i) {
    if constexpr (kBf16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
    else return reinterpret_cast<const float*>(base)[i];
  }
  __device__ __forceinline__ static void clear(void* base, int64_t i) {
    if constexpr (kBf16) *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(base) + i) = make_uint4(0, 0, 0, 0);
    else *reinterpret_cast<float4*>(reinterpret_cast<float*>(base) + i) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __device__ __forceinline__ static void clear1(void* base, int64_t i) {
    if constexpr (kBf16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(0.f);
    else reinterpret_cast<float*>(base)[i] = 0.f;
  }
};

// Element range [b, e) of piece j of shard s: shards of S elements from lo, pieces of P.
__device__ __forceinline__ void piece_range(const Args& a, int s, int j, int64_t S, int64_t P, int64_t& b,
                                            int64_t& e) {
  const int64_t s0 = min(a.hi, a.lo + static_cast<int64_t>(s) * S);
  const int64_t s1 = min(a.hi, s0 + S);
  b = min(s1, s0 + static_cast<int64_t>(j) * P);
  e = min(s1, b + P);
}

__device__ __forceinline__ float my_scale(const Args& a) {
  float scale = 1.f / static_cast<float>(a.world);
  if (a.cov) {
    const float cn = a.cov[1];
    scale = (cn > 0.f ? a.cov[0] / cn : 0.f) / static_cast<float>(a.world);
  }
  return scale;
}

template <typename G>
__device__ __forceinline__ void clear_range(void* grad, int64_t b, int64_t e) {
  constexpr int VE = G::VE;
  for (int64_t i = b + static_cast<int64_t>(threadIdx.x) * VE; i < e; i += static_cast<int64_t>(kThreads) * VE) {
    if (i + VE <= e) G::clear(grad, i);
    else
      for (int64_t q = i; q < e; ++q) G::clear1(grad, q);
  }
}

// ------------------------------------------------------------------ kShard
template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1) ar_shard_kernel(Args a) {
  using G = GradVec<kBf16>;
  constexpr int VE = G::VE;
  const int j = blockIdx.x, nj = gridDim.x;
  const int W = a.world, r = a.rank;
  const int64_t step = a.counters[3];
  const uint32_t tag = static_cast<uint32_t>(step + 1);
  const int par = static_cast<int>(step & 1);
  const AdamK k = adam_constants(a);
  const int64_t S = (ceil_div(a.hi - a.lo, static_cast<int64_t>(W)) + 7) / 8 * 8;
  const int64_t P = (ceil_div(S, static_cast<int64_t>(nj)) + 7) / 8 * 8;
  __shared__ float s_w[kMaxRanks];
  __shared__ int s_fail;
  __shared__ const float* s_param[kMaxRanks];
  __shared__ const float* s_scale[kMaxRanks];
  __shared__ const void* s_grad[kMaxRanks];
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p)
    if (threadIdx.x == p) {
      s_param[p] = p < W ? a.param_peer[p] : nullptr;
      s_scale[p] = p < W ? a.scale_peer[p] : nullptr;
      s_grad[p] = p < W ? a.grad_peer[p] : nullptr;
    }

  // 1. this CTA's part of the gradient is ready on this rank: publish the scale, flag
  //    every owner (owner s reads piece j of shard s from here)
  if (threadIdx.x == 0) {
    s_fail = 0;
    a.scale_local[par] = my_scale(a);
    fence_acq_rel_sys();
    for (int p = 0; p < W; ++p) st_relaxed_sys(ready_flag(a.flags_peer[p], r, j), tag);
  }
  __syncthreads();
  // 2. wait until every rank's piece j of shard r is ready; read the ranks' scales
  if (threadIdx.x < W) {
    if (wait_tag(ready_flag(a.flags_local, threadIdx.x, j), tag, a.timeout_ns, a.err))
      s_w[threadIdx.x] = ld_relaxed_sys_f32(s_scale[threadIdx.x] + par);
    else
      s_fail = 1;
  }
  __syncthreads();
  if (s_fail) return;
  float w[kMaxRanks];
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p) w[p] = p < W ? s_w[p] : 0.f;

  // 3. reduce-scatter of piece j of the own shard (rank order: every owner computes the
  //    same sum the one-shot path would), Adam on it
  int64_t b, e;
  piece_range(a, r, j, S, P, b, e);
  const int64_t vstride = static_cast<int64_t>(kThreads) * VE;
  for (int64_t base = b + static_cast<int64_t>(threadIdx.x) * VE; base < e; base += vstride * kU) {
    float acc[kU][VE];
#pragma unroll
    for (int u = 0; u < kU; ++u)
#pragma unroll
      for (int q = 0; q < VE; ++q) acc[u][q] = 0.f;
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) {
      if (p >= W) break;
      float x[kU][VE];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = base + u * vstride;
        if (i + VE <= e) G::load(a.grad_peer[p], i, x[u]);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = base + u * vstride;
        if (i + VE <= e)
#pragma unroll
          for (int q = 0; q < VE; ++q) acc[u][q] += w[p] * x[u][q];
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * vstride;
      if (i + VE <= e) {
#pragma unroll
        for (int q = 0; q < VE; q += 4) adam4(a, k, i + q, &acc[u][q]);
      } else if (i < e) {
        for (int64_t q = i; q < e; ++q) {
          float s1 = 0.f;
          for (int p = 0; p < W; ++p) s1 += s_w[p] * G::load1(s_grad[p], q);
          finish_scalar(a, k, q, s1);
        }
      }
    }
  }
  // 4. piece j of shard r is updated: flag every other rank
  __syncthreads();
  if (threadIdx.x == 0) {
    fence_acq_rel_sys();
    for (int p = 0; p < W; ++p)
      if (p != r) st_relaxed_sys(done_flag(a.flags_peer[p], r, j), tag);
  }
  // 5. all-gather: piece j of every other shard from its owner (rotated start, so that
  //    the ranks read different owners at any one time)
  for (int d = 1; d < W; ++d) {
    const int s = (r + d) % W;
    if (threadIdx.x == 0 && !wait_tag(done_flag(a.flags_local, s, j), tag, a.timeout_ns, a.err)) s_fail = 1;
    __syncthreads();
    if (s_fail) return;
    piece_range(a, s, j, S, P, b, e);
    const float* src = s_param[s];
    const int64_t fstride = static_cast<int64_t>(kThreads) * 4;
    for (int64_t base = b + static_cast<int64_t>(threadIdx.x) * 4; base < e; base += fstride * kU) {
      float4 x[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = base + u * fstride;
        if (i + 4 <= e) x[u] = *reinterpret_cast<const float4*>(src + i);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = base + u * fstride;
        if (i + 4 <= e) {
          *reinterpret_cast<float4*>(a.param + i) = x[u];
          if (a.wbf) {
            __nv_bfloat162 lo = __floats2bfloat162_rn(x[u].x, x[u].y), hi = __floats2bfloat162_rn(x[u].z, x[u].w);
            uint2 wv;
            wv.x = *reinterpret_cast<uint32_t*>(&lo);
            wv.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(a.wbf + i) = wv;
          }
        } else if (i < e) {
          for (int64_t q = i; q < e; ++q) {
            const float pv = src[q];
            a.param[q] = pv;
            if (a.wbf) a.wbf[q] = __float2bfloat16_rn(pv);
          }
        }
      }
    }
  }
  // 6. every owner has read its piece j of this rank's gradient: clear them
  for (int s = 0; s < W; ++s) {
    piece_range(a, s, j, S, P, b, e);
    clear_range<G>(a.grad, b, e);
  }
}

// ------------------------------------------------------------------ kOneShot
template <bool kBf16>
__global__ void __launch_bounds__(kThreads, 1) ar_oneshot_kernel(Args a) {
  using G = GradVec<kBf16>;
  constexpr int VE = G::VE;
  const int j = blockIdx.x, nj = gridDim.x;
  const int W = a.world, r = a.rank;
  const int64_t step = a.counters[3];
  const uint32_t tag = static_cast<uint32_t>(step + 1);
  const int par = static_cast<int>(step & 1);
  const AdamK k = adam_constants(a);
  const int64_t P = (ceil_div(a.hi - a.lo, static_cast<int64_t>(nj)) + 7) / 8 * 8;
  const int64_t b = min(a.hi, a.lo + static_cast<int64_t>(j) * P);
  const int64_t e = min(a.hi, b + P);
  const float scale = my_scale(a);
  float* send = par ? a.slot_local[1] : a.slot_local[0];
  __shared__ int s_fail;
  __shared__ const float* s_src[kMaxRanks];
  if (threadIdx.x < kMaxRanks) s_src[threadIdx.x] = nullptr;
#pragma unroll
  for (int p = 0; p < kMaxRanks; ++p)
    if (threadIdx.x == p && p < W) s_src[p] = par ? a.slot_peer[p][1] : a.slot_peer[p][0];

  // 1. publish piece j: send = grad * c_r / W (fp32), grad = 0
  const int64_t vstride = static_cast<int64_t>(kThreads) * VE;
  for (int64_t i = b + static_cast<int64_t>(threadIdx.x) * VE; i < e; i += vstride) {
    if (i + VE <= e) {
      float x[VE];
      G::load(a.grad, i, x);
      G::clear(a.grad, i);
#pragma unroll
      for (int q = 0; q < VE; q += 4)
        *reinterpret_cast<float4*>(send + i + q) =
            make_float4(x[q] * scale, x[q + 1] * scale, x[q + 2] * scale, x[q + 3] * scale);
    } else {
      for (int64_t q = i; q < e; ++q) {
        send[q] = G::load1(a.grad, q) * scale;
        G::clear1(a.grad, q);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    s_fail = 0;
    fence_acq_rel_sys();
    for (int p = 0; p < W; ++p) st_relaxed_sys(done_flag(a.flags_peer[p], r, j), tag);
  }
  __syncthreads();
  // 2. wait for every rank's piece j
  if (threadIdx.x < W && !wait_tag(done_flag(a.flags_local, threadIdx.x, j), tag, a.timeout_ns, a.err)) s_fail = 1;
  __syncthreads();
  if (s_fail) return;
  // 3. sum the W copies in rank order (bit-identical on every rank), Adam
  const int64_t fstride = static_cast<int64_t>(kThreads) * 4;
  for (int64_t base = b + static_cast<int64_t>(threadIdx.x) * 4; base < e; base += fstride * kU) {
    float4 acc[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) acc[u] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p) {
      if (p >= W) break;
      const float* src = s_src[p];
      float4 x[kU];
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = base + u * fstride;
        if (i + 4 <= e) x[u] = *reinterpret_cast<const float4*>(src + i);
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t i = base + u * fstride;
        if (i + 4 <= e) {
          acc[u].x += x[u].x;
          acc[u].y += x[u].y;
          acc[u].z += x[u].z;
          acc[u].w += x[u].w;
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t i = base + u * fstride;
      if (i + 4 <= e) {
        if (a.do_adam) adam4(a, k, i, &acc[u].x);
        else *reinterpret_cast<float4*>(a.grad_out + i) = acc[u];
      } else if (i < e) {
        for (int64_t q = i; q < e; ++q) {
          float s1 = 0.f;
          for (int p = 0; p < W; ++p) s1 += s_src[p][q];
          finish_scalar(a, k, q, s1);
        }
      }
    }
  }
}

}  // namespace

void launch(const Args& a, int grid, cudaStream_t stream) {
  if (a.world < 1 || a.world > kMaxRanks || a.rank < 0 || a.rank >= a.world)
    throw std::invalid_argument("all-reduce: rank/world out of range");
  if (a.lo < 0 || a.hi < a.lo || (a.lo & 7)) throw std::invalid_argument("all-reduce: bucket start must be a multiple of 8");
  if (grid < 1 || grid > kMaxCtas) throw std::invalid_argument("all-reduce: grid out of range");
  if (!a.counters || !a.flags_local || !a.grad) throw std::invalid_argument("all-reduce: missing buffer");
  for (int p = 0; p < a.world; ++p)
    if (!a.flags_peer[p]) throw std::invalid_argument("all-reduce: missing peer flag page");
  if (a.do_adam && (!a.param || !a.m || !a.v)) throw std::invalid_argument("all-reduce: Adam needs param, m and v");
  if (a.hi == a.lo) return;
  if (a.mode == kShard) {
    if (!a.do_adam) throw std::invalid_argument("all-reduce: the sharded mode always runs Adam");
    if (!a.scale_local) throw std::invalid_argument("all-reduce: sharded mode needs the scale page");
    for (int p = 0; p < a.world; ++p)
      if (!a.grad_peer[p] || !a.param_peer[p] || !a.scale_peer[p])
        throw std::invalid_argument("all-reduce: sharded mode needs every rank's gradient, parameters and scale");
    if (a.grad_bf16) ar_shard_kernel<true><<<grid, kThreads, 0, stream>>>(a);
    else ar_shard_kernel<false><<<grid, kThreads, 0, stream>>>(a);
  } else {
    if (!a.slot_local[0] || !a.slot_local[1]) throw std::invalid_argument("all-reduce: one-shot needs send slots");
    for (int p = 0; p < a.world; ++p)
      if (!a.slot_peer[p][0] || !a.slot_peer[p][1]) throw std::invalid_argument("all-reduce: missing peer send slot");
    if (!a.do_adam && !a.grad_out) throw std::invalid_argument("all-reduce: grad_out needed without Adam");
    if (a.grad_bf16) ar_oneshot_kernel<true><<<grid, kThreads, 0, stream>>>(a);
    else ar_oneshot_kernel<false><<<grid, kThreads, 0, stream>>>(a);
  }
  GB_LAUNCH_CHECK();
}

}  // namespace ar
}  // namespace grappa
