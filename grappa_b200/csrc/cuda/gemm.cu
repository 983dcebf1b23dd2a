// K-GEMM: the dense projections of the GNN layers on the 5th-generation tensor
// cores.  C[m, n] = sum_k A[m, k] * B[n, k], bf16 operands, fp32 accumulation in
// tensor memory.
//
//   warp 0      TMA producer: one elected thread issues cp.async.bulk.tensor loads of
//               the A and B tiles of each 64-wide k-block into a kStages-deep ring
//               of 128B-swizzled shared-memory buffers (local HBM only, each CTA
//               loads its own tiles)
//   warp 1      allocates the accumulator in TMEM; one thread issues
//               tcgen05.mma.cta_group::1.kind::f16 (M = 128, N = BN, K = 16) and
//               releases each ring slot with tcgen05.commit
//   warps 2-5   epilogue: tcgen05.ld of the accumulator rows (warp w reads TMEM
//               lanes 32*(w%4)..+31), fused epilogue, global stores
//
// Operands may be K-major (row-major [rows][K]) or MN-major (row-major [K][rows]),
// so that the backward products dX = dY.W and dW = dY^T.X read the forward tensors
// in place, without transposes.
//
// Epilogues:
//   kStoreBf16 / kStoreF32  out = act(acc + bias) with optional dropout (Philox
//                           mask keyed by step, layer and element), stored bf16/fp32
//   kAtomicF32              out += acc (split-K over the reduction dimension; dW
//                           accumulates straight into the flat gradient buffer)
//   kCrossEntropy           the row's logits live in one thread's registers, so the
//                           softmax cross-entropy loss, its gradient
//                           (softmax - onehot)/n, the bias gradient and the
//                           correct-prediction count are computed here; the logits are
//                           never written
//
// Rows >= *M_dev (device-side row count) are not stored, so the grid can be sized
// by a static capacity and the kernel captured in a CUDA graph.  Every mbarrier
// wait is bounded by a %globaltimer deadline; on expiry the kernel sets
// kErrMmaTimeout, drains what it issued (again bounded), frees its TMEM and exits.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "grappa/rng.h"
#include "kernels.h"

namespace grappa {
namespace dev {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kThreads = 192;
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait; returns false when the deadline passed or another role aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t polls = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++polls & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitNs) return false;
    }
  }
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

// TMA store of one [box rows][64 cols] bf16 panel from 128B-swizzled shared memory.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* smem_src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(smem_u32(smem_src))
               : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// UMMA shared-memory matrix descriptor, 128B swizzle, sm_100 version field.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= 1ull << 46;
  d |= 2ull << 61;
  return d;
}

// Instruction descriptor of kind::f16 with bf16 A/B and fp32 D.
__host__ __device__ constexpr uint32_t umma_idesc(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(a_mn) << 15) |
         (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Activation backward on 32 accumulator columns of row m: keep acc * mask_scale where
// the forward output (the mask tensor) is non-zero.
__device__ __forceinline__ void apply_act_mask(const GemmArgs& a, int m, int nc, float (&v)[32]) {
  const __nv_bfloat16* hm = a.act_mask + static_cast<int64_t>(m) * a.ld_mask + nc;
  if (nc + 32 <= a.N) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
      float h[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(hm + j), h);
#pragma unroll
      for (int q = 0; q < 8; ++q) v[j + q] = h[q] != 0.f ? v[j + q] * a.mask_scale : 0.f;
    }
  } else {
    for (int j = 0; j < 32; ++j)
      v[j] = (nc + j < a.N && __bfloat162float(hm[j]) != 0.f) ? v[j] * a.mask_scale : 0.f;
  }
}

// Epilogue of one 128 x BN accumulator tile for the store and atomic modes: warp
// `quarter` drains TMEM lanes 32 * quarter + (0..31), i.e. rows m0 + 32 * quarter +
// lane, columns [c_begin, c_end) (multiples of 64 on the TMA-store path); `trow` is
// that warp's TMEM address of the tile, `stage` its 32 x (c_end - c_begin) bf16
// staging panels for the TMA store (kTmaStore), `ok` false after an aborted wait.
// attention-logit epilogue: the 32 stored values v of row m, columns nc.. (heads of
// att_feat columns), rounded to bf16 as stored, dotted with att_l / att_r per head and
// reduced into el / er (one reduction per head the chunk touches)
__device__ __forceinline__ void att_logits(const GemmArgs& a, int m, int nc, const float* v) {
  const int F = a.att_feat, H = a.att_heads;
  const bool dst = a.att_n_dst && m < *a.att_n_dst;
  int h = nc / F, bound = (h + 1) * F;
  float sl = 0.f, sr = 0.f;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int c = nc + j;
    if (c >= a.N) break;
    if (c == bound) {
      if (h < H) {
        atomicAdd(a.att_el + static_cast<int64_t>(m) * H + h, sl);
        if (dst) atomicAdd(a.att_er + static_cast<int64_t>(m) * H + h, sr);
      }
      ++h;
      bound += F;
      sl = sr = 0.f;
    }
    const float z = __bfloat162float(__float2bfloat16_rn(v[j]));
    sl = fmaf(z, __ldg(a.att_l + c), sl);
    sr = fmaf(z, __ldg(a.att_r + c), sr);
  }
  if (h < H) {
    atomicAdd(a.att_el + static_cast<int64_t>(m) * H + h, sl);
    if (dst) atomicAdd(a.att_er + static_cast<int64_t>(m) * H + h, sr);
  }
}

template <int BN, bool kTmaStore>
__device__ __forceinline__ void store_tile(const GemmArgs& a, const CUtensorMap* tmC, uint32_t trow, int m0, int n0,
                                           int M, int quarter, int lane, uint8_t* stage, bool ok, int c_begin = 0,
                                           int c_end = BN) {
  const int m = m0 + quarter * 32 + lane;
  if (kTmaStore && a.c_mode == kStoreBf16) {
    // bf16 tile through shared memory and TMA stores: each epilogue warp stages its
    // 32 rows as 64-column panels in the 128B-swizzled layout of the store's tensor
    // map (`stage`: 32 rows x BN bf16) and one lane stores them
    const uint64_t key = a.counters ? hop_key(static_cast<uint64_t>(a.counters[0]) ^ 0xD80Full,
                                              static_cast<uint64_t>(a.counters[1]),
                                              static_cast<uint64_t>(a.counters[2]), a.dropout_salt)
                                    : 0ull;
    const uint32_t thr8 = dropout_thr8(a.dropout_p);
    const float keep_scale = dropout_scale8(thr8);
    const bool live = m < M;
    // a 32-row slab that crosses the live row count stores its live rows directly,
    // so that rows >= M are never written (except the zeroed tail rows)
    const bool slab_full = m0 + quarter * 32 + 32 <= M;
    const int64_t tail_end = a.zero_tail_rows > 0
                                 ? min(static_cast<int64_t>(ceil_div(M, a.zero_tail_rows)) * a.zero_tail_rows, a.c_rows)
                                 : 0;
    const bool zero_row = !live && m < tail_end;
#pragma unroll 1
    for (int c = c_begin; c < c_end; c += 32) {
      float v[32];
      tmem_ld32(trow + c, v);
      const int nc = n0 + c;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float x = v[j];
        if (a.bias && nc + j < a.N) x += a.bias[nc + j];
        if (a.act == 1) x = fmaxf(x, 0.f);
        v[j] = live ? x : 0.f;
      }
      if (a.act_mask && live) apply_act_mask(a, m, nc, v);
      if (a.att_el && live && nc < a.N) att_logits(a, m, nc, v);
      if (a.dropout_p > 0.f && live) {
        const uint64_t base = static_cast<uint64_t>(m) * static_cast<uint64_t>(a.ldc) + static_cast<uint64_t>(nc);
        const uint32_t keep = dropout_keep_bits(key, base, 32, thr8);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = (keep >> j) & 1u ? v[j] * keep_scale : 0.f;
      }
      if (slab_full) {
        uint8_t* panel = stage + ((c - c_begin) >> 6) * 4096 + lane * 128;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int k = ((c & 63) >> 3) + q;
          *reinterpret_cast<uint4*>(panel + ((k ^ (lane & 7)) << 4)) = f32_to_bf16x8(v + 8 * q);
        }
      } else if ((live || zero_row) && ok && nc < a.N) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.C) + static_cast<int64_t>(m) * a.ldc + nc;
        if (nc + 32 <= a.ldc) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) *reinterpret_cast<uint4*>(dst + j) = f32_to_bf16x8(v + j);
        } else {
          for (int j = 0; j < 32 && nc + j < a.ldc; ++j) dst[j] = __float2bfloat16_rn(v[j]);
        }
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0 && ok && slab_full) {
      for (int p = 0; p < (c_end - c_begin) / 64; ++p)
        if (n0 + c_begin + p * 64 < a.N)
          tma_store_2d(tmC, stage + p * 4096, n0 + c_begin + p * 64, m0 + quarter * 32);
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      // the staging panels may be rewritten once the store has read them
      asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    }
    __syncwarp();
  } else {
    const uint64_t key = a.counters ? hop_key(static_cast<uint64_t>(a.counters[0]) ^ 0xD80Full,
                                              static_cast<uint64_t>(a.counters[1]),
                                              static_cast<uint64_t>(a.counters[2]), a.dropout_salt)
                                    : 0ull;
    const uint32_t thr8 = dropout_thr8(a.dropout_p);
    const float keep_scale = dropout_scale8(thr8);
    const int64_t tail_end = a.zero_tail_rows > 0
                                 ? min(static_cast<int64_t>(ceil_div(M, a.zero_tail_rows)) * a.zero_tail_rows, a.c_rows)
                                 : 0;
#pragma unroll 1
    for (int c = c_begin; c < c_end; c += 32) {
      float v[32];
      tmem_ld32(trow + c, v);
      const int nc = n0 + c;
      if (ok && m >= M && m < tail_end && nc < a.N && a.c_mode == kStoreBf16) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.C) + static_cast<int64_t>(m) * a.ldc + nc;
        for (int j = 0; j < 32 && nc + j < a.ldc; ++j) dst[j] = __float2bfloat16_rn(0.f);
        continue;
      }
      if (!ok || m >= M) continue;
      if (nc >= a.N) continue;
      if (a.c_mode == kAtomicF32) {
        float* dst = reinterpret_cast<float*>(a.C) + static_cast<int64_t>(m) * a.ldc + nc;
        if (nc + 32 <= a.N) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) red_add_v4(dst + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
          for (int j = 0; j < 32 && nc + j < a.N; ++j) atomicAdd(dst + j, v[j]);
        }
        continue;
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float x = v[j];
        if (a.bias && nc + j < a.N) x += a.bias[nc + j];
        if (a.act == 1) x = fmaxf(x, 0.f);
        v[j] = x;
      }
      if (a.act_mask) apply_act_mask(a, m, nc, v);
      if (a.att_el) att_logits(a, m, nc, v);
      if (a.dropout_p > 0.f) {
        // one Philox call covers 16 consecutive elements (byte-resolution masks)
        const uint64_t base = static_cast<uint64_t>(m) * static_cast<uint64_t>(a.ldc) + static_cast<uint64_t>(nc);
        const uint32_t keep = dropout_keep_bits(key, base, 32, thr8);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = (keep >> j) & 1u ? v[j] * keep_scale : 0.f;
      }
      if (a.c_mode == kStoreBf16) {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(a.C) + static_cast<int64_t>(m) * a.ldc + nc;
        if (nc + 32 <= a.ldc) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) *reinterpret_cast<uint4*>(dst + j) = f32_to_bf16x8(v + j);
        } else {
          for (int j = 0; j < 32 && nc + j < a.ldc; ++j) dst[j] = __float2bfloat16_rn(v[j]);
        }
      } else {
        float* dst = reinterpret_cast<float*>(a.C) + static_cast<int64_t>(m) * a.ldc + nc;
        if (nc + 32 <= a.ldc) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
          for (int j = 0; j < 32 && nc + j < a.ldc; ++j) dst[j] = v[j];
        }
      }
    }
    }
}

template <int BN>
struct Smem {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBRows = BN <= 64 ? 64 : BN;  // MN-major B needs 64-wide chunks
  static constexpr int kBBytes = kBRows * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  // ~96 KB of ring per CTA: two CTAs fit on an SM, so one CTA's epilogue overlaps the
  // other's loads and MMAs (each CTA holds at most 256 of the SM's 512 TMEM columns)
  static constexpr int kStages = (96 * 1024) / kStageBytes > 6 ? 6 : (96 * 1024) / kStageBytes;
  static constexpr int kTmemCols = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
  static constexpr int kBytes = kStages * kStageBytes + 1024 /*align*/;
};

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 2)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, GemmArgs a) {
  GB_PDL_ENTRY();
  using S = Smem<BN>;
  constexpr int kStages = S::kStages;
  constexpr bool kTmaStore = BN % 64 == 0 && 4 * 32 * BN * 2 <= kStages * S::kStageBytes;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[kStages], empty_bar[kStages], tmem_bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int M = a.M_dev ? min(*a.M_dev, a.M_cap) : a.M_cap;
  const int m0 = blockIdx.x * BM;
  // the cross-entropy epilogue also zeroes the tail rows [M, roundup(M, 64)) of its tile
  const int m_needed = a.c_mode == kCrossEntropy ? ((M + 63) / 64) * 64 : M;
  if (m0 >= m_needed) return;
  const int n0 = blockIdx.y * BN;
  // reduction range of this split (k-blocks)
  const int K = a.K_dev ? min(*a.K_dev, a.K_cap) : a.K_cap;
  const int kb_total = (K + BK - 1) / BK;
  const int kb_per = (kb_total + a.splits - 1) / a.splits;
  const int kb0 = blockIdx.z * kb_per;
  const int kb1 = min(kb_total, kb0 + kb_per);
  if (kb1 <= kb0) return;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(&tmem_bar, 1);
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&tmem_slot, S::kTmemCols);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = tmem_slot;
  const int nkb = kb1 - kb0;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int i = 0; i < nkb; ++i) {
        const int s = i % kStages;
        const uint32_t ph = (i / kStages) & 1u;
        if (i >= kStages && !mbar_wait(&empty_bar[s], ph ^ 1u, &abort_flag)) {
          set_error(a.err, kErrMmaTimeout);
          abort_flag = 1;
          break;
        }
        uint8_t* sa = smem + s * S::kStageBytes;
        uint8_t* sb = sa + S::kABytes;
        const int kc = (kb0 + i) * BK;
        mbar_expect_tx(&full_bar[s], S::kABytes + (B_MN ? (BN <= 64 ? 64 : BN) : BN) * BK * 2);
        if (A_MN) {
          tma_load_2d(sa, &tmA, &full_bar[s], m0, kc);
          tma_load_2d(sa + 64 * BK * 2, &tmA, &full_bar[s], m0 + 64, kc);
        } else {
          tma_load_2d(sa, &tmA, &full_bar[s], kc, m0);
        }
        if (B_MN) {
#pragma unroll
          for (int c = 0; c < (BN + 63) / 64; ++c) tma_load_2d(sb + c * 64 * BK * 2, &tmB, &full_bar[s], n0 + c * 64, kc);
        } else {
          tma_load_2d(sb, &tmB, &full_bar[s], kc, n0);
        }
        issued = i + 1;
      }
      // on abort, wait (bounded) until the loads already issued have landed
      if (abort_flag) {
        for (int i = 0; i < issued; ++i) {
          const int s = i % kStages;
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full_bar[s], (i / kStages) & 1u) && globaltimer_ns() - t0 < kWaitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(BM, BN, A_MN, B_MN);
      for (int i = 0; i < nkb; ++i) {
        const int s = i % kStages;
        if (!mbar_wait(&full_bar[s], (i / kStages) & 1u, &abort_flag)) {
          set_error(a.err, kErrMmaTimeout);
          abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t sa = smem_u32(smem + s * S::kStageBytes);
        const uint32_t sb = sa + S::kABytes;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t da = A_MN ? umma_desc(sa + kk * 2048, 64 * BK * 2, 1024) : umma_desc(sa + kk * 32, 16, 1024);
          const uint64_t db = B_MN ? umma_desc(sb + kk * 2048, 64 * BK * 2, 1024) : umma_desc(sb + kk * 32, 16, 1024);
          umma_f16(tmem_base, da, db, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty_bar[s]);
      }
      umma_commit(&tmem_bar);
    }
  } else {
    // epilogue warps 2..5
    const int quarter = warp & 3;
    const int row_in_tile = quarter * 32 + lane;
    const int m = m0 + row_in_tile;
    const bool ok = mbar_wait(&tmem_bar, 0, &abort_flag);
    if (!ok) {
      if (lane == 0) set_error(a.err, kErrMmaTimeout);
      abort_flag = 1;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t trow = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    if (a.c_mode == kCrossEntropy) {
     if constexpr (BN <= 64) {  // only narrow tiles carry the whole row in registers
      // BN >= n_classes; the whole row is in this thread's registers
      float v[BN];
#pragma unroll
      for (int c = 0; c < BN; c += 32) {
        float t[32];
        tmem_ld32(trow + c, t);
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c + j < BN) v[c + j] = t[j];
      }
      const int n_rows = a.n_rows_dev ? *a.n_rows_dev : M;
      const int C = a.n_classes;
      const bool live = ok && m < M;
      if (ok && m >= M && m < m_needed && m < a.M_cap) {
        // rows past the count feed the split-K dW reduction: keep them zero
        __nv_bfloat16* drow = a.dlogits + static_cast<int64_t>(m) * a.ld_dl;
        for (int j = 0; j < a.ld_dl; j += 8) *reinterpret_cast<uint4*>(drow + j) = make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < BN; ++j) v[j] += (a.bias && j < C) ? a.bias[j] : 0.f;
      float mx = -INFINITY;
      int arg = 0;
#pragma unroll
      for (int j = 0; j < BN; ++j)
        if (j < C && v[j] > mx) {
          mx = v[j];
          arg = j;
        }
      float se = 0.f;
#pragma unroll
      for (int j = 0; j < BN; ++j)
        if (j < C) se += __expf(v[j] - mx);
      const float lse = mx + __logf(se);
      const int y = live ? a.labels[m] : -1;
      const float inv_n = 1.0f / static_cast<float>(n_rows > 0 ? n_rows : 1);
      float loss = 0.f;
      __nv_bfloat16* drow = a.dlogits + static_cast<int64_t>(m) * a.ld_dl;
#pragma unroll
      for (int j = 0; j < BN; j += 8) {
        float g[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int jj = j + q;
          float p = (jj < C) ? __expf(v[jj] - lse) : 0.f;
          if (jj == y) {
            loss = lse - v[jj];
            p -= 1.0f;
          }
          g[q] = live ? p * inv_n : 0.f;
        }
        const uint4 packed = f32_to_bf16x8(g);
        if (live && j < a.ld_dl) *reinterpret_cast<uint4*>(drow + j) = packed;
        if (a.dbias) {
          // bias gradient from the bf16-rounded values the dW/dX GEMMs consume,
          // reduced over the warp's 32 rows before one atomic per column
          float gr[8];
          bf16x8_to_f32(packed, gr);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float s = warp_sum(gr[q]);
            if (lane == 0 && j + q < C && s != 0.f) atomicAdd(a.dbias + j + q, s);
          }
        }
      }
      // loss and correct count reduced over the warp's 32 rows first: one atomic per
      // warp instead of one per row on the same two words
      const float lsum = warp_sum(live ? loss * inv_n : 0.f);
      const int csum = __popc(__ballot_sync(0xffffffffu, live && arg == y));
      if (lane == 0) {
        if (lsum != 0.f) atomicAdd(a.loss_sum, lsum);
        if (csum) atomicAdd(a.correct, csum);
      }
      if (live && a.pred_out) a.pred_out[m] = arg;
     }
    } else {
      store_tile<BN, kTmaStore>(a, &tmC, trow, m0, n0, M, quarter, lane, smem + quarter * (32 * BN * 2), ok);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

// ---------------------------------------------------------------- persistent variant
// One CTA per SM walks the output tiles t = blockIdx.x, blockIdx.x + grid, ... (tile
// order: N fastest, then M, then the split), so that the producer streams the
// operands of the next tile while the epilogue warps drain the previous one.  The
// accumulator is double-buffered in TMEM (2 x BN columns): the MMA thread fills
// buffer lt & 1 of local tile lt while the epilogue reads the other; acc_full[b] is
// committed by the MMA thread, acc_empty[b] is arrived by every epilogue warp.
// The ring of k-block stages continues across tiles.  Store and atomic modes only
// (the cross-entropy epilogue stays with the one-tile kernel).
template <int BN>
struct PSmem {
  static constexpr int kABytes = BM * BK * 2;
  static constexpr int kBRows = BN <= 64 ? 64 : BN;
  static constexpr int kBBytes = kBRows * BK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStageArea = BN % 64 == 0 ? 4 * 32 * BN * 2 : 0;  // TMA-store panels
  static constexpr int kRingBudget = 218 * 1024 - kStageArea;
  static constexpr int kStages = kRingBudget / kStageBytes > 8 ? 8 : kRingBudget / kStageBytes;
  static constexpr int kAccCols = BN <= 32 ? 32 : (BN <= 64 ? 64 : (BN <= 128 ? 128 : 256));
  static constexpr int kTmemCols = 2 * kAccCols;
  static constexpr int kBytes = kStages * kStageBytes + kStageArea + 1024 /*align*/;
  static_assert(kStages >= 2, "persistent GEMM: ring too small");
};

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

constexpr int kMinSplitKb = 8;

struct TileIdx {
  int m0, n0, kb0, kb1;
};
__device__ __forceinline__ TileIdx decode_tile(int t, int n_tiles, int m_tiles, int BNv, int kb_total, int kb_per) {
  TileIdx r;
  const int nt = t % n_tiles;
  const int rest = t / n_tiles;
  r.m0 = (rest % m_tiles) * BM;
  r.n0 = nt * BNv;
  r.kb0 = (rest / m_tiles) * kb_per;
  r.kb1 = min(kb_total, r.kb0 + kb_per);
  return r;
}

// epilogue warps of the persistent kernel: two per TMEM lane quarter (each drains half
// the columns) for tiles of 128 columns and more, one otherwise
template <int BN>
__host__ __device__ constexpr int p_epi_warps() { return BN % 128 == 0 ? 8 : 4; }
template <int BN>
__host__ __device__ constexpr int p_threads() { return 64 + 32 * p_epi_warps<BN>(); }

template <int BN, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(p_threads<BN>(), 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           const __grid_constant__ CUtensorMap tmC, GemmArgs a) {
  GB_PDL_ENTRY();
  using S = PSmem<BN>;
  constexpr int kStages = S::kStages;
  constexpr bool kTmaStore = BN % 64 == 0;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t full_bar[kStages], empty_bar[kStages], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int M = a.M_dev ? min(*a.M_dev, a.M_cap) : a.M_cap;
  const int K = a.K_dev ? min(*a.K_dev, a.K_cap) : a.K_cap;
  const int kb_total = (K + BK - 1) / BK;
  // the host sizes the split count by the capacity of the reduction dimension; with
  // the live length known here, keep at least kMinSplitKb k-blocks per split, so that
  // the fp32 reductions of the split-K epilogue (one per output element and split)
  // do not outweigh the MMAs
  const int splits = max(1, min(a.splits, kb_total / kMinSplitKb));
  const int kb_per = (kb_total + splits - 1) / splits;
  const int m_tiles = (M + BM - 1) / BM;
  const int n_tiles = (a.N + BN - 1) / BN;
  const int tiles = m_tiles * n_tiles * splits;

  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_area = smem + kStages * S::kStageBytes;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], p_epi_warps<BN>());
    }
    abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&tmem_slot, S::kTmemCols);
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem_base = tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool stop = false;
      for (int t = blockIdx.x; t < tiles && !stop; t += gridDim.x) {
        const TileIdx ti = decode_tile(t, n_tiles, m_tiles, BN, kb_total, kb_per);
        for (int kb = ti.kb0; kb < ti.kb1; ++kb, ++it) {
          const int s = static_cast<int>(it % kStages);
          const uint32_t ph = (it / kStages) & 1u;
          if (it >= static_cast<uint32_t>(kStages) && !mbar_wait(&empty_bar[s], ph ^ 1u, &abort_flag)) {
            set_error(a.err, kErrMmaTimeout);
            abort_flag = 1;
            stop = true;
            break;
          }
          uint8_t* sa = smem + s * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          const int kc = kb * BK;
          mbar_expect_tx(&full_bar[s], S::kABytes + (B_MN ? (BN <= 64 ? 64 : BN) : BN) * BK * 2);
          if (A_MN) {
            tma_load_2d(sa, &tmA, &full_bar[s], ti.m0, kc);
            tma_load_2d(sa + 64 * BK * 2, &tmA, &full_bar[s], ti.m0 + 64, kc);
          } else {
            tma_load_2d(sa, &tmA, &full_bar[s], kc, ti.m0);
          }
          if (B_MN) {
#pragma unroll
            for (int c = 0; c < (BN + 63) / 64; ++c)
              tma_load_2d(sb + c * 64 * BK * 2, &tmB, &full_bar[s], ti.n0 + c * 64, kc);
          } else {
            tma_load_2d(sb, &tmB, &full_bar[s], kc, ti.n0);
          }
        }
      }
      // on abort, wait (bounded) until the loads still in flight (the last kStages
      // issued at most) have landed
      if (abort_flag) {
        const uint32_t first = it > static_cast<uint32_t>(kStages) ? it - kStages : 0u;
        for (uint32_t i = first; i < it; ++i) {
          const int s = static_cast<int>(i % kStages);
          const uint64_t t0 = globaltimer_ns();
          while (!mbar_try_wait(&full_bar[s], (i / kStages) & 1u) && globaltimer_ns() - t0 < kWaitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(BM, BN, A_MN, B_MN);
      uint32_t it = 0;
      int lt = 0;
      bool stop = false;
      for (int t = blockIdx.x; t < tiles && !stop; t += gridDim.x) {
        const TileIdx ti = decode_tile(t, n_tiles, m_tiles, BN, kb_total, kb_per);
        if (ti.kb1 <= ti.kb0) continue;
        const int b = lt & 1;
        if (lt >= 2 && !mbar_wait(&acc_empty[b], ((lt >> 1) - 1) & 1u, &abort_flag)) {
          set_error(a.err, kErrMmaTimeout);
          abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(b * S::kAccCols);
        for (int kb = ti.kb0; kb < ti.kb1; ++kb, ++it) {
          const int s = static_cast<int>(it % kStages);
          if (!mbar_wait(&full_bar[s], (it / kStages) & 1u, &abort_flag)) {
            set_error(a.err, kErrMmaTimeout);
            abort_flag = 1;
            stop = true;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sa = smem_u32(smem + s * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t da = A_MN ? umma_desc(sa + kk * 2048, 64 * BK * 2, 1024) : umma_desc(sa + kk * 32, 16, 1024);
            const uint64_t db = B_MN ? umma_desc(sb + kk * 2048, 64 * BK * 2, 1024) : umma_desc(sb + kk * 32, 16, 1024);
            umma_f16(d_tmem, da, db, idesc, (kb > ti.kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[s]);
        }
        if (stop) break;
        umma_commit(&acc_full[b]);
        ++lt;
      }
    }
  } else {
    // epilogue warps 2 .. 2 + p_epi_warps - 1
    constexpr int kEpi = p_epi_warps<BN>();
    constexpr int kCols = BN / (kEpi / 4);  // columns per epilogue warp
    const int quarter = warp & 3;
    const int part = (warp - 2) / 4;
    uint8_t* stage = stage_area + (warp - 2) * (32 * kCols * 2);
    int lt = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
      const TileIdx ti = decode_tile(t, n_tiles, m_tiles, BN, kb_total, kb_per);
      if (ti.kb1 <= ti.kb0) continue;
      const int b = lt & 1;
      if (!mbar_wait(&acc_full[b], (lt >> 1) & 1u, &abort_flag)) {
        if (lane == 0) set_error(a.err, kErrMmaTimeout);
        abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t trow = tmem_base + static_cast<uint32_t>(b * S::kAccCols) + (static_cast<uint32_t>(quarter * 32) << 16);
      store_tile<BN, kTmaStore>(a, &tmC, trow, ti.m0, ti.n0, M, quarter, lane, stage, true, part * kCols,
                                (part + 1) * kCols);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      ++lt;
    }
  }
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    tmem_dealloc(tmem_base, S::kTmemCols);
  }
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    GB_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (!p || q != cudaDriverEntryPointSuccess) throw std::runtime_error("cuTensorMapEncodeTiled not available");
    fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// 2D bf16 tensor map over a row-major [rows][cols] matrix with row stride ld
// (elements); box = [64 cols, box_rows rows], 128B swizzle, zero fill outside.
CUtensorMap make_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  if ((reinterpret_cast<uintptr_t>(ptr) & 15u) != 0) throw std::invalid_argument("GEMM operand not 16-byte aligned");
  if ((ld * 2) % 16 != 0) throw std::invalid_argument("GEMM operand row stride must be a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows > 0 ? rows : 1)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string(static_cast<int>(r)));
  return m;
}

int sm_count() {
  static int sms = 0;
  if (!sms) {
    int d = 0;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

// GRAPPA_GEMM_PERSISTENT=0 selects the one-tile-per-CTA kernel (for comparisons)
bool persistent_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("GRAPPA_GEMM_PERSISTENT");
    v = (e && e[0] == '0') ? 0 : 1;
  }
  return v == 1;
}

template <int BN, bool A_MN, bool B_MN>
void launch_t(const GemmProblem& p, const GemmArgs& a, dim3 grid, cudaStream_t stream) {
  using S = Smem<BN>;
  // A: K-major -> [M rows][K cols]; MN-major -> [K rows][M cols]
  const CUtensorMap ma = A_MN ? make_map(p.A, p.a_rows, p.a_cols, p.lda, BK) : make_map(p.A, p.a_rows, p.a_cols, p.lda, BM);
  const CUtensorMap mb = B_MN ? make_map(p.B, p.b_rows, p.b_cols, p.ldb, BK) : make_map(p.B, p.b_rows, p.b_cols, p.ldb, BN);
  // output map for the TMA-store epilogue (bf16 C of c_rows x N; otherwise an unused copy of A's)
  CUtensorMap mc = ma;
  if (a.c_mode == kStoreBf16 && BN % 64 == 0) {
    if (a.c_rows <= 0) throw std::invalid_argument("bf16 GEMM output needs its row count");
    mc = make_map(a.C, a.c_rows, a.N, a.ldc, 32);
  }
  int dev = 0;
  GB_CUDA_CHECK(cudaGetDevice(&dev));
  if (a.c_mode != kCrossEntropy && persistent_enabled()) {
    using P = PSmem<BN>;
    auto kern = gemm_persistent_kernel<BN, A_MN, B_MN>;
    static int attr_device_p = -1;
    if (attr_device_p != dev) {
      GB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, P::kBytes));
      attr_device_p = dev;
    }
    const int64_t tiles = static_cast<int64_t>(grid.x) * grid.y * grid.z;
    const unsigned g = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(tiles, sm_count())));
    launch_k(kern, g, p_threads<BN>(), P::kBytes, stream, ma, mb, mc, a);
    GB_LAUNCH_CHECK();
    return;
  }
  auto kern = gemm_kernel<BN, A_MN, B_MN>;
  static int attr_device = -1;
  if (attr_device != dev) {
    GB_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kBytes));
    attr_device = dev;
  }
  launch_k(kern, grid, kThreads, S::kBytes, stream, ma, mb, mc, a);
  GB_LAUNCH_CHECK();
}

}  // namespace

void launch_gemm(const GemmProblem& p, GemmArgs a, int bn, cudaStream_t stream) {
  if (a.splits < 1) a.splits = 1;
  const dim3 grid(static_cast<unsigned>(ceil_div(a.M_cap, BM)), static_cast<unsigned>(ceil_div(a.N, bn)),
                  static_cast<unsigned>(a.splits));
  if (a.c_mode == kCrossEntropy && (a.N > bn || a.n_classes > bn)) throw std::invalid_argument("cross-entropy epilogue needs N <= BN");
  if (a.c_mode == kCrossEntropy && a.ld_dl % 8 != 0) throw std::invalid_argument("dlogits stride must be a multiple of 8");
  if (a.act_mask && (a.c_mode != kStoreBf16 || a.bias || a.act || a.dropout_p > 0.f || a.ld_mask % 8 != 0))
    throw std::invalid_argument("activation-backward epilogue: bf16 store only, no bias/activation/dropout, mask stride % 8");
  if (a.att_el && (a.c_mode != kStoreBf16 || a.bias || a.act || a.dropout_p > 0.f || a.act_mask || !a.att_l ||
                   !a.att_r || !a.att_er || a.att_heads <= 0 || a.att_feat <= 0 || a.att_heads * a.att_feat != a.N))
    throw std::invalid_argument("attention-logit epilogue: plain bf16 store of N = heads * feat, vectors and outputs given");
  if (a.zero_tail_rows > 0 && a.c_mode != kStoreBf16)
    throw std::invalid_argument("zeroed tail rows need the bf16 store mode");
#define GB_GEMM_CASE(BNV)                                                           \
  if (bn == BNV) {                                                                  \
    if (!p.a_mn && !p.b_mn) return launch_t<BNV, false, false>(p, a, grid, stream); \
    if (!p.a_mn && p.b_mn) return launch_t<BNV, false, true>(p, a, grid, stream);   \
    if (p.a_mn && p.b_mn) return launch_t<BNV, true, true>(p, a, grid, stream);     \
    return launch_t<BNV, true, false>(p, a, grid, stream);                          \
  }
  GB_GEMM_CASE(64)
  GB_GEMM_CASE(128)
  GB_GEMM_CASE(256)
#undef GB_GEMM_CASE
  if (bn == 48) {
    if (p.a_mn || p.b_mn) throw std::invalid_argument("BN=48 supports K-major operands only");
    return launch_t<48, false, false>(p, a, grid, stream);
  }
  throw std::invalid_argument("unsupported GEMM tile width");
}

}  // namespace dev
}  // namespace grappa
