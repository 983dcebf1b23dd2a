// GAT attention over a block (DGL GATConv semantics, the layer the reference
// trains, experiments/grappa/train/gat.py:12-50): with z = fc(h) (a tcgen05 GEMM
// over the source rows, z_dst = z[:n_dst] as for DGL blocks)
//
//   el[u,h] = z_u[h] . a_l[h]        er[v,h] = z_v[h] . a_r[h]
//   e_uvh   = LeakyReLU(el[u,h] + er[v,h], slope)
//   a_uvh   = softmax over the in-edges of v
//   out_v[h] = sum_u a_uvh z_u[h] + b[h]
//
// Hidden layers write ReLU(out) flattened over heads with dropout (one kernel:
// scores are never materialised per edge); the last layer writes the mean over
// heads (the logits).  The softmax statistics (max, sum) of every (v, h) are kept
// for the backward, which recomputes a_uvh from el/er instead of storing it.
//
// Work split: one warp per destination row.  Pass 1 has lane h walk the edges for
// head h (softmax statistics from the el values only); pass 2 streams the z rows,
// each lane owning 8-column chunks of the H*F row (a chunk touches at most two
// heads, so F need not be a multiple of 8).
//
// Backward (gat_bwd_edge, one warp per dst; then gat_bwd_node, one warp per src):
//   da_uvh  = dout_v[h] . z_u[h]                     (kept per edge and head)
//   de_uvh  = a_uvh (da_uvh - sum_u' a_u'vh da_u'vh) * LeakyReLU'(x)
//   del[u,h] += de, der[v,h] += de, dz_u[h] += a_uvh dout_v[h]   (fp32 reductions)
//   dz_u[h] += del[u,h] a_l[h] + der[u,h] a_r[h];  da_l += del z;  da_r += der z
// dz is staged to bf16 for the dW / dX GEMMs and the fp32 accumulators are cleared.
//
// Input layer (no dX wanted): dz is only needed for dW = dz^T x, and
//   dW[hF+f, k] = sum_v dout_v[hF+f] y_v[h, k] + a_l[hF+f] xl[h, k] + a_r[hF+f] xr[h, k]
// with y_v[h] = sum_u a_uvh x_u (an attention-weighted sum of the layer's INPUT rows,
// per destination), xl[h] = sum_u del[u,h] x_u and xr[h] = sum_{u<n_dst} der[u,h] x_u.
// The edge kernel then writes y (n_dst rows of H * in) instead of scattering the
// H*F-wide dz over the sources with fp32 reductions, the node kernel reduces xl/xr,
// a GEMM forms dout^T y and gat_dw_combine adds its diagonal head blocks and the two
// rank-1 terms into dW.
#include <algorithm>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "grappa/rng.h"
#include "kernels.h"

namespace grappa {
namespace dev {

namespace {

constexpr int kMaxHeads = 8;
constexpr int kThreads = 256;

int sms() {
  static int s = 0;
  if (!s) {
    int d = 0;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&s, cudaDevAttrMultiProcessorCount, d);
    if (s <= 0) s = 148;
  }
  return s;
}
int grid_warps(int rows, int per_sm = 16) {
  const int64_t want = ceil_div(rows > 0 ? rows : 1, kThreads / 32);
  return static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(sms()) * per_sm));
}

__device__ __forceinline__ void red_add_v4f(float* p, float a, float b, float c, float d) {
  // no "memory" clobber: the reduced buffer is not read in the same launch, and a
  // compiler barrier here would serialise the edge loop's loads behind every reduction
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d));
}
__device__ __forceinline__ float leaky(float x, float s) { return x > 0.f ? x : x * s; }
// column of z that virtual column c reads (a.zmod > 0: one row shared by every head)
__device__ __forceinline__ int zcol(const GatArgs& a, int c) { return a.zmod > 0 ? c % a.zmod : c; }

// Column sums of per-lane partials (lane owns columns (lane + 32 q) * 8 + j, the
// same in every warp) over the block's warps in shared memory, then one atomic per
// column per block: the column gradients (bias, attention vectors) would otherwise
// take one contended atomic per warp and column.  Called by every thread.
// One shared scratch per kernel for every block_col_atomic instantiation (a static
// __shared__ array inside the template would be allocated once per instantiation).
__device__ __forceinline__ float (*col_scratch())[1024] {
  __shared__ float s[kThreads / 32][1024];
  return s;
}

template <int CPL>
__device__ void block_col_atomic(const float (&v)[CPL][8], float* dst, int HF) {
  float (*s)[1024] = col_scratch();
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
  for (int q = 0; q < CPL; ++q)
#pragma unroll
    for (int j = 0; j < 8; ++j) s[w][(lane + 32 * q) * 8 + j] = v[q][j];
  __syncthreads();
  for (int c = threadIdx.x; c < HF; c += blockDim.x) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < kThreads / 32; ++k) t += s[k][c];
    if (t != 0.f) atomicAdd(dst + c, t);
  }
  __syncthreads();
}

// ------------------------------------------------------------------ scores
template <int CPL>
__global__ void __launch_bounds__(kThreads) gat_scores_kernel(GatArgs a) {
  GB_PDL_ENTRY();
  const int n_src = a.n_src_ptr ? min(*a.n_src_ptr, a.cap_src) : a.cap_src;
  const int n_dst = a.n_dst_ptr ? min(*a.n_dst_ptr, a.cap_dst) : a.cap_dst;
  const int HF = a.heads * a.feat;
  const int lane = threadIdx.x & 31;
  const int warps_total = (gridDim.x * kThreads) >> 5;
  // fast path: heads of F % 8 == 0 columns with F / 8 lanes per head (a power of two
  // below 32): every 8-column chunk lies in one head, reduced by a segmented shuffle
  const int g = a.feat / 8;
  const bool seg = a.feat % 8 == 0 && g < 32 && (g & (g - 1)) == 0;
  if (seg) {
    for (int r = (blockIdx.x * kThreads + threadIdx.x) >> 5; r < n_src; r += warps_total) {
      const bool is_dst = r < n_dst;
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c0 = (lane + 32 * q) * 8;
        float sl = 0.f, sr = 0.f;
        if (c0 < HF) {
          float f[8], al[8], ar[8];
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(r) * a.ldz + zcol(a, c0)), f);
          *reinterpret_cast<float4*>(al) = __ldg(reinterpret_cast<const float4*>(a.attn_l + c0));
          *reinterpret_cast<float4*>(al + 4) = __ldg(reinterpret_cast<const float4*>(a.attn_l + c0 + 4));
          *reinterpret_cast<float4*>(ar) = __ldg(reinterpret_cast<const float4*>(a.attn_r + c0));
          *reinterpret_cast<float4*>(ar + 4) = __ldg(reinterpret_cast<const float4*>(a.attn_r + c0 + 4));
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            sl += f[j] * al[j];
            sr += f[j] * ar[j];
          }
        }
        for (int off = 1; off < g; off <<= 1) {
          sl += __shfl_xor_sync(0xffffffffu, sl, off);
          sr += __shfl_xor_sync(0xffffffffu, sr, off);
        }
        if (c0 < HF && (lane & (g - 1)) == 0) {
          const int h = c0 / a.feat;
          a.el[static_cast<int64_t>(r) * a.heads + h] = sl;
          if (is_dst) a.er[static_cast<int64_t>(r) * a.heads + h] = sr;
        }
      }
    }
    return;
  }
  for (int r = (blockIdx.x * kThreads + threadIdx.x) >> 5; r < n_src; r += warps_total) {
    float pl[kMaxHeads], pr[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) pl[h] = pr[h] = 0.f;
    const bool is_dst = r < n_dst;
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c0 = (lane + 32 * q) * 8;
      if (c0 >= HF) continue;
      float f[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(r) * a.ldz + zcol(a, c0)), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + j;
        if (c >= HF) break;
        const int h = c / a.feat;
#pragma unroll
        for (int hh = 0; hh < kMaxHeads; ++hh)
          if (hh == h) {
            pl[hh] += f[j] * a.attn_l[c];
            if (is_dst) pr[hh] += f[j] * a.attn_r[c];
          }
      }
    }
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) {
      if (h >= a.heads) break;
      const float sl = warp_sum(pl[h]);
      const float sr = warp_sum(pr[h]);
      if (lane == 0) {
        a.el[static_cast<int64_t>(r) * a.heads + h] = sl;
        if (is_dst) a.er[static_cast<int64_t>(r) * a.heads + h] = sr;
      }
    }
  }
}

// ------------------------------------------------------------------ forward
// One pass over the in-edges of a destination with an online softmax: the edges are
// taken 32 at a time (one coalesced load of their source ids, then lane t loads the
// el row of edge t), every head's running max m and denominator s are updated from the
// batch's scores by warp reductions, the accumulated rows are rescaled by exp(m_old -
// m_new), and the z rows of the batch are added with the weights exp(x - m), four
// edges' rows in flight per lane.  The output is acc / s (+ bias); m and s are kept
// for the backward, which recomputes the attention from them.
template <int HM>
__device__ __forceinline__ float pick_head(const float (&v)[HM], int h) {
  float r = 0.f;
#pragma unroll
  for (int hh = 0; hh < HM; ++hh)
    if (hh == h) r = v[hh];
  return r;
}

// HM: the head count rounded up to 4 or kMaxHeads (sizes the per-head register arrays);
// EU_: edges whose z rows are in flight together (0: 4 for CPL 1, else 2); MINB: CTAs
// per SM the registers are capped for (occupancy against registers per lane)
// SEGF: F % 8 == 0, so every 8-column chunk lies in one head (no per-element head pick)
template <int CPL, int HM, int EU_ = 0, int MINB = 1, bool SEGF = false>
__global__ void __launch_bounds__(kThreads, MINB) gat_fwd_kernel(GatArgs a) {
  GB_PDL_ENTRY();
  extern __shared__ float s_row[];  // mean_heads: [warps][HF]
  __shared__ float s_w[kThreads / 32][32][HM];  // the batch's edge weights, per head
  __shared__ int s_u[kThreads / 32][32];        // the batch's source rows
  const int n_dst = a.n_dst_ptr ? min(*a.n_dst_ptr, a.cap_dst) : a.cap_dst;
  const int H = a.heads, F = a.feat, HF = H * F;
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int warps_total = (gridDim.x * kThreads) >> 5;
  const int out_w = a.mean_heads ? F : HF;
  const int rows_end = a.zero_tail_rows > 0 ? min(a.cap_dst, static_cast<int>(ceil_div(n_dst, a.zero_tail_rows) * a.zero_tail_rows)) : n_dst;
  uint64_t key = 0;
  uint32_t thr = 0;
  float ks = 1.f;
  if (a.dropout_p > 0.f) {
    key = hop_key(static_cast<uint64_t>(a.counters[0]) ^ 0xD80Full, static_cast<uint64_t>(a.counters[1]),
                  static_cast<uint64_t>(a.counters[2]), a.dropout_salt);
    thr = dropout_thr8(a.dropout_p);
    ks = dropout_scale8(thr);
  }
  constexpr int EU = EU_ > 0 ? EU_ : (CPL <= 1 ? 4 : 2);  // edges whose z rows are in flight together
  int h0[CPL], h1[CPL];
  uint32_t in0[CPL];  // bit j: column c0 + j belongs to head h0 (else to h1)
#pragma unroll
  for (int q = 0; q < CPL; ++q) {
    const int c0 = (lane + 32 * q) * 8;
    h0[q] = min(c0 / F, H - 1);
    h1[q] = min(h0[q] + 1, H - 1);
    in0[q] = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if ((c0 + j) / F == h0[q]) in0[q] |= 1u << j;
  }
  for (int v = (blockIdx.x * kThreads + threadIdx.x) >> 5; v < rows_end; v += warps_total) {
    if (v >= n_dst) {
      for (int c = lane * 8; c < a.ldo; c += 256)
        *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(v) * a.ldo + c) = make_uint4(0, 0, 0, 0);
      continue;
    }
    const int beg = a.indptr[v], end = a.indptr[v + 1];
    float er[HM], m[HM], sden[HM];
#pragma unroll
    for (int h = 0; h < HM; ++h) {
      er[h] = h < H ? a.er[static_cast<int64_t>(v) * H + h] : 0.f;
      m[h] = -INFINITY;
      sden[h] = 0.f;
    }
    float acc[CPL][8];
#pragma unroll
    for (int q = 0; q < CPL; ++q)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[q][j] = 0.f;
    for (int cb = beg; cb < end; cb += 32) {
      const int cnt = min(32, end - cb);
      const bool mine = lane < cnt;
      const int my_u = mine ? a.indices[cb + lane] : 0;
      float x[HM];
      if (HM == 4 && H == 4) {
        float4 e4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (mine) e4 = *reinterpret_cast<const float4*>(a.el + static_cast<int64_t>(my_u) * 4);
        x[0] = e4.x;
        x[1] = e4.y;
        x[2] = e4.z;
        x[3] = e4.w;
      } else {
#pragma unroll
        for (int h = 0; h < HM; ++h) x[h] = (mine && h < H) ? a.el[static_cast<int64_t>(my_u) * H + h] : 0.f;
      }
      float sc[HM];
#pragma unroll
      for (int h = 0; h < HM; ++h) {
        if (h >= H) {
          sc[h] = 1.f;
          continue;
        }
        const float xs = mine ? leaky(x[h] + er[h], a.slope) : -INFINITY;
        float bm = xs;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o));
        const float nm = fmaxf(m[h], bm);
        sc[h] = __expf(m[h] - nm);  // 0 on the first batch (m = -inf)
        const float w = mine ? __expf(xs - nm) : 0.f;
        s_w[wib][lane][h] = w;
        sden[h] = sden[h] * sc[h] + warp_sum(w);
        m[h] = nm;
      }
      s_u[wib][lane] = my_u;
      __syncwarp();
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const float s0 = pick_head<HM>(sc, h0[q]), s1 = pick_head<HM>(sc, h1[q]);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[q][j] *= (SEGF || ((in0[q] >> j) & 1u)) ? s0 : s1;
      }
      for (int k = 0; k < cnt; k += EU) {
        uint4 zv[EU][CPL];
        float wt0[EU][CPL], wt1[EU][CPL];
#pragma unroll
        for (int t = 0; t < EU; ++t) {
          const bool ok = k + t < cnt;
          const int u = s_u[wib][ok ? k + t : 0];
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            const int c0 = (lane + 32 * q) * 8;
            wt0[t][q] = ok ? s_w[wib][k + t][h0[q]] : 0.f;
            wt1[t][q] = (!SEGF && ok) ? s_w[wib][k + t][h1[q]] : 0.f;
            zv[t][q] = make_uint4(0, 0, 0, 0);
            if (ok && c0 < HF) zv[t][q] = *reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(u) * a.ldz + zcol(a, c0));
          }
        }
#pragma unroll
        for (int t = 0; t < EU; ++t)
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            float f[8];
            bf16x8_to_f32(zv[t][q], f);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[q][j] = fmaf((SEGF || ((in0[q] >> j) & 1u)) ? wt0[t][q] : wt1[t][q], f[j], acc[q][j]);
          }
      }
      __syncwarp();  // the batch's weights are read before the next batch writes them
    }
    // normalise by the softmax denominators; keep the statistics for the backward
    if (lane < H) {
      a.smax[static_cast<int64_t>(v) * H + lane] = pick_head<HM>(m, lane);
      a.ssum[static_cast<int64_t>(v) * H + lane] = pick_head<HM>(sden, lane);
    }
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const float d0 = pick_head<HM>(sden, h0[q]), d1 = pick_head<HM>(sden, h1[q]);
      const float i0 = d0 > 0.f ? 1.f / d0 : 0.f, i1 = d1 > 0.f ? 1.f / d1 : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[q][j] *= (SEGF || ((in0[q] >> j) & 1u)) ? i0 : i1;
    }
    if (!a.mean_heads) {
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c0 = (lane + 32 * q) * 8;
        if (c0 >= a.ldo) continue;
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int c = c0 + j;
          float x = c < HF ? acc[q][j] + (a.bias ? a.bias[c] : 0.f) : 0.f;
          if (a.act == 1) x = fmaxf(x, 0.f);
          o[j] = x;
        }
        if (a.dropout_p > 0.f) {
          const uint64_t base = static_cast<uint64_t>(v) * static_cast<uint64_t>(a.ldo) + static_cast<uint64_t>(c0);
          const uint32_t keep = dropout_keep_bits(key, base, 8, thr);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = (keep >> j) & 1u ? o[j] * ks : 0.f;
        }
        *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(v) * a.ldo + c0) = f32_to_bf16x8(o);
      }
    } else {
      float* row = s_row + wib * HF;
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c0 = (lane + 32 * q) * 8;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (c0 + j < HF) row[c0 + j] = acc[q][j] + (a.bias ? a.bias[c0 + j] : 0.f);
      }
      __syncwarp();
      const float inv_h = 1.f / static_cast<float>(H);
      for (int f = lane; f < a.ldo; f += 32) {
        float t = 0.f;
        if (f < out_w)
          for (int h = 0; h < H; ++h) t += row[h * F + f];
        a.out[static_cast<int64_t>(v) * a.ldo + f] = __float2bfloat16_rn(t * inv_h);
      }
      __syncwarp();
    }
  }
}

// ------------------------------------------------------------------ backward, per destination
// SEG: every 8-column chunk lies in one head and a head spans a power-of-two group of
// lanes (F a power of two in [8, 256]): the per-head dot products of an edge are then
// a butterfly inside each lane group (log2(F / 8) shuffles) instead of H full warp
// reductions, and no per-element head arithmetic is needed.  Otherwise the generic
// path handles chunks that straddle two heads.
struct HeadMap {
  int h0[4];      // head of chunk q (CPL <= 4)
  int lph;        // lanes per head (SEG)
  int src_q, src_lane;  // lane h (< H): chunk and lane where the sum of head h ends up
};

template <int CPL, bool SEG>
__device__ __forceinline__ HeadMap head_map(int lane, int H, int F) {
  HeadMap m;
#pragma unroll
  for (int q = 0; q < CPL; ++q) m.h0[q] = min((lane + 32 * q) * 8 / F, H - 1);
  m.lph = SEG ? F / 8 : 32;
  const int chunk = SEG ? lane * (F / 8) : 0;  // first chunk of head `lane`
  m.src_q = chunk / 32;
  m.src_lane = chunk % 32;
  return m;
}

// da of one edge for head `lane` (lanes >= H get 0): sum over the head's columns of
// go * z, z given as the lane's bf16 chunks.
template <int CPL, bool SEG>
__device__ __forceinline__ float edge_head_dot(const float (&go)[CPL][8], const uint4 (&zv)[CPL], const HeadMap& m,
                                               int lane, int H, int F, int HF) {
  if constexpr (SEG) {
    float part[CPL];
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      float f[8];
      bf16x8_to_f32(zv[q], f);
      float t = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) t = fmaf(go[q][j], f[j], t);
      part[q] = t;
    }
    for (int off = 1; off < m.lph; off <<= 1)
#pragma unroll
      for (int q = 0; q < CPL; ++q) part[q] += __shfl_xor_sync(0xffffffffu, part[q], off);
    float da = 0.f;
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const float t = __shfl_sync(0xffffffffu, part[q], m.src_lane);
      if (q == m.src_q) da = t;
    }
    return lane < H ? da : 0.f;
  } else {
    float p[kMaxHeads];
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) p[h] = 0.f;
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c0 = (lane + 32 * q) * 8;
      if (c0 >= HF) continue;
      float f[8];
      bf16x8_to_f32(zv[q], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int h = (c0 + j) / F;
        const float t = go[q][j] * f[j];
#pragma unroll
        for (int hh = 0; hh < kMaxHeads; ++hh)
          if (hh == h) p[hh] += t;
      }
    }
    float da_mine = 0.f;
#pragma unroll
    for (int h = 0; h < kMaxHeads; ++h) {
      if (h >= H) break;
      const float t = warp_sum(p[h]);
      if (lane == h) da_mine = t;
    }
    return da_mine;
  }
}

// resident blocks per SM the edge kernel is compiled for: two (128 registers: four
// edges' rows in flight per warp), one for wide heads x features
template <int CPL, int CPLY>
constexpr int bwd_min_blocks() { return CPL + CPLY <= 3 ? 2 : 1; }

// MINB > 0: registers capped for MINB CTAs per SM (the occupancy variants)
template <int CPL, int CPLY, bool SEG, int MINB = 0>
__global__ void __launch_bounds__(kThreads, MINB > 0 ? MINB : bwd_min_blocks<CPL, CPLY>()) gat_bwd_edge_kernel(GatArgs a) {
  GB_PDL_ENTRY();
  const int n_dst = a.n_dst_ptr ? min(*a.n_dst_ptr, a.cap_dst) : a.cap_dst;
  const int H = a.heads, F = a.feat, HF = H * F;
  const int IN = a.in_dim, HIN = H * a.in_dim;  // input-layer mode (CPLY > 0)
  const int lane = threadIdx.x & 31;
  const int warps_total = (gridDim.x * kThreads) >> 5;
  const float inv_h = a.mean_heads ? 1.f / static_cast<float>(H) : 1.f;
  const HeadMap hm = head_map<CPL, SEG>(lane, H, F);
  constexpr int NY = CPLY > 0 ? CPLY : 1;
  constexpr int EU = CPL == 1 && NY <= 2 ? 4 : 2;  // edges per pass-A iteration
  int hy[NY], ky[NY];  // head and input column of the lane's y chunks
#pragma unroll
  for (int q = 0; q < NY; ++q) {
    const int c0 = (lane + 32 * q) * 8;
    hy[q] = CPLY > 0 ? min(c0 / max(IN, 1), H - 1) : 0;
    ky[q] = c0 - hy[q] * IN;
  }
  float y[NY][8];
#pragma unroll
  for (int q = 0; q < NY; ++q)
#pragma unroll
    for (int j = 0; j < 8; ++j) y[q][j] = 0.f;
  float bsum[CPL][8];
#pragma unroll
  for (int q = 0; q < CPL; ++q)
#pragma unroll
    for (int j = 0; j < 8; ++j) bsum[q][j] = 0.f;
  for (int v = (blockIdx.x * kThreads + threadIdx.x) >> 5; v < n_dst; v += warps_total) {
    const int beg = a.indptr[v], end = a.indptr[v + 1];
    float go[CPL][8];
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c0 = (lane + 32 * q) * 8;
      if (!a.mean_heads && c0 + 8 <= HF) {
        float t[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.dout + static_cast<int64_t>(v) * a.lddo + c0), t);
#pragma unroll
        for (int j = 0; j < 8; ++j) go[q][j] = t[j];
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int c = c0 + j;
          float g = 0.f;
          if (c < HF) {
            const int col = a.mean_heads ? c % F : c;
            g = __bfloat162float(a.dout[static_cast<int64_t>(v) * a.lddo + col]) * inv_h;
          }
          go[q][j] = g;
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) bsum[q][j] += go[q][j];
    }
    float m = 0.f, s = 1.f, er_h = 0.f;
    if (lane < H) {
      m = a.smax[static_cast<int64_t>(v) * H + lane];
      s = a.ssum[static_cast<int64_t>(v) * H + lane];
      er_h = a.er[static_cast<int64_t>(v) * H + lane];
    }
    const float inv_s = 1.f / s;
    // The in-edges are taken 32 at a time: one coalesced load of their source ids,
    // broadcast by shuffles, so no row load waits behind an index load.
    // pass A: da per edge and head, S_h = sum a da, EU edges per iteration with all
    // their row loads issued together; in input-layer mode also y_v = sum a x_u
    float S = 0.f;
    for (int cb = beg; cb < end; cb += 32) {
      const int cnt = min(32, end - cb);
      const int my_idx = lane < cnt ? a.indices[cb + lane] : 0;
      for (int k = 0; k < cnt; k += EU) {
        int uu[EU];
        float elv[EU];
        uint4 zv[EU][CPL];
#pragma unroll
        for (int t = 0; t < EU; ++t) {
          uu[t] = __shfl_sync(0xffffffffu, my_idx, min(k + t, 31));
          const bool ok = k + t < cnt;
          elv[t] = 0.f;
          if (ok && lane < H) elv[t] = a.el[static_cast<int64_t>(uu[t]) * H + lane];
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            const int c0 = (lane + 32 * q) * 8;
            zv[t][q] = make_uint4(0, 0, 0, 0);
            if (ok && c0 < HF)
              zv[t][q] = *reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(uu[t]) * a.ldz + zcol(a, c0));
          }
        }
        uint4 xv[CPLY > 0 ? EU : 1][NY];
        if constexpr (CPLY > 0) {
#pragma unroll
          for (int t = 0; t < EU; ++t)
#pragma unroll
            for (int q = 0; q < CPLY; ++q) {
              const int c0 = (lane + 32 * q) * 8;
              xv[t][q] = make_uint4(0, 0, 0, 0);
              if (k + t < cnt && c0 < HIN)
                xv[t][q] = *reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(uu[t]) * a.ldx + ky[q]);
            }
        }
        float alv[EU];
#pragma unroll
        for (int t = 0; t < EU; ++t) {
          const float da = edge_head_dot<CPL, SEG>(go, zv[t], hm, lane, H, F, HF);
          alv[t] = 0.f;
          if (lane < H && k + t < cnt) {
            alv[t] = __expf(leaky(elv[t] + er_h, a.slope) - m) * inv_s;
            a.edge_scratch[static_cast<int64_t>(cb + k + t) * H + lane] = da;
            S += alv[t] * da;
          }
        }
        if constexpr (CPLY > 0) {
          // y_v[h, k] += a_uvh x_u[k]; an 8-column chunk of the [H, IN] row lies in one head
#pragma unroll
          for (int q = 0; q < CPLY; ++q) {
            const int c0 = (lane + 32 * q) * 8;
            float at[EU];
#pragma unroll
            for (int t = 0; t < EU; ++t) at[t] = __shfl_sync(0xffffffffu, alv[t], hy[q]);
            if (c0 >= HIN) continue;
#pragma unroll
            for (int t = 0; t < EU; ++t) {
              float f[8];
              bf16x8_to_f32(xv[t][q], f);
#pragma unroll
              for (int j = 0; j < 8; ++j) y[q][j] = fmaf(at[t], f[j], y[q][j]);
            }
          }
        }
      }
    }
    // pass B: score gradients and (dz mode) the transposed weighted sum.  Lane l
    // fetches the el row and the pass-A da values of edge l of the chunk (one round
    // trip for up to 32 edges); lane h takes those of head h by shuffles.
    float der_acc = 0.f;
    for (int cb = beg; cb < end; cb += 32) {
      const int cnt = min(32, end - cb);
      const int my_idx = lane < cnt ? a.indices[cb + lane] : 0;
      float elc[kMaxHeads], dac[kMaxHeads];
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h) elc[h] = dac[h] = 0.f;
      if (lane < cnt) {
        if (H == 4) {
          const float4 e4 = *reinterpret_cast<const float4*>(a.el + static_cast<int64_t>(my_idx) * 4);
          const float4 d4 = *reinterpret_cast<const float4*>(a.edge_scratch + static_cast<int64_t>(cb + lane) * 4);
          elc[0] = e4.x; elc[1] = e4.y; elc[2] = e4.z; elc[3] = e4.w;
          dac[0] = d4.x; dac[1] = d4.y; dac[2] = d4.z; dac[3] = d4.w;
        } else {
#pragma unroll
          for (int h = 0; h < kMaxHeads; ++h)
            if (h < H) {
              elc[h] = a.el[static_cast<int64_t>(my_idx) * H + h];
              dac[h] = a.edge_scratch[static_cast<int64_t>(cb + lane) * H + h];
            }
        }
      }
      for (int k = 0; k < cnt; ++k) {
        const int u = __shfl_sync(0xffffffffu, my_idx, k);
        float el_m = 0.f, da_m = 0.f;
#pragma unroll
        for (int h = 0; h < kMaxHeads; ++h) {
          if (h >= H) break;
          const float t1 = __shfl_sync(0xffffffffu, elc[h], k);
          const float t2 = __shfl_sync(0xffffffffu, dac[h], k);
          if (lane == h) {
            el_m = t1;
            da_m = t2;
          }
        }
        float al = 0.f;
        if (lane < H) {
          const float x = leaky(el_m + er_h, a.slope);
          al = __expf(x - m) * inv_s;
          const float de = al * (da_m - S);
          const float dx = x > 0.f ? de : de * a.slope;
          atomicAdd(a.del + static_cast<int64_t>(u) * H + lane, dx);
          der_acc += dx;
        }
        if (CPLY == 0 && a.dz) {
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            const int c0 = (lane + 32 * q) * 8;
            const float a0 = __shfl_sync(0xffffffffu, al, hm.h0[q]);
            float a1 = a0;
            if constexpr (!SEG) a1 = __shfl_sync(0xffffffffu, al, min(hm.h0[q] + 1, H - 1));
            if (c0 >= HF) continue;
            float tv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) tv[j] = (SEG || (c0 + j) / F == hm.h0[q] ? a0 : a1) * go[q][j];
            float* d = a.dz + static_cast<int64_t>(u) * a.lddz + c0;
            if (c0 + 8 <= HF) {
              red_add_v4f(d, tv[0], tv[1], tv[2], tv[3]);
              red_add_v4f(d + 4, tv[4], tv[5], tv[6], tv[7]);
            } else {
              for (int j = 0; j < 8 && c0 + j < HF; ++j) atomicAdd(d + j, tv[j]);
            }
          }
        }
      }
    }
    if (lane < H) a.der[static_cast<int64_t>(v) * H + lane] = der_acc;
    if constexpr (CPLY > 0) {
#pragma unroll
      for (int q = 0; q < CPLY; ++q) {
        const int c0 = (lane + 32 * q) * 8;
        if (c0 < HIN)
          *reinterpret_cast<uint4*>(a.y + static_cast<int64_t>(v) * a.ldy + c0) = f32_to_bf16x8(y[q]);
#pragma unroll
        for (int j = 0; j < 8; ++j) y[q][j] = 0.f;
      }
    }
  }
  if (a.dbias) block_col_atomic<CPL>(bsum, a.dbias, HF);
}

// ------------------------------------------------------------------ backward, per source
// A streaming pass over the source rows, kNodeRows rows per warp iteration with every
// load of the iteration issued before the first use (the kernel is latency-bound:
// a few KB per warp in flight is what keeps HBM busy).  dz mode: dz_u += del a_l +
// der a_r, staged to bf16 and cleared; input-layer mode (CPLY > 0): the xl / xr row
// reductions instead.  Both: the attention-vector gradients da_l += del z,
// da_r += der z.  del is cleared for the next step after its rows are consumed.
constexpr int kNodeRows = 4;

template <int CPL, int CPLY, bool SEG, int MINB = 0>
__global__ void __launch_bounds__(kThreads, MINB > 0 ? MINB : 1) gat_bwd_node_kernel(GatArgs a) {
  GB_PDL_ENTRY();
  const int n_src = a.n_src_ptr ? min(*a.n_src_ptr, a.cap_src) : a.cap_src;
  const int n_dst = a.n_dst_ptr ? min(*a.n_dst_ptr, a.cap_dst) : a.cap_dst;
  const int H = a.heads, F = a.feat, HF = H * F;
  const int IN = a.in_dim, HIN = H * a.in_dim;
  const int lane = threadIdx.x & 31;
  const int warps_total = (gridDim.x * kThreads) >> 5;
  const HeadMap hm = head_map<CPL, SEG>(lane, H, F);
  constexpr bool DZ = CPLY == 0;
  constexpr int NY = CPLY > 0 ? CPLY : 1;
  constexpr int R = kNodeRows;
  const int rows_end =
      DZ && a.zero_tail_rows > 0
          ? min(a.cap_src, static_cast<int>(ceil_div(n_src, a.zero_tail_rows) * a.zero_tail_rows))
          : n_src;
  int hy[NY], ky[NY];
#pragma unroll
  for (int q = 0; q < NY; ++q) {
    const int c0 = (lane + 32 * q) * 8;
    hy[q] = CPLY > 0 ? min(c0 / max(IN, 1), H - 1) : 0;
    ky[q] = c0 - hy[q] * IN;
  }
  // z is read only for the attention-vector gradients (da_l = sum del z); the input
  // layer gets them as W xl instead (gat_in_dw) and passes none
  const bool want_g = a.dattn_l || a.dattn_r;
  float gl[CPL][8], gr[CPL][8], xl[NY][8], xr[NY][8];
#pragma unroll
  for (int q = 0; q < CPL; ++q)
#pragma unroll
    for (int j = 0; j < 8; ++j) gl[q][j] = gr[q][j] = 0.f;
#pragma unroll
  for (int q = 0; q < NY; ++q)
#pragma unroll
    for (int j = 0; j < 8; ++j) xl[q][j] = xr[q][j] = 0.f;
  const int first = (blockIdx.x * kThreads + threadIdx.x) >> 5;
  for (int u0 = R * first; u0 < rows_end; u0 += R * warps_total) {
    // ---- loads of the R rows
    float dl[R], dr[R];
    uint4 zv[R][CPL];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int u = u0 + i;
      dl[i] = dr[i] = 0.f;
      if (lane < H && u < n_src) {
        dl[i] = a.del[static_cast<int64_t>(u) * H + lane];
        if (u < n_dst) dr[i] = a.der[static_cast<int64_t>(u) * H + lane];
      }
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c0 = (lane + 32 * q) * 8;
        zv[i][q] = make_uint4(0, 0, 0, 0);
        if (want_g && u < n_src && c0 < HF)
          zv[i][q] = *reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(u) * a.ldz + zcol(a, c0));
      }
    }
    float4 dv[DZ ? R : 1][CPL][2];
    uint4 xv[DZ ? 1 : R][NY];
    if constexpr (DZ) {
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int q = 0; q < CPL; ++q) {
          const int c0 = (lane + 32 * q) * 8;
          const float* d = a.dz + static_cast<int64_t>(u0 + i) * a.lddz + c0;
          dv[i][q][0] = dv[i][q][1] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (a.dz && u0 + i < n_src && c0 < HF) {
            if (c0 + 8 <= HF) {
              dv[i][q][0] = *reinterpret_cast<const float4*>(d);
              dv[i][q][1] = *reinterpret_cast<const float4*>(d + 4);
            } else {
              float t[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
              for (int j = 0; j < 8 && c0 + j < HF; ++j) t[j] = d[j];
              dv[i][q][0] = make_float4(t[0], t[1], t[2], t[3]);
              dv[i][q][1] = make_float4(t[4], t[5], t[6], t[7]);
            }
          }
        }
    } else {
#pragma unroll
      for (int i = 0; i < R; ++i)
#pragma unroll
        for (int q = 0; q < NY; ++q) {
          const int c0 = (lane + 32 * q) * 8;
          xv[i][q] = make_uint4(0, 0, 0, 0);
          if (u0 + i < n_src && c0 < HIN)
            xv[i][q] = *reinterpret_cast<const uint4*>(a.x + static_cast<int64_t>(u0 + i) * a.ldx + ky[q]);
        }
    }
    // ---- arithmetic and stores
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int u = u0 + i;
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c0 = (lane + 32 * q) * 8;
        const int ha = hm.h0[q];
        const float dla = __shfl_sync(0xffffffffu, dl[i], ha), dra = __shfl_sync(0xffffffffu, dr[i], ha);
        float dlb = dla, drb = dra;
        if constexpr (!SEG) {
          const int hb = min(ha + 1, H - 1);
          dlb = __shfl_sync(0xffffffffu, dl[i], hb);
          drb = __shfl_sync(0xffffffffu, dr[i], hb);
        }
        if (u >= rows_end) continue;
        if (DZ && a.dz_bf16 && c0 >= a.lddzb) continue;
        float o[8];
        if (u < n_src && c0 < HF) {
          float zf[8];
          bf16x8_to_f32(zv[i][q], zf);
          float dvf[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          if constexpr (DZ) {
            *reinterpret_cast<float4*>(dvf) = dv[i][q][0];
            *reinterpret_cast<float4*>(dvf + 4) = dv[i][q][1];
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const bool fa = SEG || (c0 + j) / F == ha;
            const float cl = fa ? dla : dlb, cr = fa ? dra : drb;
            gl[q][j] = fmaf(cl, zf[j], gl[q][j]);
            gr[q][j] = fmaf(cr, zf[j], gr[q][j]);
            if constexpr (DZ) {
              const bool in = c0 + j < HF;
              o[j] = in ? dvf[j] + cl * __ldg(a.attn_l + min(c0 + j, HF - 1)) +
                              cr * __ldg(a.attn_r + min(c0 + j, HF - 1))
                        : 0.f;
            }
          }
          if (DZ && a.dz) {
            float* d = a.dz + static_cast<int64_t>(u) * a.lddz + c0;
            if (c0 + 8 <= HF) {
              *reinterpret_cast<float4*>(d) = make_float4(0.f, 0.f, 0.f, 0.f);
              *reinterpret_cast<float4*>(d + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
              for (int j = 0; j < 8 && c0 + j < HF; ++j) d[j] = 0.f;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = 0.f;
        }
        if (DZ && a.dz_bf16) *reinterpret_cast<uint4*>(a.dz_bf16 + static_cast<int64_t>(u) * a.lddzb + c0) = f32_to_bf16x8(o);
      }
      if constexpr (!DZ) {
#pragma unroll
        for (int q = 0; q < NY; ++q) {
          const int c0 = (lane + 32 * q) * 8;
          const float dlq = __shfl_sync(0xffffffffu, dl[i], hy[q]), drq = __shfl_sync(0xffffffffu, dr[i], hy[q]);
          if (u >= n_src || c0 >= HIN) continue;
          float f[8];
          bf16x8_to_f32(xv[i][q], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            xl[q][j] = fmaf(dlq, f[j], xl[q][j]);
            xr[q][j] = fmaf(drq, f[j], xr[q][j]);
          }
        }
      }
      if (lane < H && u < n_src) a.del[static_cast<int64_t>(u) * H + lane] = 0.f;
    }
  }
  if (a.dattn_l) block_col_atomic<CPL>(gl, a.dattn_l, HF);
  if (a.dattn_r) block_col_atomic<CPL>(gr, a.dattn_r, HF);
  if constexpr (!DZ) {
    block_col_atomic<NY>(xl, a.xl, HIN);
    block_col_atomic<NY>(xr, a.xr, HIN);
  }
}

// dW[r, k] += T[r, h * IN + k] + a_l[r] xl[h, k] + a_r[r] xr[h, k], h = r / F
__global__ void gat_dw_combine_kernel(const float* T, int64_t ldt, const float* xl, const float* xr,
                                      const float* attn_l, const float* attn_r, int H, int F, int IN, float* dw,
                                      int64_t ldw) {
  GB_PDL_ENTRY();
  const int total = H * F * IN;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int r = i / IN, k = i % IN, h = r / F;
    dw[static_cast<int64_t>(r) * ldw + k] +=
        T[static_cast<int64_t>(r) * ldt + h * IN + k] + attn_l[r] * xl[h * IN + k] + attn_r[r] * xr[h * IN + k];
  }
}

// wl/wr (fp32 [H * IN]) and the block-diagonal Wbd (bf16 [rows, H * IN]) of the input
// layer's projection-after-aggregation form (see launch_gat_in_prep)
__global__ void gat_in_prep_kernel(const __nv_bfloat16* w, int64_t ldw, const float* attn_l, const float* attn_r,
                                   int H, int F, int IN, int rows, float* wl, float* wr, __nv_bfloat16* wbd,
                                   int64_t ldwbd) {
  GB_PDL_ENTRY();
  const int HIN = H * IN;
  const int64_t total = static_cast<int64_t>(rows) * HIN;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total + 2 * HIN;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    if (i < total) {
      const int r = static_cast<int>(i / HIN), c = static_cast<int>(i % HIN);
      const int h = c / IN, k = c % IN;
      const bool on = r < H * F && r / F == h;
      wbd[static_cast<int64_t>(r) * ldwbd + c] = on ? w[static_cast<int64_t>(r) * ldw + k] : __float2bfloat16_rn(0.f);
    } else {
      const int j = static_cast<int>(i - total);  // [0, 2 HIN)
      const bool left = j < HIN;
      const int c = left ? j : j - HIN;
      const int h = c / IN, k = c % IN;
      const float* av = left ? attn_l : attn_r;
      float t = 0.f;
      for (int f = 0; f < F; ++f)
        t += __bfloat162float(w[static_cast<int64_t>(h * F + f) * ldw + k]) * av[h * F + f];
      (left ? wl : wr)[c] = t;
    }
  }
}

// dW[r, k] += T[r, h*IN + k] + a_l[r] xl[h, k] + a_r[r] xr[h, k] for r < H*F (h = r / F);
// dattn_l[r] += W[r, :] . xl[h, :], dattn_r[r] += W[r, :] . xr[h, :]
__global__ void gat_in_dw_kernel(const float* T, int64_t ldt, const float* xl, const float* xr, const float* attn_l,
                                 const float* attn_r, const float* w, int64_t ldw_in, int H, int F, int IN, float* dw,
                                 int64_t ldw, float* dattn_l, float* dattn_r) {
  GB_PDL_ENTRY();
  const int HF = H * F;
  const int total = HF * IN;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int r = i / IN, k = i % IN, h = r / F;
    dw[static_cast<int64_t>(r) * ldw + k] +=
        T[static_cast<int64_t>(r) * ldt + h * IN + k] + attn_l[r] * xl[h * IN + k] + attn_r[r] * xr[h * IN + k];
  }
  if (!dattn_l && !dattn_r) return;
  // da_l[r] += W[r, :] . xl[h], one warp per row (lanes split the row, then a warp sum)
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < HF; r += warps) {
    const int h = r / F;
    float tl = 0.f, tr = 0.f;
    for (int k = lane; k < IN; k += 32) {
      const float wv = w[static_cast<int64_t>(r) * ldw_in + k];
      tl = fmaf(wv, xl[h * IN + k], tl);
      tr = fmaf(wv, xr[h * IN + k], tr);
    }
    tl = warp_sum(tl);
    tr = warp_sum(tr);
    if (lane == 0) {
      if (dattn_l) dattn_l[r] += tl;
      if (dattn_r) dattn_r[r] += tr;
    }
  }
}

// out[c] += sum over live rows of x[r, c]: one thread per column, rows split over blocks
__global__ void col_sum_bf16_kernel(const __nv_bfloat16* x, int64_t ldx, const int32_t* n_ptr, int cap_rows, int cols,
                                    float* out) {
  GB_PDL_ENTRY();
  const int n = n_ptr ? min(*n_ptr, cap_rows) : cap_rows;
  const int rows_per = (n + gridDim.y - 1) / gridDim.y;
  const int r0 = blockIdx.y * rows_per, r1 = min(n, r0 + rows_per);
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x) {
    float t = 0.f;
    for (int r = r0; r < r1; ++r) t += __bfloat162float(x[static_cast<int64_t>(r) * ldx + c]);
    if (t != 0.f) atomicAdd(out + c, t);
  }
}

int cpl_for(int hf) { return (hf + 255) / 256; }

void check(const GatArgs& a) {
  if (a.heads <= 0 || a.heads > kMaxHeads) throw std::invalid_argument("gat: 1..8 heads");
  if (a.zmod > 0 && (a.zmod != a.feat || a.zmod % 8 != 0))
    throw std::invalid_argument("gat: shared-row mode needs feat == zmod, a multiple of 8");
  const int hf = a.heads * a.feat;
  if (hf > 1024) throw std::invalid_argument("gat: heads * feat <= 1024");
  if (a.ldz % 8 != 0) throw std::invalid_argument("gat: z stride % 8");
}

}  // namespace

#define GAT_DISPATCH(KERNEL, GRID, SMEM)                                               \
  do {                                                                                 \
    const int cpl = cpl_for(a.heads * a.feat);                                         \
    if (cpl <= 1) launch_k(KERNEL<1>, GRID, kThreads, SMEM, stream, a);                      \
    else if (cpl <= 2) launch_k(KERNEL<2>, GRID, kThreads, SMEM, stream, a);                 \
    else launch_k(KERNEL<4>, GRID, kThreads, SMEM, stream, a);                               \
    GB_LAUNCH_CHECK();                                                                 \
  } while (0)

// GRAPPA_GAT_OCC = 2 (default) or 3: the forward (3 CTAs per SM) and the backward node
// pass (2; with 3 also the edge pass) of the common shapes (one 8-column chunk per
// lane) capped in registers for occupancy; 0: the registers the compiler picks.  On the
// 111M-node GAT workload: 0.938 s/epoch with 0, 0.855 with 2, 1.139 with 3 (spills).
static int gat_occ() {
  static const int v = [] {
    const char* e = std::getenv("GRAPPA_GAT_OCC");
    return e ? std::atoi(e) : 2;
  }();
  return v;
}

void launch_gat_scores(const GatArgs& a, cudaStream_t stream) {
  check(a);
  GAT_DISPATCH(gat_scores_kernel, grid_warps(a.cap_src), 0);
}

void launch_gat_fwd(const GatArgs& a, cudaStream_t stream) {
  check(a);
  if (a.ldo % 8 != 0) throw std::invalid_argument("gat: out stride % 8");
  if (a.dropout_p > 0.f && !a.counters) throw std::invalid_argument("gat: dropout needs the step counters");
  const size_t smem = a.mean_heads ? (kThreads / 32) * a.heads * a.feat * sizeof(float) : 0;
  const int grid = grid_warps(a.cap_dst);
  const int cpl = cpl_for(a.heads * a.feat);
#define GAT_FWD(C)                                                                      \
  do {                                                                                  \
    if (a.heads <= 4) launch_k(gat_fwd_kernel<C, 4>, grid, kThreads, smem, stream, a);        \
    else launch_k(gat_fwd_kernel<C, kMaxHeads>, grid, kThreads, smem, stream, a);            \
  } while (0)
  // variants of the common case (<= 4 heads, H * F <= 256) picked by GRAPPA_GAT_FWD
  // ("eu,minb": 4,1 default; 8,1; 4,3; 8,2)
  static const int variant = [] {
    const char* e = std::getenv("GRAPPA_GAT_FWD");
    if (!e) return 0;
    const std::string v(e);
    return v == "8,1" ? 1 : v == "4,3" ? 2 : v == "8,2" ? 3 : 0;
  }();
  const int occ = gat_occ();
  if (cpl <= 1 && a.heads <= 4 && variant > 0) {
    if (variant == 1) launch_k(gat_fwd_kernel<1, 4, 8, 1>, grid, kThreads, smem, stream, a);
    else if (variant == 2) launch_k(gat_fwd_kernel<1, 4, 4, 3>, grid, kThreads, smem, stream, a);
    else launch_k(gat_fwd_kernel<1, 4, 8, 2>, grid, kThreads, smem, stream, a);
  } else if (cpl <= 1 && a.heads <= 4 && occ >= 2) {
    // register cap for 3 CTAs per SM; heads of a multiple of 8 columns skip the head picks
    if (a.feat % 8 == 0) launch_k(gat_fwd_kernel<1, 4, 4, 3, true>, grid, kThreads, smem, stream, a);
    else launch_k(gat_fwd_kernel<1, 4, 4, 3>, grid, kThreads, smem, stream, a);
  } else if (cpl <= 1) GAT_FWD(1);
  else if (cpl <= 2) GAT_FWD(2);
  else GAT_FWD(4);
#undef GAT_FWD
  GB_LAUNCH_CHECK();
}

bool seg_heads(int F) { return F >= 8 && F <= 256 && (F & (F - 1)) == 0; }

// EMB / NMB: CTAs per SM the edge / node pass registers are capped for (0: default)
template <int CPL, int CPLY, bool SEG, int EMB, int NMB>
void gat_bwd_launch(const GatArgs& a, cudaStream_t stream) {
  constexpr int mb = EMB > 0 ? EMB : bwd_min_blocks<CPL, CPLY>();
  launch_k(gat_bwd_edge_kernel<CPL, CPLY, SEG, EMB>, grid_warps(a.cap_dst, mb), kThreads, 0, stream, a);
  GB_LAUNCH_CHECK();
  launch_k(gat_bwd_node_kernel<CPL, CPLY, SEG, NMB>,
           grid_warps(static_cast<int>(ceil_div(a.cap_src, kNodeRows)), NMB > 0 ? NMB : 1), kThreads, 0, stream, a);
  GB_LAUNCH_CHECK();
}

template <int CPL, int CPLY, bool SEG>
void gat_bwd_pair(const GatArgs& a, cudaStream_t stream) {
  // one 8-column chunk per lane: the node pass capped for 2 CTAs per SM (128 registers
  // instead of 178-184); with GRAPPA_GAT_OCC=3 both passes for 3
  if constexpr (CPL == 1 && SEG && (CPLY == 0 || CPLY == 2)) {
    const int occ = gat_occ();
    if (occ == 2) return gat_bwd_launch<CPL, CPLY, SEG, 0, 2>(a, stream);
    if (occ >= 3) return gat_bwd_launch<CPL, CPLY, SEG, 3, 3>(a, stream);
  }
  if constexpr (CPL == 4 && !SEG && CPLY == 0) {
    // wide last layer (H * F up to 1024): GRAPPA_GAT_OCC_LAST=2 caps its edge pass for
    // 2 CTAs per SM (219 -> 128 registers)
    static const int last = [] {
      const char* e = std::getenv("GRAPPA_GAT_OCC_LAST");
      return e ? std::atoi(e) : 0;
    }();
    if (last == 2) return gat_bwd_launch<CPL, CPLY, SEG, 2, 0>(a, stream);
  }
  gat_bwd_launch<CPL, CPLY, SEG, 0, 0>(a, stream);
}

template <int CPLY>
void gat_bwd_cpl(const GatArgs& a, cudaStream_t stream) {
  const int cpl = cpl_for(a.heads * a.feat);
  const bool seg = seg_heads(a.feat);
  if (cpl <= 1) seg ? gat_bwd_pair<1, CPLY, true>(a, stream) : gat_bwd_pair<1, CPLY, false>(a, stream);
  else if (cpl <= 2) seg ? gat_bwd_pair<2, CPLY, true>(a, stream) : gat_bwd_pair<2, CPLY, false>(a, stream);
  else seg ? gat_bwd_pair<4, CPLY, true>(a, stream) : gat_bwd_pair<4, CPLY, false>(a, stream);
}

void launch_gat_bwd(const GatArgs& a, cudaStream_t stream) {
  check(a);
  if (a.lddz % 4 != 0 || a.lddzb % 8 != 0) throw std::invalid_argument("gat: gradient strides");
  if (!a.mean_heads && a.lddo % 8 != 0) throw std::invalid_argument("gat: dout stride % 8");
  gat_bwd_cpl<0>(a, stream);
}

void launch_gat_bwd_input(const GatArgs& a, cudaStream_t stream) {
  check(a);
  if (a.mean_heads) throw std::invalid_argument("gat input-layer backward: hidden layers only");
  if (a.in_dim <= 0 || a.in_dim % 8 != 0 || a.ldx % 8 != 0 || a.ldy % 8 != 0)
    throw std::invalid_argument("gat input-layer backward: in_dim and strides must be multiples of 8");
  const int hin = a.heads * a.in_dim;
  if (hin > 1024) throw std::invalid_argument("gat input-layer backward: heads * in <= 1024");
  if (!a.x || !a.y || !a.xl || !a.xr) throw std::invalid_argument("gat input-layer backward: x, y, xl, xr needed");
  if (a.lddo % 8 != 0) throw std::invalid_argument("gat: dout stride % 8");
  const int cply = cpl_for(hin);
  if (cply <= 1) gat_bwd_cpl<1>(a, stream);
  else if (cply <= 2) gat_bwd_cpl<2>(a, stream);
  else gat_bwd_cpl<4>(a, stream);
}

void launch_gat_in_prep(const __nv_bfloat16* w, int64_t ldw, const float* attn_l, const float* attn_r, int heads,
                        int feat, int in_dim, int rows, float* wl, float* wr, __nv_bfloat16* wbd, int64_t ldwbd,
                        cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(rows) * heads * in_dim + 2 * heads * in_dim;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(total, 256), sms() * 4)));
  launch_k(gat_in_prep_kernel, grid, 256, 0, stream, w, ldw, attn_l, attn_r, heads, feat, in_dim, rows, wl, wr, wbd, ldwbd);
  GB_LAUNCH_CHECK();
}

void launch_gat_in_dw(const float* T, int64_t ldt, const float* xl, const float* xr, const float* attn_l,
                      const float* attn_r, const float* w, int64_t ldw_in, int heads, int feat, int in_dim, float* dw,
                      int64_t ldw, float* dattn_l, float* dattn_r, cudaStream_t stream) {
  const int total = std::max(heads * feat * in_dim, heads * feat * 32);
  const int grid = std::max(1, std::min((total + 255) / 256, sms() * 4));
  launch_k(gat_in_dw_kernel, grid, 256, 0, stream, T, ldt, xl, xr, attn_l, attn_r, w, ldw_in, heads, feat, in_dim, dw, ldw,
                                             dattn_l, dattn_r);
  GB_LAUNCH_CHECK();
}

void launch_col_sum_bf16(const __nv_bfloat16* x, int64_t ldx, const int32_t* n_ptr, int cap_rows, int cols, float* out,
                         cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>(std::max(1, (cols + 255) / 256)),
                  static_cast<unsigned>(std::max(1, std::min(sms() * 2, (cap_rows + 255) / 256))));
  launch_k(col_sum_bf16_kernel, grid, 256, 0, stream, x, ldx, n_ptr, cap_rows, cols, out);
  GB_LAUNCH_CHECK();
}

void launch_gat_dw_combine(const float* T, int64_t ldt, const float* xl, const float* xr, const float* attn_l,
                           const float* attn_r, int heads, int feat, int in_dim, float* dw, int64_t ldw,
                           cudaStream_t stream) {
  const int total = heads * feat * in_dim;
  const int grid = std::max(1, std::min((total + 255) / 256, sms() * 4));
  launch_k(gat_dw_combine_kernel, grid, 256, 0, stream, T, ldt, xl, xr, attn_l, attn_r, heads, feat, in_dim, dw, ldw);
  GB_LAUNCH_CHECK();
}

}  // namespace dev
}  // namespace grappa
