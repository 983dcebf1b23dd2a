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
#include <algorithm>

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

// Column sums of per-lane partials (lane owns columns (lane + 32 q) * 8 + j, the
// same in every warp) over the block's warps in shared memory, then one atomic per
// column per block: the column gradients (bias, attention vectors) would otherwise
// take one contended atomic per warp and column.  Called by every thread.
template <int CPL>
__device__ void block_col_atomic(const float (&v)[CPL][8], float* dst, int HF) {
  __shared__ float s[kThreads / 32][1024];
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
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(r) * a.ldz + c0), f);
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
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(r) * a.ldz + c0), f);
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
template <int CPL>
__global__ void __launch_bounds__(kThreads) gat_fwd_kernel(GatArgs a) {
  extern __shared__ float s_row[];  // mean_heads: [warps][HF]
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
    thr = static_cast<uint32_t>(static_cast<double>(a.dropout_p) * 4294967296.0);
    ks = 1.f / (1.f - a.dropout_p);
  }
  for (int v = (blockIdx.x * kThreads + threadIdx.x) >> 5; v < rows_end; v += warps_total) {
    if (v >= n_dst) {
      for (int c = lane * 8; c < a.ldo; c += 256)
        *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(v) * a.ldo + c) = make_uint4(0, 0, 0, 0);
      continue;
    }
    const int beg = a.indptr[v], end = a.indptr[v + 1];
    // pass 1: lane h owns head h
    float m = -INFINITY, s = 0.f, er_h = 0.f;
    if (lane < H) {
      er_h = a.er[static_cast<int64_t>(v) * H + lane];
      for (int e = beg; e < end; ++e) {
        const int u = a.indices[e];
        const float x = leaky(a.el[static_cast<int64_t>(u) * H + lane] + er_h, a.slope);
        if (x > m) {
          s = s * __expf(m - x) + 1.f;
          m = x;
        } else {
          s += __expf(x - m);
        }
      }
      a.smax[static_cast<int64_t>(v) * H + lane] = m;
      a.ssum[static_cast<int64_t>(v) * H + lane] = s;
    }
    // pass 2: weighted sum of z rows
    float acc[CPL][8];
    int h0[CPL];
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      h0[q] = min(((lane + 32 * q) * 8) / F, H - 1);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[q][j] = 0.f;
    }
    for (int e = beg; e < end; ++e) {
      const int u = a.indices[e];
      // attention of every head for this edge, computed by lane h and broadcast
      float al = 0.f;
      if (lane < H) {
        const float x = leaky(a.el[static_cast<int64_t>(u) * H + lane] + er_h, a.slope);
        al = __expf(x - m) / s;
      }
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c0 = (lane + 32 * q) * 8;
        const float a0 = __shfl_sync(0xffffffffu, al, h0[q]);
        const float a1 = __shfl_sync(0xffffffffu, al, min(h0[q] + 1, H - 1));
        if (c0 >= HF) continue;
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(u) * a.ldz + c0), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int h = (c0 + j) / F;
          acc[q][j] += (h == h0[q] ? a0 : a1) * f[j];
        }
      }
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
          float x = c < HF ? acc[q][j] + a.bias[c] : 0.f;
          if (a.act == 1) x = fmaxf(x, 0.f);
          o[j] = x;
        }
        if (a.dropout_p > 0.f) {
          const uint64_t base = static_cast<uint64_t>(v) * static_cast<uint64_t>(a.ldo) + static_cast<uint64_t>(c0);
          const U4 r0 = index_draw4(key, base >> 2, 0);
          const U4 r1 = index_draw4(key, (base >> 2) + 1, 0);
          const uint32_t w[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = w[j] >= thr ? o[j] * ks : 0.f;
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
          if (c0 + j < HF) row[c0 + j] = acc[q][j] + a.bias[c0 + j];
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
template <int CPL>
__global__ void __launch_bounds__(kThreads) gat_bwd_edge_kernel(GatArgs a) {
  const int n_dst = a.n_dst_ptr ? min(*a.n_dst_ptr, a.cap_dst) : a.cap_dst;
  const int H = a.heads, F = a.feat, HF = H * F;
  const int lane = threadIdx.x & 31;
  const int warps_total = (gridDim.x * kThreads) >> 5;
  const float inv_h = a.mean_heads ? 1.f / static_cast<float>(H) : 1.f;
  float bsum[CPL][8];
#pragma unroll
  for (int q = 0; q < CPL; ++q)
#pragma unroll
    for (int j = 0; j < 8; ++j) bsum[q][j] = 0.f;
  for (int v = (blockIdx.x * kThreads + threadIdx.x) >> 5; v < n_dst; v += warps_total) {
    const int beg = a.indptr[v], end = a.indptr[v + 1];
    float go[CPL][8];
    int h0[CPL];
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c0 = (lane + 32 * q) * 8;
      h0[q] = min(c0 / F, H - 1);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + j;
        float g = 0.f;
        if (c < HF) {
          const int col = a.mean_heads ? c % F : c;
          g = __bfloat162float(a.dout[static_cast<int64_t>(v) * a.lddo + col]) * inv_h;
        }
        go[q][j] = g;
        bsum[q][j] += g;
      }
    }
    float m = 0.f, s = 1.f, er_h = 0.f;
    if (lane < H) {
      m = a.smax[static_cast<int64_t>(v) * H + lane];
      s = a.ssum[static_cast<int64_t>(v) * H + lane];
      er_h = a.er[static_cast<int64_t>(v) * H + lane];
    }
    // pass A: da per edge and head, S_h = sum a da
    float S = 0.f;
    for (int e = beg; e < end; ++e) {
      const int u = a.indices[e];
      float p[kMaxHeads];
#pragma unroll
      for (int h = 0; h < kMaxHeads; ++h) p[h] = 0.f;
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c0 = (lane + 32 * q) * 8;
        if (c0 >= HF) continue;
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(u) * a.ldz + c0), f);
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
      if (lane < H) {
        const float x = leaky(a.el[static_cast<int64_t>(u) * H + lane] + er_h, a.slope);
        const float al = __expf(x - m) / s;
        a.edge_scratch[static_cast<int64_t>(e) * H + lane] = da_mine;
        S += al * da_mine;
      }
    }
    // pass B: score gradients and the transposed weighted sum
    float der_acc = 0.f;
    for (int e = beg; e < end; ++e) {
      const int u = a.indices[e];
      float al = 0.f;
      if (lane < H) {
        const float x = leaky(a.el[static_cast<int64_t>(u) * H + lane] + er_h, a.slope);
        al = __expf(x - m) / s;
        const float de = al * (a.edge_scratch[static_cast<int64_t>(e) * H + lane] - S);
        const float dx = x > 0.f ? de : de * a.slope;
        atomicAdd(a.del + static_cast<int64_t>(u) * H + lane, dx);
        der_acc += dx;
      }
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c0 = (lane + 32 * q) * 8;
        const float a0 = __shfl_sync(0xffffffffu, al, h0[q]);
        const float a1 = __shfl_sync(0xffffffffu, al, min(h0[q] + 1, H - 1));
        if (c0 >= HF) continue;
        float t[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) t[j] = ((c0 + j) / F == h0[q] ? a0 : a1) * go[q][j];
        float* d = a.dz + static_cast<int64_t>(u) * a.lddz + c0;
        if (c0 + 8 <= HF) {
          red_add_v4f(d, t[0], t[1], t[2], t[3]);
          red_add_v4f(d + 4, t[4], t[5], t[6], t[7]);
        } else {
          for (int j = 0; j < 8 && c0 + j < HF; ++j) atomicAdd(d + j, t[j]);
        }
      }
    }
    if (lane < H) a.der[static_cast<int64_t>(v) * H + lane] = der_acc;
  }
  if (a.dbias) block_col_atomic<CPL>(bsum, a.dbias, HF);
}

// ------------------------------------------------------------------ backward, per source
template <int CPL>
__global__ void __launch_bounds__(kThreads) gat_bwd_node_kernel(GatArgs a) {
  const int n_src = a.n_src_ptr ? min(*a.n_src_ptr, a.cap_src) : a.cap_src;
  const int n_dst = a.n_dst_ptr ? min(*a.n_dst_ptr, a.cap_dst) : a.cap_dst;
  const int H = a.heads, F = a.feat, HF = H * F;
  const int lane = threadIdx.x & 31;
  const int warps_total = (gridDim.x * kThreads) >> 5;
  const int rows_end = a.zero_tail_rows > 0 ? min(a.cap_src, static_cast<int>(ceil_div(n_src, a.zero_tail_rows) * a.zero_tail_rows)) : n_src;
  float gl[CPL][8], gr[CPL][8];
#pragma unroll
  for (int q = 0; q < CPL; ++q)
#pragma unroll
    for (int j = 0; j < 8; ++j) gl[q][j] = gr[q][j] = 0.f;
  for (int u = (blockIdx.x * kThreads + threadIdx.x) >> 5; u < rows_end; u += warps_total) {
    if (u >= n_src) {
      for (int c = lane * 8; c < a.lddzb; c += 256)
        *reinterpret_cast<uint4*>(a.dz_bf16 + static_cast<int64_t>(u) * a.lddzb + c) = make_uint4(0, 0, 0, 0);
      continue;
    }
    float dl = 0.f, dr = 0.f;
    if (lane < H) {
      float* pl = a.del + static_cast<int64_t>(u) * H + lane;
      dl = *pl;
      *pl = 0.f;
      if (u < n_dst) dr = a.der[static_cast<int64_t>(u) * H + lane];
    }
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c0 = (lane + 32 * q) * 8;
      const int ha = min(c0 / F, H - 1);
      const int hb = min(ha + 1, H - 1);
      const float dla = __shfl_sync(0xffffffffu, dl, ha), dlb = __shfl_sync(0xffffffffu, dl, hb);
      const float dra = __shfl_sync(0xffffffffu, dr, ha), drb = __shfl_sync(0xffffffffu, dr, hb);
      if (c0 >= a.lddzb) continue;
      float o[8];
      if (c0 < HF) {
        // all loads of the chunk first (16-byte vectors), then the arithmetic, then the
        // stores: no load waits behind a store that might alias it
        float zf[8], dv[8], al[8], ar[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.z + static_cast<int64_t>(u) * a.ldz + c0), zf);
        float* d = a.dz + static_cast<int64_t>(u) * a.lddz + c0;
        const bool full = c0 + 8 <= HF;
        if (full) {
          *reinterpret_cast<float4*>(dv) = *reinterpret_cast<const float4*>(d);
          *reinterpret_cast<float4*>(dv + 4) = *reinterpret_cast<const float4*>(d + 4);
          *reinterpret_cast<float4*>(al) = __ldg(reinterpret_cast<const float4*>(a.attn_l + c0));
          *reinterpret_cast<float4*>(al + 4) = __ldg(reinterpret_cast<const float4*>(a.attn_l + c0 + 4));
          *reinterpret_cast<float4*>(ar) = __ldg(reinterpret_cast<const float4*>(a.attn_r + c0));
          *reinterpret_cast<float4*>(ar + 4) = __ldg(reinterpret_cast<const float4*>(a.attn_r + c0 + 4));
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const bool in = c0 + j < HF;
            dv[j] = in ? d[j] : 0.f;
            al[j] = in ? a.attn_l[c0 + j] : 0.f;
            ar[j] = in ? a.attn_r[c0 + j] : 0.f;
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int c = c0 + j;
          const bool first = c / F == ha;
          const float cl = first ? dla : dlb, cr = first ? dra : drb;
          o[j] = c < HF ? dv[j] + cl * al[j] + cr * ar[j] : 0.f;
          if (c < HF) {
            gl[q][j] += cl * zf[j];
            gr[q][j] += cr * zf[j];
          }
        }
        if (full) {
          *reinterpret_cast<float4*>(d) = make_float4(0.f, 0.f, 0.f, 0.f);
          *reinterpret_cast<float4*>(d + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
          for (int j = 0; j < 8 && c0 + j < HF; ++j) d[j] = 0.f;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = 0.f;
      }
      *reinterpret_cast<uint4*>(a.dz_bf16 + static_cast<int64_t>(u) * a.lddzb + c0) = f32_to_bf16x8(o);
    }
  }
  if (a.dattn_l) block_col_atomic<CPL>(gl, a.dattn_l, HF);
  if (a.dattn_r) block_col_atomic<CPL>(gr, a.dattn_r, HF);
}

int cpl_for(int hf) { return (hf + 255) / 256; }

void check(const GatArgs& a) {
  if (a.heads <= 0 || a.heads > kMaxHeads) throw std::invalid_argument("gat: 1..8 heads");
  const int hf = a.heads * a.feat;
  if (hf > 1024) throw std::invalid_argument("gat: heads * feat <= 1024");
  if (a.ldz % 8 != 0) throw std::invalid_argument("gat: z stride % 8");
}

}  // namespace

#define GAT_DISPATCH(KERNEL, GRID, SMEM)                                               \
  do {                                                                                 \
    const int cpl = cpl_for(a.heads * a.feat);                                         \
    if (cpl <= 1) KERNEL<1><<<GRID, kThreads, SMEM, stream>>>(a);                      \
    else if (cpl <= 2) KERNEL<2><<<GRID, kThreads, SMEM, stream>>>(a);                 \
    else KERNEL<4><<<GRID, kThreads, SMEM, stream>>>(a);                               \
    GB_LAUNCH_CHECK();                                                                 \
  } while (0)

void launch_gat_scores(const GatArgs& a, cudaStream_t stream) {
  check(a);
  GAT_DISPATCH(gat_scores_kernel, grid_warps(a.cap_src), 0);
}

void launch_gat_fwd(const GatArgs& a, cudaStream_t stream) {
  check(a);
  if (a.ldo % 8 != 0) throw std::invalid_argument("gat: out stride % 8");
  if (a.dropout_p > 0.f && !a.counters) throw std::invalid_argument("gat: dropout needs the step counters");
  const size_t smem = a.mean_heads ? (kThreads / 32) * a.heads * a.feat * sizeof(float) : 0;
  GAT_DISPATCH(gat_fwd_kernel, grid_warps(a.cap_dst), smem);
}

void launch_gat_bwd(const GatArgs& a, cudaStream_t stream) {
  check(a);
  if (a.lddz % 4 != 0 || a.lddzb % 8 != 0) throw std::invalid_argument("gat: gradient strides");
  GAT_DISPATCH(gat_bwd_edge_kernel, grid_warps(a.cap_dst, 4), 0);
  GAT_DISPATCH(gat_bwd_node_kernel, grid_warps(a.cap_src, 4), 0);
}

}  // namespace dev
}  // namespace grappa
