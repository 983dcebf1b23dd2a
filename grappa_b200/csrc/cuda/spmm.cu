// K-SpMM: neighbour aggregation over a block in CSR-by-dst form, bf16 rows in,
// fp32 accumulation, bf16 out, and its transpose for the backward pass.
//
// Forward, for every destination v < n_dst (one warp per row, 16-byte vector
// loads; for narrow rows the warp splits into groups that each walk a different
// edge, and the groups are reduced with shuffles):
//   kAggMean      agg_v = 1/deg_v * sum_e h[src_e]                 (SAGEConv 'mean')
//   kAggSum       agg_v = sum_e h[src_e] (+ self_scale * h_v)      (GINConv 'sum', eps)
//   kAggGcn       agg_v = dnorm_v * sum_e snorm[src_e] * h[src_e]  (GraphConv norm='both';
//                 dnorm_v = max(in_deg_v,1)^-1/2 from the block, snorm = max(out_deg,1)^-1/2)
//   kAggWeighted  agg_v = sum_e w_e n[src_e] / max(sum_e w_e, 1)   (PinSAGE WeightedSAGEConv)
// The aggregate is written at column agg_col of the output row, and the dst row
// itself can be copied at column self_col, producing the concatenated operand
// [h_v | agg_v] of one GEMM that replaces SAGEConv's fc_self + fc_neigh.
// The source rows can be addressed through src_map (local src -> table row),
// which lets the first layer aggregate straight from the resident feature table
// (no gathered copy of the input features is materialised).
//
// An optional epilogue adds a bias, applies ReLU and dropout to the aggregate
// (GraphConv when the projection runs before the aggregation).
//
// Backward: dsrc[src_e] += coef_e * dagg_v with vector fp32 reductions
// (red.global.add.v4.f32), plus the gradient of the self block to the dst rows.
#include "common.cuh"
#include "grappa/rng.h"
#include "kernels.h"

#include <algorithm>

namespace grappa {
namespace dev {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void red_add_v4f(float* p, float a, float b, float c, float d) {
  // no "memory" clobber: dsrc is not read in the same launch (see aggregate_bwd_kernel)
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d));
}

__host__ __device__ __forceinline__ int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

template <int CPL>
__global__ void __launch_bounds__(kThreads) aggregate_kernel(AggArgs a) {
  GB_PDL_ENTRY();
  const int n_dst = a.n_dst_ptr ? *a.n_dst_ptr : a.n_dst;
  const int chunks = a.dim >> 3;
  const int lpe = CPL == 1 ? next_pow2(chunks) : 32;  // lanes per edge
  const int groups = 32 / lpe;
  const int lane = threadIdx.x & 31;
  const int g = lane / lpe;
  const int sub = lane % lpe;
  const int warps_total = (gridDim.x * kThreads) >> 5;
  const int wg = (blockIdx.x * kThreads + threadIdx.x) >> 5;
  const int tail = a.zero_tail_rows > 0 ? min(a.cap_rows, static_cast<int>(ceil_div(n_dst, a.zero_tail_rows) * a.zero_tail_rows)) : n_dst;
  for (int row = wg; row < tail; row += warps_total) {
    if (row >= n_dst) {
      // zero rows past the count so that a split-K reduction over this buffer sees zeros
      const uint4 z = make_uint4(0, 0, 0, 0);
      for (int c = lane; c < chunks; c += 32) {
        *reinterpret_cast<uint4*>(a.out + row * a.out_stride + a.agg_col + c * 8) = z;
        if (a.self_col >= 0) *reinterpret_cast<uint4*>(a.out + row * a.out_stride + a.self_col + c * 8) = z;
      }
      continue;
    }
    const int beg = a.indptr[row];
    const int end = a.indptr[row + 1];
    float acc[CPL][8];
#pragma unroll
    for (int q = 0; q < CPL; ++q)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[q][j] = 0.f;
    float wsum = 0.f;
    int e = beg + g;
    // four, then two edges per group per iteration for memory-level parallelism
    for (; e + 3 * groups < end; e += 4 * groups) {
      int u[4];
      float w[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        u[t] = a.indices[e + t * groups];
        w[t] = 1.f;
        if (a.mode == kAggWeighted) w[t] = a.edge_w[e + t * groups];
      }
      int64_t rr[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        rr[t] = a.src_map ? a.src_map[u[t]] : u[t];
        if (a.mode == kAggGcn) w[t] = a.src_norm[u[t]];
        wsum += w[t];
      }
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = sub + q * lpe;
        if (c < chunks) {
          uint4 x[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) x[t] = *reinterpret_cast<const uint4*>(a.src + rr[t] * a.src_stride + c * 8);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            float f[8];
            bf16x8_to_f32(x[t], f);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[q][j] += w[t] * f[j];
          }
        }
      }
    }
    for (; e + groups < end; e += 2 * groups) {
      const int u0 = a.indices[e], u1 = a.indices[e + groups];
      const int64_t r0 = a.src_map ? a.src_map[u0] : u0;
      const int64_t r1 = a.src_map ? a.src_map[u1] : u1;
      float w0 = 1.f, w1 = 1.f;
      if (a.mode == kAggGcn) {
        w0 = a.src_norm[u0];
        w1 = a.src_norm[u1];
      } else if (a.mode == kAggWeighted) {
        w0 = a.edge_w[e];
        w1 = a.edge_w[e + groups];
      }
      wsum += w0 + w1;
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = sub + q * lpe;
        if (c < chunks) {
          const uint4 x0 = *reinterpret_cast<const uint4*>(a.src + r0 * a.src_stride + c * 8);
          const uint4 x1 = *reinterpret_cast<const uint4*>(a.src + r1 * a.src_stride + c * 8);
          float f0[8], f1[8];
          bf16x8_to_f32(x0, f0);
          bf16x8_to_f32(x1, f1);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[q][j] += w0 * f0[j] + w1 * f1[j];
        }
      }
    }
    for (; e < end; e += groups) {
      const int u0 = a.indices[e];
      const int64_t r0 = a.src_map ? a.src_map[u0] : u0;
      float w0 = 1.f;
      if (a.mode == kAggGcn) w0 = a.src_norm[u0];
      else if (a.mode == kAggWeighted) w0 = a.edge_w[e];
      wsum += w0;
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = sub + q * lpe;
        if (c < chunks) {
          const uint4 x0 = *reinterpret_cast<const uint4*>(a.src + r0 * a.src_stride + c * 8);
          float f0[8];
          bf16x8_to_f32(x0, f0);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[q][j] += w0 * f0[j];
        }
      }
    }
    // reduce the edge groups
    for (int off = lpe; off < 32; off <<= 1) {
      wsum += __shfl_xor_sync(0xffffffffu, wsum, off);
#pragma unroll
      for (int q = 0; q < CPL; ++q)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[q][j] += __shfl_xor_sync(0xffffffffu, acc[q][j], off);
    }
    const int deg = end - beg;
    float scale = 1.f;
    if (a.mode == kAggMean) scale = deg > 0 ? 1.f / static_cast<float>(deg) : 0.f;
    else if (a.mode == kAggGcn) scale = a.dst_norm ? a.dst_norm[row] : rsqrtf(static_cast<float>(deg > 1 ? deg : 1));
    else if (a.mode == kAggWeighted) scale = 1.f / fmaxf(wsum, 1.f);
    if (g == 0) {
      const int64_t rs = a.src_map ? a.src_map[row] : row;
      uint64_t key = 0;
      uint32_t thr = 0;
      float keep_scale = 1.f;
      if (a.dropout_p > 0.f) {
        key = hop_key(static_cast<uint64_t>(a.counters[0]) ^ 0xD80Full, static_cast<uint64_t>(a.counters[1]),
                      static_cast<uint64_t>(a.counters[2]), a.dropout_salt);
        thr = dropout_thr8(a.dropout_p);
        keep_scale = dropout_scale8(thr);
      }
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = sub + q * lpe;
        if (c >= chunks) continue;
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = acc[q][j] * scale;
        if (a.self_col >= 0 || a.self_scale != 0.f) {
          const uint4 xs = *reinterpret_cast<const uint4*>(a.src + rs * a.src_stride + c * 8);
          if (a.self_col >= 0) *reinterpret_cast<uint4*>(a.out + row * a.out_stride + a.self_col + c * 8) = xs;
          if (a.self_scale != 0.f) {
            float fs[8];
            bf16x8_to_f32(xs, fs);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] += a.self_scale * fs[j];
          }
        }
        if (a.bias) {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] += a.bias[c * 8 + j];
        }
        if (a.act == 1) {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = fmaxf(o[j], 0.f);
        }
        if (a.dropout_p > 0.f) {
          const uint64_t base = static_cast<uint64_t>(row) * static_cast<uint64_t>(a.out_stride) +
                                static_cast<uint64_t>(a.agg_col + c * 8);
          const uint32_t keep = dropout_keep_bits(key, base, 8, thr);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = (keep >> j) & 1u ? o[j] * keep_scale : 0.f;
        }
        *reinterpret_cast<uint4*>(a.out + row * a.out_stride + a.agg_col + c * 8) = f32_to_bf16x8(o);
      }
    }
  }
}

template <int CPL>
__global__ void __launch_bounds__(kThreads) aggregate_bwd_kernel(AggBwdArgs a) {
  GB_PDL_ENTRY();
  const int n_dst = a.n_dst_ptr ? *a.n_dst_ptr : a.n_dst;
  const int chunks = a.dim >> 3;
  const int lpe = CPL == 1 ? next_pow2(chunks) : 32;
  const int groups = 32 / lpe;
  const int lane = threadIdx.x & 31;
  const int g = lane / lpe;
  const int sub = lane % lpe;
  const int warps_total = (gridDim.x * kThreads) >> 5;
  const int wg = (blockIdx.x * kThreads + threadIdx.x) >> 5;
  for (int row = wg; row < n_dst; row += warps_total) {
    const int beg = a.indptr[row];
    const int end = a.indptr[row + 1];
    const int deg = end - beg;
    float go[CPL][8];
    float wsum = 0.f;
    if (a.mode == kAggWeighted) {
      for (int e = beg + lane; e < end; e += 32) wsum += a.edge_w[e];
      wsum = warp_sum(wsum);
    }
    float scale = 1.f;
    if (a.mode == kAggMean) scale = deg > 0 ? 1.f / static_cast<float>(deg) : 0.f;
    else if (a.mode == kAggGcn) scale = a.dst_norm ? a.dst_norm[row] : rsqrtf(static_cast<float>(deg > 1 ? deg : 1));
    else if (a.mode == kAggWeighted) scale = 1.f / fmaxf(wsum, 1.f);
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = sub + q * lpe;
      if (c < chunks) {
        const uint4 x = *reinterpret_cast<const uint4*>(a.dout + row * a.dout_stride + a.agg_col + c * 8);
        bf16x8_to_f32(x, go[q]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) go[q][j] = 0.f;
      }
    }
    // self contributions go to the dst row (the first n_dst src rows)
    if (g == 0 && (a.self_col >= 0 || a.self_scale != 0.f)) {
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = sub + q * lpe;
        if (c >= chunks) continue;
        float s[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] = a.self_scale * go[q][j];
        if (a.self_col >= 0) {
          const uint4 x = *reinterpret_cast<const uint4*>(a.dout + row * a.dout_stride + a.self_col + c * 8);
          float f[8];
          bf16x8_to_f32(x, f);
#pragma unroll
          for (int j = 0; j < 8; ++j) s[j] += f[j];
        }
        float* d = a.dsrc + static_cast<int64_t>(row) * a.dsrc_stride + c * 8;
        red_add_v4f(d, s[0], s[1], s[2], s[3]);
        red_add_v4f(d + 4, s[4], s[5], s[6], s[7]);
      }
    }
    for (int e = beg + g; e < end; e += groups) {
      const int u = a.indices[e];
      float w = scale;
      if (a.mode == kAggGcn) w *= a.src_norm[u];
      else if (a.mode == kAggWeighted) w *= a.edge_w[e];
#pragma unroll
      for (int q = 0; q < CPL; ++q) {
        const int c = sub + q * lpe;
        if (c >= chunks) continue;
        float* d = a.dsrc + static_cast<int64_t>(u) * a.dsrc_stride + c * 8;
        red_add_v4f(d, w * go[q][0], w * go[q][1], w * go[q][2], w * go[q][3]);
        red_add_v4f(d + 4, w * go[q][4], w * go[q][5], w * go[q][6], w * go[q][7]);
      }
    }
  }
}

// Mean-aggregation backward gathered by source with the activation backward fused
// (see AggBwdGatherArgs).  One warp per source row, lane l owning 8-column chunks
// l, l + 32, ...; the row's transposed edges are read 32 at a time (one coalesced
// load of their destinations, with the destinations' degrees), then four rows of the
// output gradient are in flight per lane.  Column sums of dy go to dbias with one
// atomic per column and block.
template <int CPL>
__global__ void __launch_bounds__(kThreads) aggregate_bwd_gather_kernel(AggBwdGatherArgs a) {
  GB_PDL_ENTRY();
  __shared__ float s_col[kThreads / 32][CPL * 256];
  const int n_src = min(*a.n_src_ptr, a.cap_rows);
  const int n_dst = *a.n_dst_ptr;
  const int chunks = a.dim >> 3;
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  const int warps_total = (gridDim.x * kThreads) >> 5;
  const int rows_end = min(a.cap_rows, static_cast<int>(ceil_div(n_src, 64) * 64));
  float bsum[CPL][8];
#pragma unroll
  for (int q = 0; q < CPL; ++q)
#pragma unroll
    for (int j = 0; j < 8; ++j) bsum[q][j] = 0.f;
  for (int u = (blockIdx.x * kThreads + threadIdx.x) >> 5; u < rows_end; u += warps_total) {
    __nv_bfloat16* dyrow = a.dy + static_cast<int64_t>(u) * a.dy_stride;
    if (u >= n_src) {
      for (int c = lane; c < chunks; c += 32) *reinterpret_cast<uint4*>(dyrow + c * 8) = make_uint4(0, 0, 0, 0);
      continue;
    }
    float acc[CPL][8];
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = lane + 32 * q;
      if (u < n_dst && c < chunks) {
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.dout + static_cast<int64_t>(u) * a.dout_stride + a.self_col +
                                                        c * 8), acc[q]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[q][j] = 0.f;
      }
    }
    const int beg = a.tptr[u], end = a.tptr[u + 1];
    for (int cb = beg; cb < end; cb += 32) {
      const int cnt = min(32, end - cb);
      int my_v = 0;
      float my_w = 0.f;
      if (lane < cnt) {
        my_v = a.tdst[cb + lane];
        if (my_v >= 0 && my_v < n_dst) {
          const int d = a.indptr[my_v + 1] - a.indptr[my_v];
          my_w = d > 0 ? 1.f / static_cast<float>(d) : 0.f;
        } else {
          my_v = 0;
          set_error(a.err, kErrBadIndex);
        }
      }
      for (int k = 0; k < cnt; k += 4) {
        uint4 x[4][CPL];
        float w[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int v = __shfl_sync(0xffffffffu, my_v, min(k + t, 31));
          w[t] = __shfl_sync(0xffffffffu, my_w, min(k + t, 31));
          if (k + t >= cnt) w[t] = 0.f;
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            const int c = lane + 32 * q;
            x[t][q] = make_uint4(0, 0, 0, 0);
            if (k + t < cnt && c < chunks)
              x[t][q] = *reinterpret_cast<const uint4*>(a.dout + static_cast<int64_t>(v) * a.dout_stride + a.agg_col +
                                                        c * 8);
          }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
          for (int q = 0; q < CPL; ++q) {
            float f[8];
            bf16x8_to_f32(x[t][q], f);
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[q][j] = fmaf(w[t], f[j], acc[q][j]);
          }
      }
    }
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = lane + 32 * q;
      if (c >= chunks) continue;
      float h[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.mask + static_cast<int64_t>(u) * a.mask_stride + c * 8), h);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        acc[q][j] = h[j] != 0.f ? acc[q][j] * a.scale : 0.f;
        bsum[q][j] += acc[q][j];
      }
      *reinterpret_cast<uint4*>(dyrow + c * 8) = f32_to_bf16x8(acc[q]);
    }
  }
  if (a.dbias) {
#pragma unroll
    for (int q = 0; q < CPL; ++q)
#pragma unroll
      for (int j = 0; j < 8; ++j) s_col[wib][(lane + 32 * q) * 8 + j] = bsum[q][j];
    __syncthreads();
    for (int c = threadIdx.x; c < a.dim; c += blockDim.x) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kThreads / 32; ++w) t += s_col[w][c];
      if (t != 0.f) atomicAdd(a.dbias + c, t);
    }
  }
}

__global__ void out_degree_kernel(const int32_t* indices, const int32_t* n_edges_ptr, float* deg) {
  GB_PDL_ENTRY();
  const int n_e = *n_edges_ptr;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n_e; e += gridDim.x * blockDim.x)
    atomicAdd(deg + indices[e], 1.f);
}
__global__ void rsqrt_clear_kernel(float* deg, const int32_t* n_ptr, int cap, float* out) {
  GB_PDL_ENTRY();
  const int n = n_ptr ? *n_ptr : cap;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float d = deg[i];
    out[i] = rsqrtf(d > 1.f ? d : 1.f);
    deg[i] = 0.f;  // leave the scratch zeroed for the next call
  }
}

int sm_count() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

int grid_for_rows(int cap_rows) {
  const int64_t want = ceil_div(cap_rows > 0 ? cap_rows : 1, kThreads / 32);
  return static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(sm_count()) * 16));
}

}  // namespace

void launch_aggregate(const AggArgs& args, int cap_dst, cudaStream_t stream) {
  AggArgs a = args;
  a.cap_rows = cap_dst;
  if (a.dim % 8 != 0) throw std::invalid_argument("aggregate: dim must be a multiple of 8");
  if (a.src_stride % 8 != 0 || a.out_stride % 8 != 0 || a.agg_col % 8 != 0 || (a.self_col >= 0 && a.self_col % 8 != 0))
    throw std::invalid_argument("aggregate: strides and column offsets must be multiples of 8 elements");
  if (a.dropout_p > 0.f && !a.counters) throw std::invalid_argument("aggregate: dropout needs the step counters");
  const int rows = a.zero_tail_rows > 0 ? static_cast<int>(ceil_div(cap_dst, a.zero_tail_rows) * a.zero_tail_rows) : cap_dst;
  const int grid = grid_for_rows(rows);
  const int chunks = a.dim / 8;
  if (chunks <= 32) launch_k(aggregate_kernel<1>, grid, kThreads, 0, stream, a);
  else if (chunks <= 64) launch_k(aggregate_kernel<2>, grid, kThreads, 0, stream, a);
  else if (chunks <= 128) launch_k(aggregate_kernel<4>, grid, kThreads, 0, stream, a);
  else throw std::invalid_argument("aggregate: dim > 1024 not supported");
  GB_LAUNCH_CHECK();
}

void launch_aggregate_bwd(const AggBwdArgs& a, int cap_dst, cudaStream_t stream) {
  if (a.dim % 8 != 0 || a.dsrc_stride % 4 != 0) throw std::invalid_argument("aggregate_bwd: bad dim/stride");
  const int grid = grid_for_rows(cap_dst);
  const int chunks = a.dim / 8;
  if (chunks <= 32) launch_k(aggregate_bwd_kernel<1>, grid, kThreads, 0, stream, a);
  else if (chunks <= 64) launch_k(aggregate_bwd_kernel<2>, grid, kThreads, 0, stream, a);
  else if (chunks <= 128) launch_k(aggregate_bwd_kernel<4>, grid, kThreads, 0, stream, a);
  else throw std::invalid_argument("aggregate_bwd: dim > 1024 not supported");
  GB_LAUNCH_CHECK();
}

void launch_aggregate_bwd_gather(const AggBwdGatherArgs& a, cudaStream_t stream) {
  if (a.dim % 8 != 0 || a.dout_stride % 8 != 0 || a.dy_stride % 8 != 0 || a.mask_stride % 8 != 0 ||
      a.self_col % 8 != 0 || a.agg_col % 8 != 0)
    throw std::invalid_argument("aggregate_bwd_gather: dims, strides and columns must be multiples of 8");
  const int grid = grid_for_rows(a.cap_rows);
  const int chunks = a.dim / 8;
  if (chunks <= 32) launch_k(aggregate_bwd_gather_kernel<1>, grid, kThreads, 0, stream, a);
  else if (chunks <= 64) launch_k(aggregate_bwd_gather_kernel<2>, grid, kThreads, 0, stream, a);
  else throw std::invalid_argument("aggregate_bwd_gather: dim > 512 not supported");
  GB_LAUNCH_CHECK();
}

void launch_src_norm(const int32_t* indices, const int32_t* n_edges_ptr, int cap_edges, const int32_t* n_src_ptr,
                     int cap_src, float* deg_scratch, float* src_norm, cudaStream_t stream) {
  const int g1 = static_cast<int>(std::min<int64_t>(ceil_div(cap_edges > 0 ? cap_edges : 1, 256), sm_count() * 8));
  launch_k(out_degree_kernel, g1, 256, 0, stream, indices, n_edges_ptr, deg_scratch);
  GB_LAUNCH_CHECK();
  const int g2 = static_cast<int>(std::min<int64_t>(ceil_div(cap_src > 0 ? cap_src : 1, 256), sm_count() * 8));
  launch_k(rsqrt_clear_kernel, g2, 256, 0, stream, deg_scratch, n_src_ptr, cap_src, src_norm);
  GB_LAUNCH_CHECK();
}

}  // namespace dev
}  // namespace grappa
