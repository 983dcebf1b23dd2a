// Fused last layer of GraphSAGE-mean with the softmax cross-entropy loss (the
// reference's SAGEConv output layer and F.cross_entropy, experiments/grappa/train/
// sage.py and t10n_train.py): one warp per destination row v of the last block
//
//   x_v    = [h_v | mean_{u in N(v)} h_u]                      (bf16, kept for dW)
//   z_v    = x_v W^T + b                                      (C <= 64 classes)
//   loss  += (logsumexp(z_v) - z_v[y_v]) / n,   correct += [argmax z_v == y_v]
//   dz_v   = (softmax(z_v) - onehot(y_v)) / n                  (bf16, kept for dW)
//   db    += dz_v,      dx_v = dz_v W                          (bf16)
//
// The layer's rows are few (one per seed, about a thousand) and narrow (C classes), so
// a tensor-core tile would run on a handful of SMs; here every SM takes rows, W sits
// in shared memory, and the aggregation, the logits, the loss, its gradient and the
// input gradient of the layer are one kernel instead of an aggregation, a GEMM with a
// cross-entropy epilogue and a dX GEMM.  The per-class partial dot products of a row
// are reduced across the warp by a transposing butterfly (31 shuffles per 32
// classes), after which lane c holds class c (and class 32 + c).
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "grappa/rng.h"
#include "kernels.h"

namespace grappa {
namespace dev {

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// v[i] summed over the warp, scattered: afterwards lane l's v[0] is the total of index l
__device__ __forceinline__ void transpose_reduce32(float (&v)[32], int lane) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) {
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < off; ++i) {
      const float send = upper ? v[i] : v[i + off];
      const float keep = upper ? v[i + off] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
    }
  }
}

// NC: classes rounded up to 32 or 64
template <int NC>
__global__ void __launch_bounds__(kThreads) sage_head_kernel(SageHeadArgs a) {
  GB_PDL_ENTRY();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* s_w = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [NC][2 ip]
  __shared__ float s_db[64];
  __shared__ float s_loss;
  __shared__ int s_correct;
  const int ip = a.ip, K = 2 * ip, C = a.n_classes;
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  // W (and zero rows past C) into shared memory, 16 bytes per thread and step
  const int kc = K / 8;
  for (int i = threadIdx.x; i < NC * kc; i += kThreads) {
    const int c = i / kc, k8 = i % kc;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (c < C) v = *reinterpret_cast<const uint4*>(a.w + static_cast<int64_t>(c) * a.ldw + k8 * 8);
    *reinterpret_cast<uint4*>(s_w + c * K + k8 * 8) = v;
  }
  if (threadIdx.x < 64) s_db[threadIdx.x] = 0.f;
  if (threadIdx.x == 0) {
    s_loss = 0.f;
    s_correct = 0;
  }
  __syncthreads();

  const int n = min(*a.n_dst_ptr, a.cap_dst);
  const float inv_n = 1.0f / static_cast<float>(n > 0 ? n : 1);
  const int tail = min(a.cap_dst, static_cast<int>(ceil_div(n, 64) * 64));
  const bool has_cols = lane * 8 < ip;  // lane owns columns [8 lane, 8 lane + 8) of each half
  const int c0 = lane * 8;
  const int warps_total = gridDim.x * kWarps;
  float db_a = 0.f, db_b = 0.f;
  float loss_acc = 0.f;
  int correct_acc = 0;
  for (int v = blockIdx.x * kWarps + wib; v < tail; v += warps_total) {
    if (v >= n) {
      // rows past the count feed the split-K dW reduction: zero gradient rows
      for (int j = lane; j < a.ld_dl; j += 32) a.dl[static_cast<int64_t>(v) * a.ld_dl + j] = __float2bfloat16_rn(0.f);
      continue;
    }
    // ---- aggregation: self row and the mean of the in-neighbours' rows
    const int beg = a.indptr[v], end = a.indptr[v + 1];
    float xs[8], xa[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) xs[j] = xa[j] = 0.f;
    if (has_cols) {
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(v) * a.ldh + c0), xs);
      int e = beg;
      for (; e + 3 < end; e += 4) {
        uint4 r[4];
#pragma unroll
        for (int t = 0; t < 4; ++t)
          r[t] = *reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(a.indices[e + t]) * a.ldh + c0);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          float f[8];
          bf16x8_to_f32(r[t], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) xa[j] += f[j];
        }
      }
      for (; e < end; ++e) {
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(a.indices[e]) * a.ldh + c0), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) xa[j] += f[j];
      }
      const float sc = end > beg ? 1.f / static_cast<float>(end - beg) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) xa[j] *= sc;
      // the stored (bf16) operand is what the logits and the dW GEMM use
      const uint4 ps = f32_to_bf16x8(xs), pa = f32_to_bf16x8(xa);
      bf16x8_to_f32(ps, xs);
      bf16x8_to_f32(pa, xa);
      __nv_bfloat16* xr = a.x + static_cast<int64_t>(v) * a.ldx;
      *reinterpret_cast<uint4*>(xr + c0) = ps;
      *reinterpret_cast<uint4*>(xr + ip + c0) = pa;
    }
    // ---- logits: per-class partial dot products, then a transposing reduction
    float za, zb = -INFINITY;
    {
      float p[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        float t = 0.f;
        if (has_cols && c < C) {
          float ws[8], wa[8];
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_w + c * K + c0), ws);
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_w + c * K + ip + c0), wa);
#pragma unroll
          for (int j = 0; j < 8; ++j) t = fmaf(xs[j], ws[j], fmaf(xa[j], wa[j], t));
        }
        p[c] = t;
      }
      transpose_reduce32(p, lane);
      za = lane < C ? p[0] + (a.bias ? a.bias[lane] : 0.f) : -INFINITY;
    }
    if constexpr (NC > 32) {
      float p[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        float t = 0.f;
        if (has_cols && 32 + c < C) {
          float ws[8], wa[8];
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_w + (32 + c) * K + c0), ws);
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_w + (32 + c) * K + ip + c0), wa);
#pragma unroll
          for (int j = 0; j < 8; ++j) t = fmaf(xs[j], ws[j], fmaf(xa[j], wa[j], t));
        }
        p[c] = t;
      }
      transpose_reduce32(p, lane);
      zb = 32 + lane < C ? p[0] + (a.bias ? a.bias[32 + lane] : 0.f) : -INFINITY;
    }
    // ---- softmax cross-entropy (argmax: the first class of the largest logit)
    float mx = fmaxf(za, zb);
    int arg = za >= zb ? lane : 32 + lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, mx, o);
      const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
      if (om > mx || (om == mx && oa < arg)) {
        mx = om;
        arg = oa;
      }
    }
    const float ea = lane < C ? __expf(za - mx) : 0.f;
    const float eb = 32 + lane < C ? __expf(zb - mx) : 0.f;
    const float lse = mx + __logf(warp_sum(ea + eb));
    const int y = a.labels[v];
    const float zy = __shfl_sync(0xffffffffu, y < 32 ? za : zb, y & 31);
    if (lane == 0) {
      loss_acc += (lse - zy) * inv_n;
      correct_acc += arg == y;
      if (a.pred_out) a.pred_out[v] = arg;
    }
    float ga = lane < C ? (__expf(za - lse) - (lane == y ? 1.f : 0.f)) * inv_n : 0.f;
    float gb = 32 + lane < C ? (__expf(zb - lse) - (32 + lane == y ? 1.f : 0.f)) * inv_n : 0.f;
    ga = __bfloat162float(__float2bfloat16_rn(ga));
    gb = __bfloat162float(__float2bfloat16_rn(gb));
    db_a += ga;
    db_b += gb;
    __nv_bfloat16* dlr = a.dl + static_cast<int64_t>(v) * a.ld_dl;
    if (lane < a.ld_dl) dlr[lane] = __float2bfloat16_rn(ga);
    if (32 + lane < a.ld_dl) dlr[32 + lane] = __float2bfloat16_rn(gb);
    // ---- input gradient of the layer: dx_v = dz_v W
    if (a.dx) {
      // every lane takes part in the shuffles (class c lives in lane c % 32); the lanes
      // that own columns accumulate
      float ds[8], da[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) ds[j] = da[j] = 0.f;
#pragma unroll 4
      for (int c = 0; c < C; ++c) {
        const float g = __shfl_sync(0xffffffffu, c < 32 ? ga : gb, c & 31);
        if (has_cols) {
          float ws[8], wa[8];
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_w + c * K + c0), ws);
          bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_w + c * K + ip + c0), wa);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            ds[j] = fmaf(g, ws[j], ds[j]);
            da[j] = fmaf(g, wa[j], da[j]);
          }
        }
      }
      if (has_cols) {
        __nv_bfloat16* dxr = a.dx + static_cast<int64_t>(v) * a.lddx;
        *reinterpret_cast<uint4*>(dxr + c0) = f32_to_bf16x8(ds);
        *reinterpret_cast<uint4*>(dxr + ip + c0) = f32_to_bf16x8(da);
      }
    }
  }
  // ---- block totals, one global atomic per class / counter per CTA
  if (a.dbias) {
    if (lane < C && db_a != 0.f) atomicAdd(&s_db[lane], db_a);
    if (32 + lane < C && db_b != 0.f) atomicAdd(&s_db[32 + lane], db_b);
  }
  if (lane == 0) {
    if (loss_acc != 0.f) atomicAdd(&s_loss, loss_acc);
    if (correct_acc) atomicAdd(&s_correct, correct_acc);
  }
  __syncthreads();
  if (a.dbias && threadIdx.x < C && s_db[threadIdx.x] != 0.f) atomicAdd(a.dbias + threadIdx.x, s_db[threadIdx.x]);
  if (threadIdx.x == 0) {
    if (a.loss_sum && s_loss != 0.f) atomicAdd(a.loss_sum, s_loss);
    if (a.correct && s_correct) atomicAdd(a.correct, s_correct);
  }
}

// ---------------------------------------------------------------- tile version
// 16 destination rows per CTA (8 warps).  The two contractions of the layer run as
// warp-level bf16 MMAs (m16n8k16, fp32 accumulation) on operands staged in shared
// memory: logits Z[16 x C] = X[16 x 2ip] W^T (the k-steps split over the warps, the
// partial tiles summed through shared memory) and dX[16 x 2ip] = dZ[16 x C] W (the
// n-tiles split over the warps).  Aggregation and the softmax cross-entropy run as in
// the row version, two rows per warp; W is copied into shared memory with cp.async
// while the rows are aggregated.
constexpr int kTileRows = 16;

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void ldsm_x4(uint32_t a, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(a));
}
__device__ __forceinline__ void ldsm_x2(uint32_t a, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(a));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t a, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(a));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// shared-memory layout of the tile kernel (row strides padded by 8 elements: ldmatrix
// rows of one 8x8 matrix fall into distinct 16-byte bank groups)
struct HeadTileLayout {
  int K, ldk, KC, ldc, NT;
  size_t w_off, x_off, z_off, d_off, bytes;
  __host__ __device__ HeadTileLayout(int ip, int C) {
    K = 2 * ip;
    ldk = K + 8;
    NT = (C + 7) / 8;           // n-tiles of the logits
    KC = ((NT * 8 + 15) / 16) * 16;  // classes padded to whole k-steps of the dX product
    ldc = KC + 8;
    w_off = 0;                                                    // W   [KC][ldk] bf16
    x_off = w_off + static_cast<size_t>(KC) * ldk * 2;           // X   [16][ldk] bf16 (then dX)
    z_off = x_off + static_cast<size_t>(kTileRows) * ldk * 2;    // Z   [kWarps][16][NT*8] f32
    d_off = z_off + static_cast<size_t>(kWarps) * kTileRows * NT * 8 * 4;  // dZ [16][ldc] bf16
    bytes = d_off + static_cast<size_t>(kTileRows) * ldc * 2;
  }
};

__global__ void __launch_bounds__(kThreads) sage_head_tile_kernel(SageHeadArgs a) {
  GB_PDL_ENTRY();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __shared__ float s_db[64];
  __shared__ float s_loss;
  __shared__ int s_correct;
  const int ip = a.ip, C = a.n_classes;
  const HeadTileLayout L(ip, C);
  const int K = L.K, ldk = L.ldk, NT = L.NT, KC = L.KC, ldc = L.ldc;
  __nv_bfloat16* s_w = reinterpret_cast<__nv_bfloat16*>(smem_raw + L.w_off);
  __nv_bfloat16* s_x = reinterpret_cast<__nv_bfloat16*>(smem_raw + L.x_off);
  float* s_z = reinterpret_cast<float*>(smem_raw + L.z_off);
  __nv_bfloat16* s_d = reinterpret_cast<__nv_bfloat16*>(smem_raw + L.d_off);
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int n = min(*a.n_dst_ptr, a.cap_dst);
  const int tail = min(a.cap_dst, static_cast<int>(ceil_div(n, 64) * 64));
  const int r0 = blockIdx.x * kTileRows;
  if (r0 >= tail) return;
  // ---- W into shared memory (cp.async, overlapping the aggregation); rows >= C zero
  const int kc8 = K / 8;
  for (int i = threadIdx.x; i < KC * kc8; i += kThreads) {
    const int c = i / kc8, k8 = i % kc8;
    __nv_bfloat16* dst = s_w + c * ldk + k8 * 8;
    if (c < C) {
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)),
                   "l"(a.w + static_cast<int64_t>(c) * a.ldw + k8 * 8));
    } else {
      *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
    }
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  if (threadIdx.x < 64) s_db[threadIdx.x] = 0.f;
  if (threadIdx.x == 0) {
    s_loss = 0.f;
    s_correct = 0;
  }
  for (int i = threadIdx.x; i < kTileRows * (ldc / 8); i += kThreads)
    *reinterpret_cast<uint4*>(s_d + (i / (ldc / 8)) * ldc + (i % (ldc / 8)) * 8) = make_uint4(0, 0, 0, 0);
  // ---- aggregation: rows 2 wib, 2 wib + 1 of the tile
  const bool has_cols = lane * 8 < ip;
  const int c0 = lane * 8;
  for (int rr = 0; rr < 2; ++rr) {
    const int t = 2 * wib + rr, v = r0 + t;
    uint4 ps = make_uint4(0, 0, 0, 0), pa = make_uint4(0, 0, 0, 0);
    if (v < n && has_cols) {
      const int beg = a.indptr[v], end = a.indptr[v + 1];
      float xs[8], xa[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) xa[j] = 0.f;
      const uint4 self = *reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(v) * a.ldh + c0);
      int e = beg;
      for (; e + 3 < end; e += 4) {
        uint4 r[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          r[q] = *reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(a.indices[e + q]) * a.ldh + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[8];
          bf16x8_to_f32(r[q], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) xa[j] += f[j];
        }
      }
      for (; e < end; ++e) {
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(a.indices[e]) * a.ldh + c0), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) xa[j] += f[j];
      }
      const float sc = end > beg ? 1.f / static_cast<float>(end - beg) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) xa[j] *= sc;
      bf16x8_to_f32(self, xs);
      ps = f32_to_bf16x8(xs);
      pa = f32_to_bf16x8(xa);
      __nv_bfloat16* xr = a.x + static_cast<int64_t>(v) * a.ldx;
      *reinterpret_cast<uint4*>(xr + c0) = ps;
      *reinterpret_cast<uint4*>(xr + ip + c0) = pa;
    }
    if (has_cols) {  // rows past the count enter the products as zeros
      *reinterpret_cast<uint4*>(s_x + t * ldk + c0) = ps;
      *reinterpret_cast<uint4*>(s_x + t * ldk + ip + c0) = pa;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // ---- logits: warp wib takes k-steps wib, wib + 8, ...; partial tiles to s_z
  {
    const int g = lane >> 2, tq = lane & 3;
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[j][q] = 0.f;
    const int ksteps = K / 16;
    for (int ks = wib; ks < ksteps; ks += kWarps) {
      const int k0 = ks * 16;
      uint32_t x0, x1, x2, x3;
      ldsm_x4(smem_addr(s_x + (lane & 15) * ldk + k0 + (lane >> 4) * 8), x0, x1, x2, x3);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (j >= NT) break;
        uint32_t b0, b1;
        const int l16 = lane & 15;
        ldsm_x2(smem_addr(s_w + (j * 8 + (l16 & 7)) * ldk + k0 + (l16 >> 3) * 8), b0, b1);
        mma_bf16(acc[j], x0, x1, x2, x3, b0, b1);
      }
    }
    float* zw = s_z + wib * kTileRows * NT * 8;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= NT) break;
      const int col = j * 8 + tq * 2;
      zw[g * NT * 8 + col] = acc[j][0];
      zw[g * NT * 8 + col + 1] = acc[j][1];
      zw[(g + 8) * NT * 8 + col] = acc[j][2];
      zw[(g + 8) * NT * 8 + col + 1] = acc[j][3];
    }
  }
  __syncthreads();
  // ---- softmax cross-entropy, two rows per warp (lane c: class c and 32 + c)
  const float inv_n = 1.0f / static_cast<float>(n > 0 ? n : 1);
  float db_a = 0.f, db_b = 0.f, loss_acc = 0.f;
  int correct_acc = 0;
  const int ZW = NT * 8;
  for (int rr = 0; rr < 2; ++rr) {
    const int t = 2 * wib + rr, v = r0 + t;
    if (v >= tail) continue;
    __nv_bfloat16* dlr = a.dl + static_cast<int64_t>(v) * a.ld_dl;
    if (v >= n) {
      for (int j = lane; j < a.ld_dl; j += 32) dlr[j] = __float2bfloat16_rn(0.f);
      continue;
    }
    float za = -INFINITY, zb = -INFINITY;
    if (lane < C) {
      float s = a.bias ? a.bias[lane] : 0.f;
      for (int w = 0; w < kWarps; ++w) s += s_z[(w * kTileRows + t) * ZW + lane];
      za = s;
    }
    if (32 + lane < C) {
      float s = a.bias ? a.bias[32 + lane] : 0.f;
      for (int w = 0; w < kWarps; ++w) s += s_z[(w * kTileRows + t) * ZW + 32 + lane];
      zb = s;
    }
    float mx = fmaxf(za, zb);
    int arg = za >= zb ? lane : 32 + lane;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, mx, o);
      const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
      if (om > mx || (om == mx && oa < arg)) {
        mx = om;
        arg = oa;
      }
    }
    const float ea = lane < C ? __expf(za - mx) : 0.f;
    const float eb = 32 + lane < C ? __expf(zb - mx) : 0.f;
    const float lse = mx + __logf(warp_sum(ea + eb));
    const int y = a.labels[v];
    const float zy = __shfl_sync(0xffffffffu, y < 32 ? za : zb, y & 31);
    if (lane == 0) {
      loss_acc += (lse - zy) * inv_n;
      correct_acc += arg == y;
      if (a.pred_out) a.pred_out[v] = arg;
    }
    float ga = lane < C ? (__expf(za - lse) - (lane == y ? 1.f : 0.f)) * inv_n : 0.f;
    float gb = 32 + lane < C ? (__expf(zb - lse) - (32 + lane == y ? 1.f : 0.f)) * inv_n : 0.f;
    const __nv_bfloat16 ha = __float2bfloat16_rn(ga), hb = __float2bfloat16_rn(gb);
    db_a += __bfloat162float(ha);
    db_b += __bfloat162float(hb);
    if (lane < a.ld_dl) dlr[lane] = ha;
    if (32 + lane < a.ld_dl) dlr[32 + lane] = hb;
    if (lane < KC) s_d[t * ldc + lane] = ha;
    if (32 + lane < KC) s_d[t * ldc + 32 + lane] = hb;
  }
  if (a.dbias) {
    if (lane < C && db_a != 0.f) atomicAdd(&s_db[lane], db_a);
    if (32 + lane < C && db_b != 0.f) atomicAdd(&s_db[32 + lane], db_b);
  }
  if (lane == 0) {
    if (loss_acc != 0.f) atomicAdd(&s_loss, loss_acc);
    if (correct_acc) atomicAdd(&s_correct, correct_acc);
  }
  __syncthreads();
  // ---- dX = dZ W: warp wib takes n-tiles wib, wib + 8, ... of the 2 ip columns; the
  // bf16 result is staged in the X tile, then stored as 16-byte rows
  if (a.dx || a.dsrc) {
    const int g = lane >> 2, tq = lane & 3;
    const int l16 = lane & 15;
    const int kst = KC / 16;
    uint32_t da[4][4];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      if (s >= kst) break;
      ldsm_x4(smem_addr(s_d + (lane & 15) * ldc + s * 16 + (lane >> 4) * 8), da[s][0], da[s][1], da[s][2], da[s][3]);
    }
    for (int nt = wib; nt < K / 8; nt += kWarps) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        if (s >= kst) break;
        uint32_t b0, b1;
        ldsm_x2_t(smem_addr(s_w + (s * 16 + l16) * ldk + nt * 8), b0, b1);
        mma_bf16(acc, da[s][0], da[s][1], da[s][2], da[s][3], b0, b1);
      }
      const int col = nt * 8 + tq * 2;
      *reinterpret_cast<uint32_t*>(s_x + g * ldk + col) = pack_bf16x2(acc[0], acc[1]);
      *reinterpret_cast<uint32_t*>(s_x + (g + 8) * ldk + col) = pack_bf16x2(acc[2], acc[3]);
    }
    __syncthreads();
    if (a.dx) {
      for (int i = threadIdx.x; i < kTileRows * kc8; i += kThreads) {
        const int t = i / kc8, k8 = i % kc8, v = r0 + t;
        if (v < n)
          *reinterpret_cast<uint4*>(a.dx + static_cast<int64_t>(v) * a.lddx + k8 * 8) =
              *reinterpret_cast<const uint4*>(s_x + t * ldk + k8 * 8);
      }
    }
    if (a.dsrc && has_cols) {
      // the aggregation's backward from the bf16 dx rows: self half to the row itself,
      // neighbour half / deg to every in-neighbour (two rows per warp, 8 columns a lane)
      for (int rr = 0; rr < 2; ++rr) {
        const int t = 2 * wib + rr, v = r0 + t;
        if (v >= n) continue;
        const int beg = a.indptr[v], end = a.indptr[v + 1];
        const float sc = end > beg ? 1.f / static_cast<float>(end - beg) : 0.f;
        float fs[8], fa[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_x + t * ldk + c0), fs);
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_x + t * ldk + ip + c0), fa);
        float* d = a.dsrc + static_cast<int64_t>(v) * a.ld_dsrc + c0;
        red_add_v4(d, fs[0], fs[1], fs[2], fs[3]);
        red_add_v4(d + 4, fs[4], fs[5], fs[6], fs[7]);
#pragma unroll
        for (int j = 0; j < 8; ++j) fa[j] *= sc;
        for (int e = beg; e < end; ++e) {
          float* du = a.dsrc + static_cast<int64_t>(a.indices[e]) * a.ld_dsrc + c0;
          red_add_v4(du, fa[0], fa[1], fa[2], fa[3]);
          red_add_v4(du + 4, fa[4], fa[5], fa[6], fa[7]);
        }
      }
    }
  }
  if (a.dbias && threadIdx.x < C && s_db[threadIdx.x] != 0.f) atomicAdd(a.dbias + threadIdx.x, s_db[threadIdx.x]);
  if (threadIdx.x == 0) {
    if (a.loss_sum && s_loss != 0.f) atomicAdd(a.loss_sum, s_loss);
    if (a.correct && s_correct) atomicAdd(a.correct, s_correct);
  }
}

// ---------------------------------------------------------------- middle layers
// A hidden GraphSAGE layer as 16-row tiles, each tile split over two CTAs by output
// columns (blockIdx.y), so that the CTA's slice of W fits in shared memory:
//   forward   H[v, n] = dropout(relu([h_v | mean h_u] . W[n] + b[n])) for its 128
//             columns n (the aggregation is done by both CTAs of a tile; half 0 also
//             stores the aggregated rows X for the weight gradient)
//   backward  dX = dY W for its half of the 2 ip input columns, reduced straight into
//             the previous layer's fp32 gradient rows: the self half to dsrc[v], the
//             neighbour half / deg(v) to dsrc[u] of every in-neighbour u
// (an aggregation and a tcgen05 GEMM, and a dX GEMM and an aggregation backward, are
// replaced; the block has a few thousand rows, so a 128-row tensor-core tile would
// leave most SMs idle).
constexpr int kFwdCols = 128;  // output columns per forward CTA

struct LayerTileLayout {
  int ip, K, ldk, op, ldo;
  size_t w_off, x_off, bytes;
};
__host__ __device__ inline LayerTileLayout fwd_layout(int ip) {
  LayerTileLayout L;
  L.ip = ip;
  L.K = 2 * ip;
  L.ldk = L.K + 8;
  L.op = 0;
  L.ldo = 0;
  L.w_off = 0;                                                    // W slice [128][ldk]
  L.x_off = static_cast<size_t>(kFwdCols) * L.ldk * 2;            // X tile  [16][ldk]
  L.bytes = L.x_off + static_cast<size_t>(kTileRows) * L.ldk * 2;
  return L;
}
__host__ __device__ inline LayerTileLayout bwd_layout(int ip, int op) {
  LayerTileLayout L;
  L.ip = ip;
  L.K = op;                 // reduction over the layer's outputs
  L.ldk = ip + 8;           // W half [op][ldk]
  L.op = op;
  L.ldo = op + 8;           // dY tile [16][ldo], then the dX half [16][ldk]
  L.w_off = 0;
  L.x_off = static_cast<size_t>(op) * L.ldk * 2;
  const size_t dy = static_cast<size_t>(kTileRows) * L.ldo * 2, dx = static_cast<size_t>(kTileRows) * L.ldk * 2;
  L.bytes = L.x_off + (dy > dx ? dy : dx);
  return L;
}

__global__ void __launch_bounds__(kThreads) sage_fwd_tile_kernel(SageLayerArgs a) {
  GB_PDL_ENTRY();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int ip = a.ip;
  const LayerTileLayout L = fwd_layout(ip);
  const int K = L.K, ldk = L.ldk;
  __nv_bfloat16* s_w = reinterpret_cast<__nv_bfloat16*>(smem_raw + L.w_off);
  __nv_bfloat16* s_x = reinterpret_cast<__nv_bfloat16*>(smem_raw + L.x_off);
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int n = min(*a.n_dst_ptr, a.cap_dst);
  const int r0 = blockIdx.x * kTileRows;
  const int n0 = blockIdx.y * kFwdCols;
  if (r0 >= n) return;
  // W rows n0 .. n0 + 127 into shared memory
  const int kc8 = K / 8;
  for (int i = threadIdx.x; i < kFwdCols * kc8; i += kThreads) {
    const int c = i / kc8, k8 = i % kc8;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(s_w + c * ldk + k8 * 8)),
                 "l"(a.w + static_cast<int64_t>(n0 + c) * a.ldw + k8 * 8));
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  // aggregation: rows 2 wib, 2 wib + 1 of the tile
  const bool has_cols = lane * 8 < ip;
  const int c0 = lane * 8;
  for (int rr = 0; rr < 2; ++rr) {
    const int t = 2 * wib + rr, v = r0 + t;
    uint4 ps = make_uint4(0, 0, 0, 0), pa = make_uint4(0, 0, 0, 0);
    if (v < n && has_cols) {
      const int beg = a.indptr[v], end = a.indptr[v + 1];
      float xa[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) xa[j] = 0.f;
      ps = *reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(v) * a.ldh + c0);
      int e = beg;
      for (; e + 3 < end; e += 4) {
        uint4 r[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          r[q] = *reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(a.indices[e + q]) * a.ldh + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[8];
          bf16x8_to_f32(r[q], f);
#pragma unroll
          for (int j = 0; j < 8; ++j) xa[j] += f[j];
        }
      }
      for (; e < end; ++e) {
        float f[8];
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(a.indices[e]) * a.ldh + c0), f);
#pragma unroll
        for (int j = 0; j < 8; ++j) xa[j] += f[j];
      }
      const float sc = end > beg ? 1.f / static_cast<float>(end - beg) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) xa[j] *= sc;
      pa = f32_to_bf16x8(xa);
      if (blockIdx.y == 0) {
        __nv_bfloat16* xr = a.x + static_cast<int64_t>(v) * a.ldx;
        *reinterpret_cast<uint4*>(xr + c0) = ps;
        *reinterpret_cast<uint4*>(xr + ip + c0) = pa;
      }
    }
    if (has_cols) {
      *reinterpret_cast<uint4*>(s_x + t * ldk + c0) = ps;
      *reinterpret_cast<uint4*>(s_x + t * ldk + ip + c0) = pa;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // Z[16 x 128] = X W_slice^T: warp wib takes n-tiles 2 wib, 2 wib + 1
  const int g = lane >> 2, tq = lane & 3, l16 = lane & 15;
  float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
  for (int ks = 0; ks < K / 16; ++ks) {
    const int k0 = ks * 16;
    uint32_t x0, x1, x2, x3;
    ldsm_x4(smem_addr(s_x + (lane & 15) * ldk + k0 + (lane >> 4) * 8), x0, x1, x2, x3);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      uint32_t b0, b1;
      ldsm_x2(smem_addr(s_w + ((2 * wib + j) * 8 + (l16 & 7)) * ldk + k0 + (l16 >> 3) * 8), b0, b1);
      mma_bf16(acc[j], x0, x1, x2, x3, b0, b1);
    }
  }
  // bias, ReLU, dropout (byte-resolution mask of the output element index), bf16 store
  uint64_t key = 0;
  uint32_t thr8 = 0;
  float ks = 1.f;
  if (a.dropout_p > 0.f) {
    key = hop_key(static_cast<uint64_t>(a.counters[0]) ^ 0xD80Full, static_cast<uint64_t>(a.counters[1]),
                  static_cast<uint64_t>(a.counters[2]), a.dropout_salt);
    thr8 = dropout_thr8(a.dropout_p);
    ks = dropout_scale8(thr8);
  }
#pragma unroll
  for (int j = 0; j < 2; ++j) {
    const int col = n0 + (2 * wib + j) * 8 + tq * 2;
#pragma unroll
    for (int hrow = 0; hrow < 2; ++hrow) {
      const int v = r0 + g + 8 * hrow;
      if (v >= n) continue;
      float o0 = acc[j][2 * hrow] + (a.bias ? a.bias[col] : 0.f);
      float o1 = acc[j][2 * hrow + 1] + (a.bias ? a.bias[col + 1] : 0.f);
      if (a.act == 1) {
        o0 = fmaxf(o0, 0.f);
        o1 = fmaxf(o1, 0.f);
      }
      if (a.dropout_p > 0.f) {
        const uint64_t idx = static_cast<uint64_t>(v) * static_cast<uint64_t>(a.ldo) + static_cast<uint64_t>(col);
        const uint32_t keep = dropout_keep_bits(key, idx, 2, thr8);
        o0 = (keep & 1u) ? o0 * ks : 0.f;
        o1 = (keep & 2u) ? o1 * ks : 0.f;
      }
      *reinterpret_cast<uint32_t*>(a.out + static_cast<int64_t>(v) * a.ldo + col) = pack_bf16x2(o0, o1);
    }
  }
}

__global__ void __launch_bounds__(kThreads) sage_bwd_tile_kernel(SageLayerArgs a) {
  GB_PDL_ENTRY();
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int ip = a.ip, op = a.op;
  const LayerTileLayout L = bwd_layout(ip, op);
  const int ldk = L.ldk, ldo = L.ldo;
  __nv_bfloat16* s_w = reinterpret_cast<__nv_bfloat16*>(smem_raw + L.w_off);  // [op][ldk]: W[:, half]
  __nv_bfloat16* s_t = reinterpret_cast<__nv_bfloat16*>(smem_raw + L.x_off);  // dY tile, then dX half
  const int lane = threadIdx.x & 31, wib = threadIdx.x >> 5;
  const int n = min(*a.n_dst_ptr, a.cap_dst);
  const int r0 = blockIdx.x * kTileRows;
  const int half = blockIdx.y;  // 0: self columns [0, ip), 1: neighbour columns [ip, 2 ip)
  if (r0 >= n) return;
  const int ic8 = ip / 8;
  for (int i = threadIdx.x; i < op * ic8; i += kThreads) {
    const int k = i / ic8, c8 = i % ic8;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(s_w + k * ldk + c8 * 8)),
                 "l"(a.w + static_cast<int64_t>(k) * a.ldw + half * ip + c8 * 8));
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  const int oc8 = op / 8;
  for (int i = threadIdx.x; i < kTileRows * oc8; i += kThreads) {
    const int t = i / oc8, c8 = i % oc8, v = r0 + t;
    uint4 d = make_uint4(0, 0, 0, 0);
    if (v < n) d = *reinterpret_cast<const uint4*>(a.dy + static_cast<int64_t>(v) * a.lddy + c8 * 8);
    *reinterpret_cast<uint4*>(s_t + t * ldo + c8 * 8) = d;
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // dX half [16 x ip] = dY [16 x op] W[:, half]: warp wib takes n-tiles wib, wib + 8, ...
  const int g = lane >> 2, tq = lane & 3, l16 = lane & 15;
  const int ntiles = ip / 8, ksteps = op / 16;
  float acc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[j][q] = 0.f;
  for (int ks = 0; ks < ksteps; ++ks) {
    const int k0 = ks * 16;
    uint32_t d0, d1, d2, d3;
    ldsm_x4(smem_addr(s_t + (lane & 15) * ldo + k0 + (lane >> 4) * 8), d0, d1, d2, d3);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int nt = wib + 8 * j;
      if (nt >= ntiles) break;
      uint32_t b0, b1;
      ldsm_x2_t(smem_addr(s_w + (k0 + l16) * ldk + nt * 8), b0, b1);
      mma_bf16(acc[j], d0, d1, d2, d3, b0, b1);
    }
  }
  __syncthreads();  // every warp has read the dY tile: its buffer takes the dX half
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int nt = wib + 8 * j;
    if (nt >= ntiles) break;
    const int col = nt * 8 + tq * 2;
    *reinterpret_cast<uint32_t*>(s_t + g * ldk + col) = pack_bf16x2(acc[j][0], acc[j][1]);
    *reinterpret_cast<uint32_t*>(s_t + (g + 8) * ldk + col) = pack_bf16x2(acc[j][2], acc[j][3]);
  }
  __syncthreads();
  // the aggregation's backward from the bf16 dX rows, two rows per warp, 8 columns a lane
  const bool has_cols = lane * 8 < ip;
  const int c0 = lane * 8;
  if (!has_cols) return;
  for (int rr = 0; rr < 2; ++rr) {
    const int t = 2 * wib + rr, v = r0 + t;
    if (v >= n) continue;
    float f[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(s_t + t * ldk + c0), f);
    if (half == 0) {
      float* d = a.dsrc + static_cast<int64_t>(v) * a.ld_dsrc + c0;
      red_add_v4(d, f[0], f[1], f[2], f[3]);
      red_add_v4(d + 4, f[4], f[5], f[6], f[7]);
    } else {
      const int beg = a.indptr[v], end = a.indptr[v + 1];
      const float sc = end > beg ? 1.f / static_cast<float>(end - beg) : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] *= sc;
      for (int e = beg; e < end; ++e) {
        float* du = a.dsrc + static_cast<int64_t>(a.indices[e]) * a.ld_dsrc + c0;
        red_add_v4(du, f[0], f[1], f[2], f[3]);
        red_add_v4(du + 4, f[4], f[5], f[6], f[7]);
      }
    }
  }
}

}  // namespace

bool sage_layer_tile_supported(int ip, int op) {
  return ip > 0 && ip % 16 == 0 && ip <= 256 && op > 0 && op % kFwdCols == 0 && op <= 256 &&
         fwd_layout(ip).bytes <= 200 * 1024 && bwd_layout(ip, op).bytes <= 200 * 1024;
}

void launch_sage_layer_fwd(const SageLayerArgs& a, cudaStream_t stream) {
  if (!sage_layer_tile_supported(a.ip, a.op)) throw std::invalid_argument("sage layer tile: unsupported shape");
  if (a.ldh % 8 || a.ldx % 8 || a.ldw % 8 || a.ldo % 2) throw std::invalid_argument("sage layer tile: strides");
  if (a.dropout_p > 0.f && !a.counters) throw std::invalid_argument("sage layer tile: dropout needs the counters");
  const LayerTileLayout L = fwd_layout(a.ip);
  GB_CUDA_CHECK(cudaFuncSetAttribute(sage_fwd_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(L.bytes)));
  const dim3 grid(static_cast<unsigned>(ceil_div(a.cap_dst > 0 ? a.cap_dst : 1, kTileRows)),
                  static_cast<unsigned>(a.op / kFwdCols));
  launch_k(sage_fwd_tile_kernel, grid, kThreads, L.bytes, stream, a);
  GB_LAUNCH_CHECK();
}

void launch_sage_layer_bwd(const SageLayerArgs& a, cudaStream_t stream) {
  if (!sage_layer_tile_supported(a.ip, a.op)) throw std::invalid_argument("sage layer tile: unsupported shape");
  if (a.lddy % 8 || a.ldw % 8 || a.ld_dsrc % 4 || !a.dsrc) throw std::invalid_argument("sage layer tile: strides");
  const LayerTileLayout L = bwd_layout(a.ip, a.op);
  GB_CUDA_CHECK(cudaFuncSetAttribute(sage_bwd_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(L.bytes)));
  const dim3 grid(static_cast<unsigned>(ceil_div(a.cap_dst > 0 ? a.cap_dst : 1, kTileRows)), 2u);
  launch_k(sage_bwd_tile_kernel, grid, kThreads, L.bytes, stream, a);
  GB_LAUNCH_CHECK();
}

bool sage_head_supported(int ip, int n_classes) {
  return ip > 0 && ip % 8 == 0 && ip <= 256 && n_classes > 0 && n_classes <= 64;
}

void launch_sage_head(const SageHeadArgs& a, cudaStream_t stream) {
  // GRAPPA_SAGE_HEAD_TILE=0: the row version (no fused aggregation backward)
  static const bool tile = [] {
    const char* e = std::getenv("GRAPPA_SAGE_HEAD_TILE");
    return !(e && e[0] == '0');
  }();
  if (!sage_head_supported(a.ip, a.n_classes)) throw std::invalid_argument("sage head: ip % 8, ip <= 256, <= 64 classes");
  if (a.dsrc && (a.ld_dsrc % 4 || !tile))
    throw std::invalid_argument("sage head: the fused aggregation backward needs the tile kernel and ld_dsrc % 4");
  if (a.ldh % 8 || a.ldx % 8 || a.ldw % 8 || (a.dx && a.lddx % 8))
    throw std::invalid_argument("sage head: row strides must be multiples of 8 elements");
  if (a.ld_dl < a.n_classes) throw std::invalid_argument("sage head: dlogits row shorter than the classes");
  if (tile) {
    const HeadTileLayout L(a.ip, a.n_classes);
    GB_CUDA_CHECK(cudaFuncSetAttribute(sage_head_tile_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(L.bytes)));
    const int tiles = static_cast<int>(ceil_div(a.cap_dst > 0 ? a.cap_dst : 1, kTileRows));
    launch_k(sage_head_tile_kernel, tiles, kThreads, L.bytes, stream, a);
    GB_LAUNCH_CHECK();
    return;
  }
  const int nc = a.n_classes <= 32 ? 32 : 64;
  const size_t smem = static_cast<size_t>(nc) * 2 * a.ip * sizeof(__nv_bfloat16);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int want = static_cast<int>(ceil_div(a.cap_dst > 0 ? a.cap_dst : 1, kWarps));
  const int grid = std::max(1, std::min(want, sms));
  if (nc == 32) {
    GB_CUDA_CHECK(cudaFuncSetAttribute(sage_head_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
    launch_k(sage_head_kernel<32>, grid, kThreads, smem, stream, a);
  } else {
    GB_CUDA_CHECK(cudaFuncSetAttribute(sage_head_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem)));
    launch_k(sage_head_kernel<64>, grid, kThreads, smem, stream, a);
  }
  GB_LAUNCH_CHECK();
}

}  // namespace dev
}  // namespace grappa
