// Row-wise network ops around the GEMMs and aggregations: softmax cross-entropy,
// BatchNorm1d (+ReLU), row L2 normalisation, dropout and fp32 -> bf16 staging.
// All of them read the live row count from device memory so that a captured
// step graph replays them with the sizes of the current batch.
//
// Reference math (DGL/PyTorch modules the reference trains with):
//   CrossEntropyLoss              experiments/grappa/train/t10n_train.py:157
//   GIN MLP / BatchNorm1d + ReLU  experiments/grappa/train/gin.py:22-37,101-110
//   PinSAGE z / |z|               experiments/grappa/train/pinsage.py:40-48
#include <algorithm>

#include "common.cuh"
#include "grappa/rng.h"
#include "kernels.h"

namespace grappa {
namespace dev {

namespace {

int grid_1d(int64_t work, int threads, int per_sm) {
  static int sms = 0;
  if (!sms) {
    int d = 0;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d);
    if (sms <= 0) sms = 148;
  }
  const int64_t want = ceil_div(work > 0 ? work : 1, threads);
  return static_cast<int>(std::min<int64_t>(want, static_cast<int64_t>(sms) * per_sm));
}

__device__ __forceinline__ int live_rows(const int32_t* p, int cap) { return p ? min(*p, cap) : cap; }
__device__ __forceinline__ int tail_rows(int n, int cap, int zt) {
  return zt > 0 ? min(cap, static_cast<int>(ceil_div(n, zt) * zt)) : n;
}

// ------------------------------------------------------------------ cross-entropy
template <int CPL>
__global__ void __launch_bounds__(256) cross_entropy_kernel(CeArgs a) {
  GB_PDL_ENTRY();
  const int n = live_rows(a.n_rows_ptr, a.cap_rows);
  const int rows_end = tail_rows(n, a.cap_rows, a.zero_tail_rows);
  const int n_sel = a.n_sel_ptr ? *a.n_sel_ptr : n;
  const float inv_n = 1.f / static_cast<float>(n_sel > 0 ? n_sel : 1);
  const int lane = threadIdx.x & 31;
  const int warps_total = (gridDim.x * blockDim.x) >> 5;
  const int C = a.n_classes;
  float bsum[CPL];
#pragma unroll
  for (int q = 0; q < CPL; ++q) bsum[q] = 0.f;
  float loss_acc = 0.f;
  int correct = 0;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows_end; r += warps_total) {
    __nv_bfloat16* drow = a.dlogits + static_cast<int64_t>(r) * a.ld_dl;
    const bool live = r < n && (!a.row_mask || a.row_mask[r]);
    if (!live) {
      for (int c = lane; c < a.ld_dl; c += 32) drow[c] = __float2bfloat16_rn(0.f);
      continue;
    }
    const __nv_bfloat16* lrow = a.logits + static_cast<int64_t>(r) * a.ld;
    float v[CPL];
    float mx = -INFINITY;
    int arg = 0;
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = lane + 32 * q;
      v[q] = c < C ? __bfloat162float(lrow[c]) : -INFINITY;
      if (v[q] > mx) {
        mx = v[q];
        arg = c;
      }
    }
    // warp argmax (ties: smaller class index, as torch.argmax)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float om = __shfl_xor_sync(0xffffffffu, mx, o);
      const int oa = __shfl_xor_sync(0xffffffffu, arg, o);
      if (om > mx || (om == mx && oa < arg)) {
        mx = om;
        arg = oa;
      }
    }
    float se = 0.f;
#pragma unroll
    for (int q = 0; q < CPL; ++q)
      if (lane + 32 * q < C) se += __expf(v[q] - mx);
    se = warp_sum(se);
    const float lse = mx + __logf(se);
    const int y = a.labels[r];
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = lane + 32 * q;
      if (c >= a.ld_dl) continue;
      float p = c < C ? __expf(v[q] - lse) : 0.f;
      if (c == y) {
        loss_acc += (lse - v[q]) * inv_n;
        p -= 1.f;
      }
      const __nv_bfloat16 gb = __float2bfloat16_rn(p * inv_n);
      drow[c] = gb;
      bsum[q] += __bfloat162float(gb);
    }
    if (lane == 0 && arg == y) ++correct;
  }
  if (a.dbias) {
#pragma unroll
    for (int q = 0; q < CPL; ++q) {
      const int c = lane + 32 * q;
      if (c < C && bsum[q] != 0.f) atomicAdd(a.dbias + c, bsum[q]);
    }
  }
  loss_acc = warp_sum(loss_acc);
  if (lane == 0) {
    if (loss_acc != 0.f) atomicAdd(a.loss_sum, loss_acc);
    if (correct) atomicAdd(a.correct, correct);
  }
}

// ------------------------------------------------------------------ BatchNorm
// column sums of x and x^2 over the live rows: one thread per column pair, the
// block's rows strided over the grid
__global__ void bn_stats_kernel(BnArgs a) {
  GB_PDL_ENTRY();
  const int n = live_rows(a.n_ptr, a.cap);
  const int pairs = a.dim >> 1;
  for (int cp = threadIdx.x; cp < pairs; cp += blockDim.x) {
    float s0 = 0.f, s1 = 0.f, q0 = 0.f, q1 = 0.f;
    for (int r = blockIdx.x; r < n; r += gridDim.x) {
      const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162*>(a.x + static_cast<int64_t>(r) * a.ldx + 2 * cp);
      const float2 f = __bfloat1622float2(x);
      s0 += f.x;
      s1 += f.y;
      q0 += f.x * f.x;
      q1 += f.y * f.y;
    }
    atomicAdd(a.sums + 2 * cp, s0);
    atomicAdd(a.sums + 2 * cp + 1, s1);
    atomicAdd(a.sums + a.dim + 2 * cp, q0);
    atomicAdd(a.sums + a.dim + 2 * cp + 1, q1);
  }
}

__device__ __forceinline__ void bn_moments(const float* sums, int dim, int c, int n, float eps, float* mean,
                                           float* rstd, float* var_b) {
  const float inv = 1.f / static_cast<float>(n > 0 ? n : 1);
  const float m = sums[c] * inv;
  const float v = fmaxf(sums[dim + c] * inv - m * m, 0.f);
  *mean = m;
  *var_b = v;
  *rstd = rsqrtf(v + eps);
}

__global__ void bn_apply_kernel(BnArgs a) {
  GB_PDL_ENTRY();
  extern __shared__ float sh[];  // [2 * dim]: scale, shift
  const int n = live_rows(a.n_ptr, a.cap);
  for (int c = threadIdx.x; c < a.dim; c += blockDim.x) {
    float mean, rstd, var;
    if (a.training) {
      bn_moments(a.sums, a.dim, c, n, a.eps, &mean, &rstd, &var);
      if (blockIdx.x == 0 && a.running_mean && c < a.stat_dim) {
        const float unb = n > 1 ? var * static_cast<float>(n) / static_cast<float>(n - 1) : var;
        a.running_mean[c] = (1.f - a.momentum) * a.running_mean[c] + a.momentum * mean;
        a.running_var[c] = (1.f - a.momentum) * a.running_var[c] + a.momentum * unb;
      }
    } else {
      mean = c < a.stat_dim ? a.running_mean[c] : 0.f;
      rstd = rsqrtf((c < a.stat_dim ? a.running_var[c] : 1.f) + a.eps);
    }
    const float sc = a.gamma[c] * rstd;
    sh[c] = sc;
    sh[a.dim + c] = a.beta[c] - mean * sc;
  }
  if (a.training && blockIdx.x == 0 && threadIdx.x == 0 && a.num_batches) *a.num_batches += 1;
  __syncthreads();
  const int rows_end = tail_rows(n, a.cap, a.zero_tail_rows);
  const int pairs = a.dim >> 1;
  const int64_t total = static_cast<int64_t>(rows_end) * pairs;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / pairs);
    const int cp = static_cast<int>(i % pairs);
    __nv_bfloat162* yp = reinterpret_cast<__nv_bfloat162*>(a.y + static_cast<int64_t>(r) * a.ldy + 2 * cp);
    if (r >= n) {
      *yp = __floats2bfloat162_rn(0.f, 0.f);
      continue;
    }
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(a.x + static_cast<int64_t>(r) * a.ldx + 2 * cp));
    float y0 = f.x * sh[2 * cp] + sh[a.dim + 2 * cp];
    float y1 = f.y * sh[2 * cp + 1] + sh[a.dim + 2 * cp + 1];
    if (a.act == 1) {
      y0 = fmaxf(y0, 0.f);
      y1 = fmaxf(y1, 0.f);
    }
    *yp = __floats2bfloat162_rn(y0, y1);
  }
}

// g = dy * relu'(y); column sums of g and g * xhat
__global__ void bn_bwd_reduce_kernel(BnBwdArgs a) {
  GB_PDL_ENTRY();
  const int n = live_rows(a.n_ptr, a.cap);
  for (int c = threadIdx.x; c < a.dim; c += blockDim.x) {
    float mean, rstd, var;
    bn_moments(a.sums, a.dim, c, n, a.eps, &mean, &rstd, &var);
    float sg = 0.f, sgx = 0.f;
    for (int r = blockIdx.x; r < n; r += gridDim.x) {
      float g = a.dy_bf16 ? __bfloat162float(a.dy_bf16[static_cast<int64_t>(r) * a.lddy + c])
                          : a.dy[static_cast<int64_t>(r) * a.lddy + c];
      if (a.y && __bfloat162float(a.y[static_cast<int64_t>(r) * a.ldy + c]) == 0.f) g = 0.f;
      const float xh = (__bfloat162float(a.x[static_cast<int64_t>(r) * a.ldx + c]) - mean) * rstd;
      sg += g;
      sgx += g * xh;
    }
    atomicAdd(a.bsums + c, sg);
    atomicAdd(a.bsums + a.dim + c, sgx);
  }
}

__global__ void bn_bwd_apply_kernel(BnBwdArgs a) {
  GB_PDL_ENTRY();
  const int n = live_rows(a.n_ptr, a.cap);
  const float inv_n = 1.f / static_cast<float>(n > 0 ? n : 1);
  if (blockIdx.x == 0) {
    for (int c = threadIdx.x; c < a.dim; c += blockDim.x) {
      if (a.dbeta) a.dbeta[c] += a.bsums[c];
      if (a.dgamma) a.dgamma[c] += a.bsums[a.dim + c];
    }
  }
  const int rows_end = tail_rows(n, a.cap, a.zero_tail_rows);
  const int64_t total = static_cast<int64_t>(rows_end) * a.dim;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / a.dim);
    const int c = static_cast<int>(i % a.dim);
    __nv_bfloat16* dxp = a.dx + static_cast<int64_t>(r) * a.lddx + c;
    if (r >= n) {
      *dxp = __float2bfloat16_rn(0.f);
      continue;
    }
    float mean, rstd, var;
    bn_moments(a.sums, a.dim, c, n, a.eps, &mean, &rstd, &var);
    float g;
    if (a.dy_bf16) {
      g = __bfloat162float(a.dy_bf16[static_cast<int64_t>(r) * a.lddy + c]);
    } else {
      float* dyp = a.dy + static_cast<int64_t>(r) * a.lddy + c;
      g = *dyp;
      if (a.clear_dy) *dyp = 0.f;
    }
    if (a.y && __bfloat162float(a.y[static_cast<int64_t>(r) * a.ldy + c]) == 0.f) g = 0.f;
    const float xh = (__bfloat162float(a.x[static_cast<int64_t>(r) * a.ldx + c]) - mean) * rstd;
    const float d = a.gamma[c] * rstd * (g - inv_n * a.bsums[c] - xh * inv_n * a.bsums[a.dim + c]);
    *dxp = __float2bfloat16_rn(d);
  }
}

// ------------------------------------------------------------------ L2 normalisation
__global__ void l2norm_fwd_kernel(const __nv_bfloat16* z, int64_t ldz, int dim, const int32_t* n_ptr, int cap,
                                  __nv_bfloat16* y, int64_t ldy, float* norms) {
  GB_PDL_ENTRY();
  const int n = live_rows(n_ptr, cap);
  const int lane = threadIdx.x & 31;
  const int warps_total = (gridDim.x * blockDim.x) >> 5;
  const int rows_end = tail_rows(n, cap, 64);
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < rows_end; r += warps_total) {
    if (r >= n) {
      for (int c = lane * 8; c < dim; c += 256)
        *reinterpret_cast<uint4*>(y + static_cast<int64_t>(r) * ldy + c) = make_uint4(0, 0, 0, 0);
      continue;
    }
    float ss = 0.f;
    for (int c = lane * 8; c < dim; c += 256) {
      float f[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(z + static_cast<int64_t>(r) * ldz + c), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += f[j] * f[j];
    }
    ss = warp_sum(ss);
    float nr = sqrtf(ss);
    if (nr == 0.f) nr = 1.f;
    const float inv = 1.f / nr;
    if (lane == 0) norms[r] = nr;
    for (int c = lane * 8; c < dim; c += 256) {
      float f[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(z + static_cast<int64_t>(r) * ldz + c), f);
#pragma unroll
      for (int j = 0; j < 8; ++j) f[j] *= inv;
      *reinterpret_cast<uint4*>(y + static_cast<int64_t>(r) * ldy + c) = f32_to_bf16x8(f);
    }
  }
}

__global__ void l2norm_bwd_kernel(const __nv_bfloat16* y, int64_t ldy, float* dy, const __nv_bfloat16* dyb,
                                  int64_t lddy, const float* norms, int dim, const int32_t* n_ptr, int cap, float* dz,
                                  int64_t lddz) {
  GB_PDL_ENTRY();
  const int n = live_rows(n_ptr, cap);
  const int lane = threadIdx.x & 31;
  const int warps_total = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n; r += warps_total) {
    float dot = 0.f;
    for (int c = lane * 8; c < dim; c += 256) {
      float f[8], g[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(y + static_cast<int64_t>(r) * ldy + c), f);
      if (dyb) {
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(dyb + static_cast<int64_t>(r) * lddy + c), g);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) g[j] = dy[static_cast<int64_t>(r) * lddy + c + j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) dot += f[j] * g[j];
    }
    dot = warp_sum(dot);
    const float inv = 1.f / norms[r];
    for (int c = lane * 8; c < dim; c += 256) {
      float f[8], g[8];
      bf16x8_to_f32(*reinterpret_cast<const uint4*>(y + static_cast<int64_t>(r) * ldy + c), f);
      if (dyb) {
        bf16x8_to_f32(*reinterpret_cast<const uint4*>(dyb + static_cast<int64_t>(r) * lddy + c), g);
      } else {
        float* gp = dy + static_cast<int64_t>(r) * lddy + c;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          g[j] = gp[j];
          gp[j] = 0.f;
        }
      }
      float* o = dz + static_cast<int64_t>(r) * lddz + c;
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (g[j] - f[j] * dot) * inv;
    }
  }
}

__global__ void add_bf16_rows_kernel(float* dst, int64_t ldd, const __nv_bfloat16* src, int64_t lds, int dim,
                                     const int32_t* n_ptr, int cap) {
  GB_PDL_ENTRY();
  const int n = live_rows(n_ptr, cap);
  const int chunks = dim >> 3;
  const int64_t total = static_cast<int64_t>(n) * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / chunks);
    const int c = static_cast<int>(i % chunks) * 8;
    float f[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(src + static_cast<int64_t>(r) * lds + c), f);
    float* d = dst + static_cast<int64_t>(r) * ldd + c;
#pragma unroll
    for (int j = 0; j < 8; ++j) d[j] += f[j];
  }
}

// ------------------------------------------------------------------ dropout
__device__ __forceinline__ uint64_t dropout_key(const int64_t* counters, uint32_t salt) {
  return hop_key(static_cast<uint64_t>(counters[0]) ^ 0xD80Full, static_cast<uint64_t>(counters[1]),
                 static_cast<uint64_t>(counters[2]), salt);
}

__global__ void dropout_rows_kernel(const __nv_bfloat16* in, int64_t ldi, __nv_bfloat16* out, int64_t ldo, int dim,
                                    int64_t ld_mask, const int32_t* n_ptr, int cap, float p, const int64_t* counters,
                                    uint32_t salt) {
  GB_PDL_ENTRY();
  const int n = live_rows(n_ptr, cap);
  const int rows_end = tail_rows(n, cap, 64);
  const int chunks = dim >> 3;
  const uint64_t key = dropout_key(counters, salt);
  const uint32_t thr = dropout_thr8(p);
  const float ks = dropout_scale8(thr);
  const int64_t total = static_cast<int64_t>(rows_end) * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / chunks);
    const int c = static_cast<int>(i % chunks) * 8;
    uint4* op = reinterpret_cast<uint4*>(out + static_cast<int64_t>(r) * ldo + c);
    if (r >= n) {
      *op = make_uint4(0, 0, 0, 0);
      continue;
    }
    float f[8];
    bf16x8_to_f32(*reinterpret_cast<const uint4*>(in + static_cast<int64_t>(r) * ldi + c), f);
    const uint64_t base = static_cast<uint64_t>(r) * static_cast<uint64_t>(ld_mask) + static_cast<uint64_t>(c);
    const uint32_t keep = dropout_keep_bits(key, base, 8, thr);
#pragma unroll
    for (int j = 0; j < 8; ++j) f[j] = (keep >> j) & 1u ? f[j] * ks : 0.f;
    *op = f32_to_bf16x8(f);
  }
}

__global__ void dropout_grad_kernel(float* g, int64_t ldg, int dim, int64_t ld_mask, const int32_t* n_ptr, int cap,
                                    float p, const int64_t* counters, uint32_t salt) {
  GB_PDL_ENTRY();
  const int n = live_rows(n_ptr, cap);
  const int chunks = dim >> 3;
  const uint64_t key = dropout_key(counters, salt);
  const uint32_t thr = dropout_thr8(p);
  const float ks = dropout_scale8(thr);
  const int64_t total = static_cast<int64_t>(n) * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / chunks);
    const int c = static_cast<int>(i % chunks) * 8;
    float* gp = g + static_cast<int64_t>(r) * ldg + c;
    const uint64_t base = static_cast<uint64_t>(r) * static_cast<uint64_t>(ld_mask) + static_cast<uint64_t>(c);
    const uint32_t keep = dropout_keep_bits(key, base, 8, thr);
#pragma unroll
    for (int j = 0; j < 8; ++j) gp[j] = (keep >> j) & 1u ? gp[j] * ks : 0.f;
  }
}

__global__ void f32_to_bf16_rows_kernel(float* src, int64_t lds, __nv_bfloat16* dst, int64_t ldd, int dim,
                                        const int32_t* n_ptr, int cap, bool clear, int zt) {
  GB_PDL_ENTRY();
  const int n = live_rows(n_ptr, cap);
  const int rows_end = tail_rows(n, cap, zt);
  const int chunks = dim >> 3;
  const int64_t total = static_cast<int64_t>(rows_end) * chunks;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / chunks);
    const int c = static_cast<int>(i % chunks) * 8;
    uint4* dp = reinterpret_cast<uint4*>(dst + static_cast<int64_t>(r) * ldd + c);
    if (r >= n) {
      *dp = make_uint4(0, 0, 0, 0);
      continue;
    }
    float* sp = src + static_cast<int64_t>(r) * lds + c;
    const float4 a = *reinterpret_cast<float4*>(sp);
    const float4 b = *reinterpret_cast<float4*>(sp + 4);
    const float f[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    *dp = f32_to_bf16x8(f);
    if (clear) {
      *reinterpret_cast<float4*>(sp) = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(sp + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
}

}  // namespace

void launch_cross_entropy(const CeArgs& a, cudaStream_t stream) {
  if (a.n_classes <= 0 || a.n_classes > 1024) throw std::invalid_argument("cross_entropy: 1..1024 classes");
  const int grid = grid_1d(static_cast<int64_t>(a.cap_rows) * 32, 256, 8);
  const int cpl = (std::max(a.n_classes, static_cast<int32_t>(a.ld_dl)) + 31) / 32;
  if (cpl <= 1) launch_k(cross_entropy_kernel<1>, grid, 256, 0, stream, a);
  else if (cpl <= 2) launch_k(cross_entropy_kernel<2>, grid, 256, 0, stream, a);
  else if (cpl <= 4) launch_k(cross_entropy_kernel<4>, grid, 256, 0, stream, a);
  else if (cpl <= 8) launch_k(cross_entropy_kernel<8>, grid, 256, 0, stream, a);
  else if (cpl <= 16) launch_k(cross_entropy_kernel<16>, grid, 256, 0, stream, a);
  else launch_k(cross_entropy_kernel<32>, grid, 256, 0, stream, a);
  GB_LAUNCH_CHECK();
}

void launch_batchnorm_fwd(const BnArgs& a, cudaStream_t stream) {
  if (a.dim % 8 != 0 || a.ldx % 2 != 0 || a.ldy % 8 != 0) throw std::invalid_argument("batchnorm: dim % 8");
  if (a.training) {
    const int g = grid_1d(static_cast<int64_t>(a.cap) * 256 / 64, 256, 4);
    launch_k(bn_stats_kernel, g, 256, 0, stream, a);
    GB_LAUNCH_CHECK();
  }
  const int g2 = grid_1d(static_cast<int64_t>(a.cap) * (a.dim / 2), 256, 8);
  launch_k(bn_apply_kernel, g2, 256, 2 * a.dim * sizeof(float), stream, a);
  GB_LAUNCH_CHECK();
}

void launch_batchnorm_bwd(const BnBwdArgs& a, cudaStream_t stream) {
  const int g = grid_1d(static_cast<int64_t>(a.cap) * 256 / 64, 256, 4);
  launch_k(bn_bwd_reduce_kernel, g, 256, 0, stream, a);
  GB_LAUNCH_CHECK();
  const int g2 = grid_1d(static_cast<int64_t>(a.cap) * a.dim, 256, 8);
  launch_k(bn_bwd_apply_kernel, g2, 256, 0, stream, a);
  GB_LAUNCH_CHECK();
}

void launch_l2norm_fwd(const __nv_bfloat16* z, int64_t ldz, int32_t dim, const int32_t* n_ptr, int cap,
                       __nv_bfloat16* y, int64_t ldy, float* norms, cudaStream_t stream) {
  if (dim % 8 != 0) throw std::invalid_argument("l2norm: dim % 8");
  launch_k(l2norm_fwd_kernel, grid_1d(static_cast<int64_t>(cap) * 32, 256, 8), 256, 0, stream, z, ldz, dim, n_ptr, cap, y,
                                                                                         ldy, norms);
  GB_LAUNCH_CHECK();
}

void launch_l2norm_bwd(const __nv_bfloat16* y, int64_t ldy, float* dy, const __nv_bfloat16* dy_bf16, int64_t lddy,
                       const float* norms, int32_t dim, const int32_t* n_ptr, int cap, float* dz, int64_t lddz,
                       cudaStream_t stream) {
  if (dim % 8 != 0) throw std::invalid_argument("l2norm: dim % 8");
  launch_k(l2norm_bwd_kernel, grid_1d(static_cast<int64_t>(cap) * 32, 256, 8), 256, 0, stream, y, ldy, dy, dy_bf16, lddy,
                                                                                         norms, dim, n_ptr, cap, dz,
                                                                                         lddz);
  GB_LAUNCH_CHECK();
}

void launch_add_bf16_rows(float* dst, int64_t ldd, const __nv_bfloat16* src, int64_t lds, int32_t dim,
                          const int32_t* n_ptr, int cap, cudaStream_t stream) {
  if (dim % 8 != 0 || lds % 8 != 0) throw std::invalid_argument("add_bf16_rows: alignment");
  launch_k(add_bf16_rows_kernel, grid_1d(static_cast<int64_t>(cap) * (dim / 8), 256, 8), 256, 0, stream, dst, ldd, src, lds,
                                                                                                   dim, n_ptr, cap);
  GB_LAUNCH_CHECK();
}

void launch_dropout_rows(const __nv_bfloat16* in, int64_t ldi, __nv_bfloat16* out, int64_t ldo, int32_t dim,
                         int64_t ld_mask, const int32_t* n_ptr, int cap, float p, const int64_t* counters,
                         uint32_t salt, cudaStream_t stream) {
  if (dim % 8 != 0 || ld_mask % 8 != 0) throw std::invalid_argument("dropout_rows: dim and ld_mask % 8");
  launch_k(dropout_rows_kernel, grid_1d(static_cast<int64_t>(cap) * (dim / 8), 256, 8), 256, 0, stream, 
      in, ldi, out, ldo, dim, ld_mask, n_ptr, cap, p, counters, salt);
  GB_LAUNCH_CHECK();
}

void launch_dropout_grad(float* g, int64_t ldg, int32_t dim, int64_t ld_mask, const int32_t* n_ptr, int cap, float p,
                         const int64_t* counters, uint32_t salt, cudaStream_t stream) {
  if (dim % 8 != 0 || ld_mask % 8 != 0) throw std::invalid_argument("dropout_grad: dim and ld_mask % 8");
  launch_k(dropout_grad_kernel, grid_1d(static_cast<int64_t>(cap) * (dim / 8), 256, 8), 256, 0, stream, 
      g, ldg, dim, ld_mask, n_ptr, cap, p, counters, salt);
  GB_LAUNCH_CHECK();
}

void launch_f32_to_bf16_rows(float* src, int64_t lds, __nv_bfloat16* dst, int64_t ldd, int32_t dim,
                             const int32_t* n_ptr, int cap, bool clear, int32_t zero_tail_rows, cudaStream_t stream) {
  if (dim % 8 != 0 || lds % 4 != 0 || ldd % 8 != 0) throw std::invalid_argument("f32_to_bf16_rows: alignment");
  launch_k(f32_to_bf16_rows_kernel, grid_1d(static_cast<int64_t>(cap) * (dim / 8), 256, 8), 256, 0, stream, 
      src, lds, dst, ldd, dim, n_ptr, cap, clear, zero_tail_rows);
  GB_LAUNCH_CHECK();
}

}  // namespace dev
}  // namespace grappa
