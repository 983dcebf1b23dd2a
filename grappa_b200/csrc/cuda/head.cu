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

#include "common.cuh"
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

}  // namespace

bool sage_head_supported(int ip, int n_classes) {
  return ip > 0 && ip % 8 == 0 && ip <= 256 && n_classes > 0 && n_classes <= 64;
}

void launch_sage_head(const SageHeadArgs& a, cudaStream_t stream) {
  if (!sage_head_supported(a.ip, a.n_classes)) throw std::invalid_argument("sage head: ip % 8, ip <= 256, <= 64 classes");
  if (a.ldh % 8 || a.ldx % 8 || a.ldw % 8 || (a.dx && a.lddx % 8))
    throw std::invalid_argument("sage head: row strides must be multiples of 8 elements");
  if (a.ld_dl < a.n_classes) throw std::invalid_argument("sage head: dlogits row shorter than the classes");
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
