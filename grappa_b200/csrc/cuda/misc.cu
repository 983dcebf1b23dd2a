// Element-wise and gather kernels of the training step, the synthetic-data
// generators, and the fused Adam update.
#include <cstdlib>

#include "common.cuh"
#include "grappa/rng.h"
#include "kernels.h"

#include <algorithm>

namespace grappa {
namespace dev {

namespace {

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

int grid_1d(int64_t n, int threads, int per_sm = 8) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(n > 0 ? n : 1, threads), int64_t(sm_count()) * per_sm)));
}

// ---------------------------------------------------------------- act_bwd
// One row chunk of act_bwd: g = dh * scale, masked by h > 0 when h is given (ReLU),
// rounded to bf16 (the value the GEMMs consume), accumulated into colsum.
__device__ __forceinline__ uint4 act_bwd_chunk(const ActBwdArgs& a, const float4& d0, const float4& d1, const uint4& hv,
                                              float (&colsum)[8]) {
  float g[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
  if (a.h) {
    float h[8];
    bf16x8_to_f32(hv, h);
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = h[j] != 0.f ? g[j] * a.scale : 0.f;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] *= a.scale;
  }
  const uint4 packed = f32_to_bf16x8(g);
  bf16x8_to_f32(packed, g);
#pragma unroll
  for (int j = 0; j < 8; ++j) colsum[j] += g[j];
  return packed;
}

// Two rows per iteration with both rows' loads issued first: the kernel streams dH
// (fp32, cleared for the next step), H and dY once and is bound by the latency of
// those loads at one row in flight per thread.
__global__ void act_bwd_kernel(ActBwdArgs a, int chunks) {
  GB_PDL_ENTRY();
  extern __shared__ float s_col[];  // [blockDim.x * 8]
  const int n = a.n_ptr ? *a.n_ptr : a.n;
  const int rpb = blockDim.x / chunks;
  const int c = threadIdx.x % chunks;
  const int r_in = threadIdx.x / chunks;
  const int tail = static_cast<int>(ceil_div(n, 64) * 64);
  const int rows_end = min(tail, a.cap_rows > 0 ? a.cap_rows : tail);
  const int rstride = gridDim.x * rpb;
  float colsum[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int r0 = blockIdx.x * rpb + r_in; r0 < rows_end; r0 += 2 * rstride) {
    const int rr[2] = {r0, r0 + rstride};
    float4 d[2][2];
    uint4 hv[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      d[k][0] = d[k][1] = make_float4(0.f, 0.f, 0.f, 0.f);
      if (rr[k] < n) {
        const float* dh = a.dh + static_cast<int64_t>(rr[k]) * a.dh_stride + c * 8;
        d[k][0] = *reinterpret_cast<const float4*>(dh);
        d[k][1] = *reinterpret_cast<const float4*>(dh + 4);
        if (a.h) hv[k] = *reinterpret_cast<const uint4*>(a.h + static_cast<int64_t>(rr[k]) * a.h_stride + c * 8);
      }
    }
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int r = rr[k];
      if (r >= rows_end) continue;
      uint4 out = make_uint4(0, 0, 0, 0);
      if (r < n) {
        float* dh = a.dh + static_cast<int64_t>(r) * a.dh_stride + c * 8;
        *reinterpret_cast<float4*>(dh) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(dh + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        out = act_bwd_chunk(a, d[k][0], d[k][1], hv[k], colsum);
      }
      *reinterpret_cast<uint4*>(a.dy + static_cast<int64_t>(r) * a.dy_stride + c * 8) = out;
    }
  }
  if (!a.dbias) return;
#pragma unroll
  for (int j = 0; j < 8; ++j) s_col[threadIdx.x * 8 + j] = colsum[j];
  __syncthreads();
  for (int t = threadIdx.x; t < chunks * 8; t += blockDim.x) {
    const int cc = t / 8, j = t % 8;
    float s = 0.f;
    for (int q = 0; q < rpb; ++q) s += s_col[(q * chunks + cc) * 8 + j];
    if (s != 0.f) atomicAdd(a.dbias + cc * 8 + j, s);
  }
}

// ---------------------------------------------------------------- gathers
template <bool F32>
__global__ void gather_rows_kernel(const void* table, int64_t ts, int dim, const int32_t* ids, const int32_t* n_ptr,
                                   int n_static, __nv_bfloat16* out, int64_t os) {
  GB_PDL_ENTRY();
  const int n = n_ptr ? *n_ptr : n_static;
  const int chunks = dim >> 3;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; r < n; r += warps) {
    const int64_t src = ids[r];
    for (int c = lane; c < chunks; c += 32) {
      uint4 v;
      if (F32) {
        const float* t = reinterpret_cast<const float*>(table) + src * ts + c * 8;
        const float4 x = *reinterpret_cast<const float4*>(t);
        const float4 y = *reinterpret_cast<const float4*>(t + 4);
        const float f[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
        v = f32_to_bf16x8(f);
      } else {
        v = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(table) + src * ts + c * 8);
      }
      *reinterpret_cast<uint4*>(out + r * os + c * 8) = v;
    }
  }
}

template <typename T>
__global__ void gather_scalar_kernel(const T* table, const int32_t* ids, const int32_t* n_ptr, int n_static, T* out) {
  GB_PDL_ENTRY();
  const int n = n_ptr ? *n_ptr : n_static;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) out[i] = table[ids[i]];
}

// ---------------------------------------------------------------- generators
__global__ void rmat_kernel(int64_t n, int scale, uint64_t ta, uint64_t tb, uint64_t tc, uint64_t key, int64_t e0,
                            int64_t count, int64_t* keys) {
  GB_PDL_ENTRY();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t e = static_cast<uint64_t>(e0 + i);
    uint64_t u = 0, v = 0;
    U4 r{0, 0, 0, 0};
    for (int l = 0; l < scale; ++l) {
      if ((l & 3) == 0) r = index_draw4(key, e, static_cast<uint32_t>(l >> 2));
      const uint64_t x = u4_word(r, l & 3);
      const uint64_t bu = x >= tb ? 1u : 0u;
      const uint64_t bv = ((x >= ta && x < tb) || x >= tc) ? 1u : 0u;
      u = (u << 1) | bu;
      v = (v << 1) | bv;
    }
    int64_t out = -1;
    if (u < static_cast<uint64_t>(n) && v < static_cast<uint64_t>(n) && u != v) {
      const uint64_t lo = u < v ? u : v, hi = u < v ? v : u;
      out = static_cast<int64_t>(lo * static_cast<uint64_t>(n) + hi);
    }
    keys[i] = out;
  }
}

__global__ void shuffle_keys_kernel(const int64_t* ids, int64_t n, uint64_t k, int64_t* keys) {
  GB_PDL_ENTRY();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    keys[i] = static_cast<int64_t>(mix64(static_cast<uint64_t>(ids[i]) ^ k) >> 1);
}

// Box-Muller transform of Philox uniforms (standard normal samples).
__global__ void normal_kernel(float* out, int64_t n, uint64_t key) {
  GB_PDL_ENTRY();
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; 2 * i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const U4 r = index_draw4(key, static_cast<uint64_t>(i), 7u);
    const float u1 = (static_cast<float>(r.x >> 8) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>(r.y >> 8) * (1.0f / 16777216.0f);
    const float rad = sqrtf(-2.0f * logf(u1));
    float s, c;
    sincospif(2.0f * u2, &s, &c);
    out[2 * i] = rad * c;
    if (2 * i + 1 < n) out[2 * i + 1] = rad * s;
  }
}

// Rows [row0, row0 + rows) of the [*, d] matrix whose flat element i is the normal
// value of index i (the stream of normal_kernel), as bf16 rows of stride ld (columns
// past d zeroed).  d is even, so a Box-Muller pair never straddles two rows.
__global__ void normal_rows_kernel(__nv_bfloat16* out, int64_t ld, int64_t row0, int64_t rows, int d,
                                   uint64_t key) {
  GB_PDL_ENTRY();
  const int64_t pairs_per_row = d / 2;
  const int64_t total = rows * pairs_per_row;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = t / pairs_per_row;
    const int c = static_cast<int>(t % pairs_per_row) * 2;
    const uint64_t pair = static_cast<uint64_t>(((row0 + r) * d + c) >> 1);
    const U4 q = index_draw4(key, pair, 7u);
    const float u1 = (static_cast<float>(q.x >> 8) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>(q.y >> 8) * (1.0f / 16777216.0f);
    const float rad = sqrtf(-2.0f * logf(u1));
    float sn, cs;
    sincospif(2.0f * u2, &sn, &cs);
    __nv_bfloat162* o = reinterpret_cast<__nv_bfloat162*>(out + r * ld + c);
    *o = __floats2bfloat162_rn(rad * cs, rad * sn);
    if (c + 2 == d)
      for (int64_t z = d; z < ld; ++z) out[r * ld + z] = __float2bfloat16_rn(0.f);
  }
}

__global__ void dropout_mask_kernel(uint8_t* mask, int64_t rows, int64_t cols, int64_t ld, uint32_t thr,
                                    const int64_t* counters, uint32_t salt) {
  GB_PDL_ENTRY();
  const uint64_t key = hop_key(static_cast<uint64_t>(counters[0]) ^ 0xD80Full, static_cast<uint64_t>(counters[1]),
                               static_cast<uint64_t>(counters[2]), salt);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < rows * cols;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const uint64_t idx = static_cast<uint64_t>(r) * static_cast<uint64_t>(ld) + static_cast<uint64_t>(c);
    mask[i] = static_cast<uint8_t>(dropout_keep_bits(key, idx, 1, thr) & 1u);
  }
}

// ---------------------------------------------------------------- Adam
// Same update as torch.optim.Adam (no amsgrad): m = b1 m + (1-b1) g,
// v = b2 v + (1-b2) g^2, p -= lr/bc1 * m / (sqrt(v)/sqrt(bc2) + eps).
__device__ __forceinline__ float adam_elem(const AdamArgs& a, float g, float& p, float& m, float& v, float step_size,
                                           float inv_sqrt_bc2) {
  if (a.weight_decay != 0.f) g += a.weight_decay * p;
  m = a.beta1 * m + (1.f - a.beta1) * g;
  v = a.beta2 * v + (1.f - a.beta2) * g * g;
  p -= step_size * m / (sqrtf(v) * inv_sqrt_bc2 + a.eps);
  return p;
}

// VEC: four elements per thread with 16-byte loads, all issued before the
// arithmetic (the update is one streaming pass over g, p, m and v); the elements
// past the last multiple of four, and buffers that are not 16-byte aligned, take the
// scalar path.
template <bool VEC>
__global__ void adam_kernel(AdamArgs a) {
  GB_PDL_ENTRY();
  const float t = static_cast<float>(*a.step + 1);
  const float bc1 = 1.f - powf(a.beta1, t);
  const float bc2 = 1.f - powf(a.beta2, t);
  const float step_size = a.lr / bc1;
  const float inv_sqrt_bc2 = rsqrtf(bc2);
  const float gs = a.grad_scale * (a.grad_scale_dev ? *a.grad_scale_dev : 1.f);
  const int64_t tid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  const int64_t nthreads = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int64_t scalar_from = 0;
  if (VEC) {
    const int64_t n4 = a.n / 4;
    scalar_from = n4 * 4;
    for (int64_t q = tid; q < n4; q += nthreads) {
      float4 g = reinterpret_cast<const float4*>(a.grad)[q];
      float4 p = reinterpret_cast<const float4*>(a.param)[q];
      float4 m = reinterpret_cast<const float4*>(a.m)[q];
      float4 v = reinterpret_cast<const float4*>(a.v)[q];
      if (a.clear_grad) reinterpret_cast<float4*>(a.grad)[q] = make_float4(0.f, 0.f, 0.f, 0.f);
      adam_elem(a, g.x * gs, p.x, m.x, v.x, step_size, inv_sqrt_bc2);
      adam_elem(a, g.y * gs, p.y, m.y, v.y, step_size, inv_sqrt_bc2);
      adam_elem(a, g.z * gs, p.z, m.z, v.z, step_size, inv_sqrt_bc2);
      adam_elem(a, g.w * gs, p.w, m.w, v.w, step_size, inv_sqrt_bc2);
      reinterpret_cast<float4*>(a.param)[q] = p;
      reinterpret_cast<float4*>(a.m)[q] = m;
      reinterpret_cast<float4*>(a.v)[q] = v;
      if (a.param_bf16) {
        __nv_bfloat16 w[4] = {__float2bfloat16_rn(p.x), __float2bfloat16_rn(p.y), __float2bfloat16_rn(p.z),
                              __float2bfloat16_rn(p.w)};
        reinterpret_cast<uint2*>(a.param_bf16)[q] = *reinterpret_cast<uint2*>(w);
      }
    }
  }
  for (int64_t i = scalar_from + tid; i < a.n; i += nthreads) {
    const float g = a.grad[i] * gs;
    if (a.clear_grad) a.grad[i] = 0.f;
    float p = a.param[i], m = a.m[i], v = a.v[i];
    adam_elem(a, g, p, m, v, step_size, inv_sqrt_bc2);
    a.m[i] = m;
    a.v[i] = v;
    a.param[i] = p;
    if (a.param_bf16) a.param_bf16[i] = __float2bfloat16_rn(p);
  }
}

// counters = [seed, epoch, step_in_epoch, global_step, gen, adam_t]
__global__ void sampler_counters_kernel(const int64_t* main, int64_t* dst, int64_t step_offset) {
  GB_PDL_ENTRY();
  dst[0] = main[0];
  dst[1] = main[1];
  dst[2] = main[2] + step_offset;
  dst[3] = main[3] + step_offset;
  dst[4] += 1;  // the sampler's own compaction generation
  dst[5] = main[5];
}

__global__ void step_end_kernel(int64_t* counters, const int64_t* ring_slot, float* fstats, int nf, int32_t* istats,
                                int ni) {
  GB_PDL_ENTRY();
  if (ring_slot) {
    float* ring = reinterpret_cast<float*>(static_cast<uintptr_t>(*ring_slot));
    if (ring && fstats) ring[counters[2]] = fstats[2];
  }
  for (int i = 0; i < nf; ++i) fstats[i] = 0.f;
  for (int i = 0; i < ni; ++i) istats[i] = 0;
  counters[2] += 1;
  counters[3] += 1;
  counters[4] += 1;
  counters[5] += 1;
}

__global__ void sample_prologue_kernel(SamplePrologueArgs a) {
  GB_PDL_ENTRY();
  const int64_t row = a.main[2] + a.step_offset;
  const int32_t* table =
      a.table_slot ? reinterpret_cast<const int32_t*>(static_cast<uintptr_t>(*a.table_slot)) : nullptr;
  const int n = table ? (row >= 0 && row < a.n_rows ? a.count_table[row] : 0) : *a.n_seeds;
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    a.dst[0] = a.main[0];
    a.dst[1] = a.main[1];
    a.dst[2] = a.main[2] + a.step_offset;
    a.dst[3] = a.main[3] + a.step_offset;
    a.dst[4] += 1;  // the sampler's own compaction generation
    a.dst[5] = a.main[5];
    if (a.cov) {
      a.cov[0] = 0.f;
      a.cov[1] = 0.f;
    }
  }
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < a.B; i += gridDim.x * blockDim.x) {
    int32_t s;
    if (table) {
      s = i < n ? table[row * a.B + i] : 0;
      a.seeds[i] = s;
    } else {
      s = a.seeds[i];
    }
    if (i < n) {
      if (a.seed_labels) a.seed_labels[i] = a.labels[s];
      if (a.seed_gideg) a.seed_gideg[i] = a.gideg[s];
    }
  }
  // every block derived n itself; one writes it (the table-less path only reads it)
  if (table && blockIdx.x == 0 && threadIdx.x == 0) *a.n_seeds = n;
}

}  // namespace

void launch_act_bwd(const ActBwdArgs& a, cudaStream_t stream) {
  if (a.dim % 8 != 0) throw std::invalid_argument("act_bwd: dim must be a multiple of 8");
  const int chunks = a.dim / 8;
  if (chunks > 256) throw std::invalid_argument("act_bwd: dim too large");
  const int rpb = std::max(1, 256 / chunks);
  const int threads = chunks * rpb;
  const int rows = a.cap_rows > 0 ? a.cap_rows : a.n;
  // with a bias gradient every block ends with one atomic per column: fewer blocks per
  // SM than without, so that those atomics do not queue up on the same words
  // (GRAPPA_ACT_BWD_BLOCKS_PER_SM overrides the count with a bias gradient; the
  // GraphSAGE epoch measured 0.0360 s with 3, 0.0364 with 6, 0.0378 with 12)
  static const int per_sm_bias = [] {
    const char* e = std::getenv("GRAPPA_ACT_BWD_BLOCKS_PER_SM");
    const int v = e ? std::atoi(e) : 3;
    return v > 0 ? v : 3;
  }();
  const int per_sm = a.dbias ? per_sm_bias : 8;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(ceil_div(rows, rpb), int64_t(sm_count()) * per_sm)));
  launch_k(act_bwd_kernel, grid, threads, threads * 8 * sizeof(float), stream, a, chunks);
  GB_LAUNCH_CHECK();
}

void launch_gather_rows_bf16(const void* table, bool table_f32, int64_t table_stride, int32_t dim, const int32_t* ids,
                             const int32_t* n_ptr, int32_t n, int cap, __nv_bfloat16* out, int64_t out_stride,
                             cudaStream_t stream) {
  if (dim % 8 != 0) throw std::invalid_argument("gather: dim must be a multiple of 8");
  const int grid = grid_1d(static_cast<int64_t>(cap) * 32, 256, 16);
  if (table_f32)
    launch_k(gather_rows_kernel<true>, grid, 256, 0, stream, table, table_stride, dim, ids, n_ptr, n, out, out_stride);
  else
    launch_k(gather_rows_kernel<false>, grid, 256, 0, stream, table, table_stride, dim, ids, n_ptr, n, out, out_stride);
  GB_LAUNCH_CHECK();
}

void launch_gather_i32(const int32_t* table, const int32_t* ids, const int32_t* n_ptr, int n, int cap, int32_t* out,
                       cudaStream_t stream) {
  launch_k(gather_scalar_kernel<int32_t>, grid_1d(cap, 256), 256, 0, stream, table, ids, n_ptr, n, out);
  GB_LAUNCH_CHECK();
}
void launch_gather_i64(const int64_t* table, const int32_t* ids, const int32_t* n_ptr, int n, int cap, int64_t* out,
                       cudaStream_t stream) {
  launch_k(gather_scalar_kernel<int64_t>, grid_1d(cap, 256), 256, 0, stream, table, ids, n_ptr, n, out);
  GB_LAUNCH_CHECK();
}

void launch_rmat_candidates(int64_t n, int scale, double a, double b, double c, uint64_t seed, int64_t e_begin,
                            int64_t count, int64_t* keys, cudaStream_t stream) {
  const uint64_t ta = static_cast<uint64_t>(a * 4294967296.0);
  const uint64_t tb = static_cast<uint64_t>((a + b) * 4294967296.0);
  const uint64_t tc = static_cast<uint64_t>((a + b + c) * 4294967296.0);
  launch_k(rmat_kernel, grid_1d(count, 256, 32), 256, 0, stream, n, scale, ta, tb, tc, mix64(seed ^ 0x524D4154ull), e_begin,
                                                          count, keys);
  GB_LAUNCH_CHECK();
}

void launch_shuffle_keys(const int64_t* ids, int64_t n, uint64_t seed, uint64_t epoch, int64_t* keys,
                         cudaStream_t stream) {
  const uint64_t k = mix64(mix64(seed ^ 0x5348554646ull) ^ epoch);
  launch_k(shuffle_keys_kernel, grid_1d(n, 256, 16), 256, 0, stream, ids, n, k, keys);
  GB_LAUNCH_CHECK();
}

void launch_normal_fill(float* out, int64_t n, uint64_t seed, cudaStream_t stream) {
  launch_k(normal_kernel, grid_1d((n + 1) / 2, 256, 32), 256, 0, stream, out, n, mix64(seed ^ 0x4E4F524Dull));
  GB_LAUNCH_CHECK();
}

void launch_normal_rows_bf16(__nv_bfloat16* out, int64_t ld, int64_t row0, int64_t rows, int d, uint64_t seed,
                             cudaStream_t stream) {
  if (d % 2 != 0) throw std::invalid_argument("normal_rows: d must be even");
  launch_k(normal_rows_kernel, grid_1d(rows * (d / 2), 256, 32), 256, 0, stream, out, ld, row0, rows, d,
                                                                          mix64(seed ^ 0x4E4F524Dull));
  GB_LAUNCH_CHECK();
}

void launch_dropout_mask(uint8_t* mask, int64_t rows, int64_t cols, int64_t ld, float p, const int64_t* counters,
                         uint32_t salt, cudaStream_t stream) {
  const uint32_t thr = dropout_thr8(p);
  launch_k(dropout_mask_kernel, grid_1d(rows * cols, 256, 16), 256, 0, stream, mask, rows, cols, ld, thr, counters, salt);
  GB_LAUNCH_CHECK();
}

void launch_adam(const AdamArgs& a, cudaStream_t stream) {
  const bool vec = ((reinterpret_cast<uintptr_t>(a.grad) | reinterpret_cast<uintptr_t>(a.param) |
                     reinterpret_cast<uintptr_t>(a.m) | reinterpret_cast<uintptr_t>(a.v)) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(a.param_bf16) & 7u) == 0;
  if (vec)
    launch_k(adam_kernel<true>, grid_1d((a.n + 3) / 4, 256, 4), 256, 0, stream, a);
  else
    launch_k(adam_kernel<false>, grid_1d(a.n, 256, 4), 256, 0, stream, a);
  GB_LAUNCH_CHECK();
}

void launch_sampler_counters(const int64_t* main, int64_t* dst, int64_t step_offset, cudaStream_t stream) {
  launch_k(sampler_counters_kernel, 1, 1, 0, stream, main, dst, step_offset);
  GB_LAUNCH_CHECK();
}

void launch_step_end(int64_t* counters, const int64_t* ring_slot, float* fstats, int nf, int32_t* istats, int ni,
                     cudaStream_t stream) {
  launch_k(step_end_kernel, 1, 1, 0, stream, counters, ring_slot, fstats, fstats ? nf : 0, istats, istats ? ni : 0);
  GB_LAUNCH_CHECK();
}

void launch_sample_prologue(const SamplePrologueArgs& a, cudaStream_t stream) {
  if (a.B <= 0) throw std::invalid_argument("sample_prologue: empty batch capacity");
  if (a.table_slot && !a.count_table) throw std::invalid_argument("sample_prologue: a seed table needs its counts");
  if ((a.seed_labels && !a.labels) || (a.seed_gideg && !a.gideg))
    throw std::invalid_argument("sample_prologue: gathered outputs need their tables");
  const int threads = 1024;
  const int blocks = static_cast<int>(std::min<int64_t>(8, (a.B + threads - 1) / threads));
  launch_k(sample_prologue_kernel, blocks, threads, 0, stream, a);
  GB_LAUNCH_CHECK();
}

}  // namespace dev
}  // namespace grappa
