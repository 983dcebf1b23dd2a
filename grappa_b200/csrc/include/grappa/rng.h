// Counter-based random numbers shared bit-for-bit by the C++ host code and the
// sm_100a kernels, so that every sampling decision the GPU makes can be replayed
// exactly on the CPU (the oracle used by the tests).
//
// Philox4x32-10 is the generator published by Salmon, Moraes, Dror and Shaw,
// "Parallel random numbers: as easy as 1, 2, 3" (SC'11); the multipliers and
// Weyl increments below are the ones given in that paper.  splitmix64's
// finaliser (Steele, Lea, Flood, "Fast splittable pseudorandom number
// generators", OOPSLA'14) is used to derive keys from (seed, epoch, step, hop).
//
// The reference seeds its C++ RNG from std::random_device (csrc/base/random.h:21-31)
// and shuffles with an unseeded torch.randperm (t10n/sampler.py:148-151); here
// every stream is a pure function of explicit counters.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define GB_HD __host__ __device__ __forceinline__
#else
#define GB_HD inline
#endif

namespace grappa {

struct U4 {
  uint32_t x, y, z, w;
};

GB_HD uint32_t mulhi32(uint32_t a, uint32_t b) {
#if defined(__CUDA_ARCH__)
  return __umulhi(a, b);
#else
  return static_cast<uint32_t>((static_cast<uint64_t>(a) * b) >> 32);
#endif
}

GB_HD U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
#if defined(__CUDACC__)
#pragma unroll
#endif
  for (int r = 0; r < 10; ++r) {
    const uint32_t hi0 = mulhi32(0xD2511F53u, c.x);
    const uint32_t lo0 = 0xD2511F53u * c.x;
    const uint32_t hi1 = mulhi32(0xCD9E8D57u, c.z);
    const uint32_t lo1 = 0xCD9E8D57u * c.z;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

GB_HD uint32_t u4_word(const U4& v, int i) {
  return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w));
}

GB_HD uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// Key of one sampling hop.  Every rank, the GPU sampler and the CPU oracle
// derive the same key from the same (seed, epoch, step, hop).
GB_HD uint64_t hop_key(uint64_t seed, uint64_t epoch, uint64_t step, uint64_t hop) {
  uint64_t k = mix64(seed);
  k = mix64(k ^ (epoch * 0x100000001B3ull));
  k = mix64(k ^ (step * 0xC2B2AE3D27D4EB4Full));
  k = mix64(k ^ (hop + 0x165667B19E3779F9ull));
  return k;
}

// The t-th 32-bit draw of node `nid` under key `key`.
GB_HD uint32_t node_draw(uint64_t key, uint64_t nid, uint32_t t) {
  const U4 c{static_cast<uint32_t>(nid), static_cast<uint32_t>(nid >> 32), t >> 2, 0x5A3Cu};
  const U4 r = philox4x32_10(c, static_cast<uint32_t>(key), static_cast<uint32_t>(key >> 32));
  return u4_word(r, static_cast<int>(t & 3u));
}

// Uniform integer in [0, n) from a 32-bit draw (multiply-shift range reduction,
// D. Lemire, "Fast random integer generation in an interval", TOMACS 2019,
// without the rejection step; the bias is below n / 2^32).
GB_HD uint32_t draw_below(uint32_t r, uint32_t n) { return mulhi32(r, n); }

// Four 32-bit draws for an element index (edge generation, dropout masks, features).
GB_HD U4 index_draw4(uint64_t key, uint64_t idx, uint32_t salt) {
  const U4 c{static_cast<uint32_t>(idx), static_cast<uint32_t>(idx >> 32), salt, 0xC0FFEEu};
  return philox4x32_10(c, static_cast<uint32_t>(key), static_cast<uint32_t>(key >> 32));
}

// Dropout masks at byte resolution: the probability is quantised to t / 256
// (t = round(p * 256)) and element idx is kept iff byte idx % 16 of the 16-byte draw of
// group idx / 16 is >= t, so one Philox call serves 16 elements; kept values are scaled
// by 256 / (256 - t), which keeps the expectation exact for the quantised probability.
constexpr uint32_t kDropoutSalt = 0x44u;
GB_HD uint32_t dropout_thr8(float p) {
  int t = static_cast<int>(p * 256.0f + 0.5f);
  return static_cast<uint32_t>(t < 0 ? 0 : (t > 255 ? 255 : t));
}
GB_HD float dropout_scale8(uint32_t thr8) { return 256.0f / static_cast<float>(256u - thr8); }
// bit b: byte b of the draw is >= thr8
GB_HD uint32_t keep16(const U4& r, uint32_t thr8) {
  uint32_t k = 0;
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
  for (int i = 0; i < 4; ++i)
    for (int b = 0; b < 4; ++b)
      if (((w[i] >> (8 * b)) & 0xFFu) >= thr8) k |= 1u << (4 * i + b);
  return k;
}
// keep bits of the n <= 32 consecutive elements base .. base + n - 1 (bit j: base + j)
GB_HD uint32_t dropout_keep_bits(uint64_t key, uint64_t base, int n, uint32_t thr8) {
  uint64_t g = base >> 4;
  const int off = static_cast<int>(base & 15u);
  uint64_t acc = static_cast<uint64_t>(keep16(index_draw4(key, g, kDropoutSalt), thr8)) >> off;
  int have = 16 - off;
  while (have < n) {
    ++g;
    acc |= static_cast<uint64_t>(keep16(index_draw4(key, g, kDropoutSalt), thr8)) << have;
    have += 16;
  }
  return n >= 32 ? static_cast<uint32_t>(acc) : static_cast<uint32_t>(acc & ((1ull << n) - 1));
}

// Uniform float in [0, 1) from the top 24 bits of a draw.
GB_HD float u01(uint32_t r) { return static_cast<float>(r >> 8) * (1.0f / 16777216.0f); }

// Hash partitioner: partition id of a global node id.
GB_HD int32_t hash_part(uint64_t nid, uint64_t seed, int32_t n_part) {
  return static_cast<int32_t>(mix64(nid ^ mix64(seed ^ 0x7061727469ull)) % static_cast<uint64_t>(n_part));
}

// Sampling of `k` distinct in-neighbour offsets out of `d` (d > k) for node
// `nid`: the offsets are the first k distinct values of the sequence
//   o_t = draw_below(node_draw(key, nid, t), d),  t = 0, 1, 2, ...
// taken in order of first appearance.  The first k distinct values of an i.i.d.
// uniform sequence form a uniform random k-subset, which is the distribution the
// reference draws with a sparse Fisher-Yates shuffle (csrc/base/random.h:38-141).
// After kMaxDraws draws the remaining slots take the smallest unused offsets in
// increasing order (never reached in practice: it needs kMaxDraws draws to miss
// one of the d > k values).
constexpr uint32_t kMaxDraws = 32u * 64u;

}  // namespace grappa
