// K-AR: the coverage-weighted gradient all-reduce fused with Adam, over NVLink peer
// memory (IPC-mapped buffers, ordinary 16-byte loads and stores, release/acquire
// flags at system scope).  One launch per gradient bucket, so that a bucket is
// reduced while the backward pass still computes the earlier layers' gradients.
//
// The reference scales each rank's DDP bucket by c_r / W and sums it with an NCCL
// all-reduce, then runs torch.optim.Adam (t10n/grad.py:6-24,
// experiments/grappa/train/t10n_train.py:103-114,159-162,248).  Here one kernel per
// bucket does the scaling, the bf16 -> fp32 cast of bf16 gradients, the reduction and
// the Adam update.  Two modes:
//
//   kOneShot  every rank copies its scaled bucket into a send slot (fp32, parity
//             double-buffered), raises a flag at every peer, reads all W copies and
//             runs Adam on the whole bucket.  One flag round trip: for small buckets.
//   kShard    reduce-scatter -> Adam on the owned shard -> all-gather.  Rank s owns
//             shard s of the bucket; it reads shard s of every rank's gradient
//             straight from the peers' gradient buffers (no copy), sums c_p/W-weighted
//             in rank order, updates its fp32 master weights, moments and bf16 copy
//             of the shard, and raises a flag; every rank then pulls the other shards'
//             updated fp32 master weights from their owners and writes its bf16
//             copy.  Each rank moves (W-1)/W of the gradient plus (W-1)/W of the fp32
//             parameters and does 1/W of the Adam work.  The Adam moments of a shard
//             live only on its owner (sync_moments gathers them for checkpoints).
//
// Work split: CTA j of every rank handles piece j of every shard (the same grid on
// every rank), and all flags are per (rank, CTA), so no CTA waits for another CTA
// of its own rank.  Flags carry the tag step + 1 and are compared wrap-safe with
// >=; every wait is bounded by a %globaltimer deadline, after which the CTA sets
// kErrPeerTimeout in the error word and returns.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace grappa {
namespace ar {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 160;                               // grid limit of one bucket launch
constexpr int kFlagWords = 2 * kMaxRanks * kMaxCtas;        // ready[rank][cta], done[rank][cta]
constexpr int64_t kFlagPageBytes = kFlagWords * 4;          // one page per bucket
enum Mode : int32_t { kOneShot = 0, kShard = 1 };

struct Args {
  int32_t rank = 0, world = 1;
  int32_t mode = kShard;
  bool grad_bf16 = false;                // gradient element type (fp32 or bf16)
  int64_t lo = 0, hi = 0;                // bucket [lo, hi) in elements; lo a multiple of 8
  // gradient: this rank's (cleared over [lo, hi) before the kernel returns) and every
  // rank's peer mapping (kShard reads the peers' buffers directly)
  void* grad = nullptr;
  const void* grad_peer[kMaxRanks] = {};
  // kOneShot send slots (fp32, scaled): this rank's [2] and every rank's [W][2]
  float* slot_local[2] = {nullptr, nullptr};
  const float* slot_peer[kMaxRanks][2] = {};
  // parameters: fp32 master (peer-mapped for kShard), moments, bf16 working copy
  float* param = nullptr;
  const float* param_peer[kMaxRanks] = {};
  float* m = nullptr;
  float* v = nullptr;
  __nv_bfloat16* wbf = nullptr;
  // this rank's published c_r / W ([2], by step parity) and every rank's mapping
  float* scale_local = nullptr;
  const float* scale_peer[kMaxRanks] = {};
  // the bucket's flag page: this rank's and every rank's mapping
  uint32_t* flags_local = nullptr;
  uint32_t* flags_peer[kMaxRanks] = {};
  const float* cov = nullptr;            // [sum, count] of this rank's coverage ratios (null: weight 1)
  const int64_t* counters = nullptr;     // [seed, epoch, step, global_step, gen, adam_t]
  float lr = 1e-3f, beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, weight_decay = 0.f;
  bool do_adam = true;                   // false (kOneShot only): write the reduced gradient to grad_out
  float* grad_out = nullptr;
  int32_t* err = nullptr;
  int64_t timeout_ns = 10000000000ll;
};

// grid: CTAs of the launch (1..kMaxCtas; the same on every rank)
void launch(const Args& a, int grid, cudaStream_t stream);

}  // namespace ar
}  // namespace grappa
