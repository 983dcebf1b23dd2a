// Argument blocks and launchers of the sm_100a kernels (no torch types here; the
// torch bindings live in bindings.cpp).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace grappa {
namespace dev {

// ---------------------------------------------------------------- sampling (S1)
struct SampleHopArgs {
  const int64_t* indptr = nullptr;   // graph CSC by dst, [n_graph_nodes + 1]
  const int32_t* indices = nullptr;  // graph sources
  int64_t n_graph_nodes = 0;
  const int32_t* dst_nid = nullptr;  // block destinations (graph ids)
  const int32_t* n_dst_ptr = nullptr;  // device count, or null to use n_dst
  int32_t n_dst = 0;
  const uint8_t* frontier = nullptr;   // null: every dst samples
  int32_t fanout = 0;                  // < 0: all neighbours
  bool replace = false;
  const int64_t* counters = nullptr;   // device [seed, epoch, step, ...]
  int32_t hop = 0;
  const int64_t* gideg = nullptr;      // per dst global in-degree (seed hop) or null
  float* cov_accum = nullptr;          // device [sum, count]
  int32_t* out_indptr = nullptr;       // [cap_dst + 1]
  int32_t* out_nbr = nullptr;          // [cap_edges]
  int32_t cap_edges = 0;
  int32_t* n_edges_out = nullptr;
  unsigned long long* scan_scratch = nullptr;
  int32_t* err = nullptr;
  // optional: the first pass of the block compaction (compact.cu K1) fused into the
  // hop — map[dst_nid[i]] and map[out_nbr[e]] take the atomicMin of this call's tag
  // word (from counters[4] and slot = hop) with positions i and n_dst + e, and
  // src_nid[i] = dst_nid[i], src_sampled[i] = 0 for the destinations
  unsigned long long* map = nullptr;   // dense [map_nodes]
  int64_t map_nodes = 0;
  int32_t* src_nid = nullptr;
  uint8_t* src_sampled = nullptr;
};
void launch_sample_hop(const SampleHopArgs& a, int cap_dst, cudaStream_t stream);
int sample_scan_scratch_words(int cap_dst);

// PinSAGE hop: random walks with restart + top-k visited (walk.cu)
struct WalkHopArgs {
  const int64_t* indptr = nullptr;
  const int32_t* indices = nullptr;
  int64_t n_graph_nodes = 0;
  const int32_t* dst_nid = nullptr;
  const int32_t* n_dst_ptr = nullptr;
  int32_t n_dst = 0;
  int32_t length = 0;              // steps per walk
  uint32_t restart_thr = 0;        // stop when the draw is below this (restart_prob * 2^32)
  int32_t num_walks = 0;
  int32_t num_neighbors = 0;
  const int64_t* counters = nullptr;
  int32_t hop = 0;
  int32_t* out_indptr = nullptr;
  int32_t* out_nbr = nullptr;
  float* out_w = nullptr;
  int32_t cap_edges = 0;
  int32_t* n_edges_out = nullptr;
  unsigned long long* scan_scratch = nullptr;
  int32_t* err = nullptr;
};
void launch_walk_hop(const WalkHopArgs& a, int cap_dst, cudaStream_t stream);
int walk_scan_scratch_words(int cap_dst);

// ---------------------------------------------------------------- compaction (S2)
struct CompactArgs {
  const int32_t* dst_nid = nullptr;
  const int32_t* n_dst_ptr = nullptr;
  const int32_t* nbr = nullptr;
  const int32_t* n_edges_ptr = nullptr;
  unsigned long long* map = nullptr;  // dense [n_graph_nodes]
  int64_t n_graph_nodes = 0;
  int32_t* src_nid = nullptr;         // [cap_src]
  uint8_t* src_sampled = nullptr;     // [cap_src]
  int32_t* indices = nullptr;         // [cap_edges]
  int32_t* n_src_out = nullptr;
  int32_t cap_src = 0;
  unsigned long long* scan_scratch = nullptr;
  int32_t* err = nullptr;
  // optional transpose of the block (launch_block_transpose): K3 counts the edges of
  // every local src (t_cnt, zero before; the transpose clears it again) and stores
  // each edge's rank among its source's edges (t_rank)
  int32_t* t_cnt = nullptr;
  int32_t* t_rank = nullptr;
};
// gen: device generation counter; tags are derived on the device from (*gen, slot)
// so that a captured graph keeps drawing fresh tags (slot < 16 per generation).
// run_k3 = false: the edge rewrite is left to launch_compact_edges after the last hop
void launch_compact(const CompactArgs& a, int cap_dst, int cap_edges, const int64_t* gen, int slot, int num_sms,
                    cudaStream_t stream, bool k1_done = false, bool run_k3 = true);
// the edge rewrite (K3: indices[e] = local index of nbr[e]) of several hops in one launch
struct CompactEdgesArgs {
  static constexpr int kMaxHops = 8;
  struct Hop {
    const int32_t* nbr = nullptr;
    const int32_t* n_edges_ptr = nullptr;
    int32_t* indices = nullptr;
    int32_t cap_src = 0;
  };
  Hop hops[kMaxHops];
  int32_t n_hops = 0;
  const unsigned long long* map = nullptr;
  int64_t n_graph_nodes = 0;
};
void launch_compact_edges(const CompactEdgesArgs& a, int64_t cap_edges_total, int num_sms, cudaStream_t stream);
int compact_scan_scratch_words(int cap_edges);

// The block's edges grouped by source (CSR by local src): tptr[n_src + 1] from an
// exclusive scan of t_cnt (cleared as it is read), tdst[k] = the destination of the
// k-th edge of its source (edge order within a source: t_rank).  A one-CTA scan (the
// blocks that need it are the inner hops: tens of thousands of nodes at most) and a
// fill with one warp per destination.
void launch_block_transpose(const int32_t* indptr, const int32_t* indices, const int32_t* n_dst_ptr,
                            const int32_t* n_src_ptr, int32_t* t_cnt, const int32_t* t_rank, int32_t* tptr,
                            int32_t* tdst, int cap_src, int cap_edges, int32_t* err, cudaStream_t stream);

// ---------------------------------------------------------------- GEMM
enum GemmMode : int { kStoreBf16 = 0, kStoreF32 = 1, kAtomicF32 = 2, kCrossEntropy = 3 };

struct GemmProblem {
  // physical row-major shapes; K-major A is [M][K], MN-major A is [K][M]
  const void* A = nullptr;
  int64_t a_rows = 0, a_cols = 0, lda = 0;
  bool a_mn = false;
  const void* B = nullptr;
  int64_t b_rows = 0, b_cols = 0, ldb = 0;
  bool b_mn = false;
};

struct GemmArgs {
  int32_t M_cap = 0;
  const int32_t* M_dev = nullptr;
  int32_t N = 0;
  int32_t K_cap = 0;
  const int32_t* K_dev = nullptr;
  int32_t splits = 1;
  void* C = nullptr;
  int64_t ldc = 0;
  int32_t c_mode = kStoreBf16;
  const float* bias = nullptr;
  int32_t act = 0;  // 1: ReLU
  float dropout_p = 0.f;
  const int64_t* counters = nullptr;
  uint32_t dropout_salt = 0;
  // cross-entropy epilogue
  const int32_t* labels = nullptr;
  int32_t n_classes = 0;
  __nv_bfloat16* dlogits = nullptr;
  int64_t ld_dl = 0;
  float* loss_sum = nullptr;
  int32_t* correct = nullptr;
  int32_t* pred_out = nullptr;
  const int32_t* n_rows_dev = nullptr;
  float* dbias = nullptr;              // cross-entropy epilogue: += column sums of the gradient
  int32_t* err = nullptr;
  int64_t c_rows = 0;                  // rows of C (bf16 stores go through a TMA store of that extent)
  // activation backward fused into a bf16 store (no bias, ReLU or dropout then):
  // out = mask[m, n] != 0 ? acc * mask_scale : 0, with mask the layer's forward output
  // (ReLU + dropout leave exact zeros where the gradient is cut)
  const __nv_bfloat16* act_mask = nullptr;
  int64_t ld_mask = 0;
  float mask_scale = 1.f;
  // > 0: rows [M, roundup(M, zero_tail_rows)) of C (below c_rows) are written as zeros,
  // so that a later split-K GEMM over whole 64-row blocks reads zeros past the live rows
  int32_t zero_tail_rows = 0;
  // GAT attention logits of a bf16 z = x W^T store (no bias, activation or dropout):
  // el[m, h] += sum_f bf16(z[m, hF+f]) att_l[hF+f], and er the same with att_r for
  // rows m < *att_n_dst; el / er are zeroed by the caller
  const float* att_l = nullptr;
  const float* att_r = nullptr;
  float* att_el = nullptr;
  float* att_er = nullptr;
  int32_t att_heads = 0, att_feat = 0;
  const int32_t* att_n_dst = nullptr;
};
void launch_gemm(const GemmProblem& p, GemmArgs a, int bn, cudaStream_t stream);

// ---------------------------------------------------------------- fused SAGE head (head.cu)
struct SageHeadArgs {
  const int32_t* indptr = nullptr;      // last block, CSR by destination
  const int32_t* indices = nullptr;
  const int32_t* n_dst_ptr = nullptr;
  int32_t cap_dst = 0;
  const __nv_bfloat16* h = nullptr;     // source rows (the previous layer's output), ip columns used
  int64_t ldh = 0;
  int32_t ip = 0;                       // multiple of 8, <= 256
  const __nv_bfloat16* w = nullptr;     // [n_classes][2 ip]: self half, then neighbour half
  int64_t ldw = 0;
  const float* bias = nullptr;
  int32_t n_classes = 0;                // <= 64
  const int32_t* labels = nullptr;      // per destination row
  __nv_bfloat16* x = nullptr;           // [cap, 2 ip] out: [h_v | mean h_u]
  int64_t ldx = 0;
  __nv_bfloat16* dl = nullptr;          // [cap, ld_dl] out: dlogits, rows to the next multiple of 64 zeroed
  int64_t ld_dl = 0;
  __nv_bfloat16* dx = nullptr;          // [cap, 2 ip] out: dlogits W (null: forward only)
  int64_t lddx = 0;
  // tile version: the mean aggregation's backward of dx, fused: dsrc[v] += dx[v, :ip],
  // dsrc[u] += dx[v, ip:] / deg(v) for the in-neighbours u (fp32 reductions; the rows
  // of the previous layer's output, zero before)
  float* dsrc = nullptr;
  int64_t ld_dsrc = 0;
  float* loss_sum = nullptr;
  int32_t* correct = nullptr;
  float* dbias = nullptr;
  int32_t* pred_out = nullptr;
};
bool sage_head_supported(int ip, int n_classes);

// hidden GraphSAGE layer as 16-row MMA tiles (head.cu): forward = aggregation + X W^T +
// bias / ReLU / dropout; backward = dY W reduced into the previous layer's fp32
// gradient rows through the aggregation's transpose
struct SageLayerArgs {
  const int32_t* indptr = nullptr;
  const int32_t* indices = nullptr;
  const int32_t* n_dst_ptr = nullptr;
  int32_t cap_dst = 0;
  int32_t ip = 0, op = 0;               // input width (of each half of X), output width
  const __nv_bfloat16* w = nullptr;     // [op][2 ip]
  int64_t ldw = 0;
  // forward
  const __nv_bfloat16* h = nullptr;     // source rows, ip columns used
  int64_t ldh = 0;
  const float* bias = nullptr;
  int32_t act = 1;
  float dropout_p = 0.f;
  const int64_t* counters = nullptr;
  uint32_t dropout_salt = 0;
  __nv_bfloat16* x = nullptr;           // [cap, 2 ip] aggregated rows (for dW)
  int64_t ldx = 0;
  __nv_bfloat16* out = nullptr;         // [cap, op]
  int64_t ldo = 0;
  // backward
  const __nv_bfloat16* dy = nullptr;    // [cap, op]
  int64_t lddy = 0;
  float* dsrc = nullptr;                // previous layer's fp32 gradient rows
  int64_t ld_dsrc = 0;
};
bool sage_layer_tile_supported(int ip, int op);
void launch_sage_layer_fwd(const SageLayerArgs& a, cudaStream_t stream);
void launch_sage_layer_bwd(const SageLayerArgs& a, cudaStream_t stream);
void launch_sage_head(const SageHeadArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- aggregation (K-SpMM)
enum AggMode : int { kAggMean = 0, kAggSum = 1, kAggGcn = 2, kAggWeighted = 3 };

struct AggArgs {
  const int32_t* indptr = nullptr;   // block CSR by dst [n_dst + 1]
  const int32_t* indices = nullptr;  // local src index per edge
  const int32_t* n_dst_ptr = nullptr;
  int32_t n_dst = 0;
  const __nv_bfloat16* src = nullptr;  // source rows
  int64_t src_stride = 0;
  const int32_t* src_map = nullptr;  // local src -> row of src (null: identity)
  int32_t dim = 0;                   // feature width (multiple of 8)
  int32_t mode = kAggMean;
  const float* edge_w = nullptr;     // kAggWeighted
  const float* src_norm = nullptr;   // kAggGcn: per local src
  const float* dst_norm = nullptr;   // kAggGcn: per dst (null: computed from the block in-degree)
  __nv_bfloat16* out = nullptr;
  int64_t out_stride = 0;
  int32_t agg_col = 0;               // column of the aggregate in out
  int32_t self_col = -1;             // >= 0: also copy the dst row here
  float self_scale = 0.f;            // != 0: out_agg += self_scale * self (GIN)
  int32_t zero_tail_rows = 0;        // write zeros in rows [n_dst, roundup(n_dst, this)) below cap_rows
  int32_t cap_rows = 0;              // rows of the output buffer (set by the launcher)
  // optional epilogue on the aggregate (GraphConv with the projection applied first):
  // out = dropout(act(agg + bias)); the dropout mask of element (r, c) is the Philox
  // draw of index r * out_stride + c (c counted from agg_col), as in the GEMM epilogue
  const float* bias = nullptr;
  int32_t act = 0;                   // 1: ReLU
  float dropout_p = 0.f;
  const int64_t* counters = nullptr;
  uint32_t dropout_salt = 0;
  int32_t* err = nullptr;
};
void launch_aggregate(const AggArgs& a, int cap_dst, cudaStream_t stream);

struct AggBwdArgs {
  const int32_t* indptr = nullptr;
  const int32_t* indices = nullptr;
  const int32_t* n_dst_ptr = nullptr;
  int32_t n_dst = 0;
  const __nv_bfloat16* dout = nullptr;  // gradient of the aggregation output
  int64_t dout_stride = 0;
  int32_t agg_col = 0;
  int32_t self_col = -1;                // >= 0: add this gradient block to the dst rows
  float self_scale = 0.f;               // GIN: the aggregate's gradient also flows to self
  int32_t dim = 0;
  int32_t mode = kAggMean;
  const float* edge_w = nullptr;
  const float* src_norm = nullptr;
  const float* dst_norm = nullptr;
  float* dsrc = nullptr;                // fp32 accumulation [n_src][dim], must start at 0
  int64_t dsrc_stride = 0;
  int32_t* err = nullptr;
};
void launch_aggregate_bwd(const AggBwdArgs& a, int cap_dst, cudaStream_t stream);

// Mean-aggregation backward gathered by source, with the previous layer's ReLU/dropout
// backward fused: for every local src u of the block
//   g_u = [u < n_dst] dout[u, self_col:] + sum_{v: u in N(v)} dout[v, agg_col:] / deg_v
//   dy_u = mask[u] != 0 ? g_u * scale : 0       (bf16), dbias += sum_u dy_u
// over the transposed block (tptr/tdst); rows [n_src, roundup(n_src, 64)) of dy are
// zeroed.  Replaces aggregate_bwd (fp32 scatter) + act_bwd for GraphSAGE.
struct AggBwdGatherArgs {
  const int32_t* indptr = nullptr;      // block CSR by dst (degrees)
  const int32_t* tptr = nullptr;        // transposed block [n_src + 1]
  const int32_t* tdst = nullptr;
  const int32_t* n_dst_ptr = nullptr;
  const int32_t* n_src_ptr = nullptr;
  const __nv_bfloat16* dout = nullptr;  // [n_dst, >= max(self_col, agg_col) + dim]
  int64_t dout_stride = 0;
  int32_t self_col = 0, agg_col = 0;
  int32_t dim = 0;
  const __nv_bfloat16* mask = nullptr;  // the previous layer's forward output [cap_rows, mask_stride]
  int64_t mask_stride = 0;
  float scale = 1.f;
  __nv_bfloat16* dy = nullptr;          // [cap_rows, dy_stride]
  int64_t dy_stride = 0;
  float* dbias = nullptr;
  int32_t cap_rows = 0;
  int32_t* err = nullptr;
};
void launch_aggregate_bwd_gather(const AggBwdGatherArgs& a, cudaStream_t stream);

// GCN normalisation: out-degree of every local src of a block (clamped >= 1) ^ -1/2
void launch_src_norm(const int32_t* indices, const int32_t* n_edges_ptr, int cap_edges, const int32_t* n_src_ptr,
                     int cap_src, float* deg_scratch, float* src_norm, cudaStream_t stream);

// ---------------------------------------------------------------- elementwise / misc
// dY = (h != 0) ? dh * scale : 0  (ReLU + dropout backward from the stored output),
// fp32 dh read and cleared (so the accumulation buffer starts at 0 next time);
// rows [n, roundup(n, 64)) of dY are zeroed for the split-K GEMM; the column sums of
// dY are added to dbias.
struct ActBwdArgs {
  float* dh = nullptr;
  int64_t dh_stride = 0;
  const __nv_bfloat16* h = nullptr;  // forward output (null: identity activation)
  int64_t h_stride = 0;
  __nv_bfloat16* dy = nullptr;
  int64_t dy_stride = 0;
  const int32_t* n_ptr = nullptr;
  int32_t n = 0;
  int32_t dim = 0;
  float scale = 1.f;
  float* dbias = nullptr;
  int32_t cap_rows = 0;
};
void launch_act_bwd(const ActBwdArgs& a, cudaStream_t stream);

void launch_gather_rows_bf16(const void* table, bool table_f32, int64_t table_stride, int32_t dim,
                             const int32_t* ids, const int32_t* n_ptr, int32_t n, int cap,
                             __nv_bfloat16* out, int64_t out_stride, cudaStream_t stream);
void launch_gather_i32(const int32_t* table, const int32_t* ids, const int32_t* n_ptr, int n, int cap,
                       int32_t* out, cudaStream_t stream);
void launch_gather_i64(const int64_t* table, const int32_t* ids, const int32_t* n_ptr, int n, int cap,
                       int64_t* out, cudaStream_t stream);

void launch_rmat_candidates(int64_t n, int scale, double a, double b, double c, uint64_t seed, int64_t e_begin,
                            int64_t count, int64_t* keys, cudaStream_t stream);
void launch_shuffle_keys(const int64_t* ids, int64_t n, uint64_t seed, uint64_t epoch, int64_t* keys,
                         cudaStream_t stream);
void launch_normal_fill(float* out, int64_t n, uint64_t seed, cudaStream_t stream);
void launch_normal_rows_bf16(__nv_bfloat16* out, int64_t ld, int64_t row0, int64_t rows, int d, uint64_t seed,
                             cudaStream_t stream);
void launch_dropout_mask(uint8_t* mask, int64_t rows, int64_t cols, int64_t ld, float p, const int64_t* counters,
                         uint32_t salt, cudaStream_t stream);

// ---------------------------------------------------------------- optimizer
struct AdamArgs {
  float* param = nullptr;     // fp32 master weights
  float* m = nullptr;
  float* v = nullptr;
  float* grad = nullptr;
  bool clear_grad = true;     // zero the gradient after reading it
  __nv_bfloat16* param_bf16 = nullptr;  // working copy (may be null)
  int64_t n = 0;
  float lr = 1e-3f, beta1 = 0.9f, beta2 = 0.999f, eps = 1e-8f, weight_decay = 0.f;
  const int64_t* step = nullptr;  // device count of completed optimizer steps
  float grad_scale = 1.f;
  const float* grad_scale_dev = nullptr;  // multiplies grad_scale when given
};
void launch_adam(const AdamArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- loss / normalisation (nn.cu)
// Softmax cross-entropy over bf16 logits rows (one warp per row): loss, gradient
// (softmax - onehot) / n_sel, correct count and the bias gradient (column sums).
// Rows with row_mask == 0 (or >= *n_rows_ptr) get a zero gradient; rows up to
// roundup(n, zero_tail_rows) are written so split-K reductions see zeros.
struct CeArgs {
  const __nv_bfloat16* logits = nullptr;
  int64_t ld = 0;
  int32_t n_classes = 0;
  const int32_t* labels = nullptr;
  const int32_t* n_rows_ptr = nullptr;
  int32_t cap_rows = 0;
  const uint8_t* row_mask = nullptr;
  const int32_t* n_sel_ptr = nullptr;  // denominator of the mean (null: the row count)
  __nv_bfloat16* dlogits = nullptr;
  int64_t ld_dl = 0;
  float* dbias = nullptr;
  float* loss_sum = nullptr;
  int32_t* correct = nullptr;
  int32_t zero_tail_rows = 64;
};
void launch_cross_entropy(const CeArgs& a, cudaStream_t stream);

// BatchNorm1d over the live rows (training: batch statistics, biased variance for
// the normalisation, unbiased for the running estimate; eval: running estimates),
// optionally followed by ReLU.  sums[2 * dim] must be zero before the forward and is
// kept for the backward.
struct BnArgs {
  const __nv_bfloat16* x = nullptr;
  int64_t ldx = 0;
  int32_t dim = 0;
  const int32_t* n_ptr = nullptr;
  int32_t cap = 0;
  float* sums = nullptr;
  const float* gamma = nullptr;
  const float* beta = nullptr;
  float* running_mean = nullptr;     // [stat_dim] (columns past it are padding)
  float* running_var = nullptr;
  int32_t stat_dim = 0;
  int64_t* num_batches = nullptr;
  float momentum = 0.1f, eps = 1e-5f;
  bool training = true;
  int32_t act = 1;
  __nv_bfloat16* y = nullptr;
  int64_t ldy = 0;
  int32_t zero_tail_rows = 64;
};
void launch_batchnorm_fwd(const BnArgs& a, cudaStream_t stream);
// Backward of (ReLU o BatchNorm): dy is fp32 (cleared after reading when clear_dy),
// dx written as bf16; dgamma / dbeta accumulated (+=).  bsums[2 * dim] zero before.
struct BnBwdArgs {
  const __nv_bfloat16* x = nullptr;
  int64_t ldx = 0;
  const __nv_bfloat16* y = nullptr;   // forward output (ReLU mask); null: no activation
  int64_t ldy = 0;
  float* dy = nullptr;
  const __nv_bfloat16* dy_bf16 = nullptr;  // alternative bf16 gradient (e.g. from the loss)
  int64_t lddy = 0;
  bool clear_dy = true;
  int32_t dim = 0;
  const int32_t* n_ptr = nullptr;
  int32_t cap = 0;
  const float* sums = nullptr;
  float* bsums = nullptr;
  const float* gamma = nullptr;
  float* dgamma = nullptr;
  float* dbeta = nullptr;
  float eps = 1e-5f;
  __nv_bfloat16* dx = nullptr;
  int64_t lddx = 0;
  int32_t zero_tail_rows = 64;
};
void launch_batchnorm_bwd(const BnBwdArgs& a, cudaStream_t stream);

// Row L2 normalisation (PinSAGE): y = z / |z| (|z| == 0 -> 1); norms kept for the
// backward, dz = (dy - y (y . dy)) / |z| with dy fp32 (cleared after reading) or bf16,
// dz fp32.
void launch_l2norm_fwd(const __nv_bfloat16* z, int64_t ldz, int32_t dim, const int32_t* n_ptr, int cap,
                       __nv_bfloat16* y, int64_t ldy, float* norms, cudaStream_t stream);
void launch_l2norm_bwd(const __nv_bfloat16* y, int64_t ldy, float* dy, const __nv_bfloat16* dy_bf16, int64_t lddy,
                       const float* norms, int32_t dim, const int32_t* n_ptr, int cap, float* dz, int64_t lddz,
                       cudaStream_t stream);
// dst[r, :dim] += src[r, :dim] for r < *n_ptr (fp32 += bf16)
void launch_add_bf16_rows(float* dst, int64_t ldd, const __nv_bfloat16* src, int64_t lds, int32_t dim,
                          const int32_t* n_ptr, int cap, cudaStream_t stream);

// Dropout on a bf16 matrix: out = in * keep / (1 - p) with the Philox mask of index
// r * ld_mask + c (the GEMM epilogue's rule); grad variant scales an fp32 gradient
// in place with the same mask.  Rows >= *n_ptr are written as zeros (out) / skipped.
void launch_dropout_rows(const __nv_bfloat16* in, int64_t ldi, __nv_bfloat16* out, int64_t ldo, int32_t dim,
                         int64_t ld_mask, const int32_t* n_ptr, int cap, float p, const int64_t* counters,
                         uint32_t salt, cudaStream_t stream);
void launch_dropout_grad(float* g, int64_t ldg, int32_t dim, int64_t ld_mask, const int32_t* n_ptr, int cap, float p,
                         const int64_t* counters, uint32_t salt, cudaStream_t stream);
// fp32 -> bf16 rows (clears the fp32 source when clear), rows past *n_ptr zeroed
// up to roundup(n, zero_tail_rows)
void launch_f32_to_bf16_rows(float* src, int64_t lds, __nv_bfloat16* dst, int64_t ldd, int32_t dim,
                             const int32_t* n_ptr, int cap, bool clear, int32_t zero_tail_rows, cudaStream_t stream);

// ---------------------------------------------------------------- GAT (gat.cu)
// Attention logits of every source row: el[u, h] = z_u[h] . a_l[h] and, for the
// first n_dst rows, er[v, h] = z_v[h] . a_r[h] (z: bf16 [n_src, H*F]).
struct GatArgs {
  const int32_t* indptr = nullptr;
  const int32_t* indices = nullptr;
  const int32_t* n_dst_ptr = nullptr;
  const int32_t* n_src_ptr = nullptr;
  int32_t cap_dst = 0, cap_src = 0;
  int32_t heads = 0, feat = 0;        // H, F (H * F <= 1024, F % 8 == 0)
  const __nv_bfloat16* z = nullptr;
  int64_t ldz = 0;
  const float* attn_l = nullptr;      // [H * F]
  const float* attn_r = nullptr;
  const float* bias = nullptr;        // [H * F]
  float* el = nullptr;                // [cap_src, H]
  float* er = nullptr;                // [cap_dst, H]
  float* smax = nullptr;              // [cap_dst, H] softmax max, kept for the backward
  float* ssum = nullptr;              // [cap_dst, H] softmax denominator
  float slope = 0.2f;
  // forward output: hidden layers write act(out) flattened [n_dst, H*F] with dropout;
  // the last layer writes the mean over heads [n_dst, F]
  bool mean_heads = false;
  int32_t act = 1;
  float dropout_p = 0.f;
  const int64_t* counters = nullptr;
  uint32_t dropout_salt = 0;
  __nv_bfloat16* out = nullptr;
  int64_t ldo = 0;
  // backward
  const __nv_bfloat16* dout = nullptr;  // [n_dst, H*F] (or [n_dst, F] with mean_heads)
  int64_t lddo = 0;
  float* edge_scratch = nullptr;        // [cap_edges, H]
  float* del = nullptr;                 // [cap_src, H] (zero before)
  float* der = nullptr;                 // [cap_dst, H]
  float* dz = nullptr;                  // fp32 [cap_src, H*F] (zero before)
  int64_t lddz = 0;
  float* dbias = nullptr;
  float* dattn_l = nullptr;
  float* dattn_r = nullptr;
  __nv_bfloat16* dz_bf16 = nullptr;     // GEMM operand of the backward projections
  int64_t lddzb = 0;
  int32_t zero_tail_rows = 64;
  int32_t* err = nullptr;
  // input-layer backward (launch_gat_bwd_input: no dz, see gat.cu)
  const __nv_bfloat16* x = nullptr;     // [cap_src, ldx] the layer's input rows
  int64_t ldx = 0;
  int32_t in_dim = 0;                   // width of x used by the projection (multiple of 8)
  __nv_bfloat16* y = nullptr;           // [cap_dst, ldy >= H * in_dim]
  int64_t ldy = 0;
  float* xl = nullptr;                  // [H * in_dim] (zero before)
  float* xr = nullptr;                  // [H * in_dim] (zero before)
  // > 0: z is a row of zmod columns shared by every head (column c of the H * F
  // "virtual" row reads z[c % zmod], F = zmod): the GAT input layer then runs on its
  // input rows x, with the projection applied after the aggregation (gat.cu)
  int32_t zmod = 0;
};
void launch_gat_scores(const GatArgs& a, cudaStream_t stream);
void launch_gat_fwd(const GatArgs& a, cudaStream_t stream);
void launch_gat_bwd(const GatArgs& a, cudaStream_t stream);
void launch_gat_bwd_input(const GatArgs& a, cudaStream_t stream);
void launch_gat_dw_combine(const float* T, int64_t ldt, const float* xl, const float* xr, const float* attn_l,
                           const float* attn_r, int heads, int feat, int in_dim, float* dw, int64_t ldw,
                           cudaStream_t stream);
// Input layer with the projection after the aggregation:
//   wl[h, k] = sum_f W[hF+f, k] a_l[hF+f],  wr likewise (fp32 [H * in_dim] each), and the
//   block-diagonal weight Wbd[hF+f, h*in_dim + k] = W[hF+f, k] (bf16 [rows, H * in_dim]),
// so that el = x . wl, er = x . wr and out = y Wbd^T with y_v[h] = sum_u a_uvh x_u.
void launch_gat_in_prep(const __nv_bfloat16* w, int64_t ldw, const float* attn_l, const float* attn_r, int heads,
                        int feat, int in_dim, int rows, float* wl, float* wr, __nv_bfloat16* wbd, int64_t ldwbd,
                        cudaStream_t stream);
// Its weight and attention gradients from T = dout^T y, xl, xr (as launch_gat_dw_combine)
// plus dattn_l[r] += W[r, :] . xl[h(r), :], dattn_r[r] += W[r, :] . xr[h(r), :].
void launch_gat_in_dw(const float* T, int64_t ldt, const float* xl, const float* xr, const float* attn_l,
                      const float* attn_r, const float* w, int64_t ldw_in, int heads, int feat, int in_dim, float* dw,
                      int64_t ldw, float* dattn_l, float* dattn_r, cudaStream_t stream);
// dbias[c] += sum over the live rows of x[r, c] (bf16 rows)
void launch_col_sum_bf16(const __nv_bfloat16* x, int64_t ldx, const int32_t* n_ptr, int cap_rows, int cols,
                         float* out, cudaStream_t stream);

// counters = [seed, epoch, step_in_epoch, global_step, gen, adam_t]: advance the step.
// With ring_slot (a device int64 holding the address of a float ring, 0 for none) the
// step's loss fstats[2] is stored at ring[step_in_epoch] first (the ring may be pinned
// host memory: a device -> host write); fstats[0..nf) and istats[0..ni) are then
// cleared for the next step (nf = ni = 0 keeps them).
void launch_step_end(int64_t* counters, const int64_t* ring_slot, float* fstats, int nf, int32_t* istats, int ni,
                     cudaStream_t stream);

// Step prologue of a sampler: its counters for the step step_offset ahead of the
// main ones (as launch_sampler_counters), its coverage sums cleared, and the step's
// seeds.  With table_slot (a device int64 holding the address of an int32 [n_rows, B]
// seed table, which may be pinned host memory read over PCIe; 0 = seeds already in
// place) row main[step] + step_offset is copied into seeds and its count
// count_table[row] (0 past the last row) into *n_seeds.  Then the labels (int32) and
// global in-degrees (int64, optional) of the seeds are gathered.
struct SamplePrologueArgs {
  const int64_t* main = nullptr;
  int64_t* dst = nullptr;
  int64_t step_offset = 0;
  float* cov = nullptr;
  const int64_t* table_slot = nullptr;
  const int32_t* count_table = nullptr;
  int32_t n_rows = 0;
  int32_t B = 0;
  int32_t* seeds = nullptr;
  int32_t* n_seeds = nullptr;
  const int32_t* labels = nullptr;
  int32_t* seed_labels = nullptr;
  const int64_t* gideg = nullptr;
  int64_t* seed_gideg = nullptr;
};
void launch_sample_prologue(const SamplePrologueArgs& a, cudaStream_t stream);
// The counters a sampler draws with for the step step_offset ahead of the main
// counters (seed, epoch, step + offset), with its own compaction generation (+1).
void launch_sampler_counters(const int64_t* main, int64_t* dst, int64_t step_offset, cudaStream_t stream);

}  // namespace dev
}  // namespace grappa
