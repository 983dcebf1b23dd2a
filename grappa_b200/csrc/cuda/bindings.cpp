// torch bindings of the sm_100a kernels (module grappa_b200._cuda).  Every entry
// point checks device, dtype and contiguity and launches on the current stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <optional>

#include "cuda_check.h"
#include "allreduce.h"
#include "kernels.h"
#include "peer.h"

namespace d = grappa::dev;
using at::Tensor;
using OptT = std::optional<Tensor>;

namespace {

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

template <typename T>
T* ptr(const Tensor& t, at::ScalarType st, const char* name) {
  check_cuda(t, name);
  TORCH_CHECK(t.scalar_type() == st, name, " has dtype ", t.scalar_type(), ", expected ", st);
  return reinterpret_cast<T*>(t.data_ptr());
}

template <typename T>
T* optr(const OptT& t, at::ScalarType st, const char* name) {
  if (!t.has_value() || !t->defined()) return nullptr;
  return ptr<T>(*t, st, name);
}

// 2-D operand whose rows may be strided (row stride = stride(0)) but whose
// columns are contiguous
template <typename T>
T* ptr2d(const Tensor& t, at::ScalarType st, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, " must be 2-D with contiguous rows");
  TORCH_CHECK(t.scalar_type() == st, name, " has dtype ", t.scalar_type(), ", expected ", st);
  return reinterpret_cast<T*>(t.data_ptr());
}

int num_sms() {
  static int n = 0;
  if (!n) n = at::cuda::getCurrentDeviceProperties()->multiProcessorCount;
  return n;
}

// --------------------------------------------------------------------------- S1 / S2
void sample_hop(Tensor indptr, Tensor indices, Tensor dst_nid, OptT n_dst_dev, int64_t n_dst, OptT frontier,
                int64_t fanout, bool replace, Tensor counters, int64_t hop, OptT gideg, OptT cov_accum,
                Tensor out_indptr, Tensor out_nbr, Tensor n_edges_out, Tensor scan_scratch, Tensor err,
                int64_t cap_dst, OptT map, OptT src_nid, OptT src_sampled) {
  c10::cuda::CUDAGuard g(indptr.device());
  d::SampleHopArgs a;
  a.indptr = ptr<int64_t>(indptr, at::kLong, "indptr");
  a.indices = ptr<int32_t>(indices, at::kInt, "indices");
  a.n_graph_nodes = indptr.numel() - 1;
  a.dst_nid = ptr<int32_t>(dst_nid, at::kInt, "dst_nid");
  a.n_dst_ptr = optr<int32_t>(n_dst_dev, at::kInt, "n_dst_dev");
  a.n_dst = static_cast<int32_t>(n_dst);
  a.frontier = optr<uint8_t>(frontier, at::kByte, "frontier");
  a.fanout = static_cast<int32_t>(fanout);
  a.replace = replace;
  a.counters = ptr<int64_t>(counters, at::kLong, "counters");
  a.hop = static_cast<int32_t>(hop);
  a.gideg = optr<int64_t>(gideg, at::kLong, "gideg");
  a.cov_accum = optr<float>(cov_accum, at::kFloat, "cov_accum");
  a.out_indptr = ptr<int32_t>(out_indptr, at::kInt, "out_indptr");
  a.out_nbr = ptr<int32_t>(out_nbr, at::kInt, "out_nbr");
  a.cap_edges = static_cast<int32_t>(out_nbr.numel());
  a.n_edges_out = ptr<int32_t>(n_edges_out, at::kInt, "n_edges_out");
  a.scan_scratch = reinterpret_cast<unsigned long long*>(ptr<int64_t>(scan_scratch, at::kLong, "scan_scratch"));
  a.err = ptr<int32_t>(err, at::kInt, "err");
  TORCH_CHECK(out_indptr.numel() >= cap_dst + 1, "out_indptr too small");
  TORCH_CHECK(dst_nid.numel() >= cap_dst, "dst_nid smaller than cap_dst");
  TORCH_CHECK(!a.frontier || frontier->numel() >= cap_dst, "frontier smaller than cap_dst");
  TORCH_CHECK(!a.gideg || gideg->numel() >= cap_dst, "gideg smaller than cap_dst");
  // exactly sized: the scan numbers its launches by the grid size (common.cuh LookBack)
  TORCH_CHECK(scan_scratch.numel() == d::sample_scan_scratch_words(static_cast<int>(cap_dst)),
              "scan_scratch must hold exactly sample_scratch_words(capacity) words and be used with that capacity only");
  if (map.has_value()) {
    TORCH_CHECK(src_nid.has_value() && src_sampled.has_value(), "fused compaction needs map, src_nid and src_sampled");
    TORCH_CHECK(counters.numel() >= 6 && hop >= 0 && hop < 16, "fused compaction: counters[4] and hop slot");
    a.map = reinterpret_cast<unsigned long long*>(ptr<int64_t>(*map, at::kLong, "map"));
    a.map_nodes = map->numel();
    a.src_nid = ptr<int32_t>(*src_nid, at::kInt, "src_nid");
    a.src_sampled = ptr<uint8_t>(*src_sampled, at::kByte, "src_sampled");
    TORCH_CHECK(src_nid->numel() >= cap_dst && src_sampled->numel() >= cap_dst, "src buffers smaller than cap_dst");
  }
  d::launch_sample_hop(a, static_cast<int>(cap_dst), stream());
}

int64_t sample_scratch_words(int64_t cap_dst) { return d::sample_scan_scratch_words(static_cast<int>(cap_dst)); }
int64_t compact_scratch_words(int64_t cap_e) { return d::compact_scan_scratch_words(static_cast<int>(cap_e)); }

void compact(Tensor dst_nid, Tensor n_dst_dev, Tensor nbr, Tensor n_edges_dev, Tensor map, Tensor src_nid,
             Tensor src_sampled, Tensor indices, Tensor n_src_out, Tensor scan_scratch, Tensor err, int64_t cap_dst,
             int64_t cap_edges, Tensor counters, int64_t slot, bool k1_done, OptT t_cnt, OptT t_rank, bool run_k3) {
  c10::cuda::CUDAGuard g(dst_nid.device());
  TORCH_CHECK(slot >= 0 && slot < 16, "slot must be in [0, 16)");
  TORCH_CHECK(counters.numel() >= 6, "counters needs 6 entries");
  d::CompactArgs a;
  a.dst_nid = ptr<int32_t>(dst_nid, at::kInt, "dst_nid");
  a.n_dst_ptr = ptr<int32_t>(n_dst_dev, at::kInt, "n_dst_dev");
  a.nbr = ptr<int32_t>(nbr, at::kInt, "nbr");
  a.n_edges_ptr = ptr<int32_t>(n_edges_dev, at::kInt, "n_edges_dev");
  a.map = reinterpret_cast<unsigned long long*>(ptr<int64_t>(map, at::kLong, "map"));
  a.n_graph_nodes = map.numel();
  a.src_nid = ptr<int32_t>(src_nid, at::kInt, "src_nid");
  a.src_sampled = ptr<uint8_t>(src_sampled, at::kByte, "src_sampled");
  a.indices = ptr<int32_t>(indices, at::kInt, "indices");
  a.n_src_out = ptr<int32_t>(n_src_out, at::kInt, "n_src_out");
  a.cap_src = static_cast<int32_t>(std::min(src_nid.numel(), src_sampled.numel()));
  a.scan_scratch = reinterpret_cast<unsigned long long*>(ptr<int64_t>(scan_scratch, at::kLong, "scan_scratch"));
  a.err = ptr<int32_t>(err, at::kInt, "err");
  a.t_cnt = optr<int32_t>(t_cnt, at::kInt, "t_cnt");
  a.t_rank = optr<int32_t>(t_rank, at::kInt, "t_rank");
  TORCH_CHECK(!a.t_cnt || (a.t_rank && t_cnt->numel() >= a.cap_src && t_rank->numel() >= cap_edges),
              "the transpose counters need t_cnt[cap_src] and t_rank[cap_edges]");
  TORCH_CHECK(nbr.numel() >= cap_edges && indices.numel() >= cap_edges, "edge buffers smaller than cap_edges");
  TORCH_CHECK(dst_nid.numel() >= cap_dst && a.cap_src >= cap_dst, "dst/src buffers smaller than cap_dst");
  // exactly sized: the scan numbers its launches by the grid size (common.cuh LookBack)
  TORCH_CHECK(scan_scratch.numel() == d::compact_scan_scratch_words(static_cast<int>(cap_edges)),
              "scan_scratch must hold exactly compact_scratch_words(capacity) words and be used with that capacity only");
  const int64_t* gen = ptr<int64_t>(counters, at::kLong, "counters") + 4;
  TORCH_CHECK(run_k3 || !a.t_cnt, "the transpose counters are made by K3: run it with the hop");
  d::launch_compact(a, static_cast<int>(cap_dst), static_cast<int>(cap_edges), gen, static_cast<int>(slot), num_sms(),
                    stream(), k1_done, run_k3);
}

// K3 of several hops after the last hop's K2 (see compact.cu)
void compact_edges(std::vector<Tensor> nbr, std::vector<Tensor> n_edges_dev, std::vector<Tensor> indices,
                   std::vector<int64_t> cap_src, Tensor map) {
  c10::cuda::CUDAGuard g(map.device());
  const size_t n = nbr.size();
  TORCH_CHECK(n >= 1 && n <= static_cast<size_t>(d::CompactEdgesArgs::kMaxHops) && n_edges_dev.size() == n &&
                  indices.size() == n && cap_src.size() == n,
              "compact_edges: one nbr, count, indices and capacity per hop (1..8 hops)");
  d::CompactEdgesArgs a;
  int64_t total = 0;
  for (size_t h = 0; h < n; ++h) {
    TORCH_CHECK(indices[h].numel() >= nbr[h].numel(), "compact_edges: indices shorter than nbr");
    a.hops[h].nbr = ptr<int32_t>(nbr[h], at::kInt, "nbr");
    a.hops[h].n_edges_ptr = ptr<int32_t>(n_edges_dev[h], at::kInt, "n_edges_dev");
    a.hops[h].indices = ptr<int32_t>(indices[h], at::kInt, "indices");
    a.hops[h].cap_src = static_cast<int32_t>(cap_src[h]);
    total = std::max<int64_t>(total, nbr[h].numel());
  }
  a.n_hops = static_cast<int32_t>(n);
  a.map = reinterpret_cast<const unsigned long long*>(ptr<int64_t>(map, at::kLong, "map"));
  a.n_graph_nodes = map.numel();
  d::launch_compact_edges(a, total, num_sms(), stream());
}

void block_transpose(Tensor indptr, Tensor indices, Tensor n_dst_dev, Tensor n_src_dev, Tensor t_cnt, Tensor t_rank,
                     Tensor tptr, Tensor tdst, Tensor err) {
  c10::cuda::CUDAGuard g(indptr.device());
  const int cap_src = static_cast<int>(std::min(t_cnt.numel(), tptr.numel() - 1));
  const int cap_e = static_cast<int>(std::min(t_rank.numel(), tdst.numel()));
  d::launch_block_transpose(ptr<int32_t>(indptr, at::kInt, "indptr"), ptr<int32_t>(indices, at::kInt, "indices"),
                            ptr<int32_t>(n_dst_dev, at::kInt, "n_dst"), ptr<int32_t>(n_src_dev, at::kInt, "n_src"),
                            ptr<int32_t>(t_cnt, at::kInt, "t_cnt"), ptr<int32_t>(t_rank, at::kInt, "t_rank"),
                            ptr<int32_t>(tptr, at::kInt, "tptr"), ptr<int32_t>(tdst, at::kInt, "tdst"), cap_src, cap_e,
                            ptr<int32_t>(err, at::kInt, "err"), stream());
}

void aggregate_bwd_gather(Tensor indptr, Tensor tptr, Tensor tdst, Tensor n_dst_dev, Tensor n_src_dev, Tensor dout,
                          int64_t self_col, int64_t agg_col, int64_t dim, Tensor mask, double scale, Tensor dy,
                          OptT dbias, Tensor err) {
  c10::cuda::CUDAGuard g(dout.device());
  d::AggBwdGatherArgs a;
  a.indptr = ptr<int32_t>(indptr, at::kInt, "indptr");
  a.tptr = ptr<int32_t>(tptr, at::kInt, "tptr");
  a.tdst = ptr<int32_t>(tdst, at::kInt, "tdst");
  a.n_dst_ptr = ptr<int32_t>(n_dst_dev, at::kInt, "n_dst");
  a.n_src_ptr = ptr<int32_t>(n_src_dev, at::kInt, "n_src");
  a.dout = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(dout, at::kBFloat16, "dout"));
  a.dout_stride = dout.stride(0);
  a.self_col = static_cast<int32_t>(self_col);
  a.agg_col = static_cast<int32_t>(agg_col);
  a.dim = static_cast<int32_t>(dim);
  a.mask = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(mask, at::kBFloat16, "mask"));
  a.mask_stride = mask.stride(0);
  a.scale = static_cast<float>(scale);
  a.dy = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(dy, at::kBFloat16, "dy"));
  a.dy_stride = dy.stride(0);
  a.dbias = optr<float>(dbias, at::kFloat, "dbias");
  a.cap_rows = static_cast<int32_t>(std::min(dy.size(0), mask.size(0)));
  TORCH_CHECK(tptr.numel() >= a.cap_rows + 1, "tptr needs cap_rows + 1 entries");
  TORCH_CHECK(dy.size(1) >= dim && mask.size(1) >= dim, "dy and mask need dim columns");
  a.err = ptr<int32_t>(err, at::kInt, "err");
  d::launch_aggregate_bwd_gather(a, stream());
}

// --------------------------------------------------------------------------- GEMM
void gemm(Tensor A, bool a_mn, Tensor B, bool b_mn, int64_t M_cap, OptT M_dev, int64_t N, int64_t K_cap, OptT K_dev,
          int64_t splits, Tensor C, int64_t mode, OptT bias, int64_t act, double dropout_p, OptT counters, int64_t salt,
          OptT labels, int64_t n_classes, OptT dlogits, OptT loss_sum, OptT correct, OptT pred_out, OptT n_rows_dev,
          OptT dbias, Tensor err, int64_t bn, OptT act_mask, double mask_scale, int64_t zero_tail_rows, OptT att_l,
          OptT att_r, OptT att_el, OptT att_er, int64_t att_heads, int64_t att_feat, OptT att_n_dst) {
  c10::cuda::CUDAGuard g(A.device());
  d::GemmProblem p;
  p.A = ptr2d<at::BFloat16>(A, at::kBFloat16, "A");
  p.a_rows = A.size(0);
  p.a_cols = A.size(1);
  p.lda = A.stride(0);
  p.a_mn = a_mn;
  p.B = ptr2d<at::BFloat16>(B, at::kBFloat16, "B");
  p.b_rows = B.size(0);
  p.b_cols = B.size(1);
  p.ldb = B.stride(0);
  p.b_mn = b_mn;
  d::GemmArgs a;
  a.M_cap = static_cast<int32_t>(M_cap);
  a.M_dev = optr<int32_t>(M_dev, at::kInt, "M_dev");
  a.N = static_cast<int32_t>(N);
  a.K_cap = static_cast<int32_t>(K_cap);
  a.K_dev = optr<int32_t>(K_dev, at::kInt, "K_dev");
  a.splits = static_cast<int32_t>(splits);
  a.c_mode = static_cast<int32_t>(mode);
  if (mode == d::kStoreBf16) {
    a.C = ptr2d<at::BFloat16>(C, at::kBFloat16, "C");
    a.ldc = C.stride(0);
    a.c_rows = C.size(0);
  } else if (mode != d::kCrossEntropy) {
    a.C = ptr2d<float>(C, at::kFloat, "C");
    a.ldc = C.stride(0);
  }
  a.bias = optr<float>(bias, at::kFloat, "bias");
  a.act = static_cast<int32_t>(act);
  a.dropout_p = static_cast<float>(dropout_p);
  a.counters = optr<int64_t>(counters, at::kLong, "counters");
  a.dropout_salt = static_cast<uint32_t>(salt);
  TORCH_CHECK(dropout_p == 0.0 || a.counters, "dropout needs the step counters");
  TORCH_CHECK(dropout_p == 0.0 || a.ldc % 4 == 0, "dropout needs ldc % 4 == 0");
  a.labels = optr<int32_t>(labels, at::kInt, "labels");
  a.n_classes = static_cast<int32_t>(n_classes);
  if (dlogits.has_value()) {
    a.dlogits = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(*dlogits, at::kBFloat16, "dlogits"));
    a.ld_dl = dlogits->stride(0);
  }
  a.loss_sum = optr<float>(loss_sum, at::kFloat, "loss_sum");
  a.correct = optr<int32_t>(correct, at::kInt, "correct");
  a.pred_out = optr<int32_t>(pred_out, at::kInt, "pred_out");
  a.n_rows_dev = optr<int32_t>(n_rows_dev, at::kInt, "n_rows_dev");
  a.dbias = optr<float>(dbias, at::kFloat, "dbias");
  a.err = ptr<int32_t>(err, at::kInt, "err");
  if (act_mask.has_value()) {
    a.act_mask = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(*act_mask, at::kBFloat16, "act_mask"));
    a.ld_mask = act_mask->stride(0);
    TORCH_CHECK(act_mask->size(0) >= a.M_cap, "act_mask needs M_cap rows");
  }
  a.mask_scale = static_cast<float>(mask_scale);
  a.zero_tail_rows = static_cast<int32_t>(zero_tail_rows);
  if (att_el.has_value()) {
    a.att_l = optr<float>(att_l, at::kFloat, "att_l");
    a.att_r = optr<float>(att_r, at::kFloat, "att_r");
    a.att_el = optr<float>(att_el, at::kFloat, "att_el");
    a.att_er = optr<float>(att_er, at::kFloat, "att_er");
    a.att_heads = static_cast<int32_t>(att_heads);
    a.att_feat = static_cast<int32_t>(att_feat);
    a.att_n_dst = optr<int32_t>(att_n_dst, at::kInt, "att_n_dst");
    TORCH_CHECK(att_el->numel() >= M_cap * att_heads, "att_el too small");
    TORCH_CHECK(att_l.has_value() && att_l->numel() >= N && att_r.has_value() && att_r->numel() >= N,
                "attention vectors too small");
  }
  if (mode == d::kCrossEntropy)
    TORCH_CHECK(a.labels && a.dlogits && a.loss_sum && a.correct, "cross-entropy epilogue needs labels/dlogits/loss/correct");
  d::launch_gemm(p, a, static_cast<int>(bn), stream());
}

// --------------------------------------------------------------------------- aggregation
void aggregate(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t n_dst, int64_t cap_dst, Tensor src, OptT src_map,
               int64_t dim, int64_t mode, OptT edge_w, OptT src_norm, OptT dst_norm, Tensor out, int64_t agg_col,
               int64_t self_col, double self_scale, int64_t zero_tail_rows, Tensor err, OptT bias, int64_t act,
               double dropout_p, OptT counters, int64_t dropout_salt) {
  c10::cuda::CUDAGuard g(src.device());
  d::AggArgs a;
  a.bias = optr<float>(bias, at::kFloat, "bias");
  a.act = static_cast<int32_t>(act);
  a.dropout_p = static_cast<float>(dropout_p);
  a.counters = optr<int64_t>(counters, at::kLong, "counters");
  a.dropout_salt = static_cast<uint32_t>(dropout_salt);
  TORCH_CHECK(!a.bias || bias->numel() >= dim, "bias shorter than dim");
  a.indptr = ptr<int32_t>(indptr, at::kInt, "indptr");
  a.indices = ptr<int32_t>(indices, at::kInt, "indices");
  a.n_dst_ptr = optr<int32_t>(n_dst_dev, at::kInt, "n_dst_dev");
  a.n_dst = static_cast<int32_t>(n_dst);
  a.src = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(src, at::kBFloat16, "src"));
  a.src_stride = src.stride(0);
  a.src_map = optr<int32_t>(src_map, at::kInt, "src_map");
  a.dim = static_cast<int32_t>(dim);
  a.mode = static_cast<int32_t>(mode);
  a.edge_w = optr<float>(edge_w, at::kFloat, "edge_w");
  a.src_norm = optr<float>(src_norm, at::kFloat, "src_norm");
  a.dst_norm = optr<float>(dst_norm, at::kFloat, "dst_norm");
  a.out = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(out, at::kBFloat16, "out"));
  a.out_stride = out.stride(0);
  a.agg_col = static_cast<int32_t>(agg_col);
  a.self_col = static_cast<int32_t>(self_col);
  a.self_scale = static_cast<float>(self_scale);
  a.zero_tail_rows = static_cast<int32_t>(zero_tail_rows);
  a.err = ptr<int32_t>(err, at::kInt, "err");
  TORCH_CHECK(mode != d::kAggGcn || a.src_norm, "GCN aggregation needs src_norm");
  TORCH_CHECK(mode != d::kAggWeighted || a.edge_w, "weighted aggregation needs edge_w");
  TORCH_CHECK(agg_col + dim <= out.size(1) && (self_col < 0 || self_col + dim <= out.size(1)), "output too narrow");
  TORCH_CHECK(dim <= src.size(1), "dim larger than the source rows");
  TORCH_CHECK(out.size(0) >= cap_dst, "output has fewer rows than cap_dst");
  d::launch_aggregate(a, static_cast<int>(cap_dst), stream());
}

void aggregate_bwd(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t n_dst, int64_t cap_dst, Tensor dout,
                   int64_t agg_col, int64_t self_col, double self_scale, int64_t dim, int64_t mode, OptT edge_w,
                   OptT src_norm, OptT dst_norm, Tensor dsrc, Tensor err) {
  c10::cuda::CUDAGuard g(dout.device());
  d::AggBwdArgs a;
  a.indptr = ptr<int32_t>(indptr, at::kInt, "indptr");
  a.indices = ptr<int32_t>(indices, at::kInt, "indices");
  a.n_dst_ptr = optr<int32_t>(n_dst_dev, at::kInt, "n_dst_dev");
  a.n_dst = static_cast<int32_t>(n_dst);
  a.dout = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(dout, at::kBFloat16, "dout"));
  a.dout_stride = dout.stride(0);
  a.agg_col = static_cast<int32_t>(agg_col);
  a.self_col = static_cast<int32_t>(self_col);
  a.self_scale = static_cast<float>(self_scale);
  a.dim = static_cast<int32_t>(dim);
  a.mode = static_cast<int32_t>(mode);
  a.edge_w = optr<float>(edge_w, at::kFloat, "edge_w");
  a.src_norm = optr<float>(src_norm, at::kFloat, "src_norm");
  a.dst_norm = optr<float>(dst_norm, at::kFloat, "dst_norm");
  a.dsrc = ptr2d<float>(dsrc, at::kFloat, "dsrc");
  a.dsrc_stride = dsrc.stride(0);
  a.err = ptr<int32_t>(err, at::kInt, "err");
  TORCH_CHECK(dim <= dsrc.size(1), "dsrc too narrow");
  d::launch_aggregate_bwd(a, static_cast<int>(cap_dst), stream());
}

void src_norm(Tensor indices, Tensor n_edges_dev, int64_t cap_edges, OptT n_src_dev, int64_t cap_src, Tensor deg_scratch,
              Tensor out) {
  c10::cuda::CUDAGuard g(indices.device());
  d::launch_src_norm(ptr<int32_t>(indices, at::kInt, "indices"), ptr<int32_t>(n_edges_dev, at::kInt, "n_edges"),
                     static_cast<int>(cap_edges), optr<int32_t>(n_src_dev, at::kInt, "n_src"), static_cast<int>(cap_src),
                     ptr<float>(deg_scratch, at::kFloat, "deg_scratch"), ptr<float>(out, at::kFloat, "out"), stream());
}

void act_bwd(Tensor dh, OptT h, Tensor dy, OptT n_dev, int64_t n, int64_t dim, double scale, OptT dbias,
             int64_t cap_rows) {
  c10::cuda::CUDAGuard g(dh.device());
  d::ActBwdArgs a;
  a.dh = ptr2d<float>(dh, at::kFloat, "dh");
  a.dh_stride = dh.stride(0);
  if (h.has_value()) {
    a.h = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(*h, at::kBFloat16, "h"));
    a.h_stride = h->stride(0);
  }
  a.dy = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(dy, at::kBFloat16, "dy"));
  a.dy_stride = dy.stride(0);
  a.n_ptr = optr<int32_t>(n_dev, at::kInt, "n_dev");
  a.n = static_cast<int32_t>(n);
  a.dim = static_cast<int32_t>(dim);
  a.scale = static_cast<float>(scale);
  a.dbias = optr<float>(dbias, at::kFloat, "dbias");
  a.cap_rows = static_cast<int32_t>(std::min(dy.size(0), dh.size(0)));
  if (cap_rows > 0) a.cap_rows = std::min<int32_t>(a.cap_rows, static_cast<int32_t>(cap_rows));
  d::launch_act_bwd(a, stream());
}

// --------------------------------------------------------------------------- gathers / generators
void gather_rows(Tensor table, Tensor ids, OptT n_dev, int64_t n, int64_t cap, int64_t dim, Tensor out) {
  c10::cuda::CUDAGuard g(table.device());
  TORCH_CHECK(table.is_cuda() && table.dim() == 2 && table.stride(1) == 1, "table must be a 2-D CUDA tensor");
  TORCH_CHECK(table.scalar_type() == at::kBFloat16 || table.scalar_type() == at::kFloat, "table must be bf16 or fp32");
  d::launch_gather_rows_bf16(table.data_ptr(), table.scalar_type() == at::kFloat, table.stride(0), static_cast<int32_t>(dim),
                             ptr<int32_t>(ids, at::kInt, "ids"), optr<int32_t>(n_dev, at::kInt, "n_dev"),
                             static_cast<int32_t>(n), static_cast<int>(cap),
                             reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(out, at::kBFloat16, "out")),
                             out.stride(0), stream());
}

void gather_scalar(Tensor table, Tensor ids, OptT n_dev, int64_t n, int64_t cap, Tensor out) {
  c10::cuda::CUDAGuard g(table.device());
  if (table.scalar_type() == at::kInt)
    d::launch_gather_i32(ptr<int32_t>(table, at::kInt, "table"), ptr<int32_t>(ids, at::kInt, "ids"),
                         optr<int32_t>(n_dev, at::kInt, "n_dev"), static_cast<int>(n), static_cast<int>(cap),
                         ptr<int32_t>(out, at::kInt, "out"), stream());
  else
    d::launch_gather_i64(ptr<int64_t>(table, at::kLong, "table"), ptr<int32_t>(ids, at::kInt, "ids"),
                         optr<int32_t>(n_dev, at::kInt, "n_dev"), static_cast<int>(n), static_cast<int>(cap),
                         ptr<int64_t>(out, at::kLong, "out"), stream());
}

void rmat_candidates(int64_t n, int64_t scale, double a, double b, double c, int64_t seed, int64_t e0, Tensor keys) {
  c10::cuda::CUDAGuard g(keys.device());
  d::launch_rmat_candidates(n, static_cast<int>(scale), a, b, c, static_cast<uint64_t>(seed), e0, keys.numel(),
                            ptr<int64_t>(keys, at::kLong, "keys"), stream());
}

void shuffle_keys(Tensor ids, int64_t seed, int64_t epoch, Tensor keys) {
  c10::cuda::CUDAGuard g(ids.device());
  d::launch_shuffle_keys(ptr<int64_t>(ids, at::kLong, "ids"), ids.numel(), static_cast<uint64_t>(seed),
                         static_cast<uint64_t>(epoch), ptr<int64_t>(keys, at::kLong, "keys"), stream());
}

void normal_fill(Tensor out, int64_t seed) {
  c10::cuda::CUDAGuard g(out.device());
  d::launch_normal_fill(ptr<float>(out, at::kFloat, "out"), out.numel(), static_cast<uint64_t>(seed), stream());
}

void normal_rows(Tensor out, int64_t row0, int64_t d, int64_t seed) {
  c10::cuda::CUDAGuard g(out.device());
  TORCH_CHECK(out.dim() == 2 && out.size(1) >= d, "normal_rows: out must be [rows, >= d]");
  d::launch_normal_rows_bf16(reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(out, at::kBFloat16, "out")),
                             out.stride(0), row0, out.size(0), static_cast<int>(d), static_cast<uint64_t>(seed),
                             stream());
}

void dropout_mask(Tensor mask, int64_t ld, double p, Tensor counters, int64_t salt) {
  c10::cuda::CUDAGuard g(mask.device());
  d::launch_dropout_mask(ptr<uint8_t>(mask, at::kByte, "mask"), mask.size(0), mask.size(1), ld, static_cast<float>(p),
                         ptr<int64_t>(counters, at::kLong, "counters"), static_cast<uint32_t>(salt), stream());
}

// --------------------------------------------------------------------------- optimizer
void adam(Tensor param, Tensor m, Tensor v, Tensor grad, OptT param_bf16, double lr, double b1, double b2, double eps,
          double wd, Tensor counters, double grad_scale, OptT grad_scale_dev, bool clear_grad) {
  c10::cuda::CUDAGuard g(param.device());
  d::AdamArgs a;
  a.param = ptr<float>(param, at::kFloat, "param");
  a.m = ptr<float>(m, at::kFloat, "m");
  a.v = ptr<float>(v, at::kFloat, "v");
  a.grad = ptr<float>(grad, at::kFloat, "grad");
  if (param_bf16.has_value())
    a.param_bf16 = reinterpret_cast<__nv_bfloat16*>(ptr<at::BFloat16>(*param_bf16, at::kBFloat16, "param_bf16"));
  a.n = param.numel();
  TORCH_CHECK(m.numel() == a.n && v.numel() == a.n && grad.numel() == a.n, "adam buffers differ in size");
  TORCH_CHECK(!a.param_bf16 || param_bf16->numel() == a.n, "param_bf16 differs in size");
  a.lr = static_cast<float>(lr);
  a.beta1 = static_cast<float>(b1);
  a.beta2 = static_cast<float>(b2);
  a.eps = static_cast<float>(eps);
  a.weight_decay = static_cast<float>(wd);
  TORCH_CHECK(counters.numel() >= 6, "counters needs 6 entries");
  a.step = ptr<int64_t>(counters, at::kLong, "counters") + 5;
  a.grad_scale = static_cast<float>(grad_scale);
  a.grad_scale_dev = optr<float>(grad_scale_dev, at::kFloat, "grad_scale_dev");
  a.clear_grad = clear_grad;
  d::launch_adam(a, stream());
}

void zero_(Tensor t) {
  c10::cuda::CUDAGuard g(t.device());
  check_cuda(t, "t");
  GB_CUDA_CHECK(cudaMemsetAsync(t.data_ptr(), 0, t.numel() * t.element_size(), stream()));
}

void sampler_counters(Tensor main, Tensor dst, int64_t step_offset) {
  c10::cuda::CUDAGuard g(main.device());
  TORCH_CHECK(main.numel() >= 6 && dst.numel() >= 6, "counters need 6 entries");
  d::launch_sampler_counters(ptr<int64_t>(main, at::kLong, "main"), ptr<int64_t>(dst, at::kLong, "dst"), step_offset,
                             stream());
}

void step_end(Tensor counters, OptT ring_slot, OptT fstats, OptT istats) {
  c10::cuda::CUDAGuard g(counters.device());
  TORCH_CHECK(counters.numel() >= 6, "counters needs 6 entries");
  d::launch_step_end(ptr<int64_t>(counters, at::kLong, "counters"), optr<int64_t>(ring_slot, at::kLong, "ring_slot"),
                     optr<float>(fstats, at::kFloat, "fstats"), fstats ? static_cast<int>(fstats->numel()) : 0,
                     optr<int32_t>(istats, at::kInt, "istats"), istats ? static_cast<int>(istats->numel()) : 0,
                     stream());
}

void sample_prologue(Tensor main, Tensor dst, int64_t step_offset, OptT cov, OptT table_slot, OptT count_table,
                     Tensor seeds, Tensor n_seeds, OptT labels, OptT seed_labels, OptT gideg, OptT seed_gideg) {
  c10::cuda::CUDAGuard g(main.device());
  TORCH_CHECK(main.numel() >= 6 && dst.numel() >= 6, "counters need 6 entries");
  d::SamplePrologueArgs a;
  a.main = ptr<int64_t>(main, at::kLong, "main");
  a.dst = ptr<int64_t>(dst, at::kLong, "dst");
  a.step_offset = step_offset;
  a.cov = optr<float>(cov, at::kFloat, "cov");
  a.table_slot = optr<int64_t>(table_slot, at::kLong, "table_slot");
  a.count_table = optr<int32_t>(count_table, at::kInt, "count_table");
  a.n_rows = count_table ? static_cast<int32_t>(count_table->numel()) : 0;
  a.B = static_cast<int32_t>(seeds.numel());
  a.seeds = ptr<int32_t>(seeds, at::kInt, "seeds");
  a.n_seeds = ptr<int32_t>(n_seeds, at::kInt, "n_seeds");
  a.labels = optr<int32_t>(labels, at::kInt, "labels");
  a.seed_labels = optr<int32_t>(seed_labels, at::kInt, "seed_labels");
  a.gideg = optr<int64_t>(gideg, at::kLong, "gideg");
  a.seed_gideg = optr<int64_t>(seed_gideg, at::kLong, "seed_gideg");
  d::launch_sample_prologue(a, stream());
}

// --------------------------------------------------------------------------- peer memory
Tensor tensor_from_ptr(int64_t p, std::vector<int64_t> sizes, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, device);
  return at::from_blob(reinterpret_cast<void*>(p), sizes, [](void*) {}, opts);
}

template <typename T>
T* as_ptr(int64_t p) {
  return reinterpret_cast<T*>(p);
}

// K-AR plan: the argument block of every gradient bucket, built once; launch(k) enqueues
// bucket k's kernel on the current stream (the step graph captures it).
template <typename T>
T* iptr(int64_t p) {
  return reinterpret_cast<T*>(static_cast<uintptr_t>(p));
}

struct ArPlan {
  std::vector<grappa::ar::Args> args;
  std::vector<int> grids;
  int device = -1;

  int64_t add(int64_t rank, int64_t world, int64_t mode, bool grad_bf16, int64_t lo, int64_t hi, int64_t grad,
              std::vector<int64_t> grad_peer, std::vector<int64_t> slot_local, std::vector<int64_t> slot_peer,
              int64_t param, std::vector<int64_t> param_peer, OptT m, OptT v, OptT wbf, int64_t scale_local,
              std::vector<int64_t> scale_peer, int64_t flags_local, std::vector<int64_t> flags_peer, OptT cov,
              Tensor counters, double lr, double b1, double b2, double eps, double wd, bool do_adam, OptT grad_out,
              OptT err, int64_t grid, int64_t timeout_ns) {
    namespace ga = grappa::ar;
    TORCH_CHECK(world >= 1 && world <= ga::kMaxRanks && rank >= 0 && rank < world, "rank/world out of range");
    const size_t w = static_cast<size_t>(world);
    TORCH_CHECK(flags_peer.size() == w, "one flag page per rank");
    TORCH_CHECK(grad_peer.empty() || grad_peer.size() == w, "one gradient mapping per rank");
    TORCH_CHECK(param_peer.empty() || param_peer.size() == w, "one parameter mapping per rank");
    TORCH_CHECK(scale_peer.empty() || scale_peer.size() == w, "one scale mapping per rank");
    TORCH_CHECK(slot_local.empty() || (slot_local.size() == 2 && slot_peer.size() == 2 * w), "two send slots per rank");
    TORCH_CHECK(grid >= 1 && grid <= ga::kMaxCtas, "grid out of range");
    TORCH_CHECK(counters.numel() >= 6, "counters needs 6 entries");
    ga::Args a;
    a.rank = static_cast<int32_t>(rank);
    a.world = static_cast<int32_t>(world);
    a.mode = static_cast<int32_t>(mode);
    a.grad_bf16 = grad_bf16;
    a.lo = lo;
    a.hi = hi;
    a.grad = iptr<void>(grad);
    for (size_t p = 0; p < grad_peer.size(); ++p) a.grad_peer[p] = iptr<const void>(grad_peer[p]);
    if (!slot_local.empty()) {
      a.slot_local[0] = iptr<float>(slot_local[0]);
      a.slot_local[1] = iptr<float>(slot_local[1]);
      for (size_t p = 0; p < w; ++p) {
        a.slot_peer[p][0] = iptr<const float>(slot_peer[2 * p]);
        a.slot_peer[p][1] = iptr<const float>(slot_peer[2 * p + 1]);
      }
    }
    a.param = iptr<float>(param);
    for (size_t p = 0; p < param_peer.size(); ++p) a.param_peer[p] = iptr<const float>(param_peer[p]);
    a.m = optr<float>(m, at::kFloat, "m");
    a.v = optr<float>(v, at::kFloat, "v");
    a.wbf = reinterpret_cast<__nv_bfloat16*>(optr<at::BFloat16>(wbf, at::kBFloat16, "wbf"));
    a.scale_local = iptr<float>(scale_local);
    for (size_t p = 0; p < scale_peer.size(); ++p) a.scale_peer[p] = iptr<const float>(scale_peer[p]);
    a.flags_local = iptr<uint32_t>(flags_local);
    for (size_t p = 0; p < w; ++p) a.flags_peer[p] = iptr<uint32_t>(flags_peer[p]);
    a.cov = optr<float>(cov, at::kFloat, "cov");
    a.counters = ptr<int64_t>(counters, at::kLong, "counters");
    a.lr = static_cast<float>(lr);
    a.beta1 = static_cast<float>(b1);
    a.beta2 = static_cast<float>(b2);
    a.eps = static_cast<float>(eps);
    a.weight_decay = static_cast<float>(wd);
    a.do_adam = do_adam;
    a.grad_out = optr<float>(grad_out, at::kFloat, "grad_out");
    a.err = optr<int32_t>(err, at::kInt, "err");
    a.timeout_ns = timeout_ns;
    device = counters.device().index();
    args.push_back(a);
    grids.push_back(static_cast<int>(grid));
    return static_cast<int64_t>(args.size()) - 1;
  }

  // cov (optional) replaces the bound coverage tensor for this launch
  void launch(int64_t k, OptT cov) {
    TORCH_CHECK(k >= 0 && k < static_cast<int64_t>(args.size()), "bucket index out of range");
    c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
    if (cov.has_value() && cov->defined()) {
      grappa::ar::Args a = args[k];
      a.cov = ptr<float>(*cov, at::kFloat, "cov");
      grappa::ar::launch(a, grids[k], stream());
    } else {
      grappa::ar::launch(args[k], grids[k], stream());
    }
  }

  // the learning rate of every bucket (schedules); takes effect at the next capture or
  // eager launch
  void set_lr(double lr) {
    for (auto& a : args) a.lr = static_cast<float>(lr);
  }
};

void pull_rows(std::vector<int64_t> tables, int64_t table_stride, int64_t elem_bytes, int64_t row_bytes, Tensor gids,
               OptT n_dev, int64_t n, Tensor prefix, int64_t out, int64_t out_stride, int64_t out_row0, int64_t cap,
               OptT err) {
  c10::cuda::CUDAGuard g(gids.device());
  namespace pe = grappa::peer;
  pe::PullRowsArgs a;
  TORCH_CHECK(tables.size() >= 1 && tables.size() <= static_cast<size_t>(pe::kMaxRanks), "bad table list");
  for (size_t i = 0; i < tables.size(); ++i) a.tables[i] = as_ptr<const void>(tables[i]);
  a.world = static_cast<int32_t>(tables.size());
  a.table_stride = table_stride;
  a.elem_bytes = static_cast<int32_t>(elem_bytes);
  a.row_bytes = static_cast<int32_t>(row_bytes);
  a.gids = ptr<int64_t>(gids, at::kLong, "gids");
  a.n_ptr = optr<int32_t>(n_dev, at::kInt, "n_dev");
  a.n = n;
  a.prefix = ptr<int64_t>(prefix, at::kLong, "prefix");
  TORCH_CHECK(prefix.numel() == a.world + 1, "prefix needs world + 1 entries");
  a.out = as_ptr<void>(out);
  a.out_stride = out_stride;
  a.out_row0 = out_row0;
  a.err = optr<int32_t>(err, at::kInt, "err");
  pe::launch_pull_rows(a, cap, stream());
}

void peer_copy(int64_t dst, int64_t src, int64_t bytes) {
  grappa::peer::launch_copy(as_ptr<void>(dst), as_ptr<const void>(src), bytes, stream());
}

void a2a_pull(std::vector<int64_t> src, std::vector<int64_t> src_off, std::vector<int64_t> len,
              std::vector<int64_t> dst_off, int64_t dst, int64_t first) {
  namespace pe = grappa::peer;
  const size_t w = src.size();
  TORCH_CHECK(w >= 1 && w <= static_cast<size_t>(pe::kMaxRanks) && src_off.size() == w && len.size() == w &&
                  dst_off.size() == w,
              "a2a_pull: one entry per rank");
  pe::A2aArgs a;
  a.world = static_cast<int32_t>(w);
  for (size_t p = 0; p < w; ++p) {
    a.src[p] = as_ptr<const uint8_t>(src[p]);
    a.src_off[p] = src_off[p];
    a.len[p] = len[p];
    a.dst_off[p] = dst_off[p];
  }
  a.dst = as_ptr<uint8_t>(dst);
  TORCH_CHECK(first >= 0 && first < static_cast<int64_t>(w), "a2a_pull: first segment out of range");
  a.first = static_cast<int32_t>(first);
  pe::launch_a2a_pull(a, stream());
}

void peer_barrier(int64_t rank, int64_t world, int64_t flags_local, std::vector<int64_t> flags_peer, Tensor epoch,
                  int64_t timeout_ns, Tensor err) {
  c10::cuda::CUDAGuard g(epoch.device());
  namespace pe = grappa::peer;
  TORCH_CHECK(world >= 1 && world <= pe::kMaxRanks && flags_peer.size() == static_cast<size_t>(world),
              "peer_barrier: one flag array per rank");
  uint32_t* fp[pe::kMaxRanks] = {};
  for (int p = 0; p < world; ++p) fp[p] = as_ptr<uint32_t>(flags_peer[p]);
  pe::launch_peer_barrier(static_cast<int32_t>(rank), static_cast<int32_t>(world), as_ptr<uint32_t>(flags_local), fp,
                          ptr<int64_t>(epoch, at::kLong, "epoch"), timeout_ns, ptr<int32_t>(err, at::kInt, "err"),
                          stream());
}

void mark_ids(int64_t ids, OptT n_dev, int64_t n, Tensor mark) {
  c10::cuda::CUDAGuard g(mark.device());
  grappa::peer::launch_mark(as_ptr<const int32_t>(ids), optr<int32_t>(n_dev, at::kInt, "n_dev"), n,
                            ptr<uint8_t>(mark, at::kByte, "mark"), stream());
}

void iota_map(Tensor map, int64_t g0, int64_t count, int64_t base, OptT clear_mark) {
  c10::cuda::CUDAGuard g(map.device());
  TORCH_CHECK(g0 >= 0 && g0 + count <= map.numel(), "iota_map range outside the map");
  grappa::peer::launch_iota_map(ptr<int32_t>(map, at::kInt, "map"), g0, count, static_cast<int32_t>(base),
                                optr<uint8_t>(clear_mark, at::kByte, "clear_mark"), stream());
}

void mark_compact(Tensor mark, Tensor out_ids, Tensor map, int64_t base, Tensor n_out, Tensor scratch, Tensor err) {
  c10::cuda::CUDAGuard g(mark.device());
  TORCH_CHECK(map.numel() >= mark.numel(), "map smaller than mark");
  TORCH_CHECK(scratch.numel() >= grappa::peer::mark_compact_scratch_words(mark.numel()), "scratch too small");
  grappa::peer::launch_mark_compact(ptr<uint8_t>(mark, at::kByte, "mark"), mark.numel(),
                                    ptr<int64_t>(out_ids, at::kLong, "out_ids"), ptr<int32_t>(map, at::kInt, "map"),
                                    static_cast<int32_t>(base), ptr<int32_t>(n_out, at::kInt, "n_out"),
                                    reinterpret_cast<unsigned long long*>(ptr<int64_t>(scratch, at::kLong, "scratch")),
                                    out_ids.numel(), ptr<int32_t>(err, at::kInt, "err"), stream());
}

void csr_merge(int64_t indptr_a, int64_t indices_a, int64_t n_a, int64_t indptr_b, int64_t indices_b, int64_t n_b,
               Tensor map, Tensor indptr_out, Tensor indices_out, Tensor err, int64_t g0_a, int64_t g0_b) {
  c10::cuda::CUDAGuard g(map.device());
  grappa::peer::CsrMergeArgs a;
  a.indptr_a = as_ptr<const int64_t>(indptr_a);
  a.indices_a = as_ptr<const int32_t>(indices_a);
  a.n_a = n_a;
  a.indptr_b = as_ptr<const int64_t>(indptr_b);
  a.indices_b = as_ptr<const int32_t>(indices_b);
  a.n_b = n_b;
  a.map = ptr<int32_t>(map, at::kInt, "map");
  a.indptr_out = ptr<int64_t>(indptr_out, at::kLong, "indptr_out");
  a.indices_out = ptr<int32_t>(indices_out, at::kInt, "indices_out");
  a.cap_edges = indices_out.numel();
  a.n_rows_total = indptr_out.numel() - 1;
  a.err = ptr<int32_t>(err, at::kInt, "err");
  a.g0_a = g0_a;
  a.g0_b = g0_b;
  TORCH_CHECK(a.n_rows_total >= n_a + n_b, "indptr_out too short");
  TORCH_CHECK((g0_a < 0 || g0_a + n_a <= map.numel()) && (g0_b < 0 || g0_b + n_b <= map.numel()),
              "csr_merge: partition ranges outside the map");
  grappa::peer::launch_csr_merge(a, stream());
}


// --------------------------------------------------------------------------- head.cu
void sage_head(Tensor indptr, Tensor indices, Tensor n_dst_dev, int64_t cap_dst, Tensor h, int64_t ip, Tensor w,
               OptT bias, int64_t n_classes, Tensor labels, Tensor x, Tensor dl, OptT dx, Tensor loss_sum,
               Tensor correct, OptT dbias, OptT pred_out, OptT dsrc) {
  c10::cuda::CUDAGuard g(h.device());
  d::SageHeadArgs a;
  a.indptr = ptr<int32_t>(indptr, at::kInt, "indptr");
  a.indices = ptr<int32_t>(indices, at::kInt, "indices");
  a.n_dst_ptr = ptr<int32_t>(n_dst_dev, at::kInt, "n_dst_dev");
  a.cap_dst = static_cast<int32_t>(cap_dst);
  a.h = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(h, at::kBFloat16, "h"));
  a.ldh = h.stride(0);
  a.ip = static_cast<int32_t>(ip);
  a.w = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(w, at::kBFloat16, "w"));
  a.ldw = w.stride(0);
  a.bias = optr<float>(bias, at::kFloat, "bias");
  a.n_classes = static_cast<int32_t>(n_classes);
  a.labels = ptr<int32_t>(labels, at::kInt, "labels");
  a.x = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(x, at::kBFloat16, "x"));
  a.ldx = x.stride(0);
  a.dl = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(dl, at::kBFloat16, "dl"));
  a.ld_dl = dl.stride(0);
  if (dx.has_value()) {
    a.dx = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(*dx, at::kBFloat16, "dx"));
    a.lddx = dx->stride(0);
    TORCH_CHECK(dx->size(0) >= cap_dst && dx->size(1) >= 2 * ip, "sage_head: dx too small");
  }
  a.loss_sum = ptr<float>(loss_sum, at::kFloat, "loss_sum");
  a.correct = ptr<int32_t>(correct, at::kInt, "correct");
  a.dbias = optr<float>(dbias, at::kFloat, "dbias");
  a.pred_out = optr<int32_t>(pred_out, at::kInt, "pred_out");
  if (dsrc.has_value()) {
    a.dsrc = ptr2d<float>(*dsrc, at::kFloat, "dsrc");
    a.ld_dsrc = dsrc->stride(0);
    TORCH_CHECK(dsrc->size(1) >= ip && dsrc->size(0) >= h.size(0), "sage_head: dsrc too small");
  }
  TORCH_CHECK(w.size(0) >= n_classes && w.size(1) >= 2 * ip, "sage_head: w too small");
  TORCH_CHECK(x.size(0) >= cap_dst && x.size(1) >= 2 * ip, "sage_head: x too small");
  TORCH_CHECK(dl.size(0) >= cap_dst && dl.size(1) >= n_classes, "sage_head: dl too small");
  TORCH_CHECK(labels.numel() >= cap_dst, "sage_head: labels too short");
  d::launch_sage_head(a, stream());
}

void sage_layer_fwd(Tensor indptr, Tensor indices, Tensor n_dst_dev, int64_t cap_dst, Tensor h, int64_t ip, Tensor w,
                    int64_t op, OptT bias, int64_t act, double dropout_p, OptT counters, int64_t salt, Tensor x,
                    Tensor out) {
  c10::cuda::CUDAGuard g(h.device());
  d::SageLayerArgs a;
  a.indptr = ptr<int32_t>(indptr, at::kInt, "indptr");
  a.indices = ptr<int32_t>(indices, at::kInt, "indices");
  a.n_dst_ptr = ptr<int32_t>(n_dst_dev, at::kInt, "n_dst_dev");
  a.cap_dst = static_cast<int32_t>(cap_dst);
  a.ip = static_cast<int32_t>(ip);
  a.op = static_cast<int32_t>(op);
  a.w = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(w, at::kBFloat16, "w"));
  a.ldw = w.stride(0);
  a.h = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(h, at::kBFloat16, "h"));
  a.ldh = h.stride(0);
  a.bias = optr<float>(bias, at::kFloat, "bias");
  a.act = static_cast<int32_t>(act);
  a.dropout_p = static_cast<float>(dropout_p);
  a.counters = optr<int64_t>(counters, at::kLong, "counters");
  a.dropout_salt = static_cast<uint32_t>(salt);
  a.x = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(x, at::kBFloat16, "x"));
  a.ldx = x.stride(0);
  a.out = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(out, at::kBFloat16, "out"));
  a.ldo = out.stride(0);
  TORCH_CHECK(w.size(0) >= op && w.size(1) >= 2 * ip, "sage_layer_fwd: w too small");
  TORCH_CHECK(x.size(0) >= cap_dst && x.size(1) >= 2 * ip, "sage_layer_fwd: x too small");
  TORCH_CHECK(out.size(0) >= cap_dst && out.size(1) >= op, "sage_layer_fwd: out too small");
  d::launch_sage_layer_fwd(a, stream());
}

void sage_layer_bwd(Tensor indptr, Tensor indices, Tensor n_dst_dev, int64_t cap_dst, Tensor dy, int64_t ip, Tensor w,
                    int64_t op, Tensor dsrc) {
  c10::cuda::CUDAGuard g(dy.device());
  d::SageLayerArgs a;
  a.indptr = ptr<int32_t>(indptr, at::kInt, "indptr");
  a.indices = ptr<int32_t>(indices, at::kInt, "indices");
  a.n_dst_ptr = ptr<int32_t>(n_dst_dev, at::kInt, "n_dst_dev");
  a.cap_dst = static_cast<int32_t>(cap_dst);
  a.ip = static_cast<int32_t>(ip);
  a.op = static_cast<int32_t>(op);
  a.w = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(w, at::kBFloat16, "w"));
  a.ldw = w.stride(0);
  a.dy = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(dy, at::kBFloat16, "dy"));
  a.lddy = dy.stride(0);
  a.dsrc = ptr2d<float>(dsrc, at::kFloat, "dsrc");
  a.ld_dsrc = dsrc.stride(0);
  TORCH_CHECK(w.size(0) >= op && w.size(1) >= 2 * ip, "sage_layer_bwd: w too small");
  TORCH_CHECK(dy.size(0) >= cap_dst && dy.size(1) >= op, "sage_layer_bwd: dy too small");
  TORCH_CHECK(dsrc.size(1) >= ip, "sage_layer_bwd: dsrc too narrow");
  d::launch_sage_layer_bwd(a, stream());
}

// --------------------------------------------------------------------------- nn.cu
void cross_entropy(Tensor logits, int64_t n_classes, Tensor labels, OptT n_rows_dev, int64_t cap_rows, OptT row_mask,
                   OptT n_sel_dev, Tensor dlogits, OptT dbias, Tensor loss_sum, Tensor correct) {
  c10::cuda::CUDAGuard g(logits.device());
  d::CeArgs a;
  a.logits = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(logits, at::kBFloat16, "logits"));
  a.ld = logits.stride(0);
  a.n_classes = static_cast<int32_t>(n_classes);
  a.labels = ptr<int32_t>(labels, at::kInt, "labels");
  a.n_rows_ptr = optr<int32_t>(n_rows_dev, at::kInt, "n_rows_dev");
  a.cap_rows = static_cast<int32_t>(cap_rows);
  a.row_mask = optr<uint8_t>(row_mask, at::kByte, "row_mask");
  a.n_sel_ptr = optr<int32_t>(n_sel_dev, at::kInt, "n_sel_dev");
  a.dlogits = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(dlogits, at::kBFloat16, "dlogits"));
  a.ld_dl = dlogits.stride(0);
  a.dbias = optr<float>(dbias, at::kFloat, "dbias");
  a.loss_sum = ptr<float>(loss_sum, at::kFloat, "loss_sum");
  a.correct = ptr<int32_t>(correct, at::kInt, "correct");
  TORCH_CHECK(logits.size(0) >= cap_rows && dlogits.size(0) >= cap_rows, "logits rows < cap_rows");
  TORCH_CHECK(labels.numel() >= cap_rows, "labels shorter than cap_rows");
  TORCH_CHECK(dlogits.size(1) >= n_classes && logits.size(1) >= n_classes, "fewer columns than classes");
  d::launch_cross_entropy(a, stream());
}

void batchnorm_fwd(Tensor x, int64_t dim, OptT n_dev, int64_t cap, Tensor sums, Tensor gamma, Tensor beta,
                   Tensor running_mean, Tensor running_var, OptT num_batches, double momentum, double eps,
                   bool training, int64_t act, Tensor y) {
  c10::cuda::CUDAGuard g(x.device());
  d::BnArgs a;
  a.x = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(x, at::kBFloat16, "x"));
  a.ldx = x.stride(0);
  a.dim = static_cast<int32_t>(dim);
  a.n_ptr = optr<int32_t>(n_dev, at::kInt, "n_dev");
  a.cap = static_cast<int32_t>(cap);
  a.sums = ptr<float>(sums, at::kFloat, "sums");
  a.gamma = gamma.data_ptr<float>();
  a.beta = beta.data_ptr<float>();
  a.running_mean = running_mean.data_ptr<float>();
  a.running_var = running_var.data_ptr<float>();
  a.stat_dim = static_cast<int32_t>(std::min(running_mean.numel(), running_var.numel()));
  a.num_batches = optr<int64_t>(num_batches, at::kLong, "num_batches");
  a.momentum = static_cast<float>(momentum);
  a.eps = static_cast<float>(eps);
  a.training = training;
  a.act = static_cast<int32_t>(act);
  a.y = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(y, at::kBFloat16, "y"));
  a.ldy = y.stride(0);
  TORCH_CHECK(sums.numel() >= 2 * dim && gamma.numel() >= dim && beta.numel() >= dim, "batchnorm: short parameters");
  TORCH_CHECK(x.size(0) >= cap && y.size(0) >= cap, "batchnorm: fewer rows than cap");
  d::launch_batchnorm_fwd(a, stream());
}

void batchnorm_bwd(Tensor x, OptT y, Tensor dy, bool clear_dy, int64_t dim, OptT n_dev, int64_t cap, Tensor sums,
                   Tensor bsums, Tensor gamma, OptT dgamma, OptT dbeta, double eps, Tensor dx) {
  c10::cuda::CUDAGuard g(x.device());
  d::BnBwdArgs a;
  a.x = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(x, at::kBFloat16, "x"));
  a.ldx = x.stride(0);
  if (y.has_value() && y->defined()) {
    a.y = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(*y, at::kBFloat16, "y"));
    a.ldy = y->stride(0);
  }
  if (dy.scalar_type() == at::kBFloat16) {
    a.dy_bf16 = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(dy, at::kBFloat16, "dy"));
  } else {
    a.dy = ptr2d<float>(dy, at::kFloat, "dy");
  }
  a.lddy = dy.stride(0);
  a.clear_dy = clear_dy;
  a.dim = static_cast<int32_t>(dim);
  a.n_ptr = optr<int32_t>(n_dev, at::kInt, "n_dev");
  a.cap = static_cast<int32_t>(cap);
  a.sums = ptr<float>(sums, at::kFloat, "sums");
  a.bsums = ptr<float>(bsums, at::kFloat, "bsums");
  a.gamma = gamma.data_ptr<float>();
  a.dgamma = dgamma.has_value() ? dgamma->data_ptr<float>() : nullptr;
  a.dbeta = dbeta.has_value() ? dbeta->data_ptr<float>() : nullptr;
  a.eps = static_cast<float>(eps);
  a.dx = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(dx, at::kBFloat16, "dx"));
  a.lddx = dx.stride(0);
  d::launch_batchnorm_bwd(a, stream());
}

void l2norm_fwd(Tensor z, int64_t dim, OptT n_dev, int64_t cap, Tensor y, Tensor norms) {
  c10::cuda::CUDAGuard g(z.device());
  d::launch_l2norm_fwd(reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(z, at::kBFloat16, "z")), z.stride(0),
                       static_cast<int32_t>(dim), optr<int32_t>(n_dev, at::kInt, "n_dev"), static_cast<int>(cap),
                       reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(y, at::kBFloat16, "y")), y.stride(0),
                       ptr<float>(norms, at::kFloat, "norms"), stream());
}

void l2norm_bwd(Tensor y, Tensor dy, Tensor norms, int64_t dim, OptT n_dev, int64_t cap, Tensor dz) {
  c10::cuda::CUDAGuard g(y.device());
  float* dyf = nullptr;
  const __nv_bfloat16* dyb = nullptr;
  if (dy.scalar_type() == at::kBFloat16) dyb = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(dy, at::kBFloat16, "dy"));
  else dyf = ptr2d<float>(dy, at::kFloat, "dy");
  d::launch_l2norm_bwd(reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(y, at::kBFloat16, "y")), y.stride(0),
                       dyf, dyb, dy.stride(0), ptr<float>(norms, at::kFloat, "norms"), static_cast<int32_t>(dim),
                       optr<int32_t>(n_dev, at::kInt, "n_dev"), static_cast<int>(cap), ptr2d<float>(dz, at::kFloat, "dz"),
                       dz.stride(0), stream());
}

void add_bf16_rows(Tensor dst, Tensor src, int64_t dim, OptT n_dev, int64_t cap) {
  c10::cuda::CUDAGuard g(dst.device());
  d::launch_add_bf16_rows(ptr2d<float>(dst, at::kFloat, "dst"), dst.stride(0),
                          reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(src, at::kBFloat16, "src")),
                          src.stride(0), static_cast<int32_t>(dim), optr<int32_t>(n_dev, at::kInt, "n_dev"),
                          static_cast<int>(cap), stream());
}

void dropout_rows(Tensor in, Tensor out, int64_t dim, int64_t ld_mask, OptT n_dev, int64_t cap, double p,
                  Tensor counters, int64_t salt) {
  c10::cuda::CUDAGuard g(in.device());
  d::launch_dropout_rows(reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(in, at::kBFloat16, "in")),
                         in.stride(0), reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(out, at::kBFloat16, "out")),
                         out.stride(0), static_cast<int32_t>(dim), ld_mask, optr<int32_t>(n_dev, at::kInt, "n_dev"),
                         static_cast<int>(cap), static_cast<float>(p), ptr<int64_t>(counters, at::kLong, "counters"),
                         static_cast<uint32_t>(salt), stream());
}

void dropout_grad(Tensor gr, int64_t dim, int64_t ld_mask, OptT n_dev, int64_t cap, double p, Tensor counters,
                  int64_t salt) {
  c10::cuda::CUDAGuard g(gr.device());
  d::launch_dropout_grad(ptr2d<float>(gr, at::kFloat, "g"), gr.stride(0), static_cast<int32_t>(dim), ld_mask,
                         optr<int32_t>(n_dev, at::kInt, "n_dev"), static_cast<int>(cap), static_cast<float>(p),
                         ptr<int64_t>(counters, at::kLong, "counters"), static_cast<uint32_t>(salt), stream());
}

void f32_to_bf16_rows(Tensor src, Tensor dst, int64_t dim, OptT n_dev, int64_t cap, bool clear, int64_t zero_tail_rows) {
  c10::cuda::CUDAGuard g(src.device());
  TORCH_CHECK(src.size(0) >= cap && dst.size(0) >= cap, "f32_to_bf16_rows: fewer rows than cap");
  d::launch_f32_to_bf16_rows(ptr2d<float>(src, at::kFloat, "src"), src.stride(0),
                             reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(dst, at::kBFloat16, "dst")),
                             dst.stride(0), static_cast<int32_t>(dim), optr<int32_t>(n_dev, at::kInt, "n_dev"),
                             static_cast<int>(cap), clear, static_cast<int32_t>(zero_tail_rows), stream());
}

// --------------------------------------------------------------------------- gat.cu
d::GatArgs gat_args(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t cap_dst, OptT n_src_dev, int64_t cap_src,
                    int64_t heads, int64_t feat, Tensor z, Tensor attn_l, Tensor attn_r, Tensor el, Tensor er,
                    Tensor smax, Tensor ssum, double slope, int64_t zmod = 0) {
  d::GatArgs a;
  a.zmod = static_cast<int32_t>(zmod);
  a.indptr = ptr<int32_t>(indptr, at::kInt, "indptr");
  a.indices = ptr<int32_t>(indices, at::kInt, "indices");
  a.n_dst_ptr = optr<int32_t>(n_dst_dev, at::kInt, "n_dst_dev");
  a.cap_dst = static_cast<int32_t>(cap_dst);
  a.n_src_ptr = optr<int32_t>(n_src_dev, at::kInt, "n_src_dev");
  a.cap_src = static_cast<int32_t>(cap_src);
  a.heads = static_cast<int32_t>(heads);
  a.feat = static_cast<int32_t>(feat);
  a.z = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(z, at::kBFloat16, "z"));
  a.ldz = z.stride(0);
  a.attn_l = attn_l.data_ptr<float>();
  a.attn_r = attn_r.data_ptr<float>();
  a.el = ptr<float>(el, at::kFloat, "el");
  a.er = ptr<float>(er, at::kFloat, "er");
  a.smax = ptr<float>(smax, at::kFloat, "smax");
  a.ssum = ptr<float>(ssum, at::kFloat, "ssum");
  a.slope = static_cast<float>(slope);
  TORCH_CHECK(z.size(0) >= cap_src && z.size(1) >= (zmod > 0 ? zmod : heads * feat), "gat: z too small");
  TORCH_CHECK(el.numel() >= cap_src * heads && er.numel() >= cap_dst * heads, "gat: score buffers too small");
  TORCH_CHECK(smax.numel() >= cap_dst * heads && ssum.numel() >= cap_dst * heads, "gat: softmax buffers too small");
  TORCH_CHECK(attn_l.is_cuda() && attn_r.is_cuda() && attn_l.scalar_type() == at::kFloat, "gat: attention vectors");
  return a;
}

void gat_scores(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t cap_dst, OptT n_src_dev, int64_t cap_src,
                int64_t heads, int64_t feat, Tensor z, Tensor attn_l, Tensor attn_r, Tensor el, Tensor er, Tensor smax,
                Tensor ssum, double slope) {
  c10::cuda::CUDAGuard g(z.device());
  auto a = gat_args(indptr, indices, n_dst_dev, cap_dst, n_src_dev, cap_src, heads, feat, z, attn_l, attn_r, el, er,
                    smax, ssum, slope);
  d::launch_gat_scores(a, stream());
}

void gat_fwd(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t cap_dst, OptT n_src_dev, int64_t cap_src,
             int64_t heads, int64_t feat, Tensor z, Tensor attn_l, Tensor attn_r, Tensor el, Tensor er, Tensor smax,
             Tensor ssum, double slope, Tensor bias, bool mean_heads, int64_t act, double dropout_p, OptT counters,
             int64_t dropout_salt, Tensor out) {
  c10::cuda::CUDAGuard g(z.device());
  auto a = gat_args(indptr, indices, n_dst_dev, cap_dst, n_src_dev, cap_src, heads, feat, z, attn_l, attn_r, el, er,
                    smax, ssum, slope);
  a.bias = bias.data_ptr<float>();
  a.mean_heads = mean_heads;
  a.act = static_cast<int32_t>(act);
  a.dropout_p = static_cast<float>(dropout_p);
  a.counters = optr<int64_t>(counters, at::kLong, "counters");
  a.dropout_salt = static_cast<uint32_t>(dropout_salt);
  a.out = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(out, at::kBFloat16, "out"));
  a.ldo = out.stride(0);
  TORCH_CHECK(out.size(0) >= cap_dst && out.size(1) >= (mean_heads ? feat : heads * feat), "gat: out too small");
  d::launch_gat_fwd(a, stream());
}

void gat_bwd(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t cap_dst, OptT n_src_dev, int64_t cap_src,
             int64_t heads, int64_t feat, Tensor z, Tensor attn_l, Tensor attn_r, Tensor el, Tensor er, Tensor smax,
             Tensor ssum, double slope, bool mean_heads, Tensor dout, Tensor edge_scratch, Tensor del, Tensor der,
             Tensor dz, OptT dbias, OptT dattn_l, OptT dattn_r, Tensor dz_bf16, Tensor err) {
  c10::cuda::CUDAGuard g(z.device());
  auto a = gat_args(indptr, indices, n_dst_dev, cap_dst, n_src_dev, cap_src, heads, feat, z, attn_l, attn_r, el, er,
                    smax, ssum, slope);
  a.mean_heads = mean_heads;
  a.dout = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(dout, at::kBFloat16, "dout"));
  a.lddo = dout.stride(0);
  a.edge_scratch = ptr<float>(edge_scratch, at::kFloat, "edge_scratch");
  a.del = ptr<float>(del, at::kFloat, "del");
  a.der = ptr<float>(der, at::kFloat, "der");
  a.dz = ptr2d<float>(dz, at::kFloat, "dz");
  a.lddz = dz.stride(0);
  a.dbias = dbias.has_value() ? dbias->data_ptr<float>() : nullptr;
  a.dattn_l = dattn_l.has_value() ? dattn_l->data_ptr<float>() : nullptr;
  a.dattn_r = dattn_r.has_value() ? dattn_r->data_ptr<float>() : nullptr;
  a.dz_bf16 = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(dz_bf16, at::kBFloat16, "dz_bf16"));
  a.lddzb = dz_bf16.stride(0);
  a.err = ptr<int32_t>(err, at::kInt, "err");
  TORCH_CHECK(edge_scratch.numel() >= static_cast<int64_t>(indices.numel()) * heads, "gat: edge scratch too small");
  TORCH_CHECK(dz.size(0) >= cap_src && dz_bf16.size(0) >= cap_src, "gat: gradient buffers too small");
  d::launch_gat_bwd(a, stream());
}

void gat_bwd_input(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t cap_dst, OptT n_src_dev, int64_t cap_src,
                   int64_t heads, int64_t feat, Tensor z, Tensor attn_l, Tensor attn_r, Tensor el, Tensor er,
                   Tensor smax, Tensor ssum, double slope, Tensor dout, Tensor edge_scratch, Tensor del, Tensor der,
                   OptT dbias, OptT dattn_l, OptT dattn_r, Tensor x, int64_t in_dim, Tensor y, Tensor xl, Tensor xr,
                   Tensor err) {
  c10::cuda::CUDAGuard g(z.device());
  auto a = gat_args(indptr, indices, n_dst_dev, cap_dst, n_src_dev, cap_src, heads, feat, z, attn_l, attn_r, el, er,
                    smax, ssum, slope);
  a.dout = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(dout, at::kBFloat16, "dout"));
  a.lddo = dout.stride(0);
  a.edge_scratch = ptr<float>(edge_scratch, at::kFloat, "edge_scratch");
  a.del = ptr<float>(del, at::kFloat, "del");
  a.der = ptr<float>(der, at::kFloat, "der");
  a.dbias = dbias.has_value() ? dbias->data_ptr<float>() : nullptr;
  a.dattn_l = dattn_l.has_value() ? dattn_l->data_ptr<float>() : nullptr;
  a.dattn_r = dattn_r.has_value() ? dattn_r->data_ptr<float>() : nullptr;
  a.x = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(x, at::kBFloat16, "x"));
  a.ldx = x.stride(0);
  a.in_dim = static_cast<int32_t>(in_dim);
  a.y = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(y, at::kBFloat16, "y"));
  a.ldy = y.stride(0);
  a.xl = ptr<float>(xl, at::kFloat, "xl");
  a.xr = ptr<float>(xr, at::kFloat, "xr");
  a.err = ptr<int32_t>(err, at::kInt, "err");
  TORCH_CHECK(edge_scratch.numel() >= static_cast<int64_t>(indices.numel()) * heads, "gat: edge scratch too small");
  TORCH_CHECK(x.size(0) >= cap_src && x.size(1) >= in_dim, "gat: x too small");
  TORCH_CHECK(y.size(0) >= cap_dst && y.size(1) >= heads * in_dim, "gat: y too small");
  TORCH_CHECK(xl.numel() >= heads * in_dim && xr.numel() >= heads * in_dim, "gat: xl / xr too small");
  d::launch_gat_bwd_input(a, stream());
}

// GAT input layer with the projection after the aggregation (gat.cu): the rows are the
// layer's input x (in_dim columns, shared by every head), the attention vectors wl/wr
// (fp32 [heads * in_dim]) come from gat_in_prep
void gat_in_scores(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t cap_dst, OptT n_src_dev, int64_t cap_src,
                   int64_t heads, int64_t in_dim, Tensor x, Tensor wl, Tensor wr, Tensor el, Tensor er, Tensor smax,
                   Tensor ssum, double slope) {
  c10::cuda::CUDAGuard g(x.device());
  auto a = gat_args(indptr, indices, n_dst_dev, cap_dst, n_src_dev, cap_src, heads, in_dim, x, wl, wr, el, er, smax, ssum,
                    slope, in_dim);
  d::launch_gat_scores(a, stream());
}

void gat_in_fwd(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t cap_dst, OptT n_src_dev, int64_t cap_src,
                int64_t heads, int64_t in_dim, Tensor x, Tensor wl, Tensor wr, Tensor el, Tensor er, Tensor smax,
                Tensor ssum, double slope, Tensor y) {
  c10::cuda::CUDAGuard g(x.device());
  auto a = gat_args(indptr, indices, n_dst_dev, cap_dst, n_src_dev, cap_src, heads, in_dim, x, wl, wr, el, er, smax, ssum,
                    slope, in_dim);
  a.bias = nullptr;
  a.mean_heads = false;
  a.act = 0;
  a.out = reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(y, at::kBFloat16, "y"));
  a.ldo = y.stride(0);
  TORCH_CHECK(y.size(0) >= cap_dst && y.size(1) >= heads * in_dim, "gat_in_fwd: y too small");
  d::launch_gat_fwd(a, stream());
}

void gat_in_bwd(Tensor indptr, Tensor indices, OptT n_dst_dev, int64_t cap_dst, OptT n_src_dev, int64_t cap_src,
                int64_t heads, int64_t in_dim, Tensor x, Tensor wl, Tensor wr, Tensor el, Tensor er, Tensor smax,
                Tensor ssum, double slope, Tensor gx, Tensor edge_scratch, Tensor del, Tensor der, Tensor xl, Tensor xr,
                Tensor err) {
  c10::cuda::CUDAGuard g(x.device());
  auto a = gat_args(indptr, indices, n_dst_dev, cap_dst, n_src_dev, cap_src, heads, in_dim, x, wl, wr, el, er, smax, ssum,
                    slope, in_dim);
  a.mean_heads = false;
  a.dout = reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(gx, at::kBFloat16, "gx"));
  a.lddo = gx.stride(0);
  a.edge_scratch = ptr<float>(edge_scratch, at::kFloat, "edge_scratch");
  a.del = ptr<float>(del, at::kFloat, "del");
  a.der = ptr<float>(der, at::kFloat, "der");
  a.dattn_l = ptr<float>(xl, at::kFloat, "xl");  // sum_u del x_u: the virtual rows' "attention" gradient
  a.dattn_r = ptr<float>(xr, at::kFloat, "xr");
  a.err = ptr<int32_t>(err, at::kInt, "err");
  TORCH_CHECK(edge_scratch.numel() >= static_cast<int64_t>(indices.numel()) * heads, "gat: edge scratch too small");
  TORCH_CHECK(gx.size(0) >= cap_dst && gx.size(1) >= heads * in_dim, "gat_in_bwd: gx too small");
  TORCH_CHECK(xl.numel() >= heads * in_dim && xr.numel() >= heads * in_dim, "gat_in_bwd: xl / xr too small");
  d::launch_gat_bwd(a, stream());
}

void gat_in_prep(Tensor w, Tensor attn_l, Tensor attn_r, int64_t heads, int64_t feat, int64_t in_dim, Tensor wl,
                 Tensor wr, Tensor wbd) {
  c10::cuda::CUDAGuard g(w.device());
  TORCH_CHECK(w.size(0) >= heads * feat && w.size(1) >= in_dim, "gat_in_prep: w too small");
  TORCH_CHECK(wbd.size(0) >= heads * feat && wbd.size(1) >= heads * in_dim, "gat_in_prep: wbd too small");
  TORCH_CHECK(wl.numel() >= heads * in_dim && wr.numel() >= heads * in_dim, "gat_in_prep: wl / wr too small");
  d::launch_gat_in_prep(reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(w, at::kBFloat16, "w")), w.stride(0),
                        attn_l.data_ptr<float>(), attn_r.data_ptr<float>(), static_cast<int>(heads),
                        static_cast<int>(feat), static_cast<int>(in_dim), static_cast<int>(wbd.size(0)),
                        ptr<float>(wl, at::kFloat, "wl"), ptr<float>(wr, at::kFloat, "wr"),
                        reinterpret_cast<__nv_bfloat16*>(ptr2d<at::BFloat16>(wbd, at::kBFloat16, "wbd")), wbd.stride(0),
                        stream());
}

void gat_in_dw(Tensor T, Tensor xl, Tensor xr, Tensor attn_l, Tensor attn_r, Tensor w32, int64_t heads, int64_t feat,
               int64_t in_dim, Tensor dw, OptT dattn_l, OptT dattn_r) {
  c10::cuda::CUDAGuard g(T.device());
  TORCH_CHECK(T.size(0) >= heads * feat && T.size(1) >= heads * in_dim, "gat_in_dw: T too small");
  TORCH_CHECK(dw.size(0) >= heads * feat && dw.size(1) >= in_dim && w32.size(1) >= in_dim, "gat_in_dw: dw / w too small");
  d::launch_gat_in_dw(ptr2d<float>(T, at::kFloat, "T"), T.stride(0), ptr<float>(xl, at::kFloat, "xl"),
                      ptr<float>(xr, at::kFloat, "xr"), attn_l.data_ptr<float>(), attn_r.data_ptr<float>(),
                      ptr2d<float>(w32, at::kFloat, "w32"), w32.stride(0), static_cast<int>(heads), static_cast<int>(feat),
                      static_cast<int>(in_dim), ptr2d<float>(dw, at::kFloat, "dw"), dw.stride(0),
                      dattn_l.has_value() ? dattn_l->data_ptr<float>() : nullptr,
                      dattn_r.has_value() ? dattn_r->data_ptr<float>() : nullptr, stream());
}

void col_sum_bf16(Tensor x, OptT n_dev, int64_t cols, Tensor out) {
  c10::cuda::CUDAGuard g(x.device());
  TORCH_CHECK(x.size(1) >= cols && out.numel() >= cols, "col_sum_bf16: sizes");
  d::launch_col_sum_bf16(reinterpret_cast<const __nv_bfloat16*>(ptr2d<at::BFloat16>(x, at::kBFloat16, "x")), x.stride(0),
                         optr<int32_t>(n_dev, at::kInt, "n_dev"), static_cast<int>(x.size(0)), static_cast<int>(cols),
                         ptr<float>(out, at::kFloat, "out"), stream());
}

void gat_dw_combine(Tensor T, Tensor xl, Tensor xr, Tensor attn_l, Tensor attn_r, int64_t heads, int64_t feat,
                    int64_t in_dim, Tensor dw) {
  c10::cuda::CUDAGuard g(T.device());
  TORCH_CHECK(T.size(0) >= heads * feat && T.size(1) >= heads * in_dim, "gat_dw_combine: T too small");
  TORCH_CHECK(dw.size(0) >= heads * feat && dw.size(1) >= in_dim, "gat_dw_combine: dw too small");
  d::launch_gat_dw_combine(ptr2d<float>(T, at::kFloat, "T"), T.stride(0), ptr<float>(xl, at::kFloat, "xl"),
                           ptr<float>(xr, at::kFloat, "xr"), attn_l.data_ptr<float>(), attn_r.data_ptr<float>(),
                           static_cast<int>(heads), static_cast<int>(feat), static_cast<int>(in_dim),
                           ptr2d<float>(dw, at::kFloat, "dw"), dw.stride(0), stream());
}

void walk_hop(Tensor indptr, Tensor indices, Tensor dst_nid, OptT n_dst_dev, int64_t n_dst, int64_t length,
              double restart_prob, int64_t num_walks, int64_t num_neighbors, Tensor counters, int64_t hop,
              Tensor out_indptr, Tensor out_nbr, Tensor out_w, Tensor n_edges_out, Tensor scan_scratch, Tensor err,
              int64_t cap_dst) {
  c10::cuda::CUDAGuard g(indptr.device());
  d::WalkHopArgs a;
  a.indptr = ptr<int64_t>(indptr, at::kLong, "indptr");
  a.indices = ptr<int32_t>(indices, at::kInt, "indices");
  a.n_graph_nodes = indptr.numel() - 1;
  a.dst_nid = ptr<int32_t>(dst_nid, at::kInt, "dst_nid");
  a.n_dst_ptr = optr<int32_t>(n_dst_dev, at::kInt, "n_dst_dev");
  a.n_dst = static_cast<int32_t>(n_dst);
  a.length = static_cast<int32_t>(length);
  a.restart_thr = restart_prob >= 1.0 ? 0xFFFFFFFFu : static_cast<uint32_t>(restart_prob * 4294967296.0);
  a.num_walks = static_cast<int32_t>(num_walks);
  a.num_neighbors = static_cast<int32_t>(num_neighbors);
  a.counters = ptr<int64_t>(counters, at::kLong, "counters");
  a.hop = static_cast<int32_t>(hop);
  a.out_indptr = ptr<int32_t>(out_indptr, at::kInt, "out_indptr");
  a.out_nbr = ptr<int32_t>(out_nbr, at::kInt, "out_nbr");
  a.out_w = ptr<float>(out_w, at::kFloat, "out_w");
  a.cap_edges = static_cast<int32_t>(std::min(out_nbr.numel(), out_w.numel()));
  a.n_edges_out = ptr<int32_t>(n_edges_out, at::kInt, "n_edges_out");
  a.scan_scratch = reinterpret_cast<unsigned long long*>(ptr<int64_t>(scan_scratch, at::kLong, "scan_scratch"));
  a.err = ptr<int32_t>(err, at::kInt, "err");
  TORCH_CHECK(out_indptr.numel() >= cap_dst + 1 && dst_nid.numel() >= cap_dst, "walk_hop: buffers smaller than cap_dst");
  // exactly sized: the scan numbers its launches by the grid size (common.cuh LookBack)
  TORCH_CHECK(scan_scratch.numel() == d::walk_scan_scratch_words(static_cast<int>(cap_dst)),
              "scan_scratch must hold exactly walk_scratch_words(capacity) words and be used with that capacity only");
  d::launch_walk_hop(a, static_cast<int>(cap_dst), stream());
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  py::class_<ArPlan>(m, "ArPlan")
      .def(py::init<>())
      .def("add", &ArPlan::add, py::arg("rank"), py::arg("world"), py::arg("mode"), py::arg("grad_bf16"), py::arg("lo"),
           py::arg("hi"), py::arg("grad"), py::arg("grad_peer"), py::arg("slot_local"), py::arg("slot_peer"),
           py::arg("param"), py::arg("param_peer"), py::arg("m"), py::arg("v"), py::arg("wbf"), py::arg("scale_local"),
           py::arg("scale_peer"), py::arg("flags_local"), py::arg("flags_peer"), py::arg("cov"), py::arg("counters"),
           py::arg("lr"), py::arg("b1"), py::arg("b2"), py::arg("eps"), py::arg("wd"), py::arg("do_adam"),
           py::arg("grad_out"), py::arg("err"), py::arg("grid"), py::arg("timeout_ns"))
      .def("launch", &ArPlan::launch, py::arg("k"), py::arg("cov") = py::none())
      .def("set_lr", &ArPlan::set_lr)
      .def("__len__", [](const ArPlan& p) { return p.args.size(); });
  m.doc() = "grappa_b200 sm_100a kernels";
  m.def("sample_hop", &sample_hop, py::arg("indptr"), py::arg("indices"), py::arg("dst_nid"), py::arg("n_dst_dev"),
        py::arg("n_dst"), py::arg("frontier"), py::arg("fanout"), py::arg("replace"), py::arg("counters"),
        py::arg("hop"), py::arg("gideg"), py::arg("cov_accum"), py::arg("out_indptr"), py::arg("out_nbr"),
        py::arg("n_edges_out"), py::arg("scan_scratch"), py::arg("err"), py::arg("cap_dst"),
        py::arg("map") = py::none(), py::arg("src_nid") = py::none(), py::arg("src_sampled") = py::none());
  m.def("sample_scratch_words", &sample_scratch_words);
  m.def("compact", &compact, py::arg("dst_nid"), py::arg("n_dst_dev"), py::arg("nbr"), py::arg("n_edges_dev"),
        py::arg("map"), py::arg("src_nid"), py::arg("src_sampled"), py::arg("indices"), py::arg("n_src_out"),
        py::arg("scan_scratch"), py::arg("err"), py::arg("cap_dst"), py::arg("cap_edges"), py::arg("counters"),
        py::arg("slot"), py::arg("k1_done") = false, py::arg("t_cnt") = py::none(), py::arg("t_rank") = py::none(),
        py::arg("run_k3") = true);
  m.def("compact_edges", &compact_edges, py::arg("nbr"), py::arg("n_edges_dev"), py::arg("indices"),
        py::arg("cap_src"), py::arg("map"));
  m.def("compact_scratch_words", &compact_scratch_words);
  m.def("block_transpose", &block_transpose);
  m.def("aggregate_bwd_gather", &aggregate_bwd_gather);
  m.def("sage_head", &sage_head, py::arg("indptr"), py::arg("indices"), py::arg("n_dst_dev"), py::arg("cap_dst"),
        py::arg("h"), py::arg("ip"), py::arg("w"), py::arg("bias"), py::arg("n_classes"), py::arg("labels"), py::arg("x"),
        py::arg("dl"), py::arg("dx"), py::arg("loss_sum"), py::arg("correct"), py::arg("dbias"),
        py::arg("pred_out") = py::none(), py::arg("dsrc") = py::none());
  m.def("sage_head_fused_bwd", [] {
    const char* e = std::getenv("GRAPPA_SAGE_HEAD_TILE");
    return !(e && e[0] == '0');
  });
  m.def("sage_layer_fwd", &sage_layer_fwd);
  m.def("sage_layer_bwd", &sage_layer_bwd);
  m.def("sage_layer_tile_supported",
        [](int64_t ip, int64_t op) { return d::sage_layer_tile_supported(static_cast<int>(ip), static_cast<int>(op)); });
  m.def("sage_head_supported", [](int64_t ip, int64_t c) { return d::sage_head_supported(static_cast<int>(ip), static_cast<int>(c)); });
  m.def("gemm", &gemm, py::arg("A"), py::arg("a_mn"), py::arg("B"), py::arg("b_mn"), py::arg("M_cap"), py::arg("M_dev"),
        py::arg("N"), py::arg("K_cap"), py::arg("K_dev"), py::arg("splits"), py::arg("C"), py::arg("mode"),
        py::arg("bias"), py::arg("act"), py::arg("dropout_p"), py::arg("counters"), py::arg("salt"), py::arg("labels"),
        py::arg("n_classes"), py::arg("dlogits"), py::arg("loss_sum"), py::arg("correct"), py::arg("pred_out"),
        py::arg("n_rows_dev"), py::arg("dbias"), py::arg("err"), py::arg("bn"), py::arg("act_mask") = py::none(),
        py::arg("mask_scale") = 1.0, py::arg("zero_tail_rows") = 0, py::arg("att_l") = py::none(),
        py::arg("att_r") = py::none(), py::arg("att_el") = py::none(), py::arg("att_er") = py::none(),
        py::arg("att_heads") = 0, py::arg("att_feat") = 0, py::arg("att_n_dst") = py::none());
  m.def("aggregate", &aggregate, py::arg("indptr"), py::arg("indices"), py::arg("n_dst_dev"), py::arg("n_dst"),
        py::arg("cap_dst"), py::arg("src"), py::arg("src_map"), py::arg("dim"), py::arg("mode"), py::arg("edge_w"),
        py::arg("src_norm"), py::arg("dst_norm"), py::arg("out"), py::arg("agg_col"), py::arg("self_col"),
        py::arg("self_scale"), py::arg("zero_tail_rows"), py::arg("err"), py::arg("bias") = py::none(),
        py::arg("act") = 0, py::arg("dropout_p") = 0.0, py::arg("counters") = py::none(), py::arg("dropout_salt") = 0);
  m.def("cross_entropy", &cross_entropy);
  m.def("walk_hop", &walk_hop);
  m.def("walk_scratch_words", [](int64_t cap) { return d::walk_scan_scratch_words(static_cast<int>(cap)); });
  m.def("batchnorm_fwd", &batchnorm_fwd);
  m.def("batchnorm_bwd", &batchnorm_bwd);
  m.def("l2norm_fwd", &l2norm_fwd);
  m.def("l2norm_bwd", &l2norm_bwd);
  m.def("add_bf16_rows", &add_bf16_rows);
  m.def("dropout_rows", &dropout_rows);
  m.def("dropout_grad", &dropout_grad);
  m.def("f32_to_bf16_rows", &f32_to_bf16_rows);
  m.def("gat_scores", &gat_scores);
  m.def("gat_fwd", &gat_fwd);
  m.def("gat_bwd", &gat_bwd);
  m.def("gat_bwd_input", &gat_bwd_input);
  m.def("gat_dw_combine", &gat_dw_combine);
  m.def("gat_in_scores", &gat_in_scores);
  m.def("gat_in_fwd", &gat_in_fwd);
  m.def("gat_in_bwd", &gat_in_bwd);
  m.def("gat_in_prep", &gat_in_prep);
  m.def("gat_in_dw", &gat_in_dw);
  m.def("col_sum_bf16", &col_sum_bf16);
  m.def("aggregate_bwd", &aggregate_bwd);
  m.def("src_norm", &src_norm);
  m.def("act_bwd", &act_bwd);
  m.def("gather_rows", &gather_rows);
  m.def("gather_scalar", &gather_scalar);
  m.def("rmat_candidates", &rmat_candidates);
  m.def("shuffle_keys", &shuffle_keys);
  m.def("normal_fill", &normal_fill);
  m.def("normal_rows", &normal_rows);
  m.def("dropout_mask", &dropout_mask);
  m.def("adam", &adam);
  m.def("zero_", &zero_);
  m.def("step_end", &step_end, py::arg("counters"), py::arg("ring_slot") = py::none(), py::arg("fstats") = py::none(),
        py::arg("istats") = py::none());
  m.def("sample_prologue", &sample_prologue);
  m.def("sampler_counters", &sampler_counters);
  m.def("peer_alloc", [](int64_t bytes) { return reinterpret_cast<int64_t>(grappa::peer::alloc(bytes)); });
  m.def("peer_free", [](int64_t p) { grappa::peer::release(reinterpret_cast<void*>(p)); });
  m.def("ipc_handle", [](int64_t p) { return py::bytes(grappa::peer::ipc_handle(reinterpret_cast<void*>(p))); });
  m.def("ipc_open", [](py::bytes h) { return reinterpret_cast<int64_t>(grappa::peer::ipc_open(std::string(h))); });
  m.def("ipc_close", [](int64_t p) { grappa::peer::ipc_close(reinterpret_cast<void*>(p)); });
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("pull_rows", &pull_rows, py::arg("tables"), py::arg("table_stride"), py::arg("elem_bytes"),
        py::arg("row_bytes"), py::arg("gids"), py::arg("n_dev"), py::arg("n"), py::arg("prefix"), py::arg("out"),
        py::arg("out_stride"), py::arg("out_row0"), py::arg("cap"), py::arg("err") = py::none());
  m.def("peer_copy", &peer_copy);
  m.def("a2a_pull", &a2a_pull, py::arg("src"), py::arg("src_off"), py::arg("len"), py::arg("dst_off"), py::arg("dst"),
        py::arg("first") = 0);
  m.def("peer_barrier", &peer_barrier);
  m.def("mark_ids", &mark_ids);
  m.def("iota_map", &iota_map);
  m.def("mark_compact", &mark_compact);
  m.def("mark_compact_scratch_words", [](int64_t n) { return grappa::peer::mark_compact_scratch_words(n); });
  m.def("csr_merge", &csr_merge, py::arg("indptr_a"), py::arg("indices_a"), py::arg("n_a"), py::arg("indptr_b"),
        py::arg("indices_b"), py::arg("n_b"), py::arg("map"), py::arg("indptr_out"), py::arg("indices_out"),
        py::arg("err"), py::arg("g0_a") = -1, py::arg("g0_b") = -1);
}
