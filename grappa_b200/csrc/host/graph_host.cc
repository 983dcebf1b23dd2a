#include "graph_host.h"

#ifdef _OPENMP
#include <omp.h>
#endif

#include <algorithm>
#include <cstdint>
#include <cmath>
#include <numeric>
#include <stdexcept>

#include "grappa/rng.h"

namespace grappa {
namespace host {

CSC build_csc(const int64_t* u, const int64_t* v, int64_t n_e, int64_t n_nodes) {
  CSC g;
  if (n_nodes < 0) {
    int64_t mx = -1;
#pragma omp parallel for reduction(max : mx)
    for (int64_t i = 0; i < n_e; ++i) mx = std::max(mx, std::max(u[i], v[i]));
    n_nodes = mx + 1;
  }
  g.n_nodes = n_nodes;
  std::vector<int64_t> cnt(n_nodes + 1, 0);
  // degree histogram (atomic adds keep this simple and parallel)
#pragma omp parallel for
  for (int64_t i = 0; i < n_e; ++i) {
    if (v[i] < 0 || v[i] >= n_nodes || u[i] < 0 || u[i] >= n_nodes) continue;
#pragma omp atomic
    cnt[v[i] + 1]++;
  }
  for (int64_t i = 0; i < n_nodes; ++i) cnt[i + 1] += cnt[i];
  std::vector<int64_t> raw(cnt[n_nodes]);
  std::vector<int64_t> fill(cnt.begin(), cnt.end() - 1);
  // scatter; the order inside a segment is fixed afterwards by the sort
#pragma omp parallel for
  for (int64_t i = 0; i < n_e; ++i) {
    if (v[i] < 0 || v[i] >= n_nodes || u[i] < 0 || u[i] >= n_nodes) continue;
    int64_t pos;
#pragma omp atomic capture
    pos = fill[v[i]]++;
    raw[pos] = u[i];
  }
  std::vector<int64_t> deg(n_nodes, 0);
#pragma omp parallel for schedule(dynamic, 1024)
  for (int64_t d = 0; d < n_nodes; ++d) {
    auto b = raw.begin() + cnt[d], e = raw.begin() + cnt[d + 1];
    std::sort(b, e);
    deg[d] = std::unique(b, e) - b;
  }
  g.indptr.assign(n_nodes + 1, 0);
  for (int64_t d = 0; d < n_nodes; ++d) g.indptr[d + 1] = g.indptr[d] + deg[d];
  g.n_edges = g.indptr[n_nodes];
  g.indices.resize(g.n_edges);
#pragma omp parallel for schedule(dynamic, 1024)
  for (int64_t d = 0; d < n_nodes; ++d)
    std::copy(raw.begin() + cnt[d], raw.begin() + cnt[d] + deg[d], g.indices.begin() + g.indptr[d]);
  return g;
}

void pick_offsets(uint64_t key, uint64_t nid, uint32_t d, uint32_t k, int64_t* out) {
  uint32_t acc = 0;
  for (uint32_t t = 0; t < kMaxDraws && acc < k; ++t) {
    const int64_t o = draw_below(node_draw(key, nid, t), d);
    bool seen = false;
    for (uint32_t j = 0; j < acc; ++j)
      if (out[j] == o) {
        seen = true;
        break;
      }
    if (!seen) out[acc++] = o;
  }
  for (int64_t o = 0; o < static_cast<int64_t>(d) && acc < k; ++o) {
    bool seen = false;
    for (uint32_t j = 0; j < acc; ++j)
      if (out[j] == o) {
        seen = true;
        break;
      }
    if (!seen) out[acc++] = o;
  }
}

namespace {

// Global id -> local id during compaction: open addressing with linear probing in a
// power-of-two table at most half full (std::unordered_map's node allocations made the
// compaction the larger part of a host sampling step).
class IdMap {
 public:
  static constexpr int64_t kEmpty = INT64_MIN;
  explicit IdMap(int64_t expected) {
    size_t cap = 16;
    while (cap < static_cast<size_t>(2 * expected)) cap <<= 1;
    keys_.assign(cap, kEmpty);
    vals_.resize(cap);
    mask_ = cap - 1;
  }
  // the value of key; when absent, key is inserted with value v (first insert wins)
  int64_t find_or_insert(int64_t key, int64_t v, bool* inserted) {
    size_t h = static_cast<size_t>(grappa::mix64(static_cast<uint64_t>(key))) & mask_;
    while (true) {
      if (keys_[h] == key) {
        *inserted = false;
        return vals_[h];
      }
      if (keys_[h] == kEmpty) {
        keys_[h] = key;
        vals_[h] = v;
        *inserted = true;
        return v;
      }
      h = (h + 1) & mask_;
    }
  }

 private:
  std::vector<int64_t> keys_, vals_;
  size_t mask_ = 0;
};

}  // namespace

Block sample_hop(const CSC& g, const int64_t* dst_nid, const uint8_t* frontier, int64_t n_dst,
                 int64_t fanout, uint64_t key, const int64_t* gideg, double* cov_sum,
                 double* cov_n) {
  Block b;
  b.n_dst = n_dst;
  b.indptr.assign(n_dst + 1, 0);
  std::vector<int64_t> pick(n_dst, 0);
  double csum = 0.0, cn = 0.0;
#pragma omp parallel for reduction(+ : csum, cn)
  for (int64_t i = 0; i < n_dst; ++i) {
    const int64_t nid = dst_nid[i];
    if (frontier && !frontier[i]) continue;
    if (nid < 0 || nid >= g.n_nodes) continue;
    const int64_t d = g.degree(nid);
    pick[i] = (fanout < 0 || d <= fanout) ? d : fanout;
    if (gideg) {
      csum += coverage_ratio(d, gideg[i]);
      cn += 1.0;
    }
  }
  if (cov_sum) *cov_sum += csum;
  if (cov_n) *cov_n += cn;
  for (int64_t i = 0; i < n_dst; ++i) b.indptr[i + 1] = b.indptr[i] + pick[i];
  const int64_t n_e = b.indptr[n_dst];
  std::vector<int64_t> nbr(n_e);
#pragma omp parallel for schedule(dynamic, 64)
  for (int64_t i = 0; i < n_dst; ++i) {
    const int64_t k = pick[i];
    if (k == 0) continue;
    const int64_t nid = dst_nid[i];
    const int64_t d = g.degree(nid);
    const int64_t* nb = g.indices.data() + g.indptr[nid];
    int64_t* o = nbr.data() + b.indptr[i];
    if (k == d) {
      for (int64_t j = 0; j < d; ++j) o[j] = nb[j];
    } else {
      pick_offsets(key, static_cast<uint64_t>(nid), static_cast<uint32_t>(d), static_cast<uint32_t>(k), o);
      for (int64_t j = 0; j < k; ++j) o[j] = nb[o[j]];
    }
  }
  // compaction: dst nodes first, then new sources by first appearance
  IdMap lid(n_dst + n_e);
  b.src_nid.assign(dst_nid, dst_nid + n_dst);
  b.src_nid.reserve(static_cast<size_t>(n_dst + n_e));
  bool inserted;
  for (int64_t i = 0; i < n_dst; ++i) lid.find_or_insert(dst_nid[i], i, &inserted);
  b.indices.resize(n_e);
  for (int64_t j = 0; j < n_e; ++j) {
    const int64_t next = static_cast<int64_t>(b.src_nid.size());
    const int64_t id = lid.find_or_insert(nbr[j], next, &inserted);
    if (inserted) b.src_nid.push_back(nbr[j]);
    b.indices[j] = id;
  }
  b.n_src = static_cast<int64_t>(b.src_nid.size());
  b.src_sampled.assign(b.n_src, 0);
  for (int64_t j = 0; j < n_e; ++j) b.src_sampled[b.indices[j]] = 1;
  return b;
}

Block random_walk_topk(const CSC& g, const int64_t* seeds, int64_t n_seeds, int length,
                       double restart_prob, int num_walks, int num_neighbors, uint64_t key,
                       std::vector<float>* weights) {
  const uint32_t thr = restart_prob >= 1.0 ? 0xFFFFFFFFu : static_cast<uint32_t>(restart_prob * 4294967296.0);
  std::vector<std::vector<std::pair<int64_t, int64_t>>> top(n_seeds);
#pragma omp parallel for schedule(dynamic, 16)
  for (int64_t i = 0; i < n_seeds; ++i) {
    std::vector<int64_t> visits;
    visits.reserve(static_cast<size_t>(num_walks) * length);
    const int64_t s0 = seeds[i];
    for (int j = 0; j < num_walks; ++j) {
      int64_t cur = s0;
      const uint64_t w = static_cast<uint64_t>(i) * num_walks + j;
      for (int t = 0; t < length; ++t) {
        if (cur < 0 || cur >= g.n_nodes) break;
        const U4 r = index_draw4(key, w, static_cast<uint32_t>(t));
        if (r.x < thr) break;
        const int64_t d = g.degree(cur);
        if (d == 0) break;
        cur = g.indices[g.indptr[cur] + draw_below(r.y, static_cast<uint32_t>(d))];
        visits.push_back(cur);
      }
    }
    std::sort(visits.begin(), visits.end());
    auto& tp = top[i];
    for (size_t a = 0; a < visits.size();) {
      size_t b = a;
      while (b < visits.size() && visits[b] == visits[a]) ++b;
      tp.emplace_back(static_cast<int64_t>(b - a), visits[a]);
      a = b;
    }
    // most visited first; ties by smaller id (ids are ascending already)
    std::stable_sort(tp.begin(), tp.end(), [](const auto& x, const auto& y) { return x.first > y.first; });
    if (static_cast<int64_t>(tp.size()) > num_neighbors) tp.resize(num_neighbors);
  }
  Block b;
  b.n_dst = n_seeds;
  b.indptr.assign(n_seeds + 1, 0);
  for (int64_t i = 0; i < n_seeds; ++i) b.indptr[i + 1] = b.indptr[i] + static_cast<int64_t>(top[i].size());
  const int64_t n_e = b.indptr[n_seeds];
  IdMap lid(n_seeds + n_e);
  b.src_nid.assign(seeds, seeds + n_seeds);
  bool inserted;
  for (int64_t i = 0; i < n_seeds; ++i) lid.find_or_insert(seeds[i], i, &inserted);
  b.indices.resize(n_e);
  if (weights) weights->resize(n_e);
  for (int64_t i = 0; i < n_seeds; ++i)
    for (size_t k = 0; k < top[i].size(); ++k) {
      const int64_t e = b.indptr[i] + static_cast<int64_t>(k);
      const int64_t nid = top[i][k].second;
      const int64_t id = lid.find_or_insert(nid, static_cast<int64_t>(b.src_nid.size()), &inserted);
      if (inserted) b.src_nid.push_back(nid);
      b.indices[e] = id;
      if (weights) (*weights)[e] = static_cast<float>(top[i][k].first);
    }
  b.n_src = static_cast<int64_t>(b.src_nid.size());
  b.src_sampled.assign(b.n_src, 0);
  for (int64_t j = 0; j < n_e; ++j) b.src_sampled[b.indices[j]] = 1;
  return b;
}

void rmat_candidates(int64_t n, int scale, double a, double b, double c, uint64_t seed,
                     int64_t e_begin, int64_t e_end, int64_t* keys) {
  const uint64_t ta = static_cast<uint64_t>(a * 4294967296.0);
  const uint64_t tb = static_cast<uint64_t>((a + b) * 4294967296.0);
  const uint64_t tc = static_cast<uint64_t>((a + b + c) * 4294967296.0);
  const uint64_t key = mix64(seed ^ 0x524D4154ull);
#pragma omp parallel for schedule(static)
  for (int64_t e = e_begin; e < e_end; ++e) {
    uint64_t u = 0, v = 0;
    U4 r{0, 0, 0, 0};
    for (int l = 0; l < scale; ++l) {
      if ((l & 3) == 0) r = index_draw4(key, static_cast<uint64_t>(e), static_cast<uint32_t>(l >> 2));
      const uint64_t x = u4_word(r, l & 3);
      const uint64_t bu = (x >= tb) ? 1u : 0u;
      const uint64_t bv = (x >= ta && x < tb) || (x >= tc) ? 1u : 0u;
      u = (u << 1) | bu;
      v = (v << 1) | bv;
    }
    int64_t out = -1;
    if (u < static_cast<uint64_t>(n) && v < static_cast<uint64_t>(n) && u != v) {
      const uint64_t lo = std::min(u, v), hi = std::max(u, v);
      out = static_cast<int64_t>(lo * static_cast<uint64_t>(n) + hi);
    }
    keys[e - e_begin] = out;
  }
}

void shuffle_keys(const int64_t* ids, int64_t n, uint64_t seed, uint64_t epoch, int64_t* keys) {
  const uint64_t k = mix64(mix64(seed ^ 0x5348554646ull) ^ epoch);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i)
    keys[i] = static_cast<int64_t>(mix64(static_cast<uint64_t>(ids[i]) ^ k) >> 1);
}

}  // namespace host
}  // namespace grappa
