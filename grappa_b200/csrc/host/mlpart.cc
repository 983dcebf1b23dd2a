// Multilevel k-way partitioner (see mlpart.h).
#include "mlpart.h"

#include <algorithm>
#include <memory>
#include <utility>
#ifdef _OPENMP
#include <parallel/algorithm>
#endif
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cmath>
#include <numeric>
#include <random>
#include <stdexcept>

namespace grappa {
namespace host {

namespace {

// A vector whose resize leaves new elements uninitialised: the big per-level arrays are
// written in full by parallel passes, which then also fault their pages in (a serial
// zero fill of ~2 GB per level took 7-8 s of each contraction on a 124M-edge graph).
template <typename T>
struct NoInitAlloc : std::allocator<T> {
  template <typename U>
  struct rebind {
    using other = NoInitAlloc<U>;
  };
  NoInitAlloc() = default;
  template <typename U>
  NoInitAlloc(const NoInitAlloc<U>&) {}
  template <typename U>
  void construct(U* p) noexcept {
    ::new (static_cast<void*>(p)) U;
  }
  template <typename U, typename... A>
  void construct(U* p, A&&... a) {
    ::new (static_cast<void*>(p)) U(std::forward<A>(a)...);
  }
};
using IVec = std::vector<int64_t, NoInitAlloc<int64_t>>;

// Weighted undirected graph in CSR form (both directions stored), two vertex weights.
struct WGraph {
  int64_t n = 0;
  std::vector<int64_t> xadj;
  IVec adj;
  IVec ew;   // edge weights
  std::vector<int64_t> vw0;  // vertex weight: vertices represented
  std::vector<int64_t> vw1;  // vertex weight: training vertices represented
};

// Symmetrised CSR of the input: both directions of every edge as one key u * n + v,
// a parallel sort, then per row the runs of equal keys become one edge weighted by the
// run length (rows in parallel; deterministic, since the sorted keys are).
WGraph build_input(int64_t n, const int64_t* u, const int64_t* v, int64_t m, const int8_t* train) {
  const uint64_t N = static_cast<uint64_t>(n);
  constexpr uint64_t kNone = ~0ull;  // self-loops: sorted past every real key and dropped
  std::vector<uint64_t, NoInitAlloc<uint64_t>> keys(static_cast<size_t>(2 * m));
  bool bad = false;
#pragma omp parallel for schedule(static) reduction(|| : bad)
  for (int64_t i = 0; i < m; ++i) {
    const int64_t a = u[i], b = v[i];
    if (a < 0 || b < 0 || a >= n || b >= n) {
      bad = true;
      continue;
    }
    const bool loop = a == b;
    keys[2 * i] = loop ? kNone : static_cast<uint64_t>(a) * N + static_cast<uint64_t>(b);
    keys[2 * i + 1] = loop ? kNone : static_cast<uint64_t>(b) * N + static_cast<uint64_t>(a);
  }
  if (bad) throw std::invalid_argument("edge endpoint out of range");
#ifdef _OPENMP
  __gnu_parallel::sort(keys.begin(), keys.end());
#else
  std::sort(keys.begin(), keys.end());
#endif
  const int64_t total = std::lower_bound(keys.begin(), keys.end(), kNone) - keys.begin();
  std::vector<int64_t> rs(static_cast<size_t>(n) + 1);
  rs[n] = total;
#pragma omp parallel for schedule(static)
  for (int64_t x = 0; x < n; ++x)
    rs[x] = std::lower_bound(keys.begin(), keys.begin() + total, static_cast<uint64_t>(x) * N) - keys.begin();
  std::vector<int64_t> runs(static_cast<size_t>(n) + 1, 0);
#pragma omp parallel for schedule(dynamic, 4096)
  for (int64_t x = 0; x < n; ++x) {
    int64_t r = 0;
    for (int64_t i = rs[x]; i < rs[x + 1]; ++i) r += (i == rs[x] || keys[i] != keys[i - 1]);
    runs[x + 1] = r;
  }
  WGraph g;
  g.n = n;
  g.xadj.assign(static_cast<size_t>(n) + 1, 0);
  for (int64_t x = 0; x < n; ++x) g.xadj[x + 1] = g.xadj[x] + runs[x + 1];
  g.adj.resize(static_cast<size_t>(g.xadj[n]));
  g.ew.resize(g.adj.size());
#pragma omp parallel for schedule(dynamic, 4096)
  for (int64_t x = 0; x < n; ++x) {
    int64_t o = g.xadj[x] - 1;
    for (int64_t i = rs[x]; i < rs[x + 1]; ++i) {
      if (i == rs[x] || keys[i] != keys[i - 1]) {
        ++o;
        g.adj[o] = static_cast<int64_t>(keys[i] % N);
        g.ew[o] = 1;
      } else {
        ++g.ew[o];
      }
    }
  }
  g.vw0.assign(static_cast<size_t>(n), 1);
  g.vw1.assign(static_cast<size_t>(n), 0);
  if (train)
    for (int64_t i = 0; i < n; ++i) g.vw1[i] = train[i] ? 1 : 0;
  return g;
}

// Heavy-edge matching: visit vertices in random order, match each unmatched vertex
// with its unmatched neighbour of the heaviest edge, as long as the pair stays within
// the coarse-vertex weight cap.  cmap[v] = coarse vertex id.  (Pairing the leftover
// vertices through a shared neighbour, as METIS does for power-law graphs, coarsened the
// RMAT graphs further but raised the final cut by 9-11 %, so it is not done.)
int64_t match(const WGraph& g, std::mt19937_64& rng, std::vector<int64_t>& cmap, int64_t max_vw) {
  std::vector<int64_t> order(static_cast<size_t>(g.n));
  std::iota(order.begin(), order.end(), 0);
  std::shuffle(order.begin(), order.end(), rng);
  std::vector<int64_t> mate(static_cast<size_t>(g.n), -1);
  for (int64_t v : order) {
    if (mate[v] >= 0) continue;
    int64_t best = -1, bw = -1;
    for (int64_t e = g.xadj[v]; e < g.xadj[v + 1]; ++e) {
      const int64_t w = g.adj[e];
      if (mate[w] >= 0 || w == v || g.vw0[v] + g.vw0[w] > max_vw) continue;
      if (g.ew[e] > bw) {
        bw = g.ew[e];
        best = w;
      }
    }
    if (best >= 0) {
      mate[v] = best;
      mate[best] = v;
    } else {
      mate[v] = v;
    }
  }
  cmap.assign(static_cast<size_t>(g.n), -1);
  int64_t nc = 0;
  for (int64_t v = 0; v < g.n; ++v) {
    if (cmap[v] >= 0) continue;
    cmap[v] = nc;
    cmap[mate[v]] = nc;
    ++nc;
  }
  return nc;
}

// Coarse graph: the members of every coarse vertex (a counting sort of cmap, fine ids
// ascending), then two passes over the coarse vertices in parallel, each thread with its
// own slot array: count the distinct coarse neighbours, then write them with summed
// weights in first-seen order (the order the serial construction gives).
WGraph contract(const WGraph& g, const std::vector<int64_t>& cmap, int64_t nc) {
  WGraph c;
  c.n = nc;
  c.vw0.assign(static_cast<size_t>(nc), 0);
  c.vw1.assign(static_cast<size_t>(nc), 0);
  std::vector<int64_t> mstart(static_cast<size_t>(nc) + 1, 0);
  for (int64_t v = 0; v < g.n; ++v) {
    c.vw0[cmap[v]] += g.vw0[v];
    c.vw1[cmap[v]] += g.vw1[v];
    ++mstart[cmap[v] + 1];
  }
  for (int64_t cv = 0; cv < nc; ++cv) mstart[cv + 1] += mstart[cv];
  std::vector<int64_t> members(static_cast<size_t>(g.n));
  {
    std::vector<int64_t> pos(mstart.begin(), mstart.end() - 1);
    for (int64_t v = 0; v < g.n; ++v) members[pos[cmap[v]]++] = v;
  }
  std::vector<int64_t> cdeg(static_cast<size_t>(nc) + 1, 0);
#pragma omp parallel
  {
    std::vector<int8_t> seen(static_cast<size_t>(nc), 0);
    std::vector<int64_t> list;
#pragma omp for schedule(dynamic, 256)
    for (int64_t cv = 0; cv < nc; ++cv) {
      list.clear();
      for (int64_t i = mstart[cv]; i < mstart[cv + 1]; ++i) {
        const int64_t v = members[i];
        for (int64_t e = g.xadj[v]; e < g.xadj[v + 1]; ++e) {
          const int64_t cw = cmap[g.adj[e]];
          if (cw != cv && !seen[cw]) {
            seen[cw] = 1;
            list.push_back(cw);
          }
        }
      }
      cdeg[cv + 1] = static_cast<int64_t>(list.size());
      for (int64_t cw : list) seen[cw] = 0;
    }
  }
  c.xadj.assign(static_cast<size_t>(nc) + 1, 0);
  for (int64_t cv = 0; cv < nc; ++cv) c.xadj[cv + 1] = c.xadj[cv] + cdeg[cv + 1];
  c.adj.resize(static_cast<size_t>(c.xadj[nc]));  // uninitialised: every entry is written below
  c.ew.resize(c.adj.size());
#pragma omp parallel
  {
    std::vector<int64_t> slot(static_cast<size_t>(nc), -1);
#pragma omp for schedule(dynamic, 256)
    for (int64_t cv = 0; cv < nc; ++cv) {
      int64_t o = c.xadj[cv];
      for (int64_t i = mstart[cv]; i < mstart[cv + 1]; ++i) {
        const int64_t v = members[i];
        for (int64_t e = g.xadj[v]; e < g.xadj[v + 1]; ++e) {
          const int64_t cw = cmap[g.adj[e]];
          if (cw == cv) continue;
          if (slot[cw] < 0) {
            slot[cw] = o;
            c.adj[o] = cw;
            c.ew[o++] = g.ew[e];
          } else {
            c.ew[slot[cw]] += g.ew[e];
          }
        }
      }
      for (int64_t j = c.xadj[cv]; j < o; ++j) slot[c.adj[j]] = -1;
    }
  }
  return c;
}

struct Balance {
  int64_t k;
  double cap0, cap1;  // maximum weight of a part, per type
  std::vector<int64_t> w0, w1;
  bool fits(int64_t p, int64_t a0, int64_t a1) const {
    return static_cast<double>(w0[p] + a0) <= cap0 && static_cast<double>(w1[p] + a1) <= cap1;
  }
};

Balance make_balance(const WGraph& g, int64_t k, double imb) {
  Balance b;
  b.k = k;
  int64_t t0 = 0, t1 = 0, m0 = 0, m1 = 0;
  for (int64_t v = 0; v < g.n; ++v) {
    t0 += g.vw0[v];
    t1 += g.vw1[v];
    m0 = std::max(m0, g.vw0[v]);
    m1 = std::max(m1, g.vw1[v]);
  }
  // even share plus the allowed excess, never below one heaviest vertex above the share
  b.cap0 = std::max((1.0 + imb) * t0 / k, static_cast<double>(t0) / k + m0);
  b.cap1 = std::max((1.0 + imb) * t1 / k, static_cast<double>(t1) / k + m1);
  b.w0.assign(static_cast<size_t>(k), 0);
  b.w1.assign(static_cast<size_t>(k), 0);
  return b;
}

// Greedy graph growing on the coarsest graph: parts are grown one at a time by BFS
// from a random unassigned vertex until they reach their share; leftovers go to the
// lightest part among their neighbours' (or the lightest overall).
std::vector<int64_t> initial_partition(const WGraph& g, int64_t k, double imb, std::mt19937_64& rng) {
  std::vector<int64_t> part(static_cast<size_t>(g.n), -1);
  Balance b = make_balance(g, k, imb);
  int64_t t0 = 0;
  for (int64_t v = 0; v < g.n; ++v) t0 += g.vw0[v];
  const double share0 = static_cast<double>(t0) / k;
  std::vector<int64_t> order(static_cast<size_t>(g.n));
  std::iota(order.begin(), order.end(), 0);
  std::shuffle(order.begin(), order.end(), rng);
  size_t next = 0;
  for (int64_t p = 0; p + 1 < k; ++p) {
    std::vector<int64_t> queue;
    size_t head = 0;
    while (static_cast<double>(b.w0[p]) < share0) {
      if (head == queue.size()) {
        while (next < order.size() && part[order[next]] >= 0) ++next;
        if (next == order.size()) break;
        queue.push_back(order[next++]);  // a start that does not fit is not retried
      }
      const int64_t v = queue[head++];
      if (part[v] >= 0) continue;
      if (!b.fits(p, g.vw0[v], g.vw1[v])) continue;
      part[v] = p;
      b.w0[p] += g.vw0[v];
      b.w1[p] += g.vw1[v];
      for (int64_t e = g.xadj[v]; e < g.xadj[v + 1]; ++e)
        if (part[g.adj[e]] < 0) queue.push_back(g.adj[e]);
    }
  }
  for (int64_t v : order) {
    if (part[v] >= 0) continue;
    int64_t best = k - 1;
    if (!b.fits(best, g.vw0[v], g.vw1[v])) {
      best = 0;
      for (int64_t p = 1; p < k; ++p)
        if (b.w0[p] < b.w0[best]) best = p;
    }
    part[v] = best;
    b.w0[best] += g.vw0[v];
    b.w1[best] += g.vw1[v];
  }
  return part;
}

// Greedy boundary refinement: a vertex moves to the part it is most connected to when
// that lowers the cut and both weights of the target stay within their caps.  The first
// pass visits every vertex; later passes only the boundary vertices of the pass before
// and the neighbours of vertices that moved (an interior vertex whose neighbours kept
// their parts cannot move).
void refine(const WGraph& g, std::vector<int64_t>& part, int64_t k, double imb, int passes, std::mt19937_64& rng) {
  Balance b = make_balance(g, k, imb);
  for (int64_t v = 0; v < g.n; ++v) {
    b.w0[part[v]] += g.vw0[v];
    b.w1[part[v]] += g.vw1[v];
  }
  std::vector<int64_t> conn(static_cast<size_t>(k), 0);
  std::vector<int64_t> touched;
  std::vector<int64_t> cand(static_cast<size_t>(g.n));
  std::iota(cand.begin(), cand.end(), 0);
  std::vector<int32_t> stamp(static_cast<size_t>(g.n), -1);
  std::vector<int64_t> next;
  for (int pass = 0; pass < passes && !cand.empty(); ++pass) {
    std::shuffle(cand.begin(), cand.end(), rng);
    next.clear();
    auto keep = [&](int64_t w) {
      if (stamp[w] != pass) {
        stamp[w] = pass;
        next.push_back(w);
      }
    };
    int64_t moved = 0;
    for (int64_t v : cand) {
      const int64_t pv = part[v];
      bool boundary = false;
      touched.clear();
      for (int64_t e = g.xadj[v]; e < g.xadj[v + 1]; ++e) {
        const int64_t q = part[g.adj[e]];
        if (conn[q] == 0) touched.push_back(q);
        conn[q] += g.ew[e];
        if (q != pv) boundary = true;
      }
      if (boundary) {
        int64_t best = pv, gain = 0;
        for (int64_t q : touched) {
          if (q == pv) continue;
          const int64_t gq = conn[q] - conn[pv];
          if (gq > gain && b.fits(q, g.vw0[v], g.vw1[v])) {
            gain = gq;
            best = q;
          }
        }
        if (best != pv) {
          part[v] = best;
          b.w0[pv] -= g.vw0[v];
          b.w1[pv] -= g.vw1[v];
          b.w0[best] += g.vw0[v];
          b.w1[best] += g.vw1[v];
          ++moved;
          for (int64_t e = g.xadj[v]; e < g.xadj[v + 1]; ++e) keep(g.adj[e]);
        }
        keep(v);
      }
      for (int64_t q : touched) conn[q] = 0;
    }
    if (moved == 0) break;
    cand.swap(next);
  }
}

}  // namespace

std::vector<int64_t> multilevel_partition(int64_t n, const int64_t* u, const int64_t* v, int64_t m,
                                          const int8_t* train, const MlPartOptions& opt) {
  const int64_t k = opt.n_parts;
  if (k < 1) throw std::invalid_argument("n_parts must be >= 1");
  if (k == 1 || n == 0) return std::vector<int64_t>(static_cast<size_t>(n), 0);
  std::mt19937_64 rng(opt.seed ^ 0x5EEDull);
  // GRAPPA_MLPART_VERBOSE=1: per-phase seconds on stderr
  const bool verbose = std::getenv("GRAPPA_MLPART_VERBOSE") && std::getenv("GRAPPA_MLPART_VERBOSE")[0] == '1';
  auto t_last = std::chrono::steady_clock::now();
  auto lap = [&](const char* what, int64_t nv, int64_t ne) {
    if (!verbose) return;
    const auto now = std::chrono::steady_clock::now();
    std::fprintf(stderr, "mlpart %-10s n=%lld adj=%lld %.2f s\n", what, static_cast<long long>(nv),
                 static_cast<long long>(ne), std::chrono::duration<double>(now - t_last).count());
    t_last = now;
  };
  const int64_t stop = opt.coarsest > 0 ? opt.coarsest : std::max<int64_t>(2000, 40 * k);
  std::vector<WGraph> levels;
  std::vector<std::vector<int64_t>> maps;
  levels.push_back(build_input(n, u, v, m, train));
  lap("input", levels.back().n, static_cast<int64_t>(levels.back().adj.size()));
  // no coarse vertex heavier than 1.5x the average vertex of the target coarsest graph
  const int64_t max_vw = std::max<int64_t>(2, (3 * n) / (2 * stop));
  while (levels.back().n > stop) {
    std::vector<int64_t> cmap;
    const int64_t nc = match(levels.back(), rng, cmap, max_vw);
    lap("match", levels.back().n, static_cast<int64_t>(levels.back().adj.size()));
    if (nc > static_cast<int64_t>(0.95 * static_cast<double>(levels.back().n))) break;  // no longer shrinking
    WGraph c = contract(levels.back(), cmap, nc);
    lap("contract", c.n, static_cast<int64_t>(c.adj.size()));
    maps.push_back(std::move(cmap));
    levels.push_back(std::move(c));
  }
  // several greedy-growing starts on the coarsest graph, run in parallel, each with its
  // own generator seeded in order from the run's; the lowest cut wins (the first on ties)
  const WGraph& cg = levels.back();
  constexpr int kStarts = 8;
  std::vector<uint64_t> seeds(kStarts);
  for (auto& sd : seeds) sd = rng();
  std::vector<std::vector<int64_t>> cand(kStarts);
  std::vector<int64_t> cuts(kStarts, 0);
#pragma omp parallel for schedule(dynamic, 1)
  for (int t = 0; t < kStarts; ++t) {
    std::mt19937_64 r(seeds[t]);
    std::vector<int64_t> p = initial_partition(cg, k, opt.imbalance, r);
    refine(cg, p, k, opt.imbalance, opt.refine_passes * 2, r);
    int64_t cut = 0;
    for (int64_t x = 0; x < cg.n; ++x)
      for (int64_t e = cg.xadj[x]; e < cg.xadj[x + 1]; ++e) cut += p[x] != p[cg.adj[e]] ? cg.ew[e] : 0;
    cuts[t] = cut;
    cand[t] = std::move(p);
  }
  const int best = static_cast<int>(std::min_element(cuts.begin(), cuts.end()) - cuts.begin());
  std::vector<int64_t> part = std::move(cand[best]);
  std::vector<std::vector<int64_t>>().swap(cand);
  lap("initial", cg.n, static_cast<int64_t>(cg.adj.size()));
  for (int64_t lvl = static_cast<int64_t>(levels.size()) - 2; lvl >= 0; --lvl) {
    const std::vector<int64_t>& cmap = maps[lvl];
    std::vector<int64_t> fine(static_cast<size_t>(levels[lvl].n));
    for (int64_t x = 0; x < levels[lvl].n; ++x) fine[x] = part[cmap[x]];
    part = std::move(fine);
    refine(levels[lvl], part, k, opt.imbalance, opt.refine_passes, rng);
    lap("refine", levels[lvl].n, static_cast<int64_t>(levels[lvl].adj.size()));
  }
  return part;
}

int64_t edge_cut(int64_t n, const int64_t* u, const int64_t* v, int64_t m, const int64_t* part) {
  std::vector<std::pair<int64_t, int64_t>> e;
  e.reserve(static_cast<size_t>(m));
  for (int64_t i = 0; i < m; ++i) {
    if (u[i] == v[i] || u[i] < 0 || v[i] < 0 || u[i] >= n || v[i] >= n) continue;
    e.emplace_back(std::min(u[i], v[i]), std::max(u[i], v[i]));
  }
  std::sort(e.begin(), e.end());
  e.erase(std::unique(e.begin(), e.end()), e.end());
  int64_t cut = 0;
  for (const auto& p : e) cut += part[p.first] != part[p.second];
  return cut;
}

}  // namespace host
}  // namespace grappa
