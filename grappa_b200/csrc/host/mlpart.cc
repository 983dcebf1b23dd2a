// Multilevel k-way partitioner (see mlpart.h).
#include "mlpart.h"

#include <algorithm>
#include <cmath>
#include <numeric>
#include <random>
#include <stdexcept>

namespace grappa {
namespace host {

namespace {

// Weighted undirected graph in CSR form (both directions stored), two vertex weights.
struct WGraph {
  int64_t n = 0;
  std::vector<int64_t> xadj;
  std::vector<int64_t> adj;
  std::vector<int64_t> ew;   // edge weights
  std::vector<int64_t> vw0;  // vertex weight: vertices represented
  std::vector<int64_t> vw1;  // vertex weight: training vertices represented
};

WGraph build_input(int64_t n, const int64_t* u, const int64_t* v, int64_t m, const int8_t* train) {
  // symmetrise, drop self-loops, merge duplicates (weight = multiplicity of the pair)
  std::vector<std::pair<int64_t, int64_t>> e;
  e.reserve(static_cast<size_t>(2 * m));
  for (int64_t i = 0; i < m; ++i) {
    const int64_t a = u[i], b = v[i];
    if (a == b) continue;
    if (a < 0 || b < 0 || a >= n || b >= n) throw std::invalid_argument("edge endpoint out of range");
    e.emplace_back(a, b);
    e.emplace_back(b, a);
  }
  std::sort(e.begin(), e.end());
  WGraph g;
  g.n = n;
  g.xadj.assign(static_cast<size_t>(n + 1), 0);
  for (size_t i = 0; i < e.size(); ++i) {
    if (i > 0 && e[i] == e[i - 1]) {
      continue;
    }
    ++g.xadj[static_cast<size_t>(e[i].first + 1)];
  }
  for (int64_t i = 0; i < n; ++i) g.xadj[i + 1] += g.xadj[i];
  g.adj.resize(static_cast<size_t>(g.xadj[n]));
  g.ew.resize(g.adj.size());
  int64_t k = -1;
  for (size_t i = 0; i < e.size(); ++i) {
    if (i > 0 && e[i] == e[i - 1]) {
      ++g.ew[static_cast<size_t>(k)];
      continue;
    }
    ++k;
    g.adj[static_cast<size_t>(k)] = e[i].second;
    g.ew[static_cast<size_t>(k)] = 1;
  }
  g.vw0.assign(static_cast<size_t>(n), 1);
  g.vw1.assign(static_cast<size_t>(n), 0);
  if (train)
    for (int64_t i = 0; i < n; ++i) g.vw1[i] = train[i] ? 1 : 0;
  return g;
}

// Heavy-edge matching: visit vertices in random order, match each unmatched vertex
// with its unmatched neighbour of the heaviest edge.  cmap[v] = coarse vertex id.
int64_t match(const WGraph& g, std::mt19937_64& rng, std::vector<int64_t>& cmap) {
  std::vector<int64_t> order(static_cast<size_t>(g.n));
  std::iota(order.begin(), order.end(), 0);
  std::shuffle(order.begin(), order.end(), rng);
  std::vector<int64_t> mate(static_cast<size_t>(g.n), -1);
  for (int64_t v : order) {
    if (mate[v] >= 0) continue;
    int64_t best = -1, bw = -1;
    for (int64_t e = g.xadj[v]; e < g.xadj[v + 1]; ++e) {
      const int64_t w = g.adj[e];
      if (mate[w] >= 0 || w == v) continue;
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

WGraph contract(const WGraph& g, const std::vector<int64_t>& cmap, int64_t nc) {
  WGraph c;
  c.n = nc;
  c.vw0.assign(static_cast<size_t>(nc), 0);
  c.vw1.assign(static_cast<size_t>(nc), 0);
  std::vector<std::vector<int64_t>> members(static_cast<size_t>(nc));
  for (int64_t v = 0; v < g.n; ++v) {
    c.vw0[cmap[v]] += g.vw0[v];
    c.vw1[cmap[v]] += g.vw1[v];
    members[cmap[v]].push_back(v);
  }
  c.xadj.assign(static_cast<size_t>(nc + 1), 0);
  std::vector<int64_t> slot(static_cast<size_t>(nc), -1);
  std::vector<int64_t> nbr, wt;
  for (int64_t cv = 0; cv < nc; ++cv) {
    const size_t start = nbr.size();
    for (int64_t v : members[cv])
      for (int64_t e = g.xadj[v]; e < g.xadj[v + 1]; ++e) {
        const int64_t cw = cmap[g.adj[e]];
        if (cw == cv) continue;
        if (slot[cw] < 0) {
          slot[cw] = static_cast<int64_t>(nbr.size());
          nbr.push_back(cw);
          wt.push_back(0);
        }
        wt[slot[cw]] += g.ew[e];
      }
    for (size_t i = start; i < nbr.size(); ++i) slot[nbr[i]] = -1;
    c.xadj[cv + 1] = static_cast<int64_t>(nbr.size());
  }
  c.adj = std::move(nbr);
  c.ew = std::move(wt);
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
// that lowers the cut and both weights of the target stay within their caps.
void refine(const WGraph& g, std::vector<int64_t>& part, int64_t k, double imb, int passes, std::mt19937_64& rng) {
  Balance b = make_balance(g, k, imb);
  for (int64_t v = 0; v < g.n; ++v) {
    b.w0[part[v]] += g.vw0[v];
    b.w1[part[v]] += g.vw1[v];
  }
  std::vector<int64_t> conn(static_cast<size_t>(k), 0);
  std::vector<int64_t> touched;
  std::vector<int64_t> order(static_cast<size_t>(g.n));
  std::iota(order.begin(), order.end(), 0);
  for (int pass = 0; pass < passes; ++pass) {
    std::shuffle(order.begin(), order.end(), rng);
    int64_t moved = 0;
    for (int64_t v : order) {
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
        }
      }
      for (int64_t q : touched) conn[q] = 0;
    }
    if (moved == 0) break;
  }
}

}  // namespace

std::vector<int64_t> multilevel_partition(int64_t n, const int64_t* u, const int64_t* v, int64_t m,
                                          const int8_t* train, const MlPartOptions& opt) {
  const int64_t k = opt.n_parts;
  if (k < 1) throw std::invalid_argument("n_parts must be >= 1");
  if (k == 1 || n == 0) return std::vector<int64_t>(static_cast<size_t>(n), 0);
  std::mt19937_64 rng(opt.seed ^ 0x5EEDull);
  const int64_t stop = opt.coarsest > 0 ? opt.coarsest : std::max<int64_t>(2000, 40 * k);
  std::vector<WGraph> levels;
  std::vector<std::vector<int64_t>> maps;
  levels.push_back(build_input(n, u, v, m, train));
  while (levels.back().n > stop) {
    std::vector<int64_t> cmap;
    const int64_t nc = match(levels.back(), rng, cmap);
    if (nc > static_cast<int64_t>(0.95 * static_cast<double>(levels.back().n))) break;  // no longer shrinking
    WGraph c = contract(levels.back(), cmap, nc);
    maps.push_back(std::move(cmap));
    levels.push_back(std::move(c));
  }
  // several greedy-growing starts on the coarsest graph; keep the lowest cut
  std::vector<int64_t> part;
  int64_t best_cut = -1;
  const WGraph& cg = levels.back();
  for (int t = 0; t < 8; ++t) {
    std::vector<int64_t> p = initial_partition(cg, k, opt.imbalance, rng);
    refine(cg, p, k, opt.imbalance, opt.refine_passes * 2, rng);
    int64_t cut = 0;
    for (int64_t x = 0; x < cg.n; ++x)
      for (int64_t e = cg.xadj[x]; e < cg.xadj[x + 1]; ++e) cut += p[x] != p[cg.adj[e]] ? cg.ew[e] : 0;
    if (best_cut < 0 || cut < best_cut) {
      best_cut = cut;
      part = std::move(p);
    }
  }
  for (int64_t lvl = static_cast<int64_t>(levels.size()) - 2; lvl >= 0; --lvl) {
    const std::vector<int64_t>& cmap = maps[lvl];
    std::vector<int64_t> fine(static_cast<size_t>(levels[lvl].n));
    for (int64_t x = 0; x < levels[lvl].n; ++x) fine[x] = part[cmap[x]];
    part = std::move(fine);
    refine(levels[lvl], part, k, opt.imbalance, opt.refine_passes, rng);
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
