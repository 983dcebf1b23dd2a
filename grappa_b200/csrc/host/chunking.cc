#include "chunking.h"

#include <cstdio>
#include <stdexcept>

namespace grappa {
namespace host {

namespace {

template <typename T>
void write_file(const std::string& name, const T* data, size_t n) {
  FILE* f = std::fopen(name.c_str(), "wb");
  if (!f) throw std::runtime_error("cannot open " + name + " for writing");
  const size_t w = n ? std::fwrite(data, sizeof(T), n, f) : 0;
  std::fclose(f);
  if (w != n) throw std::runtime_error("short write to " + name);
}

template <typename T>
std::vector<T> read_file(const std::string& name) {
  FILE* f = std::fopen(name.c_str(), "rb");
  if (!f) throw std::runtime_error("cannot open " + name);
  std::fseek(f, 0, SEEK_END);
  const long bytes = std::ftell(f);
  std::fseek(f, 0, SEEK_SET);
  std::vector<T> v(static_cast<size_t>(bytes) / sizeof(T));
  const size_t r = v.empty() ? 0 : std::fread(v.data(), sizeof(T), v.size(), f);
  std::fclose(f);
  if (r != v.size()) throw std::runtime_error("short read from " + name);
  return v;
}

std::string pfile(const std::string& path, int64_t i, const char* ext) {
  return path + "/p" + std::to_string(i) + "." + ext + ".bin";
}

}  // namespace

ChunkStats chunk_build(const std::string& path, int64_t n_n, int64_t n_e, int64_t n_part,
                       const int64_t* src, const int64_t* dst, const int64_t* nid2pid) {
  if (n_part <= 0) throw std::invalid_argument("n_part must be positive");
  ChunkStats st;
  st.part_nodes.assign(n_part, 0);
  st.part_edges.assign(n_part, 0);
  st.bridge_edges.assign(n_part * n_part, 0);
  std::vector<int64_t> lid(n_n);
  std::vector<std::vector<int64_t>> oid(n_part);
  for (int64_t v = 0; v < n_n; ++v) {
    const int64_t p = nid2pid[v];
    if (p < 0 || p >= n_part) throw std::out_of_range("nid2pid out of range");
    lid[v] = st.part_nodes[p]++;
    oid[p].push_back(v);
  }
  std::vector<int64_t> ideg(n_n, 0);
  std::vector<std::vector<int64_t>> pu(n_part), pv(n_part);
  std::vector<std::vector<int64_t>> bu(n_part * n_part), bv(n_part * n_part);
  for (int64_t i = 0; i < n_e; ++i) {
    const int64_t u = src[i], v = dst[i];
    if (u < 0 || u >= n_n || v < 0 || v >= n_n) throw std::out_of_range("edge id out of range");
    ideg[v]++;
    if (u == v) continue;
    const int64_t a = nid2pid[u], b = nid2pid[v];
    if (a == b) {
      pu[a].push_back(lid[u]);
      pv[a].push_back(lid[v]);
    } else {
      bu[a * n_part + b].push_back(lid[u]);
      bv[a * n_part + b].push_back(lid[v]);
    }
  }
  for (int64_t p = 0; p < n_part; ++p) {
    for (int64_t l = 0; l < st.part_nodes[p]; ++l) {
      pu[p].push_back(l);
      pv[p].push_back(l);
    }
    st.part_edges[p] = static_cast<int64_t>(pu[p].size());
    write_file(pfile(path, p, "u"), pu[p].data(), pu[p].size());
    write_file(pfile(path, p, "v"), pv[p].data(), pv[p].size());
    write_file(pfile(path, p, "oid"), oid[p].data(), oid[p].size());
    std::vector<int64_t> pideg(oid[p].size());
    for (size_t l = 0; l < oid[p].size(); ++l) pideg[l] = ideg[oid[p][l]];
    write_file(pfile(path, p, "ideg"), pideg.data(), pideg.size());
    for (int64_t q = 0; q < n_part; ++q) {
      if (q == p) continue;
      auto& U = bu[p * n_part + q];
      auto& V = bv[p * n_part + q];
      st.bridge_edges[p * n_part + q] = static_cast<int64_t>(U.size());
      if (U.empty()) continue;
      const std::string base = path + "/b" + std::to_string(p) + "_" + std::to_string(q);
      write_file(base + ".u.bin", U.data(), U.size());
      write_file(base + ".v.bin", V.data(), V.size());
    }
  }
  return st;
}

void chunk_split_node_feat(const std::string& path, int64_t n_n, int64_t dim, int64_t n_part,
                           const float* feat) {
  for (int64_t p = 0; p < n_part; ++p) {
    auto oid = read_file<int64_t>(pfile(path, p, "oid"));
    std::vector<float> out(oid.size() * dim);
    for (size_t l = 0; l < oid.size(); ++l) {
      if (oid[l] < 0 || oid[l] >= n_n) throw std::out_of_range("oid out of range");
      std::copy(feat + oid[l] * dim, feat + (oid[l] + 1) * dim, out.begin() + l * dim);
    }
    write_file(pfile(path, p, "nfeat"), out.data(), out.size());
  }
}

void chunk_split_node_data(const std::string& path, int64_t n_n, int64_t n_part,
                           const float* label, const int8_t* train, const int8_t* valid,
                           const int8_t* test) {
  for (int64_t p = 0; p < n_part; ++p) {
    auto oid = read_file<int64_t>(pfile(path, p, "oid"));
    const size_t n = oid.size();
    std::vector<float> lab(n);
    std::vector<int8_t> tr(n), va(n), te(n);
    for (size_t l = 0; l < n; ++l) {
      const int64_t g = oid[l];
      if (g < 0 || g >= n_n) throw std::out_of_range("oid out of range");
      lab[l] = label[g];
      tr[l] = train[g];
      va[l] = valid[g];
      te[l] = test[g];
    }
    write_file(pfile(path, p, "label"), lab.data(), n);
    write_file(pfile(path, p, "train"), tr.data(), n);
    write_file(pfile(path, p, "valid"), va.data(), n);
    write_file(pfile(path, p, "test"), te.data(), n);
  }
}

}  // namespace host
}  // namespace grappa
