#include "xborder.h"

#ifdef _OPENMP
#include <omp.h>
#endif

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>

namespace grappa {
namespace host {

XBorder::XBorder(int64_t rank, int64_t n_part, std::vector<int64_t> prefix_sum)
    : rank_(rank), n_part_(n_part), nbr_idx_(rank), prefix_sum_(std::move(prefix_sum)) {
  if (static_cast<int64_t>(prefix_sum_.size()) != n_part_ + 1)
    throw std::invalid_argument("XBorder: prefix_sum must have n_part + 1 entries");
  gid_lid_.resize(n_part_);
}

int64_t XBorder::owner(int64_t gid) const {
  auto it = std::upper_bound(prefix_sum_.begin(), prefix_sum_.end(), gid);
  const int64_t p = static_cast<int64_t>(it - prefix_sum_.begin()) - 1;
  return (p < 0 || p >= n_part_) ? -1 : p;
}

void XBorder::mask_by_partition(const int64_t* ids, int64_t n, int8_t* mask) const {
  std::memset(mask, 0, static_cast<size_t>(n_part_ * n));
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const int64_t p = owner(ids[i]);
    if (p >= 0) mask[p * n + i] = 1;
  }
}

std::vector<std::vector<int64_t>> XBorder::group_by_partition(const int64_t* ids, int64_t n,
                                                              int8_t* mask) const {
  if (mask) mask_by_partition(ids, n, mask);
  std::vector<std::vector<int64_t>> out(n_part_);
#ifdef _OPENMP
  const int nt = omp_get_max_threads();
#else
  const int nt = 1;
#endif
  std::vector<std::vector<std::vector<int64_t>>> local(nt, std::vector<std::vector<int64_t>>(n_part_));
#pragma omp parallel
  {
#ifdef _OPENMP
    const int t = omp_get_thread_num();
    const int T = omp_get_num_threads();
#else
    const int t = 0, T = 1;
#endif
    const int64_t len = (n + T - 1) / T;
    const int64_t b = std::min(n, t * len), e = std::min(n, b + len);
    for (int64_t i = b; i < e; ++i) {
      const int64_t p = owner(ids[i]);
      if (p >= 0) local[t][p].push_back(ids[i]);
    }
  }
  for (int64_t p = 0; p < n_part_; ++p)
    for (int t = 0; t < nt; ++t) out[p].insert(out[p].end(), local[t][p].begin(), local[t][p].end());
  return out;
}

void XBorder::ad_hoc_clear() {
  for (auto& m : gid_lid_) m.clear();
}

void XBorder::ad_hoc_build_id_mapping(int64_t pid, const int64_t* gids, int64_t n) {
  if (pid == rank_ || pid == nbr_idx_) return;
  auto& m = gid_lid_.at(pid);
  m.reserve(m.size() + n);
  for (int64_t i = 0; i < n; ++i) m[gids[i]] = i;
}

bool XBorder::resolve(int64_t gid, int64_t* pid, int64_t* row) const {
  const int64_t p = owner(gid);
  if (p < 0) return false;
  if (p == rank_ || p == nbr_idx_) {
    *pid = p;
    *row = gid - prefix_sum_[p];
    return true;
  }
  auto it = gid_lid_[p].find(gid);
  if (it == gid_lid_[p].end()) return false;
  *pid = p;
  *row = it->second;
  return true;
}

template <typename T>
void XBorder::fill_rows(T* out, int64_t dim, const std::vector<const T*>& tables, const int64_t* ids,
                        int64_t n, const int64_t* out_idx) const {
  int64_t bad = -1;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    int64_t p, r;
    const int64_t o = out_idx ? out_idx[i] : i;
    if (!resolve(ids[i], &p, &r) || tables[p] == nullptr) {
#pragma omp critical
      bad = ids[i];
      continue;
    }
    std::memcpy(out + o * dim, tables[p] + r * dim, sizeof(T) * dim);
  }
  if (bad >= 0) throw std::out_of_range("XBorder: no row for global id " + std::to_string(bad));
}

template void XBorder::fill_rows<float>(float*, int64_t, const std::vector<const float*>&,
                                        const int64_t*, int64_t, const int64_t*) const;
template void XBorder::fill_rows<int64_t>(int64_t*, int64_t, const std::vector<const int64_t*>&,
                                          const int64_t*, int64_t, const int64_t*) const;

}  // namespace host
}  // namespace grappa
