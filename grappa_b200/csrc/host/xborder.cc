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
  // bucket width 2^s <= the smallest non-empty partition: a bucket then holds at most one
  // start of a non-empty partition, and owner() needs one table read and a compare or two
  const int64_t range = prefix_sum_[n_part_] - prefix_sum_[0];
  int64_t min_size = range;
  for (int64_t p = 0; p < n_part_; ++p) {
    const int64_t sz = prefix_sum_[p + 1] - prefix_sum_[p];
    if (sz < 0) throw std::invalid_argument("XBorder: prefix_sum must not decrease");
    if (sz > 0) min_size = std::min(min_size, sz);
  }
  if (range > 0 && n_part_ < (int64_t{1} << 31)) {
    int s = 0;
    while ((int64_t{2} << s) <= min_size) ++s;
    const int64_t buckets = ((range - 1) >> s) + 1;
    if (buckets <= (int64_t{1} << 22)) {
      lut_shift_ = s;
      lut_.resize(static_cast<size_t>(buckets));
      int64_t p = 0;
      for (int64_t b = 0; b < buckets; ++b) {
        const int64_t gid = prefix_sum_[0] + (b << s);
        while (p + 1 < n_part_ && gid >= prefix_sum_[p + 1]) ++p;
        lut_[static_cast<size_t>(b)] = static_cast<int32_t>(p);
      }
    }
  }
}

int64_t XBorder::owner(int64_t gid) const {
  if (gid < prefix_sum_[0] || gid >= prefix_sum_[n_part_]) return -1;
  if (!lut_.empty()) {
    int64_t p = lut_[static_cast<size_t>((gid - prefix_sum_[0]) >> lut_shift_)];
    while (gid >= prefix_sum_[p + 1]) ++p;  // past the one partition start inside the bucket
    return p;
  }
  if (n_part_ <= 64) {
    // count the partition starts at or below gid: no branches to mispredict on random
    // ids (a binary search spent most of its time there); empty partitions are skipped
    // as upper_bound skips them
    const int64_t* ps = prefix_sum_.data();
    int64_t p = 0;
    for (int64_t q = 1; q < n_part_; ++q) p += gid >= ps[q];
    return p;
  }
  auto it = std::upper_bound(prefix_sum_.begin(), prefix_sum_.end(), gid);
  return static_cast<int64_t>(it - prefix_sum_.begin()) - 1;
}

namespace {

int team_size() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // namespace

void XBorder::mask_by_partition(const int64_t* ids, int64_t n, int8_t* mask) const {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const int64_t p = owner(ids[i]);
    for (int64_t q = 0; q < n_part_; ++q) mask[q * n + i] = static_cast<int8_t>(q == p);
  }
}

// Two passes over contiguous slices, one slice per thread: count each slice's ids per
// owner (zeroing the slice's mask columns on the way), then, once the caller has given
// storage for every partition, write every id straight to its place in its owner's list
// (slice order = input order) and set its mask entry.
void XBorder::group_by_partition_into(const int64_t* ids, int64_t n, int8_t* mask,
                                      const std::function<int64_t*(int64_t, int64_t)>& alloc) const {
  const int nt = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(team_size(), (n + 4095) / 4096)));
  const int64_t P = n_part_;
  std::vector<int64_t> cnt(static_cast<size_t>(nt) * P, 0);
  auto slice = [&](int t, int64_t* b, int64_t* e) {
    const int64_t len = (n + nt - 1) / nt;
    *b = std::min(n, t * len);
    *e = std::min(n, *b + len);
  };
#pragma omp parallel for num_threads(nt) schedule(static, 1)
  for (int t = 0; t < nt; ++t) {
    int64_t b, e;
    slice(t, &b, &e);
    int64_t* c = cnt.data() + static_cast<size_t>(t) * P;
    if (mask)
      for (int64_t q = 0; q < P; ++q) std::memset(mask + q * n + b, 0, static_cast<size_t>(e - b));
    for (int64_t i = b; i < e; ++i) {
      const int64_t p = owner(ids[i]);
      if (p >= 0) ++c[p];
    }
  }
  std::vector<int64_t*> out(static_cast<size_t>(P));
  std::vector<int64_t> pos(static_cast<size_t>(nt) * P, 0);
  for (int64_t q = 0; q < P; ++q) {
    int64_t total = 0;
    for (int t = 0; t < nt; ++t) {
      pos[static_cast<size_t>(t) * P + q] = total;
      total += cnt[static_cast<size_t>(t) * P + q];
    }
    out[static_cast<size_t>(q)] = alloc(q, total);
  }
#pragma omp parallel for num_threads(nt) schedule(static, 1)
  for (int t = 0; t < nt; ++t) {
    int64_t b, e;
    slice(t, &b, &e);
    int64_t* w = pos.data() + static_cast<size_t>(t) * P;
    for (int64_t i = b; i < e; ++i) {
      const int64_t p = owner(ids[i]);
      if (p < 0) continue;
      out[static_cast<size_t>(p)][w[p]++] = ids[i];
      if (mask) mask[p * n + i] = 1;
    }
  }
}

std::vector<std::vector<int64_t>> XBorder::group_by_partition(const int64_t* ids, int64_t n,
                                                              int8_t* mask) const {
  std::vector<std::vector<int64_t>> out(static_cast<size_t>(n_part_));
  group_by_partition_into(ids, n, mask, [&](int64_t p, int64_t count) {
    out[static_cast<size_t>(p)].resize(static_cast<size_t>(count));
    return out[static_cast<size_t>(p)].data();
  });
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
