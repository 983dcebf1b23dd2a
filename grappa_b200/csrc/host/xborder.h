// Cross-partition id helper of the CPU path.
//
// Same interface and semantics as the reference's XBorder
// (csrc/python/py_xborder.h:17-61, csrc/python/py_xborder.cc:18-295): node ids are
// global ids laid out partition after partition (partition p owns
// [prefix_sum[p], prefix_sum[p+1])); the helper splits id lists by owner and
// gathers feature rows for a batch from the own partition, the current
// neighbour partition and a halo cache.  The GPU path replaces it with a dense
// global->working id map built at repartition time.
#pragma once
#include <cstdint>
#include <functional>
#include <unordered_map>
#include <vector>

namespace grappa {
namespace host {

class XBorder {
 public:
  XBorder(int64_t rank, int64_t n_part, std::vector<int64_t> prefix_sum);

  int64_t owner(int64_t gid) const;
  // ids grouped by owner into storage that alloc(p, count) returns for each partition
  // (called once per partition, in order, between the counting and the filling pass);
  // mask (may be null) receives the [n_part, n] 0/1 owner mask
  void group_by_partition_into(const int64_t* ids, int64_t n, int8_t* mask,
                               const std::function<int64_t*(int64_t, int64_t)>& alloc) const;
  // ids grouped by owner (in input order) and a [n_part, n] 0/1 mask
  std::vector<std::vector<int64_t>> group_by_partition(const int64_t* ids, int64_t n,
                                                       int8_t* mask) const;
  void mask_by_partition(const int64_t* ids, int64_t n, int8_t* mask) const;

  void set_nbr_idx(int64_t idx) { nbr_idx_ = idx; }
  int64_t nbr_idx() const { return nbr_idx_; }
  void ad_hoc_clear();
  // halo rows of partition pid are stored in the order of gids
  void ad_hoc_build_id_mapping(int64_t pid, const int64_t* gids, int64_t n);
  // resolve a global id to (table, row); table = partition id
  bool resolve(int64_t gid, int64_t* pid, int64_t* row) const;

  template <typename T>
  void fill_rows(T* out, int64_t dim, const std::vector<const T*>& tables, const int64_t* ids,
                 int64_t n, const int64_t* out_idx) const;

  const std::vector<int64_t>& prefix_sum() const { return prefix_sum_; }
  int64_t rank() const { return rank_; }
  int64_t n_part() const { return n_part_; }

 private:
  // owner lookup: lut_[(gid - prefix_sum_[0]) >> lut_shift_] is the owner of the first id
  // of that bucket; buckets are no wider than the smallest partition (empty when the
  // table would be too large; owner() searches then)
  std::vector<int32_t> lut_;
  int lut_shift_ = 0;
  int64_t rank_, n_part_, nbr_idx_;
  std::vector<int64_t> prefix_sum_;
  std::vector<std::unordered_map<int64_t, int64_t>> gid_lid_;
};

}  // namespace host
}  // namespace grappa
