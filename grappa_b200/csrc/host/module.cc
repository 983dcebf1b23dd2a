// Python module grappa_b200._C: the host (CPU) engine of the framework.
//
// Submodules mirror the reference's t10n._C (csrc/python/pybind11.cc:59-130):
//   graph    HostGraph, HostSampler, one-hop neighbour sampling, helpers
//   xborder  XBorder
//   c_seq    build / split_node_feat / split_node_data / print_string
//   c_dist   random_assign_pid
// plus helpers used by the synthetic data generator and the tests.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cmath>
#include <memory>
#include <optional>
#include <unordered_map>

#include "chunking.h"
#include "graph_host.h"
#include "grappa/rng.h"
#include "mlpart.h"
#include "numa.h"
#include "pipeline.h"
#include "xborder.h"

namespace py = pybind11;
using grappa::host::Block;
using grappa::host::CSC;

namespace {

template <typename T>
using arr = py::array_t<T, py::array::c_style | py::array::forcecast>;

template <typename T>
py::array_t<T> to_py(std::vector<T>&& v) {
  auto* heap = new std::vector<T>(std::move(v));
  py::capsule owner(heap, [](void* p) { delete static_cast<std::vector<T>*>(p); });
  return py::array_t<T>({static_cast<py::ssize_t>(heap->size())}, {sizeof(T)}, heap->data(), owner);
}

template <typename T>
py::array_t<T> to_py_copy(const std::vector<T>& v) {
  std::vector<T> c(v);
  return to_py(std::move(c));
}

// Host CSC of a partition.  With numa_node >= 0 its arrays are placed on that node
// (reference: csrc/python/py_graph.cc:23-34, numa_set_membind before the build; here
// a preferred-node policy for the build only).
class HostGraph {
 public:
  HostGraph(arr<int64_t> u, arr<int64_t> v, int64_t n_nodes, int numa_node) {
    if (u.size() != v.size()) throw std::invalid_argument("u and v differ in length");
    py::gil_scoped_release rel;
    grappa::host::MemPolicyScope place(numa_node);  // inactive for numa_node < 0
    numa_placed = place.active();
    csc = grappa::host::build_csc(u.data(), v.data(), static_cast<int64_t>(u.size()), n_nodes);
  }
  CSC csc;
  bool numa_placed = false;
};

struct HostBatch {
  std::vector<Block> blocks;  // hop order: the seed hop first
  double cov_sum = 0.0, cov_n = 0.0;
  std::vector<int64_t> seeds;
};

py::dict block_to_py(Block& b) {
  py::dict d;
  d["n_dst"] = b.n_dst;
  d["n_src"] = b.n_src;
  d["indptr"] = to_py_copy(b.indptr);
  d["indices"] = to_py_copy(b.indices);
  d["src_nid"] = to_py_copy(b.src_nid);
  d["src_sampled"] = to_py_copy(b.src_sampled);
  return d;
}

HostBatch sample_batch(const CSC& g, const std::vector<int64_t>& fanouts, const int64_t* seeds,
                       int64_t n_seeds, const int64_t* gideg, uint64_t seed, uint64_t epoch,
                       uint64_t step, bool repeated) {
  HostBatch hb;
  hb.seeds.assign(seeds, seeds + n_seeds);
  std::vector<int64_t> dst(seeds, seeds + n_seeds);
  std::vector<uint8_t> front;
  int hop = 0;
  for (auto it = fanouts.rbegin(); it != fanouts.rend(); ++it, ++hop) {
    const uint64_t key = grappa::hop_key(seed, epoch, step, hop);
    int64_t fan = *it;
    Block b;
    if (repeated) {
      // with replacement: fanout draws per node with at least one neighbour
      b.n_dst = static_cast<int64_t>(dst.size());
      b.indptr.assign(b.n_dst + 1, 0);
      for (int64_t i = 0; i < b.n_dst; ++i) {
        const bool f = front.empty() || front[i];
        const int64_t d = (f && dst[i] >= 0 && dst[i] < g.n_nodes) ? g.degree(dst[i]) : 0;
        b.indptr[i + 1] = b.indptr[i] + (d == 0 ? 0 : (fan < 0 ? d : fan));
        if (gideg && f) {
          hb.cov_sum += grappa::host::coverage_ratio(d, gideg[i]);
          hb.cov_n += 1.0;
        }
      }
      std::vector<int64_t> nbr(b.indptr[b.n_dst]);
      for (int64_t i = 0; i < b.n_dst; ++i) {
        const int64_t k = b.indptr[i + 1] - b.indptr[i];
        if (!k) continue;
        const int64_t d = g.degree(dst[i]);
        for (int64_t t = 0; t < k; ++t) {
          const uint32_t o = (fan < 0) ? static_cast<uint32_t>(t)
                                       : grappa::draw_below(grappa::node_draw(key, dst[i], t), d);
          nbr[b.indptr[i] + t] = g.indices[g.indptr[dst[i]] + o];
        }
      }
      // compaction with the same rule as sample_hop
      std::unordered_map<int64_t, int64_t> lid;
      b.src_nid = dst;
      for (int64_t i = 0; i < b.n_dst; ++i) lid.emplace(dst[i], i);
      b.indices.resize(nbr.size());
      for (size_t j = 0; j < nbr.size(); ++j) {
        auto f = lid.find(nbr[j]);
        if (f == lid.end()) {
          const int64_t id = static_cast<int64_t>(b.src_nid.size());
          lid.emplace(nbr[j], id);
          b.src_nid.push_back(nbr[j]);
          b.indices[j] = id;
        } else {
          b.indices[j] = f->second;
        }
      }
      b.n_src = static_cast<int64_t>(b.src_nid.size());
      b.src_sampled.assign(b.n_src, 0);
      for (auto x : b.indices) b.src_sampled[x] = 1;
    } else {
      b = grappa::host::sample_hop(g, dst.data(), front.empty() ? nullptr : front.data(),
                                   static_cast<int64_t>(dst.size()), fan, key, gideg,
                                   &hb.cov_sum, &hb.cov_n);
    }
    gideg = nullptr;  // the coverage counter covers the seed hop only
    dst = b.src_nid;
    front = b.src_sampled;
    hb.blocks.push_back(std::move(b));
  }
  return hb;
}

// Pipelined batch producer: a worker thread keeps up to two sampled batches ready
// (BatchPipeline; the reference's py_graph.cc:50-371 busy-waits, here the consumer
// sleeps on a condition variable).
class HostSampler {
 public:
  HostSampler(HostGraph* g, std::vector<int64_t> fanouts, bool repeated, bool count_resampling,
              uint64_t seed)
      : g_(g), fanouts_(std::move(fanouts)), repeated_(repeated), count_(count_resampling),
        seed_(seed), pipe_(2) {}
  ~HostSampler() { pipe_.stop(); }

  void reinit(arr<int64_t> targets, py::object gideg, int64_t batch_size, int64_t n_batch,
              int64_t epoch) {
    pipe_.stop();  // the worker reads targets_/gideg_: end it before they change
    if (batch_size <= 0) throw std::invalid_argument("batch_size must be positive");
    std::vector<int64_t> gd_new;
    if (!gideg.is_none()) {
      auto gd = gideg.cast<arr<int64_t>>();
      if (gd.size() != targets.size()) throw std::invalid_argument("gideg and targets differ in length");
      gd_new.assign(gd.data(), gd.data() + gd.size());
    }
    targets_.assign(targets.data(), targets.data() + targets.size());
    gideg_ = std::move(gd_new);
    bs_ = batch_size;
    const int64_t nb = n_batch < 0 ? (static_cast<int64_t>(targets_.size()) + bs_ - 1) / bs_ : n_batch;
    epoch_ = epoch < 0 ? epoch_ + 1 : epoch;
    const int64_t ep = epoch_, bs = bs_;
    pipe_.start(nb, [this, ep, bs](int64_t s) {
      const int64_t n = static_cast<int64_t>(targets_.size());
      const int64_t b = std::min(n, s * bs), e = std::min(n, b + bs);
      return std::make_unique<HostBatch>(sample_batch(
          g_->csc, fanouts_, targets_.data() + b, e - b,
          (count_ && !gideg_.empty()) ? gideg_.data() + b : nullptr, seed_, ep, s, repeated_));
    });
  }

  py::tuple next_batch() {
    std::unique_ptr<HostBatch> b;
    {
      py::gil_scoped_release rel;
      b = pipe_.next();
    }
    if (!b) throw py::stop_iteration();
    py::list blocks;
    for (auto& blk : b->blocks) blocks.append(block_to_py(blk));
    return py::make_tuple(to_py(std::move(b->seeds)), blocks, b->cov_sum, b->cov_n);
  }

  // Reference-compatible output: ([u_hop1, v_hop1, u_hop2, ...], [cov_sum, cov_n]) with
  // u/v as graph ids (csrc/python/py_graph.cc:345-371).
  py::tuple next_batch_coo() {
    auto t = next_batch();
    py::list blocks = t[1];
    py::list layers;
    for (auto item : blocks) {
      py::dict d = item.cast<py::dict>();
      auto indptr = d["indptr"].cast<arr<int64_t>>();
      auto indices = d["indices"].cast<arr<int64_t>>();
      auto src = d["src_nid"].cast<arr<int64_t>>();
      const int64_t n_dst = d["n_dst"].cast<int64_t>();
      std::vector<int64_t> u(indices.size()), v(indices.size());
      for (int64_t i = 0; i < n_dst; ++i)
        for (int64_t e = indptr.data()[i]; e < indptr.data()[i + 1]; ++e) {
          u[e] = src.data()[indices.data()[e]];
          v[e] = src.data()[i];
        }
      layers.append(to_py(std::move(u)));
      layers.append(to_py(std::move(v)));
    }
    std::vector<float> cnt;
    if (count_) cnt = {static_cast<float>(t[2].cast<double>()), static_cast<float>(t[3].cast<double>())};
    return py::make_tuple(layers, to_py(std::move(cnt)));
  }

  int64_t epoch() const { return epoch_; }

 private:
  HostGraph* g_;
  std::vector<int64_t> fanouts_;
  bool repeated_, count_;
  uint64_t seed_;
  std::vector<int64_t> targets_, gideg_;
  int64_t bs_ = 1, epoch_ = -1;
  grappa::host::BatchPipeline<HostBatch> pipe_;
};

template <typename T>
std::vector<const T*> table_ptrs(const std::vector<py::object>& tables, std::vector<arr<T>>* keep) {
  std::vector<const T*> tp;
  keep->reserve(tables.size());
  for (auto& t : tables) {
    if (t.is_none()) {
      tp.push_back(nullptr);
      continue;
    }
    keep->push_back(t.cast<arr<T>>());
    tp.push_back(keep->back().data());
  }
  return tp;
}

}  // namespace

PYBIND11_MODULE(_C, m) {
  m.doc() = "grappa_b200 host engine (CSC build, sampling, cross-partition ids, chunking)";
  auto mg = m.def_submodule("graph");
  py::class_<HostGraph>(mg, "HostGraph")
      .def(py::init<arr<int64_t>, arr<int64_t>, int64_t, int>(), py::arg("u"), py::arg("v"),
           py::arg("n_nodes") = -1, py::arg("numa_node") = -1)
      .def_readonly("numa_placed", &HostGraph::numa_placed)
      .def("numa_node_of_indices", [](HostGraph& g) {
        return g.csc.indices.empty() ? -1 : grappa::host::numa_node_of(g.csc.indices.data());
      })
      .def_property_readonly("n_nodes", [](HostGraph& g) { return g.csc.n_nodes; })
      .def_property_readonly("n_edges", [](HostGraph& g) { return g.csc.n_edges; })
      .def("indptr", [](HostGraph& g) { return to_py_copy(g.csc.indptr); })
      .def("indices", [](HostGraph& g) { return to_py_copy(g.csc.indices); })
      .def("in_degrees", [](HostGraph& g, arr<int64_t> ids) {
        std::vector<int64_t> out(ids.size());
        for (py::ssize_t i = 0; i < ids.size(); ++i) {
          const int64_t v = ids.data()[i];
          out[i] = (v >= 0 && v < g.csc.n_nodes) ? g.csc.degree(v) : 0;
        }
        return to_py(std::move(out));
      });
  py::class_<HostSampler>(mg, "HostSampler")
      .def(py::init<HostGraph*, std::vector<int64_t>, bool, bool, uint64_t>(), py::arg("graph"),
           py::arg("fanouts"), py::arg("repeated") = false, py::arg("count_resampling") = false,
           py::arg("seed") = 0, py::keep_alive<1, 2>())
      .def("reinit", &HostSampler::reinit, py::arg("targets"), py::arg("gideg") = py::none(),
           py::arg("batch_size"), py::arg("n_batch") = -1, py::arg("epoch") = -1)
      .def("c_reinit_from",
           [](HostSampler& s, arr<int64_t> t, int64_t bs, int64_t nb) { s.reinit(t, py::none(), bs, nb, -1); })
      .def("c_reinit_with_gideg_from",
           [](HostSampler& s, arr<int64_t> t, arr<int64_t> gd, int64_t bs, int64_t nb) {
             s.reinit(t, gd, bs, nb, -1);
           })
      .def("next_batch", &HostSampler::next_batch)
      .def("c_next_batch_py", &HostSampler::next_batch_coo)
      .def_property_readonly("epoch", &HostSampler::epoch);
  mg.def(
      "sample_batch",
      [](HostGraph& g, std::vector<int64_t> fanouts, arr<int64_t> seeds, py::object gideg,
         uint64_t seed, uint64_t epoch, uint64_t step, bool repeated) {
        const int64_t* gd = nullptr;
        arr<int64_t> gda;
        if (!gideg.is_none()) {
          gda = gideg.cast<arr<int64_t>>();
          gd = gda.data();
        }
        HostBatch hb;
        {
          py::gil_scoped_release rel;
          hb = sample_batch(g.csc, fanouts, seeds.data(), static_cast<int64_t>(seeds.size()), gd, seed,
                            epoch, step, repeated);
        }
        py::list blocks;
        for (auto& b : hb.blocks) blocks.append(block_to_py(b));
        return py::make_tuple(blocks, hb.cov_sum, hb.cov_n);
      },
      py::arg("graph"), py::arg("fanouts"), py::arg("seeds"), py::arg("gideg") = py::none(),
      py::arg("seed") = 0, py::arg("epoch") = 0, py::arg("step") = 0, py::arg("repeated") = false);
  // One-hop neighbour sampler for arbitrary seeds (reference: HostNeighborSampler,
  // csrc/python/py_graph.cc:373-390); fanout < 0 takes all neighbours.
  mg.def(
      "sample_neighbors",
      [](HostGraph& g, arr<int64_t> seeds, int64_t fanout, uint64_t key) {
        Block b = grappa::host::sample_hop(g.csc, seeds.data(), nullptr, static_cast<int64_t>(seeds.size()),
                                           fanout, key, nullptr, nullptr, nullptr);
        std::vector<int64_t> u(b.indices.size()), v(b.indices.size());
        for (int64_t i = 0; i < b.n_dst; ++i)
          for (int64_t e = b.indptr[i]; e < b.indptr[i + 1]; ++e) {
            u[e] = b.src_nid[b.indices[e]];
            v[e] = b.src_nid[i];
          }
        return py::make_tuple(to_py(std::move(u)), to_py(std::move(v)));
      },
      py::arg("graph"), py::arg("seeds"), py::arg("fanout"), py::arg("key") = 0);
  mg.def(
      "random_walk_topk",
      [](HostGraph& g, arr<int64_t> seeds, int length, double restart_prob, int num_walks, int num_neighbors,
         uint64_t key) {
        std::vector<float> w;
        Block b;
        {
          py::gil_scoped_release rel;
          b = grappa::host::random_walk_topk(g.csc, seeds.data(), static_cast<int64_t>(seeds.size()), length,
                                             restart_prob, num_walks, num_neighbors, key, &w);
        }
        py::dict d = block_to_py(b);
        d["weights"] = to_py(std::move(w));
        return d;
      },
      py::arg("graph"), py::arg("seeds"), py::arg("length"), py::arg("restart_prob") = 0.5,
      py::arg("num_walks") = 4, py::arg("num_neighbors") = 5, py::arg("key") = 0);
  mg.def("pick_offsets", [](uint64_t key, uint64_t nid, uint32_t d, uint32_t k) {
    std::vector<int64_t> out(k);
    grappa::host::pick_offsets(key, nid, d, k, out.data());
    return to_py(std::move(out));
  });
  mg.def("hop_key", &grappa::hop_key);
  mg.def("coverage_ratio", &grappa::host::coverage_ratio);
  mg.def("rmat_candidates", [](int64_t n, int scale, double a, double b, double c, uint64_t seed,
                               int64_t e0, int64_t e1) {
    std::vector<int64_t> keys(e1 - e0);
    {
      py::gil_scoped_release rel;
      grappa::host::rmat_candidates(n, scale, a, b, c, seed, e0, e1, keys.data());
    }
    return to_py(std::move(keys));
  });
  mg.def("shuffle_keys", [](arr<int64_t> ids, uint64_t seed, uint64_t epoch) {
    std::vector<int64_t> keys(ids.size());
    grappa::host::shuffle_keys(ids.data(), static_cast<int64_t>(ids.size()), seed, epoch, keys.data());
    return to_py(std::move(keys));
  });
  mg.def("hash_part", [](arr<int64_t> ids, uint64_t seed, int32_t n_part) {
    if (n_part < 1) throw std::invalid_argument("n_part must be >= 1");
    std::vector<int64_t> out(ids.size());
    for (py::ssize_t i = 0; i < ids.size(); ++i)
      out[i] = grappa::hash_part(static_cast<uint64_t>(ids.data()[i]), seed, n_part);
    return to_py(std::move(out));
  }, py::arg("ids"), py::arg("seed"), py::arg("n_part"));

  // Dropout keep-mask with the same Philox stream as the GPU kernels: element (r, c)
  // of a row-major buffer with row stride ld is kept iff byte (idx % 16) of the draw of
  // group idx / 16 (idx = r*ld + c) is >= round(p * 256) (key from seed, epoch, step, salt).
  m.def("dropout_mask", [](uint64_t seed, uint64_t epoch, uint64_t step, uint32_t salt, int64_t rows,
                           int64_t cols, int64_t ld, double p) {
    std::vector<uint8_t> mask(static_cast<size_t>(rows * cols));
    const uint64_t key = grappa::hop_key(seed ^ 0xD80Full, epoch, step, salt);
    const uint32_t thr = grappa::dropout_thr8(static_cast<float>(p));
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < rows * cols; ++i) {
      const uint64_t idx = static_cast<uint64_t>(i / cols) * static_cast<uint64_t>(ld) + static_cast<uint64_t>(i % cols);
      mask[i] = static_cast<uint8_t>(grappa::dropout_keep_bits(key, idx, 1, thr) & 1u);
    }
    return to_py(std::move(mask));
  });
  m.def("normal", [](int64_t n, uint64_t seed) {
    // Box-Muller over the same Philox stream as the GPU generator
    std::vector<float> out(n);
    const uint64_t key = grappa::mix64(seed ^ 0x4E4F524Dull);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (n + 1) / 2; ++i) {
      const grappa::U4 r = grappa::index_draw4(key, static_cast<uint64_t>(i), 7u);
      const double u1 = (static_cast<double>(r.x >> 8) + 0.5) / 16777216.0;
      const double u2 = static_cast<double>(r.y >> 8) / 16777216.0;
      const double rad = std::sqrt(-2.0 * std::log(u1));
      out[2 * i] = static_cast<float>(rad * std::cos(2.0 * M_PI * u2));
      if (2 * i + 1 < n) out[2 * i + 1] = static_cast<float>(rad * std::sin(2.0 * M_PI * u2));
    }
    return to_py(std::move(out));
  });

  // NUMA placement and bandwidth (libnuma-free; reference: test/numa_bench.c and the
  // numa_set_membind of csrc/python/py_graph.cc:23-34)
  auto mn = m.def_submodule("numa");
  mn.def("nodes", &grappa::host::numa_nodes, "online NUMA node ids");
  mn.def("node_cpus", &grappa::host::numa_node_cpus, py::arg("node"),
         "CPUs of a node that this process may run on");
  mn.def("parse_cpulist", [](const std::string& s) { return grappa::host::parse_cpulist(s.c_str()); });
  mn.def(
      "node_of", [](py::buffer b) {
        py::buffer_info info = b.request();
        return info.size == 0 ? -1 : grappa::host::numa_node_of(info.ptr);
      },
      py::arg("buffer"), "NUMA node of the buffer's first page (-1 if unknown)");
  mn.def("pin_thread", &grappa::host::pin_thread_to_node, py::arg("node"),
         "pin the calling thread to the node's CPUs");
  mn.def(
      "bandwidth",
      [](int cpu_node, int mem_node, int64_t mbytes, int threads, int reps) {
        grappa::host::Bandwidth r;
        {
          py::gil_scoped_release rel;
          r = grappa::host::memory_bandwidth(cpu_node, mem_node, static_cast<size_t>(mbytes) << 20, threads, reps);
        }
        py::dict d;
        d["cpu_node"] = cpu_node;
        d["mem_node"] = mem_node;
        d["mem_node_seen"] = r.mem_node_seen;
        d["write_gbs"] = r.write_gbs;
        d["read_gbs"] = r.read_gbs;
        return d;
      },
      py::arg("cpu_node"), py::arg("mem_node"), py::arg("mbytes") = 256, py::arg("threads") = 0, py::arg("reps") = 3);
  // with numa.MemPolicy(node): pages this thread faults in come from `node` first
  struct PyMemPolicy {
    int node;
    std::unique_ptr<grappa::host::MemPolicyScope> scope;
  };
  py::class_<PyMemPolicy>(mn, "MemPolicy")
      .def(py::init([](int node) { return PyMemPolicy{node, nullptr}; }), py::arg("node"))
      .def("__enter__", [](PyMemPolicy& p) {
        p.scope = std::make_unique<grappa::host::MemPolicyScope>(p.node);
        return p.scope->active();
      })
      .def("__exit__", [](PyMemPolicy& p, py::object, py::object, py::object) {
        p.scope.reset();
        return false;
      });

  auto mx = m.def_submodule("xborder");
  py::class_<grappa::host::XBorder>(mx, "XBorder")
      .def(py::init<int64_t, int64_t, std::vector<int64_t>>())
      .def("owner", &grappa::host::XBorder::owner)
      .def("group_by_partition",
           [](grappa::host::XBorder& x, arr<int64_t> ids, py::object mask) {
             int8_t* mp = nullptr;
             if (!mask.is_none()) {
               auto ma = mask.cast<py::array_t<int8_t>>();
               if (ma.size() != x.n_part() * ids.size()) throw std::invalid_argument("mask shape");
               mp = ma.mutable_data();
             }
             // numpy arrays left uninitialised: the parallel fill pass writes (and first
             // touches) every entry
             std::vector<py::array_t<int64_t>> arrs;
             arrs.reserve(static_cast<size_t>(x.n_part()));
             x.group_by_partition_into(ids.data(), static_cast<int64_t>(ids.size()), mp,
                                       [&](int64_t, int64_t count) {
                                         arrs.emplace_back(static_cast<py::ssize_t>(count));
                                         return arrs.back().mutable_data();
                                       });
             py::list out;
             for (auto& a : arrs) out.append(a);
             return out;
           },
           py::arg("ids"), py::arg("mask") = py::none())
      .def("mask_by_partition",
           [](grappa::host::XBorder& x, arr<int64_t> ids, py::array_t<int8_t> mask) {
             if (mask.size() != x.n_part() * ids.size()) throw std::invalid_argument("mask shape");
             x.mask_by_partition(ids.data(), static_cast<int64_t>(ids.size()), mask.mutable_data());
           })
      .def("set_nbr_idx", &grappa::host::XBorder::set_nbr_idx)
      .def_property_readonly("nbr_idx", &grappa::host::XBorder::nbr_idx)
      .def("ad_hoc_clear", &grappa::host::XBorder::ad_hoc_clear)
      .def("ad_hoc_build_id_mapping",
           [](grappa::host::XBorder& x, int64_t pid, arr<int64_t> gids) {
             x.ad_hoc_build_id_mapping(pid, gids.data(), static_cast<int64_t>(gids.size()));
           })
      .def("ad_hoc_fill_batch_feat",
           [](grappa::host::XBorder& x, py::array_t<float> out, std::vector<py::object> tables,
              arr<int64_t> ids, py::object out_idx) {
             std::vector<arr<float>> keep;
             auto tp = table_ptrs<float>(tables, &keep);
             const int64_t dim = out.ndim() == 2 ? out.shape(1) : 1;
             const int64_t* oi = nullptr;
             arr<int64_t> oia;
             if (!out_idx.is_none()) {
               oia = out_idx.cast<arr<int64_t>>();
               oi = oia.data();
             }
             x.fill_rows<float>(out.mutable_data(), dim, tp, ids.data(), static_cast<int64_t>(ids.size()), oi);
           },
           py::arg("batch_feat"), py::arg("feat_n"), py::arg("ids"), py::arg("batch_idx") = py::none())
      .def("ad_hoc_fill_batch_ideg",
           [](grappa::host::XBorder& x, py::array_t<int64_t> out, std::vector<py::object> tables,
              arr<int64_t> ids) {
             std::vector<arr<int64_t>> keep;
             auto tp = table_ptrs<int64_t>(tables, &keep);
             x.fill_rows<int64_t>(out.mutable_data(), 1, tp, ids.data(), static_cast<int64_t>(ids.size()), nullptr);
           });

  auto ms = m.def_submodule("c_seq");
  ms.def("print_string", [](const std::string& s) { py::print(s); });
  // multilevel k-way edge-cut partition balanced by node count and training nodes
  // (the reference's METIS assignment with the train mask as a balance type)
  ms.def(
      "multilevel_partition",
      [](int64_t n, arr<int64_t> u, arr<int64_t> v, int64_t n_part, std::optional<arr<int8_t>> train, uint64_t seed,
         double imbalance) {
        if (u.size() != v.size()) throw std::invalid_argument("u and v differ in length");
        if (train && train->size() != n) throw std::invalid_argument("train mask needs one entry per node");
        grappa::host::MlPartOptions opt;
        opt.n_parts = n_part;
        opt.seed = seed;
        opt.imbalance = imbalance;
        const int8_t* tr = train ? train->data() : nullptr;
        std::vector<int64_t> part;
        {
          py::gil_scoped_release rel;
          part = grappa::host::multilevel_partition(n, u.data(), v.data(), static_cast<int64_t>(u.size()), tr, opt);
        }
        return to_py(std::move(part));
      },
      py::arg("n"), py::arg("u"), py::arg("v"), py::arg("n_part"), py::arg("train") = py::none(), py::arg("seed") = 0,
      py::arg("imbalance") = 0.03);
  ms.def("edge_cut", [](int64_t n, arr<int64_t> u, arr<int64_t> v, arr<int64_t> part) {
    if (part.size() != n) throw std::invalid_argument("one part per node");
    return grappa::host::edge_cut(n, u.data(), v.data(), static_cast<int64_t>(u.size()), part.data());
  });
  ms.def("build", [](const std::string& path, int64_t n_n, int64_t n_e, int64_t feat_dim, int64_t n_part,
                     arr<int64_t> src, arr<int64_t> dst, arr<int64_t> nid2pid) {
    (void)feat_dim;
    if (src.size() < n_e || dst.size() < n_e || nid2pid.size() < n_n) throw std::invalid_argument("array sizes");
    grappa::host::ChunkStats st;
    {
      py::gil_scoped_release rel;
      st = grappa::host::chunk_build(path, n_n, n_e, n_part, src.data(), dst.data(), nid2pid.data());
    }
    py::dict d;
    d["part_nodes"] = st.part_nodes;
    d["part_edges"] = st.part_edges;
    d["bridge_edges"] = st.bridge_edges;
    return d;
  });
  ms.def("split_node_feat", [](const std::string& path, int64_t n_n, int64_t dim, int64_t n_part, arr<float> feat) {
    if (feat.size() < n_n * dim) throw std::invalid_argument("feature array too small");
    py::gil_scoped_release rel;
    grappa::host::chunk_split_node_feat(path, n_n, dim, n_part, feat.data());
  });
  ms.def("split_node_data", [](const std::string& path, int64_t n_n, int64_t n_part, arr<float> label,
                               arr<int8_t> tr, arr<int8_t> va, arr<int8_t> te) {
    if (label.size() < n_n || tr.size() < n_n || va.size() < n_n || te.size() < n_n)
      throw std::invalid_argument("node data arrays too small");
    py::gil_scoped_release rel;
    grappa::host::chunk_split_node_data(path, n_n, n_part, label.data(), tr.data(), va.data(), te.data());
  });

  auto md = m.def_submodule("c_dist");
  // Seeded partition assignment.  The reference draws an unseeded pcg32 id per
  // node (csrc/python/py_dist_chunking.cc:13-24); the assignment here is a hash
  // of (node id, seed), so every process computes the same owner for a node.
  md.def("random_assign_pid", [](int64_t n, int64_t n_part, uint64_t seed) {
    if (n_part < 1 || n_part > INT32_MAX) throw std::invalid_argument("n_part must be in [1, 2^31)");
    if (n < 0) throw std::invalid_argument("n must be >= 0");
    std::vector<int64_t> out(n);
#pragma omp parallel for
    for (int64_t i = 0; i < n; ++i) out[i] = grappa::hash_part(static_cast<uint64_t>(i), seed, static_cast<int32_t>(n_part));
    return to_py(std::move(out));
  }, py::arg("n"), py::arg("n_part"), py::arg("seed") = 0);
}
