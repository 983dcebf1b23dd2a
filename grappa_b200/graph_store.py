"""GPU-resident partition data and the working graph of one rank.

Every rank owns one partition (global node ids [prefix[r], prefix[r+1]), the
reference's id scheme, t10n/dataloader.py:242-252): the complete in-edge CSR of
its nodes (sources as global ids), their features, labels, split masks and
global in-degrees.  These arrays never change and are exported to the other
ranks through CUDA IPC.

Training samples from the *working graph*: the own partition plus, since the
last repartition, the current neighbour partition q and a halo of the sources of
their in-edges owned by other partitions (reference: load_nbr_chunk_v2,
t10n/dataloader.py:261-450).  Working node ids are [own | q | halo].  The
reference rebuilds this from chunk files on a shared filesystem; here it is
rebuilt on the GPU by pulling q's CSR and features and the halo rows straight
out of the peers' HBM (grappa_b200/csrc/cuda/peer.cu: mark / mark_compact /
csr_merge / pull_rows), with no NCCL call and no host round trip.
"""
import torch

from grappa_b200 import _native
from grappa_b200.models.flat import pad8


class OwnPartition:
    """The static arrays of one rank's partition (on its device)."""

    def __init__(self, rank, world, prefix, indptr, indices, feat, label, train_mask, val_mask, test_mask, gideg,
                 ext_src, feat_dim=None):
        self.rank, self.world = rank, world
        self.prefix = [int(x) for x in prefix]
        self.indptr = indptr          # int64 [n_r + 1]
        self.indices = indices        # int32 global source ids
        self.feat = feat              # bf16 [n_r, pad8(d)]
        self.feat_dim = int(feat_dim if feat_dim is not None else feat.shape[1])
        self.label = label            # int32 [n_r]
        self.train_mask, self.val_mask, self.test_mask = train_mask, val_mask, test_mask
        self.gideg = gideg            # int64 [n_r] global in-degree (no self-loop)
        self.ext_src = ext_src        # int32 sorted unique external sources

    @property
    def n_nodes(self):
        return self.prefix[self.rank + 1] - self.prefix[self.rank]

    @property
    def n_edges(self):
        return int(self.indices.numel())

    @property
    def n_global(self):
        return self.prefix[-1]


def partition_assignment(n, world, seed):
    """Owner of every node: a seeded hash (the benchmark configs' 'hash into partitions')."""
    if world == 1:
        return torch.zeros(n, dtype=torch.int64)
    return torch.from_numpy(_native.host().c_dist.random_assign_pid(n, world, seed))


def partition_from_global(graph, world, rank, device, part_seed=0, feat_dtype=torch.bfloat16):
    """Relabel ``graph`` (a SyntheticGraph) into partition-contiguous ids and return this
    rank's OwnPartition.  Every rank runs this on the same graph and gets the same
    relabelling; only its own rows are kept.  Each own node gets one self-loop, as
    the reference's chunk writer appends (csrc/python/py_seq_chunking.cc:110-134)."""
    device = torch.device(device)
    n = graph.n_nodes
    pid = partition_assignment(n, world, part_seed).to(device)
    order = torch.argsort(pid * n + torch.arange(n, device=device))  # (pid, id) order
    new_id = torch.empty(n, dtype=torch.int64, device=device)
    new_id[order] = torch.arange(n, dtype=torch.int64, device=device)
    counts = torch.bincount(pid, minlength=world).cpu()
    prefix = [0]
    for c in counts.tolist():
        prefix.append(prefix[-1] + c)
    lo, hi = prefix[rank], prefix[rank + 1]
    u = new_id[graph.u.to(device)]
    v = new_id[graph.v.to(device)]
    gideg_all = torch.bincount(v, minlength=n)
    sel = (v >= lo) & (v < hi)
    uu, vv = u[sel], v[sel]
    del u, v, sel
    loops = torch.arange(lo, hi, dtype=torch.int64, device=device)
    uu = torch.cat([uu, loops])
    vv = torch.cat([vv, loops]) - lo
    key, _ = torch.sort(vv * n + uu)
    indices = (key % n).to(torch.int32)
    deg = torch.bincount(key // n, minlength=hi - lo)
    indptr = torch.zeros(hi - lo + 1, dtype=torch.int64, device=device)
    indptr[1:] = torch.cumsum(deg, 0)
    del key, uu, vv
    ext = indices[(indices < lo) | (indices >= hi)]
    ext_src = torch.unique(ext).to(torch.int32)  # sorted
    own_old = order[lo:hi]  # old ids of own nodes, ascending new id
    d = graph.spec.feat_dim
    feat = torch.zeros((hi - lo, pad8(d)), dtype=feat_dtype, device=device)
    feat[:, :d] = graph.feat.to(device)[own_old].to(feat_dtype)
    label = graph.label.to(device)[own_old].to(torch.int32)
    tr = graph.train_mask.to(device)[own_old]
    va = graph.val_mask.to(device)[own_old]
    te = graph.test_mask.to(device)[own_old]
    gideg = gideg_all[lo:hi].clone()
    return OwnPartition(rank, world, prefix, indptr, indices, feat, label, tr, va, te, gideg, ext_src, feat_dim=d)


class WorkingGraph:
    """CSR (by destination, working ids) + features of [own | neighbour | halo] nodes."""

    def __init__(self, indptr, indices, feat, n_own, n_nbr, n_halo_dev, cap_nodes, nbr):
        self.indptr, self.indices, self.feat = indptr, indices, feat
        self.n_own, self.n_nbr = n_own, n_nbr
        self.n_halo_dev = n_halo_dev
        self.cap_nodes = cap_nodes
        self.nbr = nbr


class PartitionStore:
    """Own partition + working graph of one rank; ``repartition(q)`` rebuilds the working
    graph for neighbour partition q through peer memory."""

    def __init__(self, own, comm=None):
        self.own = own
        self.comm = comm
        self.rank, self.world = own.rank, own.world
        self.device = own.indices.device
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.working = None
        self._peer = None
        self.repart_log = []
        self.cap_nodes = own.n_nodes
        if self.world > 1:
            self._export()

    # -- peer exports ---------------------------------------------------------------------
    def _export(self):
        from grappa_b200.parallel.comm import PeerBuffer

        own, comm = self.own, self.comm
        cu = _native.cuda()
        arrays = {"indptr": own.indptr, "indices": own.indices, "feat": own.feat, "ext": own.ext_src}
        self._peer = {}
        for name, t in arrays.items():
            nbytes = (t.numel() * t.element_size() + 255) // 256 * 256
            pb = PeerBuffer(comm, nbytes)
            if t.numel():
                pb.tensor(t.dtype, [t.numel()]).copy_(t.reshape(-1))
            self._peer[name] = pb
        self._sizes = comm.all_gather_object(
            {"n": own.n_nodes, "e": own.n_edges, "ext": int(own.ext_src.numel())})
        self.feat_stride = int(own.feat.shape[1])
        self._prefix_dev = torch.tensor(own.prefix, dtype=torch.int64, device=self.device)
        max_n = max(s["n"] for s in self._sizes)
        max_e = max(s["e"] for s in self._sizes)
        max_ext = max(s["ext"] for s in self._sizes)
        cap_halo = min(own.n_global, int(own.ext_src.numel()) + max_ext)
        self.cap_nodes = own.n_nodes + max_n + cap_halo
        self.cap_own_nbr = own.n_nodes + max_n
        self.cap_edges = own.n_edges + max_e
        dev = self.device
        self._indptr_w = torch.zeros(self.cap_nodes + 1, dtype=torch.int64, device=dev)
        self._indices_w = torch.zeros(max(1, self.cap_edges), dtype=torch.int32, device=dev)
        self._feat_w = torch.zeros((self.cap_nodes, self.feat_stride), dtype=own.feat.dtype, device=dev)
        self._map = torch.zeros(own.n_global, dtype=torch.int32, device=dev)
        self._mark = torch.zeros(own.n_global, dtype=torch.uint8, device=dev)
        self._halo_ids = torch.zeros(max(1, cap_halo), dtype=torch.int64, device=dev)
        self._n_halo = torch.zeros(1, dtype=torch.int32, device=dev)
        self._mc_scratch = torch.zeros(cu.mark_compact_scratch_words(own.n_global), dtype=torch.int64, device=dev)
        torch.cuda.synchronize()
        comm.barrier()

    # -- working graph --------------------------------------------------------------------
    def repartition(self, nbr):
        """Rebuild the working graph for neighbour partition ``nbr`` (the rank itself for W=1)."""
        own = self.own
        if self.world == 1 or nbr == self.rank:
            self.working = WorkingGraph(own.indptr, own.indices, own.feat, own.n_nodes, 0,
                                        torch.zeros(1, dtype=torch.int32, device=self.device), own.n_nodes, self.rank)
            return self.working
        cu = _native.cuda()
        r, q = self.rank, nbr
        sz = self._sizes
        n_r, n_q = own.n_nodes, sz[q]["n"]
        peer = self._peer
        # events: start, marks + halo compaction, CSR merge, end (main stream); halo rows
        # done (second side stream); feature-copy start and end (side stream)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
        ev[0].record()
        # q's feature rows (the largest transfer, independent of the CSR and halo work)
        # stream over NVLink on a side stream while the marks, the CSR merge and the halo
        # pulls run here; the own rows are copied once (they never change)
        fs = self.feat_stride
        esz = own.feat.element_size()
        main = torch.cuda.current_stream(self.device)
        if getattr(self, "_side", None) is None:
            self._side = torch.cuda.Stream(device=self.device)
        self._side.wait_stream(main)
        with torch.cuda.stream(self._side):
            ev[5].record()
            if not getattr(self, "_own_rows_in", False):
                self._feat_w[:n_r].copy_(own.feat)
                self._own_rows_in = True
            cu.peer_copy(self._feat_w.data_ptr() + n_r * fs * esz, peer["feat"].ptrs[q], n_q * fs * esz)
            ev[6].record()
        # 1. halo = (ext_r U ext_q) \ (V_r U V_q), found by marking a dense global-id array
        cu.mark_ids(peer["ext"].ptrs[r], None, sz[r]["ext"], self._mark)
        cu.mark_ids(peer["ext"].ptrs[q], None, sz[q]["ext"], self._mark)
        cu.iota_map(self._map, own.prefix[r], n_r, 0, self._mark)
        cu.iota_map(self._map, own.prefix[q], n_q, n_r, self._mark)
        cu.mark_compact(self._mark, self._halo_ids, self._map, n_r + n_q, self._n_halo, self._mc_scratch, self.err)
        ev[1].record()
        # 2. halo feature rows from their owners, on a second side stream beside the CSR
        # merge (both need only the halo ids and the map)
        if getattr(self, "_side2", None) is None:
            self._side2 = torch.cuda.Stream(device=self.device)
        self._side2.wait_stream(main)
        tables = [peer["feat"].ptrs[p] for p in range(self.world)]
        with torch.cuda.stream(self._side2):
            cu.pull_rows(tables, fs, esz, fs * esz, self._halo_ids, self._n_halo, 0, self._prefix_dev,
                         self._feat_w.data_ptr(), fs, n_r + n_q, self._halo_ids.numel(), self.err)
            ev[3].record()
        # 3. working CSR: own in-edges, then q's in-edges pulled from q, sources translated
        # own and neighbour sources translate arithmetically (their ids are the ranges the
        # id map holds as iotas); only halo sources read the map
        cu.csr_merge(peer["indptr"].ptrs[r], peer["indices"].ptrs[r], n_r, peer["indptr"].ptrs[q],
                     peer["indices"].ptrs[q], n_q, self._map, self._indptr_w, self._indices_w, self.err,
                     g0_a=own.prefix[r], g0_b=own.prefix[q])
        ev[2].record()
        main.wait_stream(self._side)
        main.wait_stream(self._side2)
        ev[4].record()
        # bytes this rank pulls over NVLink: q's external-source list and CSR, q's feature
        # rows and the halo rows (their count is on the device until the log is read)
        pulled = sz[q]["ext"] * 4 + (n_q + 1) * 8 + sz[q]["e"] * 4 + n_q * fs * esz
        self.repart_log.append({"events": ev, "bytes_fixed": pulled, "row_bytes": fs * esz,
                                "n_halo": self._n_halo.clone(), "csr_bytes": (n_q + 1) * 8 + sz[q]["e"] * 4,
                                "feat_bytes": n_q * fs * esz})
        self.working = WorkingGraph(self._indptr_w, self._indices_w, self._feat_w, n_r, n_q, self._n_halo,
                                    self.cap_nodes, q)
        return self.working

    def repartition_stats(self, link_gbs=770.0):
        """Device time and NVLink bytes of every peer-memory repartition so far (synchronises):
        [{'ms', 'bytes', 'frac_of_link_roofline'}], the roofline being the pulled bytes at
        ``link_gbs`` GB/s (the measured peer bandwidth per direction; nominal 900)."""
        torch.cuda.synchronize(self.device)
        out = []
        for rec in self.repart_log:
            ev = rec["events"]
            ms = ev[0].elapsed_time(ev[4])
            b = rec["bytes_fixed"] + int(rec["n_halo"].item()) * rec["row_bytes"]
            t = lambda i, j: round(ev[i].elapsed_time(ev[j]), 4)  # noqa: E731
            out.append({"ms": round(ms, 4), "bytes": int(b),
                        "frac_of_link_roofline": round(b / (link_gbs * 1e9) * 1e3 / ms, 4) if ms > 0 else None,
                        "phases_ms": {"marks": t(0, 1), "csr_merge": t(1, 2), "halo_rows": t(1, 3),
                                      "feature_copy": t(5, 6), "join": round(max(t(2, 4), 0.0), 4)},
                        "csr_gbs": round(rec["csr_bytes"] / max(t(1, 2), 1e-6) / 1e6, 1),
                        "feature_gbs": round(rec["feat_bytes"] / max(t(5, 6), 1e-6) / 1e6, 1)})
        return out

    def check_errors(self):
        e = int(self.err.item())
        if e:
            raise RuntimeError(f"device error word {e:#x} raised during repartitioning")

    def close(self):
        if self._peer:
            for pb in self._peer.values():
                pb.close()
            self._peer = None


def working_graph_host(parts, rank, nbr):
    """The working graph of ``rank`` with neighbour partition ``nbr`` built from every
    rank's OwnPartition on the host (tensors on any one device): the same layout as
    ``PartitionStore.repartition`` builds over peer memory — rows [own | nbr | halo],
    halo = sorted global ids of the in-edge sources of own and nbr that neither owns,
    CSR by destination in working ids, halo rows without in-edges.  This is the oracle
    of the peer-memory path and the working graph of single-process tools."""
    own, q = parts[rank], parts[nbr]
    dev = own.indices.device
    n_r, n_q = own.n_nodes, (q.n_nodes if nbr != rank else 0)
    lo_r, lo_q = own.prefix[rank], own.prefix[nbr]
    n_global = own.n_global
    ext = own.ext_src.to(dev, torch.int64)
    if nbr != rank:
        ext = torch.cat([ext, q.ext_src.to(dev, torch.int64)])
    ext = torch.unique(ext)
    inside = ((ext >= lo_r) & (ext < lo_r + n_r)) | ((ext >= lo_q) & (ext < lo_q + n_q))
    halo = ext[~inside]
    wmap = torch.full((n_global,), -1, dtype=torch.int64, device=dev)
    wmap[lo_r:lo_r + n_r] = torch.arange(n_r, device=dev)
    if n_q:
        wmap[lo_q:lo_q + n_q] = torch.arange(n_r, n_r + n_q, device=dev)
    wmap[halo] = torch.arange(n_r + n_q, n_r + n_q + halo.numel(), device=dev)
    n_w = n_r + n_q + int(halo.numel())
    indptr = torch.zeros(n_w + 1, dtype=torch.int64, device=dev)
    deg_r = own.indptr[1:] - own.indptr[:-1]
    indptr[1:n_r + 1] = torch.cumsum(deg_r.to(dev), 0)
    pieces = [wmap[own.indices.to(dev).long()]]
    if n_q:
        deg_q = (q.indptr[1:] - q.indptr[:-1]).to(dev)
        indptr[n_r + 1:n_r + n_q + 1] = indptr[n_r] + torch.cumsum(deg_q, 0)
        pieces.append(wmap[q.indices.to(dev).long()])
    indptr[n_r + n_q + 1:] = indptr[n_r + n_q]
    indices = torch.cat(pieces).to(torch.int32)
    feats = [own.feat.to(dev)] + ([q.feat.to(dev)] if n_q else [])
    if halo.numel():
        owner = torch.bucketize(halo, torch.tensor(own.prefix[1:], device=dev), right=True)
        hf = torch.zeros((halo.numel(), own.feat.shape[1]), dtype=own.feat.dtype, device=dev)
        for p in torch.unique(owner).tolist():
            sel = owner == p
            hf[sel] = parts[p].feat.to(dev)[halo[sel] - own.prefix[p]]
        feats.append(hf)
    feat = torch.cat(feats)
    return WorkingGraph(indptr, indices, feat, n_r, n_q,
                        torch.tensor([int(halo.numel())], dtype=torch.int32, device=dev), n_w, nbr)


def next_neighbor(nbr_idx, rank, world):
    """Round-robin neighbour schedule of the reference (t10n/dataloader.py:547-553)."""
    nbr_idx = (nbr_idx + 1) % world
    if nbr_idx == rank:
        nbr_idx = (nbr_idx + 1) % world
    return nbr_idx


def partition_from_chunks(data_path, graph_name, part_method, n_part, rank, feat_dim, device,
                          feat_dtype=torch.bfloat16):
    """This rank's OwnPartition read from a chunked dataset (the reference's on-disk layout,
    grappa_b200.dataset.io_dist): the intra-partition edges p{rank}.u/v (with their
    self-loops) plus every bridge b{j}_{rank} into the partition form the complete
    in-edge CSR of the own nodes; features, labels and masks come from the p{rank}.* files.
    The global in-degree is the in-edge count without the self-loop."""
    import numpy as np

    from grappa_b200.dataset.io_dist import ChunkIO
    from grappa_b200.dataset.meta import t10n_chunk_path

    device = torch.device(device)
    io = ChunkIO(f"{data_path}/{t10n_chunk_path(graph_name, part_method, n_part)}", n_part, feat_dim)
    prefix = io.prefix
    lo, hi = prefix[rank], prefix[rank + 1]
    n = hi - lo
    us = [io.part(rank, "u") + lo]
    vs = [io.part(rank, "v")]
    for j in range(n_part):
        if j == rank:
            continue
        bu, bv = io.bridge(j, rank)
        if bu is not None:
            us.append(bu + prefix[j])
            vs.append(bv)
    u = torch.from_numpy(np.concatenate(us)).to(device)
    v = torch.from_numpy(np.concatenate(vs)).to(device)
    N = prefix[-1]
    key, _ = torch.sort(v * N + u)
    indices = (key % N).to(torch.int32)
    vv = key // N
    deg = torch.bincount(vv, minlength=n)
    indptr = torch.zeros(n + 1, dtype=torch.int64, device=device)
    indptr[1:] = torch.cumsum(deg, 0)
    loops = torch.bincount(vv[(key % N) == vv + lo], minlength=n)
    gideg = (deg - loops).to(torch.int64)
    del key, vv, u, v
    ext = indices[(indices < lo) | (indices >= hi)]
    ext_src = torch.unique(ext).to(torch.int32)
    feat = torch.zeros((n, pad8(feat_dim)), dtype=feat_dtype, device=device)
    feat[:, :feat_dim] = torch.from_numpy(io.part(rank, "nfeat")).to(device).to(feat_dtype)
    label = torch.from_numpy(io.part(rank, "label")).to(device).to(torch.int32)
    masks = [torch.from_numpy(io.part(rank, k)).to(device) for k in ("train", "valid", "test")]
    return OwnPartition(rank, n_part, prefix, indptr, indices, feat, label, masks[0], masks[1], masks[2], gideg,
                        ext_src, feat_dim=feat_dim)
