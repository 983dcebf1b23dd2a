// Peer-memory data plane over NVLink 5 / NVSwitch: IPC-exported buffers, the
// repartition pull kernels, the pull all-to-all and the device barrier (the fused
// gradient all-reduce + Adam is in allreduce.h).  No TMA copy touches peer memory here: every remote access is an
// ordinary ld/st.global through an IPC mapping.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

namespace grappa {
namespace peer {

constexpr int kMaxRanks = 8;

// ---- buffers
void* alloc(int64_t bytes);                       // cudaMalloc'd, zeroed
void release(void* p);
std::string ipc_handle(void* p);                  // 64-byte cudaIpcMemHandle_t
void* ipc_open(const std::string& handle);        // maps a peer's buffer
void ipc_close(void* p);

// ---- repartition (pull over peer memory)
struct PullRowsArgs {
  const void* tables[kMaxRanks] = {};    // per-rank row tables (peer mappings)
  int64_t table_stride = 0;              // elements
  int32_t elem_bytes = 2;
  int32_t row_bytes = 0;                 // bytes copied per row (multiple of 16)
  const int64_t* gids = nullptr;         // global ids of the rows to fetch
  const int32_t* n_ptr = nullptr;
  int64_t n = 0;
  const int64_t* prefix = nullptr;       // device [world + 1] global id ranges
  int32_t world = 1;
  void* out = nullptr;
  int64_t out_stride = 0;                // elements
  int64_t out_row0 = 0;                  // first output row
  int64_t cap = 0;                       // rows that fit in out after out_row0; n beyond it: kErrCapacity
  int32_t* err = nullptr;                // error word (kErrCapacity, kErrBadIndex); may be null
};
// A row whose global id lies outside [prefix[0], prefix[world]) is skipped and
// raises kErrBadIndex; rows past ``cap`` are dropped and raise kErrCapacity.
void launch_pull_rows(const PullRowsArgs& a, int64_t cap, cudaStream_t stream);

// contiguous copy (peer -> local), 16-byte vectors
void launch_copy(void* dst, const void* src, int64_t bytes, cudaStream_t stream);

// Pull all-to-all: this rank copies, from every rank p, the byte range
// [src_off[p], src_off[p] + len[p]) of p's (peer-mapped) send buffer into its own
// receive buffer at dst_off[p].  One launch for all peers, 16-byte P2P loads
// (all offsets and lengths multiples of 16).
struct A2aArgs {
  const uint8_t* src[kMaxRanks] = {};
  int64_t src_off[kMaxRanks] = {};
  int64_t len[kMaxRanks] = {};
  int64_t dst_off[kMaxRanks] = {};
  uint8_t* dst = nullptr;
  int32_t world = 1;
  // segment the pull starts with; the others follow in rotation.  With first =
  // (rank + 1) % world every rank reads a different peer at any one time, so that
  // no rank's outbound NVLink serves all readers at once while the others idle.
  int32_t first = 0;
};
void launch_a2a_pull(const A2aArgs& a, cudaStream_t stream);

// Device-side barrier across ranks: raise this rank's flag at every peer with the
// next tag (*epoch + 1, kept in device memory), wait (bounded by timeout_ns, then
// kErrPeerTimeout) until every peer's flag here reached it.  flags_local[world].
void launch_peer_barrier(int32_t rank, int32_t world, uint32_t* flags_local, uint32_t* const* flags_peer,
                         int64_t* epoch, int64_t timeout_ns, int32_t* err, cudaStream_t stream);

// mark[g] = 1 for g in ids (global ids)
void launch_mark(const int32_t* ids, const int32_t* n_ptr, int64_t n, uint8_t* mark, cudaStream_t stream);
// fill map[g] = base + (g - g0) for g in [g0, g0 + count) and clear mark there
void launch_iota_map(int32_t* map, int64_t g0, int64_t count, int32_t base, uint8_t* clear_mark, cudaStream_t stream);
// compact the marked global ids in increasing order: out[k] = g, map[g] = base + k, *n_out = count;
// the marks are cleared as they are consumed
void launch_mark_compact(uint8_t* mark, int64_t n_global, int64_t* out_ids, int32_t* map, int32_t base,
                         int32_t* n_out, unsigned long long* scan_scratch, int64_t cap_out, int32_t* err,
                         cudaStream_t stream);
int64_t mark_compact_scratch_words(int64_t n_global);
// working CSR: rows [0, n_a) from graph A, [n_a, n_a + n_b) from graph B (peer), sources translated
// through map (global -> working); rows after n_a + n_b are empty.
struct CsrMergeArgs {
  const int64_t* indptr_a = nullptr;
  const int32_t* indices_a = nullptr;
  int64_t n_a = 0;
  const int64_t* indptr_b = nullptr;
  const int32_t* indices_b = nullptr;
  int64_t n_b = 0;
  const int32_t* map = nullptr;
  // sources in [g0_a, g0_a + n_a) map to g - g0_a and those in [g0_b, g0_b + n_b) to
  // n_a + g - g0_b without reading the map (g0 < 0: always read the map)
  int64_t g0_a = -1, g0_b = -1;
  int64_t* indptr_out = nullptr;
  int32_t* indices_out = nullptr;
  int64_t cap_edges = 0;
  int64_t n_rows_total = 0;              // rows of indptr_out - 1
  int32_t* err = nullptr;
};
void launch_csr_merge(const CsrMergeArgs& a, cudaStream_t stream);

}  // namespace peer
}  // namespace grappa
