// Allocation-free entry point of the neighbour-sampling kernel (S1).
//
// This entry point has no counterpart in the reference (mpi-dsg/grappa samples on
// the host and has no device sampler).  It exists for callers that must not
// allocate device memory themselves: code embedded in a host application that
// owns every device allocation up front (a serving runtime with a fixed memory
// plan, for instance), and latency-critical loops where cudaMalloc/cudaFree would
// add their implicit device-wide synchronisation.  Such callers pass only their
// inputs and outputs; the kernel's scratch (the status words of its single-pass
// prefix scan) lives in a fixed, file-scope device array instead of a buffer the
// caller would have to allocate.
//
// Limits and behaviour:
//   * at most kGrappaNoAllocMaxDst (1,048,576) destination nodes per call; larger
//     requests are rejected with GRAPPA_NOALLOC_TOO_MANY_DST before anything runs;
//   * the scratch array (128 KiB) is held by every GPU that loads the library until
//     the process exits;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call before
//     any stream capture;
//   * all calls share the one array, which keeps the previous call's contents; each
//     call clears it with cudaMemsetAsync on the caller's stream before the kernel.
//     Calls that overlap on the GPU (different streams, or different host threads
//     without ordering) race on it and must be serialised by the caller;
//   * no cudaMalloc, cudaFree or allocating library routine is called.
#pragma once
#include <cstdint>

#define GRAPPA_NOALLOC_OK 0
#define GRAPPA_NOALLOC_TOO_MANY_DST 1
#define GRAPPA_NOALLOC_SETUP_FAILED 2
#define GRAPPA_NOALLOC_LAUNCH_FAILED 3
#define GRAPPA_NOALLOC_BAD_ARGUMENT 4

constexpr int kGrappaNoAllocMaxDst = 1 << 20;

extern "C" {

// One sampling hop over a CSC graph (indptr int64 [n_graph_nodes + 1], indices
// int32), for the n_dst destination nodes dst_nid; same semantics and outputs as
// the allocating launcher (grappa_b200/csrc/cuda/sample.cu, launch_sample_hop):
// out_indptr [n_dst + 1], out_nbr [cap_edges], *n_edges_out, coverage sums in
// cov_accum[2] when gideg is given.  frontier, gideg and cov_accum may be null;
// err may be null too, which turns off error reporting (capacity overflows and
// timeouts of the scan are then silent).
// dst_nid may be null when n_dst is 0 (an empty batch writes out_indptr[0] = 0 and
// *n_edges_out = 0).  counters points to device int64 [seed, epoch, step].  stream is a cudaStream_t
// (null = the legacy default stream).  Returns a GRAPPA_NOALLOC_* code.
int grappa_sample_hop_noalloc(const int64_t* indptr, const int32_t* indices, int64_t n_graph_nodes,
                              const int32_t* dst_nid, int32_t n_dst, const uint8_t* frontier, int32_t fanout,
                              int32_t replace, const int64_t* counters, int32_t hop, const int64_t* gideg,
                              float* cov_accum, int32_t* out_indptr, int32_t* out_nbr, int32_t cap_edges,
                              int32_t* n_edges_out, int32_t* err, void* stream);

// Size limit of the call above (for callers that cannot include this header).
int grappa_sample_hop_noalloc_max_dst(void);
}
