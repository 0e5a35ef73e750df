// branchcraft (B200 / sm_100a) — C++ API, a drop-in for the reference header
// include/branchcraft.hpp (same namespace, types, constants, function
// signatures and defaults). Every function is an inline wrapper over the C ABI
// of branchcraft.h, implemented by libbranchcraft.so; link with
// -lbranchcraft. Semantics follow the reference with these differences:
//   * decode() accepts splits up to 64 (the reference stops at 16);
//   * malformed device-side indices never fault: they are skipped and reported
//     through bc_last_device_error() (the reference reads or writes out of
//     bounds);
//   * packed_decode() requires strides that are multiples of 8 elements and a
//     16-byte-aligned cache (the TMA rule) and rejects others.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "branchcraft.h"

namespace branchcraft {

constexpr int kPageSize = BC_PAGE_SIZE;
constexpr int kWarpsPerBlock = 4;  // kept for source compatibility; not a launch parameter here

struct Shape {
  int batch;
  int query_heads;
  int kv_heads;
  int dim;
  int max_pages;
  int physical_pages;
};

// All pointers are device pointers. K/V: [physical_pages, 16, kv_heads, dim].
// Q: [batch, query_heads, dim]. Pages: [batch, max_pages].
// Output: FP32 [batch, query_heads, dim]. Empty sequences produce zeros.
struct Inputs {
  const half* q;
  const half* k;
  const half* v;
  const int* pages;
  const int* lengths;
  float* output;
};

// Caller allocates scratch for splits > 1: partial_a = splits*B*Hq*D floats;
// partial_ml = splits*B*Hq*2 floats. Both may be null for splits == 1.
struct Scratch {
  float* partial_a;
  float* partial_ml;
};

namespace detail {
inline bc_shape to_c(const Shape& s) {
  return bc_shape{s.batch, s.query_heads, s.kv_heads, s.dim, s.max_pages, s.physical_pages};
}
}  // namespace detail

inline cudaError_t decode(Shape shape, Inputs in, Scratch scratch, int splits,
                          cudaStream_t stream = nullptr) {
  const bc_shape s = detail::to_c(shape);
  return static_cast<cudaError_t>(bc_decode(&s, in.q, in.k, in.v, in.pages, in.lengths,
                                            in.output, scratch.partial_a, scratch.partial_ml,
                                            splits, stream));
}

inline int auto_splits(Shape shape, int max_length, int sm_count) {
  const bc_shape s = detail::to_c(shape);
  return bc_auto_splits(&s, max_length, sm_count);
}

// Draft nodes are stored in topological order, with parent[b,n] < n or -1.
// Every node attends to the request's paged prefix and its own ancestor chain
// (including itself). Draft Q: [B,N,Hq,D]; K/V: [B,N,Hkv,D].
struct TreeInputs {
  Inputs prefix;
  const half* draft_q;
  const half* draft_k;
  const half* draft_v;
  const int* parent;
  float* output;  // [B,N,Hq,D]
};

inline cudaError_t tree_verify(Shape shape, TreeInputs in, int nodes,
                               cudaStream_t stream = nullptr) {
  const bc_shape s = detail::to_c(shape);
  return static_cast<cudaError_t>(bc_tree_verify(&s, in.draft_q, in.prefix.k, in.prefix.v,
                                                 in.prefix.pages, in.prefix.lengths, in.draft_k,
                                                 in.draft_v, in.parent, in.output, nodes,
                                                 stream));
}

// Copy accepted draft nodes into physical KV destinations. `dest_pages` and
// `dest_slots` are device arrays of length accepted; `path_nodes` is the
// root-to-leaf path. The caller updates page-table metadata after completion.
inline cudaError_t commit_path(Shape shape, const half* draft_k, const half* draft_v,
                               half* cache_k, half* cache_v, const int* path_nodes,
                               const int* dest_pages, const int* dest_slots, int request,
                               int nodes, int accepted, cudaStream_t stream = nullptr) {
  const bc_shape s = detail::to_c(shape);
  return static_cast<cudaError_t>(bc_commit_path(&s, draft_k, draft_v, cache_k, cache_v,
                                                 path_nodes, dest_pages, dest_slots, request,
                                                 nodes, accepted, stream));
}

// vLLM-style packed cache. Logical shape [P,Hkv,16,2D], with runtime strides
// so either NHD or HND physical layout works without a KV copy. Q and output
// are contiguous [B,Hq,D]. Output is FP16, accumulation stays FP32.
inline cudaError_t packed_decode(Shape shape, const half* q, const half* packed_kv,
                                 const int* pages, const int* lengths, half* output,
                                 long long block_stride, long long head_stride,
                                 long long slot_stride, float scale,
                                 cudaStream_t stream = nullptr) {
  const bc_shape s = detail::to_c(shape);
  return static_cast<cudaError_t>(bc_packed_decode(&s, q, packed_kv, pages, lengths, output,
                                                   block_stride, head_stride, slot_stride,
                                                   scale, stream));
}

}  // namespace branchcraft
