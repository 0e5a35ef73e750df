// Accepted-path commit: copy draft K/V rows into physical cache slots, and the
// copy-on-write page clone that precedes it.
//   commit_kernel   <- reference src/tree_attention.cu:73-89 (commit_kernel)
//   clone_kernel    <- the torch page copy in python/branchcraft_torch/
//                      transaction.py:130-136 (self.k[fresh].copy_(self.k[old]))
// Both move 16-byte vectors; every index is range-checked on the device and a
// bad one skips its copy and sets kErrCommitIndex (the reference does not
// check and would write out of bounds).
#pragma once

#include "bc_device.cuh"

namespace bc {

// One CTA per commit entry: threads [0, n16) copy the K row, [n16, 2*n16) the V
// row; a row is kv_heads*dim halves = row16 16-byte vectors.
// Entry e takes (request, node, page, slot) = (req ? req[e] : request, ...).
template <bool VEC>
__global__ void __launch_bounds__(256)
    commit_kernel(int row_halves, int batch, int nodes, int physical_pages,
                  const __half* __restrict__ draft_k, const __half* __restrict__ draft_v,
                  __half* __restrict__ cache_k, __half* __restrict__ cache_v,
                  const int* __restrict__ req, const int* __restrict__ path,
                  const int* __restrict__ dest_pages, const int* __restrict__ dest_slots,
                  int request, unsigned* err) {
  // The next kernel may be scheduled at once (one wave: it only waits, on
  // free SMs, for this grid to finish).
  grid_launch_dependents();
  grid_dependency_wait();  // the preceding kernel of the stream has finished
  const int e = blockIdx.x;
  const int r = req ? req[e] : request;
  const int node = path[e];
  const int page = dest_pages[e];
  const int slot = dest_slots[e];
  if (r < 0 || r >= batch || node < 0 || node >= nodes || page < 0 ||
      page >= physical_pages || slot < 0 || slot >= 16) {
    if (threadIdx.x == 0) atomicOr(err, kErrCommitIndex);
    return;
  }
  const size_t src = (size_t(r) * nodes + node) * row_halves;
  const size_t dst = (size_t(page) * 16 + slot) * row_halves;
  if constexpr (VEC) {
    const int n16 = row_halves / 8;
    for (int x = threadIdx.x; x < 2 * n16; x += blockDim.x) {
      const bool is_v = x >= n16;
      const int i = is_v ? x - n16 : x;
      const uint4* s = reinterpret_cast<const uint4*>((is_v ? draft_v : draft_k) + src) + i;
      uint4* d = reinterpret_cast<uint4*>((is_v ? cache_v : cache_k) + dst) + i;
      *d = __ldg(s);
    }
  } else {
    for (int x = threadIdx.x; x < 2 * row_halves; x += blockDim.x) {
      const bool is_v = x >= row_halves;
      const int i = is_v ? x - row_halves : x;
      (is_v ? cache_v : cache_k)[dst + i] = (is_v ? draft_v : draft_k)[src + i];
    }
  }
}

// Page clone: blockIdx.y = clone index, blockIdx.z = 0 (K) / 1 (V); the page
// (16 * row_halves halves) is split over gridDim.x CTAs of 16-byte vectors.
__global__ void __launch_bounds__(256)
    clone_kernel(int page_halves, int physical_pages, __half* cache_k, __half* cache_v,
                 const int* __restrict__ src_pages, const int* __restrict__ dst_pages,
                 unsigned* err) {
  grid_launch_dependents();
  grid_dependency_wait();
  const int c = blockIdx.y;
  const int src = src_pages[c], dst = dst_pages[c];
  if (src < 0 || src >= physical_pages || dst < 0 || dst >= physical_pages) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.z == 0) atomicOr(err, kErrCommitIndex);
    return;
  }
  __half* base = blockIdx.z ? cache_v : cache_k;
  const uint4* s = reinterpret_cast<const uint4*>(base + size_t(src) * page_halves);
  uint4* d = reinterpret_cast<uint4*>(base + size_t(dst) * page_halves);
  const int n16 = page_halves / 8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += gridDim.x * blockDim.x)
    d[i] = s[i];
}

}  // namespace bc
