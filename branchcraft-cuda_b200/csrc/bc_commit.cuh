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

// Shared-memory scratch of one batch-commit task.
struct CommitScratch {
  unsigned skip;     // clone task: slots this task must not copy
  int ntargets;      // entry task: clones that take the slot's old contents
  int targets[256];
  unsigned char own[256];
};

// The batch copy-on-write commit, with the semantics of all clones first and
// then every row commit (transaction.py:114-150 per request, in request
// order), as independent tasks: tasks [0, 8 * nclones) copy a quarter page of
// K or V of one clone; task 8 * nclones + e writes commit entry e's K and V
// rows. The bytes are partitioned so that no task waits for another:
//   - a clone task skips the slots the destination's own entries write and
//     the slots that entries write in place into the clone's source page;
//   - the task of an entry writing in place into a clone source first copies
//     the slot's old contents into each clone of that page that has no entry
//     of its own for the slot, then writes its row (per 16-byte vector, the
//     read precedes the write in the same thread).
// Run by NT threads (thread index t) that `sync()` synchronises.
template <int NT, typename Sync>
__device__ __forceinline__ void commit_batch_task(
    int task, int t, Sync sync, CommitScratch& sc, int row_halves, int batch, int nodes,
    int physical_pages, const __half* __restrict__ draft_k, const __half* __restrict__ draft_v,
    __half* cache_k, __half* cache_v, const int* __restrict__ clone_src,
    const int* __restrict__ clone_dst, int nclones, const int* __restrict__ req,
    const int* __restrict__ path, const int* __restrict__ dest_pages,
    const int* __restrict__ dest_slots, int nentries, unsigned* err) {
  const int n16 = row_halves / 8;  // 16-byte vectors per slot row
  // An entry with any index out of range writes nothing (its task only sets
  // the error bit), so it neither claims a slot nor takes part in a clone.
  auto valid = [&](int f) {
    const int r = req[f], nd = path[f], pg = dest_pages[f], sl = dest_slots[f];
    return r >= 0 && r < batch && nd >= 0 && nd < nodes && pg >= 0 && pg < physical_pages &&
           sl >= 0 && sl < 16;
  };
  if (t == 0) {
    sc.skip = 0u;
    sc.ntargets = 0;
  }
  sync();
  if (task < 8 * nclones) {
    const int c = task >> 3, part = (task >> 1) & 3, kv = task & 1;
    const int src = clone_src[c], dst = clone_dst[c];
    const bool bad = src < 0 || src >= physical_pages || dst < 0 || dst >= physical_pages;
    if (bad) {
      if (t == 0 && part == 0 && kv == 0) atomicOr(err, kErrCommitIndex);
    } else {
      for (int e = t; e < nentries; e += NT) {
        const int pg = dest_pages[e], sl = dest_slots[e];
        if ((pg == dst || pg == src) && valid(e)) atomicOr(&sc.skip, 1u << sl);
      }
      if (part == 0 && kv == 0) {
        // The plan's contract: clone destinations are distinct and none is a
        // clone source (else the partitioned copies would race). A broken
        // contract is reported, not repaired.
        for (int o = t; o < nclones; o += NT)
          if (clone_src[o] == dst || (o != c && clone_dst[o] == dst)) atomicOr(err, kErrCommitIndex);
      }
    }
    sync();
    if (!bad) {
      __half* base = kv ? cache_v : cache_k;
      const uint4* sp = reinterpret_cast<const uint4*>(base + size_t(src) * 16 * row_halves);
      uint4* dp = reinterpret_cast<uint4*>(base + size_t(dst) * 16 * row_halves);
      for (int x = t; x < 4 * n16; x += NT) {
        const int sl = part * 4 + x / n16;
        if (!((sc.skip >> sl) & 1u)) dp[size_t(sl) * n16 + x % n16] = sp[size_t(sl) * n16 + x % n16];
      }
    }
    sync();  // (the scratch is reused by the caller's next task)
    return;
  }
  const int e = task - 8 * nclones;
  const int r = req[e], node = path[e], page = dest_pages[e], slot = dest_slots[e];
  const bool bad = r < 0 || r >= batch || node < 0 || node >= nodes || page < 0 ||
                   page >= physical_pages || slot < 0 || slot >= 16;
  if (bad) {
    if (t == 0) atomicOr(err, kErrCommitIndex);
    sync();
    sync();
    sync();
    return;
  }
  // Clones of this page that keep the slot's old contents: the page's clones
  // (shared memory list), minus those with an entry of their own at this
  // slot (entries scanned in parallel, one load per thread and entry).
  for (int c = t; c < nclones; c += NT) {
    const int dst = clone_dst[c];
    if (clone_src[c] == page && dst >= 0 && dst < physical_pages) {
      const int k = atomicAdd(&sc.ntargets, 1);
      sc.targets[k] = dst;  // nclones <= 256 (host)
      sc.own[k] = 0;
    }
  }
  sync();
  const int ncand = sc.ntargets;
  if (ncand > 0) {
    for (int f = t; f < nentries; f += NT) {
      if (dest_slots[f] != slot || !valid(f)) continue;
      const int pg = dest_pages[f];
      for (int k = 0; k < ncand; ++k)
        if (sc.targets[k] == pg) sc.own[k] = 1;
    }
  }
  sync();
  if (t == 0 && ncand > 0) {  // keep the clones without an entry of their own
    int n = 0;
    for (int k = 0; k < ncand; ++k)
      if (!sc.own[k]) sc.targets[n++] = sc.targets[k];
    sc.ntargets = n;
  }
  sync();
  const int nt = sc.ntargets;
  const size_t src_row = (size_t(r) * nodes + node) * n16;
  for (int x = t; x < 2 * n16; x += NT) {
    const bool is_v = x >= n16;
    const int i = is_v ? x - n16 : x;
    uint4* cache = reinterpret_cast<uint4*>(is_v ? cache_v : cache_k);
    const size_t at = (size_t(page) * 16 + slot) * n16 + i;
    if (nt > 0) {
      const uint4 old = cache[at];
      for (int k = 0; k < nt; ++k) cache[(size_t(sc.targets[k]) * 16 + slot) * n16 + i] = old;
    }
    cache[at] = __ldg(reinterpret_cast<const uint4*>(is_v ? draft_v : draft_k) + src_row + i);
  }
  sync();  // (the scratch is reused by the caller's next task)
}

// A whole batch of copy-on-write commits in one launch: CTA b runs task b
// (commit_batch_task) with its 256 threads.
__global__ void __launch_bounds__(256)
    commit_batch_kernel(int row_halves, int batch, int nodes, int physical_pages,
                        const __half* __restrict__ draft_k, const __half* __restrict__ draft_v,
                        __half* cache_k, __half* cache_v, const int* __restrict__ clone_src,
                        const int* __restrict__ clone_dst, int nclones,
                        const int* __restrict__ req, const int* __restrict__ path,
                        const int* __restrict__ dest_pages, const int* __restrict__ dest_slots,
                        int nentries, unsigned* err) {
  // One wave: the next kernel may be scheduled at once (it waits for this grid).
  grid_launch_dependents();
  grid_dependency_wait();
  __shared__ CommitScratch sc;
  commit_batch_task<256>(int(blockIdx.x), int(threadIdx.x), [] { __syncthreads(); }, sc,
                         row_halves, batch, nodes, physical_pages, draft_k, draft_v, cache_k,
                         cache_v, clone_src, clone_dst, nclones, req, path, dest_pages,
                         dest_slots, nentries, err);
}

}  // namespace bc
