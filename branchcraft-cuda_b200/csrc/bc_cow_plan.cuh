// Device-side copy-on-write commit planner: the page bookkeeping of the
// reference's PagedTreeCache.commit (python/branchcraft_torch/transaction.py:
// 114-150) for a whole batch of requests, on the GPU, producing the plan that
// the batch commit (commit_batch_task) executes.
//
// State (device arrays, updated in place): refcount[P], a free-page stack
// free_stack[0 .. *free_count) whose top is the last entry (the reference's
// free list, popped from the end: lowest page id first after
// list(range(P-1, -1, -1)), pages released by append), and each request's
// page table row and length. Request b of the batch commits path_nodes[b, 0 ..
// path_len[b]) in batch order, exactly as sequential commits would:
//   * paths are validated first (non-empty, at most `nodes` long, node ids in
//     [0, nodes)); a bad one changes nothing (status 1, the reference's
//     ValueError);
//   * a partial last page that another reference shares (refcount > 1) is
//     cloned into a freshly popped page, which replaces it in the row; the old
//     page loses a reference (and returns to the stack at 0);
//   * pages are appended (popped) until the row covers the new length;
//   * the entries place the path's nodes at positions length .. length+L-1.
// The batch is all or nothing: when the free pages run out (the reference's
// RuntimeError) the state stays as it was (status 2). The simulation runs on
// one thread over copies of refcount and the stack in shared memory, so the
// pool holds at most kCowPlanMaxPages pages.
#pragma once

#include "bc_device.cuh"

namespace bc {

constexpr int kCowPlanMaxPages = 24576;  // refcount + stack in shared memory: 192 KB
constexpr int kCowPlanThreads = 256;

enum CowPlanStatus : int { kPlanOk = 0, kPlanBadPath = 1, kPlanExhausted = 2, kPlanBadTable = 3 };

struct CowPlanParams {
  int batch, nodes, physical_pages, max_pages_in, max_pages_out;
  const int* pages_in;    // [batch, max_pages_in] page table before the commit
  const int* lengths_in;  // [batch]
  const int* path_len;    // [batch]
  const int* path_nodes;  // [batch, nodes]
  int* refcount;          // [P]
  int* free_stack;        // [P]
  int* free_count;        // [1]
  int* pages_out;         // [batch, max_pages_out] page table after the commit (-1 past the end)
  int* lengths_out;       // [batch]
  int* clone_src;         // [batch]
  int* clone_dst;         // [batch]
  int* entry_request;     // [batch * nodes]
  int* entry_node;
  int* entry_page;
  int* entry_slot;
  int* counts;            // [3]: clones, entries, status
};

__global__ void __launch_bounds__(kCowPlanThreads)
    cow_plan_kernel(const __grid_constant__ CowPlanParams p) {
  extern __shared__ int plan_smem[];
  int* rc = plan_smem;                          // refcount copy
  int* stack = plan_smem + p.physical_pages;    // free-stack copy
  __shared__ int status;
  __shared__ int nfree;
  const int tid = threadIdx.x;
  const int P = p.physical_pages;
  grid_dependency_wait();  // the preceding kernel's state and inputs are visible
  if (tid == 0) {
    status = kPlanOk;
    nfree = *p.free_count;
    if (nfree < 0 || nfree > P) status = kPlanBadTable;
  }
  __syncthreads();
  // Validation (nothing is changed when a path or a table row is bad) and the
  // rows copied to the output table; the state into shared memory.
  for (int b = tid; b < p.batch; b += kCowPlanThreads) {
    const int L = p.path_len[b], len = p.lengths_in[b];
    if (L < 1 || L > p.nodes) atomicMax(&status, kPlanBadPath);
    for (int i = 0; i < L && i < p.nodes; ++i) {
      const int node = p.path_nodes[size_t(b) * p.nodes + i];
      if (node < 0 || node >= p.nodes) atomicMax(&status, kPlanBadPath);
    }
    const int n_old = (len + kPageSize - 1) / kPageSize;
    if (len < 0 || n_old > p.max_pages_in ||
        (max(len, 0) + max(L, 0) + kPageSize - 1) / kPageSize > p.max_pages_out)
      atomicMax(&status, kPlanBadTable);
    for (int j = 0; j < n_old && j < p.max_pages_in; ++j) {
      const int pg = p.pages_in[size_t(b) * p.max_pages_in + j];
      if (pg < 0 || pg >= P) atomicMax(&status, kPlanBadTable);
    }
  }
  for (int i = tid; i < P; i += kCowPlanThreads) {
    rc[i] = p.refcount[i];
    stack[i] = p.free_stack[i];
  }
  for (int e = tid; e < p.batch * p.max_pages_out; e += kCowPlanThreads) {
    const int b = e / p.max_pages_out, j = e % p.max_pages_out;
    const int n_old = (max(p.lengths_in[b], 0) + kPageSize - 1) / kPageSize;
    p.pages_out[e] = j < n_old && j < p.max_pages_in ? p.pages_in[size_t(b) * p.max_pages_in + j]
                                                     : -1;
  }
  __syncthreads();
  if (tid == 0 && status == kPlanOk) {
    // The sequential commits, on the shared-memory copies.
    int top = nfree, ncl = 0, nent = 0;
    for (int b = 0; b < p.batch && status == kPlanOk; ++b) {
      const int len = p.lengths_in[b], L = p.path_len[b];
      const int n_old = (len + kPageSize - 1) / kPageSize;
      const int n_new = (len + L + kPageSize - 1) / kPageSize;
      int* row = p.pages_out + size_t(b) * p.max_pages_out;
      const int last = n_old > 0 ? row[n_old - 1] : -1;
      const bool copy_partial = len % kPageSize != 0 && rc[last] > 1;
      if (top < n_new - n_old + (copy_partial ? 1 : 0)) {
        status = kPlanExhausted;
        break;
      }
      if (copy_partial) {
        const int fresh = stack[--top];
        rc[fresh] = 1;
        p.clone_src[ncl] = last;
        p.clone_dst[ncl] = fresh;
        ++ncl;
        row[n_old - 1] = fresh;
        if (--rc[last] == 0) stack[top++] = last;
      }
      for (int j = n_old; j < n_new; ++j) {
        const int pg = stack[--top];
        rc[pg] = 1;
        row[j] = pg;
      }
      for (int i = 0; i < L; ++i) {
        const int pos = len + i;
        p.entry_request[nent] = b;
        p.entry_node[nent] = p.path_nodes[size_t(b) * p.nodes + i];
        p.entry_page[nent] = row[pos / kPageSize];
        p.entry_slot[nent] = pos % kPageSize;
        ++nent;
      }
      p.lengths_out[b] = len + L;
    }
    if (status == kPlanOk) {
      nfree = top;
      p.counts[0] = ncl;
      p.counts[1] = nent;
    }
  }
  __syncthreads();
  if (status == kPlanOk) {  // the new state
    for (int i = tid; i < P; i += kCowPlanThreads) {
      p.refcount[i] = rc[i];
      p.free_stack[i] = stack[i];
    }
    if (tid == 0) *p.free_count = nfree;
  } else if (tid == 0) {  // nothing to execute
    p.counts[0] = 0;
    p.counts[1] = 0;
  }
  if (tid == 0) p.counts[2] = status;
}

}  // namespace bc
