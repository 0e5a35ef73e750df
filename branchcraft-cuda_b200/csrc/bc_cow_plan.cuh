// Device-side copy-on-write commit planner: the page bookkeeping of the
// reference's PagedTreeCache.commit (python/branchcraft_torch/transaction.py:
// 114-150) for a whole batch of requests, on the GPU, producing the plan that
// the batch commit (commit_batch_task) executes.
//
// State (device arrays, read from the *_in arrays and written to the others,
// which may be the same): refcount[P], a free-page stack
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
// RuntimeError) the state stays as it was (status 2). The plan is computed in
// parallel (cow_plan_run) with O(batch) shared memory; the batch holds at most
// kCowPlanMaxBatch requests.
#pragma once

#include "bc_device.cuh"

namespace bc {

constexpr int kCowPlanMaxBatch = 256;
constexpr int kCowPlanMaxNodes = 256;  // the node cap of the entry points
constexpr int kCowPlanMaxNew = kCowPlanMaxNodes / kPageSize + 1;  // pages a commit can add
constexpr int kCowPlanThreads = 256;

enum CowPlanStatus : int { kPlanOk = 0, kPlanBadPath = 1, kPlanExhausted = 2, kPlanBadTable = 3 };

// (pages_in, lengths_in, path_len and path_nodes are read-only for the run:
// no output array may alias them; the state arrays may be updated in place)
struct CowPlanParams {
  int batch, nodes, physical_pages, max_pages_in, max_pages_out;
  const int* pages_in;    // [batch, max_pages_in] page table before the commit
  const int* lengths_in;  // [batch]
  const int* path_len;    // [batch]
  const int* path_nodes;  // [batch, nodes]
  const int* refcount_in;    // [P] state before the batch
  const int* free_stack_in;  // [P]
  const int* free_count_in;  // [1]
  int* refcount;             // [P] state after it (may be the same arrays)
  int* free_stack;           // [P]
  int* free_count;           // [1]
  int* pages_out;         // [batch, max_pages_out] page table after the commit (-1 past the end)
  int* lengths_out;       // [batch]
  int* clone_src;         // [batch]
  int* clone_dst;         // [batch]
  int* entry_request;     // [batch * nodes]
  int* entry_node;
  int* entry_page;
  int* entry_slot;
  int* counts;            // [3]: clones, entries, status ([3], [4]: see plan_flag_arrive)
};

// Shared memory of one planner run: four scalars, then per request its
// length, path length, last page, clone flag, pops, first pop, first clone
// and first entry, then the window of the free stack the batch can pop.
__host__ __device__ inline size_t cow_plan_smem_bytes(int batch) {
  return (4 + size_t(batch) * (8 + 1 + kCowPlanMaxNew)) * sizeof(int);
}

// The planner run by NT threads (index t) that `sync()` synchronises, over
// `sm` (cow_plan_smem_bytes of shared memory). Returns the status.
//
// The sequential commits are computed in parallel. A commit clones the last
// page of request b exactly when that page is partial and still shared at b's
// turn; the holders of a shared partial page all have the same length (a
// commit into such a page always clones it first), and each clone drops one
// reference, so among the batch's requests with the same last page the first
// refcount - 1 (in batch order) clone it and the rest write in place. A clone
// therefore never frees its page (its refcount stays >= 1) and nothing is
// pushed on the free stack: the batch's pops, in request order (the clone
// first, then the appended pages), are the stack entries below its top, at
// offsets given by a prefix sum of each request's pop count.
// A plan made inside the verification launch is published through
// counts[3] (0: not yet, 1: published); each of the launch's `participants`
// (the planning CTA and every CTA that waited for the flag) then arrives
// here once, after its last read of the flag, and the last one resets
// counts[3] and counts[4] to zero: the words are zero again when the launch
// ends, whatever the order in which the CTAs ran.
__device__ __forceinline__ void plan_flag_arrive(int* counts, int participants) {
  if (atom_add_acq_rel_gpu(counts + 4, 1) == participants - 1) {
    counts[3] = 0;
    counts[4] = 0;
  }
}

template <int NT, typename Sync>
__device__ __forceinline__ int cow_plan_run(const CowPlanParams& p, int t, Sync sync, int* sm) {
  const int B = p.batch, P = p.physical_pages;
  int& status = sm[0];
  int& top0 = sm[1];     // free pages before the batch
  int& total = sm[2];    // pages the batch pops
  int& window = sm[3];   // free-stack entries read (an upper bound of the pops)
  int* s_len = sm + 4;   // [B] lengths before the commit
  int* s_plen = s_len + B;
  int* s_last = s_plen + B;   // last page (-1: none)
  int* s_clone = s_last + B;  // 1: the last page is cloned
  int* s_pops = s_clone + B;  // pages popped (clone + appended)
  int* s_off = s_pops + B;    // pops of the requests before
  int* s_coff = s_off + B;    // clones of the requests before
  int* s_eoff = s_coff + B;   // entries of the requests before
  int* s_win = s_eoff + B;    // free_stack_in[top0 - window .. top0)
  if (t == 0) {
    status = kPlanOk;
    total = 0;
    window = 0;
  }
  for (int b = t; b < B; b += NT) s_last[b] = -1;
  sync();
  // First pass of loads (all independent): lengths, path lengths and nodes, the
  // free count, the page rows (copied to the output table; the row's last
  // page kept), and the state copied to the output arrays when they differ.
  if (t == 0) {
    const int nf = *p.free_count_in;
    top0 = nf;
    if (nf < 0 || nf > P) atomicMax(&status, kPlanBadTable);
  }
  for (int b = t; b < B; b += NT) {
    const int L = __ldg(p.path_len + b), len = __ldg(p.lengths_in + b);
    s_len[b] = len;
    s_plen[b] = L;
    if (L < 1 || L > p.nodes) atomicMax(&status, kPlanBadPath);
    const int n_old = (len + kPageSize - 1) / kPageSize;
    const int n_new = (max(len, 0) + max(L, 0) + kPageSize - 1) / kPageSize;
    if (len < 0 || n_old > p.max_pages_in || n_new > p.max_pages_out)
      atomicMax(&status, kPlanBadTable);
    atomicAdd(&window, 1 + max(n_new - max(n_old, 0), 0));
  }
  const int ne = B * p.nodes;
  const int h0 = t < ne ? __ldg(p.path_nodes + t) : -1;
  const int h1 = t + NT < ne ? __ldg(p.path_nodes + t + NT) : -1;
  const int h2 = t + 2 * NT < ne ? __ldg(p.path_nodes + t + 2 * NT) : -1;
  const int h3 = t + 3 * NT < ne ? __ldg(p.path_nodes + t + 3 * NT) : -1;
  auto held = [&](int e) {  // entry e's node (e = t + k * NT)
    const int k = e / NT;
    return k == 0 ? h0 : k == 1 ? h1 : k == 2 ? h2 : k == 3 ? h3 : __ldg(p.path_nodes + e);
  };
  for (int e = t; e < ne; e += NT) {
    const int node = held(e);
    if (e % p.nodes < __ldg(p.path_len + e / p.nodes) && (node < 0 || node >= p.nodes))
      atomicMax(&status, kPlanBadPath);
  }
  constexpr int kBatch = 8;  // loads issued together, then used
  const int n_rows = B * p.max_pages_out;
  for (int base = t; base < n_rows; base += NT * kBatch) {
    int len[kBatch], in[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int e = base + k * NT;
      const int b = e / p.max_pages_out, j = e % p.max_pages_out;
      len[k] = e < n_rows ? __ldg(p.lengths_in + b) : 0;
      in[k] = e < n_rows && j < p.max_pages_in
                  ? __ldg(p.pages_in + size_t(b) * p.max_pages_in + j) : -1;
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int e = base + k * NT;
      if (e >= n_rows) break;
      const int b = e / p.max_pages_out, j = e % p.max_pages_out;
      const int n_old = (max(len[k], 0) + kPageSize - 1) / kPageSize;
      int pg = -1;
      if (j < n_old && j < p.max_pages_in) {
        pg = in[k];
        if (pg < 0 || pg >= P) atomicMax(&status, kPlanBadTable);
        if (j == n_old - 1) s_last[b] = pg;
      }
      p.pages_out[e] = pg;
    }
  }
  if (p.refcount != p.refcount_in || p.free_stack != p.free_stack_in) {
    // (out of place: the state after starts as the state before)
    for (int base = t; base < P; base += NT * kBatch) {
      int a[kBatch], c[kBatch];
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int i = base + k * NT;
        a[k] = i < P ? p.refcount_in[i] : 0;
        c[k] = i < P ? p.free_stack_in[i] : 0;
      }
#pragma unroll
      for (int k = 0; k < kBatch; ++k) {
        const int i = base + k * NT;
        if (i < P) {
          p.refcount[i] = a[k];
          p.free_stack[i] = c[k];
        }
      }
    }
  }
  sync();
  // Second pass: each request's clone decision (its last page's refcount and its
  // rank among the batch's requests with the same last page), and the window
  // of the stack the batch can pop.
  const int win = min(window, max(top0, 0));
  if (status == kPlanOk) {
    for (int b = t; b < B; b += NT) {
      const int len = s_len[b], last = s_last[b];
      int clone = 0;
      if (len % kPageSize != 0 && last >= 0) {
        int rank = 0;
        for (int o = 0; o < b; ++o) rank += s_last[o] == last ? 1 : 0;
        clone = rank < p.refcount_in[last] - 1 ? 1 : 0;
      }
      const int n_old = (len + kPageSize - 1) / kPageSize;
      const int n_new = (len + s_plen[b] + kPageSize - 1) / kPageSize;
      s_clone[b] = clone;
      s_pops[b] = clone + n_new - n_old;
    }
    for (int i = t; i < win; i += NT) s_win[i] = p.free_stack_in[top0 - win + i];
  }
  sync();
  if (t == 0 && status == kPlanOk) {  // prefix sums over the requests
    int pops = 0, clones = 0, entries = 0;
    for (int b = 0; b < B; ++b) {
      s_off[b] = pops;
      s_coff[b] = clones;
      s_eoff[b] = entries;
      pops += s_pops[b];
      clones += s_clone[b];
      entries += s_plen[b];
    }
    total = pops;
    if (pops > top0) {
      status = kPlanExhausted;
    } else {
      p.counts[0] = clones;
      p.counts[1] = entries;
    }
  }
  sync();
  const int st = status;
  if (st == kPlanOk) {
    // The k-th page request b pops is the stack entry top0 - 1 - (off_b + k),
    // i.e. s_win[win - 1 - (off_b + k)].
    auto popped = [&](int b, int k) { return s_win[win - 1 - (s_off[b] + k)]; };
    for (int b = t; b < B; b += NT) {
      const int len = s_len[b], L = s_plen[b];
      const int n_old = (len + kPageSize - 1) / kPageSize;
      const int n_new = (len + L + kPageSize - 1) / kPageSize;
      int* row = p.pages_out + size_t(b) * p.max_pages_out;
      if (s_clone[b]) {
        const int fresh = popped(b, 0);
        row[n_old - 1] = fresh;
        p.clone_src[s_coff[b]] = s_last[b];
        p.clone_dst[s_coff[b]] = fresh;
        p.refcount[fresh] = 1;
        atomicSub(p.refcount + s_last[b], 1);
      }
      for (int j = n_old; j < n_new; ++j) {
        const int pg = popped(b, s_clone[b] + (j - n_old));
        row[j] = pg;
        p.refcount[pg] = 1;
      }
      p.lengths_out[b] = len + L;
    }
    for (int e = t; e < ne; e += NT) {
      const int b = e / p.nodes, i = e % p.nodes;
      if (i >= s_plen[b]) continue;
      const int len = s_len[b];
      const int n_old = (len + kPageSize - 1) / kPageSize;
      const int pos = len + i, pj = pos / kPageSize;
      int page;
      if (pj >= n_old) page = popped(b, s_clone[b] + (pj - n_old));
      else if (pj == n_old - 1) page = s_clone[b] ? popped(b, 0) : s_last[b];
      else page = __ldg(p.pages_in + size_t(b) * p.max_pages_in + pj);  // (a full page: never written)
      const int k = s_eoff[b] + i;
      p.entry_request[k] = b;
      p.entry_node[k] = held(e);
      p.entry_page[k] = page;
      p.entry_slot[k] = pos % kPageSize;
    }
    if (t == 0) *p.free_count = top0 - total;
  } else if (t == 0) {  // nothing to execute; the state after is the state before
    *p.free_count = *p.free_count_in;
    p.counts[0] = 0;
    p.counts[1] = 0;
  }
  if (t == 0) p.counts[2] = st;
  return st;
}

__global__ void __launch_bounds__(kCowPlanThreads)
    cow_plan_kernel(const __grid_constant__ CowPlanParams p) {
  extern __shared__ int plan_smem[];
  // The next kernel (the verify launch that executes this plan) may be
  // scheduled now: it runs its set-up, then waits for this grid.
  grid_launch_dependents();
  grid_dependency_wait();  // the preceding kernel's state and inputs are visible
  cow_plan_run<kCowPlanThreads>(p, int(threadIdx.x), [] { __syncthreads(); }, plan_smem);
}

}  // namespace bc
