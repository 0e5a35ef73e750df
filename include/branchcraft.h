/* branchcraft (B200 / sm_100a) — C ABI of the attention-over-paged-KV hot path.
 *
 * Every entry point takes plain pointers and sizes, launches on the caller's
 * stream (NULL = legacy default stream), allocates nothing (except
 * bc_exchange_create, which makes the multi-GPU exchange buffer) and returns a
 * cudaError_t value: 0 on success, cudaErrorInvalidValue (1) for rejected
 * arguments, otherwise the launch status. Asynchronous device faults surface at
 * the caller's next synchronisation, as with any CUDA launch.
 *
 * All tensor pointers are DEVICE pointers. FP16 data is IEEE binary16; pass it
 * as `const void*`. Layouts (row-major, innermost last):
 *   q        [batch, query_heads, dim]                 (decode)
 *   draft_q  [batch, nodes, query_heads, dim]          (tree verify)
 *   k, v     [physical_pages, 16, kv_heads, dim]       (paged cache)
 *   pages    [batch, max_pages] int32, lengths [batch] int32
 *   draft_k, draft_v [batch, nodes, kv_heads, dim], parent [batch, nodes]
 *
 * Malformed indices found on the device (page ids outside [0, physical_pages),
 * lengths outside [0, max_pages*16], cyclic or out-of-range parent pointers,
 * commit destinations out of range) never fault: the access is skipped (a
 * page outside the pool reads as zeros) and a bit is set in a per-device error
 * word that bc_last_device_error() returns.
 *
 * The library keeps, per device and for the life of the process, the device
 * addresses of its own `__device__` variables (the error word and the fixed
 * array of bc_decode_static_scratch). They belong to the device's primary
 * context: do not use the library on a device across cudaDeviceReset().
 */
#ifndef BRANCHCRAFT_H_
#define BRANCHCRAFT_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BC_PAGE_SIZE 16
#define BC_MAX_SPLITS 64
#define BC_MAX_NODES 256

/* Mirrors branchcraft::Shape (reference include/branchcraft.hpp:11-18). */
typedef struct bc_shape {
  int batch;
  int query_heads;
  int kv_heads;
  int dim; /* 64 or 128 */
  int max_pages;
  int physical_pages;
} bc_shape;

/* Device error bits returned by bc_last_device_error(). */
#define BC_ERR_PAGE_RANGE 1u
#define BC_ERR_LENGTH 2u
#define BC_ERR_PARENT 4u
#define BC_ERR_TIMEOUT 8u
#define BC_ERR_COMMIT_INDEX 16u

/* Paged GQA split-KV decode with FP32 output [batch, query_heads, dim]; empty
 * sequences give zeros. Replaces branchcraft::decode (reference
 * include/branchcraft.hpp:39-40, src/paged_gqa.cu:122-132).
 * splits in [1, BC_MAX_SPLITS] (the reference caps at 16). For splits > 1 the
 * caller provides scratch exactly as the reference documents
 * (include/branchcraft.hpp:32-36): partial_a = splits*B*Hq*D floats,
 * partial_ml = splits*B*Hq*2 floats; both NULL is rejected for splits > 1.
 * Splits <= 8 are merged on chip between the CTAs of one thread-block cluster
 * and leave the scratch untouched; larger counts go through the scratch and a
 * second (merge) launch. */
int bc_decode(const bc_shape* shape, const void* q, const void* k, const void* v,
              const int* pages, const int* lengths, float* output, float* partial_a,
              float* partial_ml, int splits, void* stream);

/* Split-count heuristic for bc_decode. Replaces branchcraft::auto_splits
 * (reference include/branchcraft.hpp:41, src/paged_gqa.cu:134-142), retuned for
 * this kernel's CTA shape (one CTA per request and KV head): the largest count,
 * at most 64 and leaving each split >= 256 keys, whose CTAs fit one wave of two
 * per SM. */
int bc_auto_splits(const bc_shape* shape, int max_length, int sm_count);

/* Paged decode with the split count chosen by the library (splits <= 0) or
 * given (1..8), merged on chip: needs no scratch. Not in the reference; backs
 * the added `paged_decode` torch schema. */
int bc_paged_decode(const bc_shape* shape, const void* q, const void* k, const void* v,
                    const int* pages, const int* lengths, float* output, int splits,
                    void* stream);

/* Ancestor-only tree verification: every (request, node, q-head) attends to the
 * request's paged prefix and to its own root-to-node chain of draft tokens
 * (never siblings), scale 1/sqrt(dim). FP32 output [batch, nodes, Hq, D].
 * nodes in [1, BC_MAX_NODES]. Parent pointers: -1 (root) or a node index;
 * chains longer than `nodes` (cycles) and indices >= nodes set BC_ERR_PARENT.
 * Replaces branchcraft::tree_verify (reference include/branchcraft.hpp:43-56,
 * src/tree_attention.cu:93-105). shape->physical_pages bounds the page ids. */
int bc_tree_verify(const bc_shape* shape, const void* draft_q, const void* prefix_k,
                   const void* prefix_v, const int* pages, const int* lengths,
                   const void* draft_k, const void* draft_v, const int* parent,
                   float* output, int nodes, void* stream);

/* As bc_tree_verify with FP16 output [batch, nodes, Hq, D] (FP32 accumulation,
 * one rounding at the end). Not in the reference. */
int bc_tree_verify_f16(const bc_shape* shape, const void* draft_q, const void* prefix_k,
                       const void* prefix_v, const int* pages, const int* lengths,
                       const void* draft_k, const void* draft_v, const int* parent,
                       void* output_f16, int nodes, void* stream);

/* Copy accepted draft nodes into physical KV slots:
 * cache_{k,v}[dest_pages[i], dest_slots[i], :, :] =
 *     draft_{k,v}[request, path_nodes[i], :, :]   for i < accepted.
 * path_nodes / dest_pages / dest_slots are device arrays of length `accepted`.
 * The caller updates page tables afterwards. Replaces branchcraft::commit_path
 * (reference include/branchcraft.hpp:58-65, src/tree_attention.cu:107-122);
 * shape->kv_heads, dim, batch and physical_pages are used. */
int bc_commit_path(const bc_shape* shape, const void* draft_k, const void* draft_v,
                   void* cache_k, void* cache_v, const int* path_nodes,
                   const int* dest_pages, const int* dest_slots, int request, int nodes,
                   int accepted, void* stream);

/* A whole batch of copy-on-write commits in one call: first every page clone
 * cache[clone_dst[c]] = cache[clone_src[c]] (K and V, all 16 slots), then every
 * entry cache[entry_page[e], entry_slot[e]] = draft[entry_request[e],
 * entry_node[e]]. All index arrays are device arrays; clone destinations are
 * distinct pages that are neither clone sources nor written by two entries at
 * the same slot. One kernel launch for up to 256 clones (the bytes each clone
 * and entry touch are partitioned, so the clones-first order needs no
 * ordering between CTAs), two beyond. Not in the reference; it is the device
 * half of PagedTreeCache.commit (python/branchcraft_torch/transaction.py:114-150)
 * for many requests. */
int bc_commit_batch(const bc_shape* shape, int nodes, const void* draft_k,
                    const void* draft_v, void* cache_k, void* cache_v, const int* clone_src,
                    const int* clone_dst, int nclones, const int* entry_request,
                    const int* entry_node, const int* entry_page, const int* entry_slot,
                    int nentries, void* stream);

/* One speculative-verification step in ONE launch: bc_tree_verify (FP32
 * output, or FP16 with output_f16 != 0) over cache_k / cache_v, and the batch
 * copy-on-write commit of bc_commit_batch (same arrays and semantics, at most
 * 256 clones) into the same cache. The commit runs concurrently with the
 * verification, so the call requires what a copy-on-write plan guarantees
 * (bc_cow.PagePool, the reference's PagedTreeCache.commit,
 * python/branchcraft_torch/transaction.py:114-150): the commit writes only
 * fresh pages (clone destinations, pages no page table of this call holds)
 * and, in place, slots at or past the length of every request whose table
 * holds that page — bytes no verified row depends on. The verification then
 * sees the cache as it was before the commit. Not in the reference (whose
 * step is tree_verify, then per request a page copy and commit_path). */
int bc_tree_verify_commit(const bc_shape* shape, const void* draft_q, void* cache_k,
                          void* cache_v, const int* pages, const int* lengths,
                          const void* draft_k, const void* draft_v, const int* parent,
                          void* output, int output_f16, int nodes, const int* clone_src,
                          const int* clone_dst, int nclones, const int* entry_request,
                          const int* entry_node, const int* entry_page, const int* entry_slot,
                          int nentries, void* stream);

/* The page bookkeeping of a batch of copy-on-write commits, on the device:
 * the refcount / free-list / clone decisions of the reference's
 * PagedTreeCache.commit (python/branchcraft_torch/transaction.py:114-150),
 * request b committing path_nodes[b, 0 .. path_len[b]) in batch order.
 * State: refcount[P], free_stack[0 .. *free_count) (the free list; its last
 * entry is popped first, released pages are pushed), read from the *_in
 * arrays and written to refcount / free_stack / free_count (the same arrays
 * for an update in place, or others to keep the state before), and, per
 * request, pages_in [batch, max_pages_in] / lengths_in [batch] (read).
 * Writes the page tables after the commit (pages_out [batch, max_pages_out],
 * -1 past each row's end; lengths_out), the plan — clone_src / clone_dst
 * (capacity batch) and entry_request / entry_node / entry_page / entry_slot
 * (capacity batch*nodes), in bc_commit_batch's format — and counts[0..2] =
 * (clones, entries, status). status 0: planned; 1: a path empty, longer than
 * `nodes` or with a node id out of range; 2: not enough free pages (the
 * reference's RuntimeError); 3: a malformed table or length. On a nonzero
 * status the state written equals the state read and the plan is empty. batch
 * at most 256. One single-CTA launch. Not in the reference (whose bookkeeping
 * is host Python). */
int bc_cow_plan(int batch, int nodes, int physical_pages, const int* pages_in,
                int max_pages_in, const int* lengths_in, const int* path_len,
                const int* path_nodes, const int* refcount_in, const int* free_stack_in,
                const int* free_count_in, int* refcount, int* free_stack, int* free_count,
                int* pages_out, int max_pages_out, int* lengths_out, int* clone_src,
                int* clone_dst, int* entry_request, int* entry_node, int* entry_page,
                int* entry_slot, int* counts, void* stream);

/* A whole speculative-verification step with no host round trip: the
 * bc_cow_plan bookkeeping of the batch's accepted paths, then the verification
 * with the planned commit executed in the same launch, as
 * bc_tree_verify_commit does (a nonzero planner status commits nothing).
 * When the verify grid, with one more cluster, is still one wave, that
 * extra cluster of the verify launch makes the plan and publishes it to the
 * others through counts[3], counting the CTAs that have read it in counts[4]
 * (so counts holds 5 ints; start [3] and [4] at zero: the launch leaves them
 * at zero, so a captured graph may be replayed); otherwise a planner launch
 * runs first. `pages` / `lengths` are the tables before the commit
 * (what the verification reads); the tables after it go to pages_out /
 * lengths_out. shape->batch at most 256. Not in the reference. */
int bc_tree_step(const bc_shape* shape, const void* draft_q, void* cache_k, void* cache_v,
                 const int* pages, const int* lengths, const void* draft_k, const void* draft_v,
                 const int* parent, void* output, int output_f16, int nodes,
                 const int* path_len, const int* path_nodes, const int* refcount_in,
                 const int* free_stack_in, const int* free_count_in, int* refcount,
                 int* free_stack, int* free_count, int* pages_out, int max_pages_out,
                 int* lengths_out, int* clone_src, int* clone_dst, int* entry_request,
                 int* entry_node, int* entry_page, int* entry_slot, int* counts, void* stream);

/* Decode straight from a packed cache with logical shape [P, Hkv, 16, 2D]:
 * K of (page, kv head, slot) starts at page*block_stride + head*head_stride +
 * slot*slot_stride elements and V at D elements after it; caller-supplied
 * softmax scale; FP16 output [B, Hq, D], FP32 accumulation. Replaces
 * branchcraft::packed_decode (reference include/branchcraft.hpp:67-74,
 * src/packed_decode.cu:64-82). Strides must be multiples of 8 elements and the
 * cache 16-byte aligned (the TMA rule); other strides are rejected. */
int bc_packed_decode(const bc_shape* shape, const void* q, const void* packed_kv,
                     const int* pages, const int* lengths, void* output,
                     long long block_stride, long long head_stride, long long slot_stride,
                     float scale, void* stream);

/* As bc_packed_decode with an explicit K->V element offset (vLLM's
 * [num_blocks, 2, 16, Hkv, D] cache: block_stride = 2*16*Hkv*D,
 * head_stride = D, slot_stride = Hkv*D, kv_offset = 16*Hkv*D) and a split
 * count (<= 0: chosen by the library; 1..8: merged on chip). Not in the
 * reference. */
int bc_packed_decode_kv(const bc_shape* shape, const void* q, const void* packed_kv,
                        const int* pages, const int* lengths, void* output,
                        long long block_stride, long long head_stride,
                        long long slot_stride, long long kv_offset, float scale, int splits,
                        void* stream);

/* FP32 merge of split partial states into out [rows, dim]:
 * partial_ml[(s*rows + r)*2 + {0,1}] = (m, l), m the natural-log running max,
 * partial_a[(s*rows + r)*dim + d] the unnormalised accumulator. Rows whose m
 * are all -inf give zeros. The same math as the reference merge_kernel
 * (src/paged_gqa.cu:76-106); used after an all-gather of per-GPU partials. */
int bc_merge_partials(int splits, int rows, int dim, const float* partial_ml,
                      const float* partial_a, float* out, void* stream);

/* As bc_merge_partials, but storing the merged STATE instead of the
 * normalised rows: out_ml[r*2 + {0,1}] = (M, L) and out_a[r*dim + d] the
 * unnormalised accumulator, each partial weighted by exp(m_s - M) — one
 * partial per row, in the layout the merge entry points read (rows whose m
 * are all -inf give M = -inf, L = 0 and zeros). A GPU holding one shard of a
 * context split reduces its many on-device splits to this one partial before
 * the all-gather, so the exchange carries rows*(dim+2) floats per rank. Not
 * in the reference; the math is its merge_kernel's (src/paged_gqa.cu:76-106). */
int bc_merge_to_partial(int splits, int rows, int dim, const float* partial_ml,
                        const float* partial_a, float* out_ml, float* out_a, void* stream);

/* bc_merge_partials over partials gathered from `world` GPUs in ONE buffer:
 * gathered holds `world` blocks back to back, block r being rank r's
 * bc_paged_decode_partial output with partial_ml and partial_a placed in one
 * allocation: splits*rows*2 (m, l) floats, then splits*rows*dim accumulator
 * floats. A single all-gather of each rank's block then feeds the merge of
 * world*splits partials into out [rows, dim]. Not in the reference; the merge
 * math is the reference merge_kernel's (src/paged_gqa.cu:76-106). */
int bc_merge_gathered(int world, int splits, int rows, int dim, const float* gathered,
                      float* out, void* stream);

/* The context-split merge fused with its exchange over peer memory, for one
 * process per GPU on GPUs with peer access (NVLink / NVSwitch): each rank's
 * kernel reduces its `splits` local partials per row (bc_paged_decode_partial
 * layout) to one state, writes it into every rank's exchange buffer with
 * peer stores, raises a flag per block of 4 rows in each, waits (at most 1 s,
 * then BC_ERR_TIMEOUT and zero rows) for the other ranks' flags, and merges
 * the world's states into out [rows, dim] — the same result on every rank, no
 * collective library call. Set up once per (world, rows, dim):
 * bc_exchange_create allocates this rank's buffer of bc_exchange_bytes (the
 * one allocation of this library; zeroed) and returns its CUDA IPC handle (64
 * bytes); the ranks exchange handles (any host channel), bc_exchange_open
 * maps each peer's buffer, and peer_buffers is a DEVICE array of the world's
 * buffer pointers in rank order (this rank's own buffer at `rank`). Every
 * rank calls bc_merge_exchange with the same epoch, counting up from 1 per
 * call; after a BC_ERR_TIMEOUT the ranks' buffers may hold a half-published
 * epoch: tear the exchange down and create it again. Teardown after every
 * rank's last call: bc_exchange_close of the
 * mapped peers, bc_exchange_destroy of the own buffer. world at most
 * BC_MAX_EXCHANGE_RANKS. Not in the reference (which has no multi-GPU path);
 * the merge math is its merge_kernel's (src/paged_gqa.cu:76-106). */
#define BC_MAX_EXCHANGE_RANKS 64
size_t bc_exchange_bytes(int world, int rows, int dim);
int bc_exchange_create(int world, int rows, int dim, void** buffer, void* ipc_handle);
int bc_exchange_open(const void* ipc_handle, void** peer_buffer);
int bc_exchange_close(void* peer_buffer);
int bc_exchange_destroy(void* buffer);
int bc_merge_exchange(int world, int rank, unsigned epoch, int splits, int rows, int dim,
                      const float* partial_ml, const float* partial_a,
                      float* const* peer_buffers, float* out, void* stream);

/* As bc_paged_decode but writing this call's un-merged state as partials
 * (m, l, acc) per (request, q-head) into partial_ml / partial_a, in the layout
 * of bc_merge_partials with rows = B*Hq: the per-GPU half of a context split
 * across GPUs. `splits` <= 0 (chosen by the library) or 1..8: the splits are
 * merged on chip and the call writes ONE partial per row (splits = 1 in that
 * layout). `splits` 9..BC_MAX_SPLITS: the call writes `splits` partials per
 * row, unmerged, for a caller that gathers them and merges all at once (for a
 * batch too small to fill the GPU with on-chip merges). Not in the reference. */
int bc_paged_decode_partial(const bc_shape* shape, const void* q, const void* k,
                            const void* v, const int* pages, const int* lengths,
                            float* partial_ml, float* partial_a, int splits, void* stream);

/* Paged split-KV decode, as bc_decode, for callers that cannot allocate device
 * memory: an attention plugin handed only its input and output buffers by an
 * engine that owns every allocation, or a latency-critical decode loop whose
 * memory plan forbids allocating per step (cudaMalloc may synchronise the
 * device and fragments the pool). Instead of caller scratch, the split
 * partials live in a fixed device array inside this library: at most
 * BC_STATIC_SCRATCH_FLOATS floats, i.e. splits * batch * query_heads *
 * (dim + 2) <= 2,097,152 (8 MiB on every GPU that loads the library, held
 * until the process exits). Larger requests return cudaErrorInvalidValue.
 * splits in [1, BC_MAX_SPLITS]; splits > 1 always merges through that array.
 * The first call on a device looks up the array's device address (with that
 * device current); make that first call before any stream capture. All calls
 * share the one array: calls that overlap on the GPU (other streams, other
 * threads) race and must be serialised by the caller. Every call rewrites all
 * the partials it reads, so nothing has to be cleared between calls.
 * No counterpart in the reference. */
#define BC_STATIC_SCRATCH_FLOATS (1 << 21)
int bc_decode_static_scratch(const bc_shape* shape, const void* q, const void* k,
                             const void* v, const int* pages, const int* lengths,
                             float* output, int splits, void* stream);

/* Self-test of the bounded waits every kernel here uses: `ctas` CTAs (with
 * smem_bytes of dynamic shared memory each, up to 200 KB, which sets how many
 * share an SM and so how many waves run) each wait on a barrier nothing
 * completes, giving up after limit_us microseconds (at most 2 s) and setting
 * BC_ERR_TIMEOUT. The first wait to give up aborts the launch: waits of later
 * waves give up at their first check, so the launch takes about one limit,
 * not one per wave. No fault, trap or unbounded spin is involved. Not in the
 * reference. */
int bc_selftest_bounded_wait(int ctas, int smem_bytes, unsigned limit_us, void* stream);

/* Returns the current device's error word (BC_ERR_* bits; 0 = clean) after
 * synchronising that device; reset != 0 clears it, and the launch abort mark
 * (a CUDA graph replays its launches with the tokens they were captured with:
 * after a BC_ERR_TIMEOUT, clear the word before replaying it). */
unsigned bc_last_device_error(int reset);

/* Library version string. */
const char* bc_version(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* BRANCHCRAFT_H_ */
