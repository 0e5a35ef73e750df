// Tree verification on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Same math as reference src/tree_attention.cu:14-71 (every draft node of a
// request attends to the request's paged prefix and to its own root-to-node
// chain, scale 1/sqrt(D), FP32 accumulation), organised as a GEMM pair:
//
//   rows  M = (request, node, q-head of the KV head's group) triples; up to
//         128 per CTA. Consecutive requests whose page tables and lengths are
//         identical (a shared prefix, found on the device) share one pass over
//         the prefix, so their rows fill the same 128-row tile;
//   keys  64-token tiles: the shared prefix pages, then the requests' draft
//         tokens (16 slots per request and node block) under the ancestor mask.
//
// Per 64-token tile:  S = Q K^T  (UMMA 128x64x16, FP16 in, FP32 in TMEM),
// softmax on S (one thread per row, reads its TMEM lane), P (FP16; FP32-exact
// output uses P = hi + lo and two MMAs) written back over S in TMEM, O += P V
// (UMMA 128xDx16, V as an MN-major operand) accumulating in TMEM. Q is an
// A operand in shared memory (staged once per CTA), P one in tensor memory:
// per tile the tensor cores read Q and K once and V once per P part.
//
// Warp roles (512 threads): two softmax warpgroups (warps 0-3 and 4-7) take
// alternate key tiles, each with its own online-softmax state and its own O
// accumulator in TMEM (thread (w & 3)*32 + lane owns row = TMEM lane of that
// index); they are merged in the epilogue. Warps 8 and 12 are the TMA
// producers of K, warps 10 and 14 those of V (pages of the page table, then
// draft K/V), each of a pair taking alternate tiles: the copy rate of paged
// boxes is bounded per issuing warp. Warp 9 allocates TMEM and issues the
// S = Q K^T MMAs, warp 11 the O += P V MMAs (one elected lane each): a
// tcgen05.mma holds its issuing thread for about its own run time (48 cycles
// for a 128x64x16 one), so one issuer per GEMM keeps the tensor pipe fed.
// Warps 13 and 15 only take part in the epilogue. After the prologue the softmax warpgroups take
// registers from the other two (setmaxnreg). K and V tiles stream through
// separate rings: a K stage is released as soon as its S = Q K^T has been
// computed, a V stage once its P V product is done, so the copies of later
// tiles are not held back by the softmax of earlier ones (5 K stages, 6 V
// stages). Four S/P buffers in TMEM let S be computed up to three tiles ahead
// of PV, so a group's next S is ready when its softmax ends.
//
// DUAL variant (requests of more than 128 rows, grids of several waves): the
// CTA runs two row tiles over the same key tiles, softmax warpgroup g owning
// row tile g and taking every key tile; (key tile, row tile) units go through
// the S/P buffers in turn, so each K/V tile copied serves twice the MMAs.
//
// The running max is kept lazily: O and l are rescaled only when a row's max
// grows by more than 2^8 (rare after the first tile), with probabilities up
// to 2^8 — the final O / l is unchanged.
//
// Splits of the key range across the CTAs of a cluster are merged through
// distributed shared memory: every CTA stages its unnormalised rows with
// their (m, l), and each row's owner CTA reads that row from every rank,
// weighs the ranks by exp2(m_c - M) / L and sums them in rank order
// (deterministic) before writing the output.
#pragma once

#include "bc_attn.cuh"
#include "bc_commit.cuh"
#include "bc_cow_plan.cuh"

namespace bc {

constexpr int kTreeRows = 128;
constexpr int kTreeTile = 64;        // keys per tile = 4 pages
constexpr int kTreeKStages = 5;
constexpr int kTreeVStages = 6;
constexpr int kTreeThreads = 512;   // 8 softmax warps, 4 TMA producers, S issuer, PV issuer, 2 idle
// Registers: launched at 128 per thread (65,536 / 512); after the prologue
// the softmax warpgroups grow and the other two shrink by the same amount
// (2 x 128 x (softmax + other) = 65,536: the whole launch budget). The
// splits are the ones with the fewest spills (none at D=64, one register's
// worth at D=128).
constexpr int kTreeLaunchRegs = 128;
template <int D>
struct TreeRegs {
  static constexpr int kSoftmax = D == 128 ? 160 : 144;
  static constexpr int kOther = 2 * kTreeLaunchRegs - kSoftmax;
  static_assert(2 * 128 * (kSoftmax + kOther) == kTreeThreads * kTreeLaunchRegs,
                "the register split must use exactly the launch budget");
  static_assert(kSoftmax % 8 == 0 && kOther % 8 == 0 && kOther >= 24 && kSoftmax <= 256,
                "setmaxnreg takes multiples of 8 in [24, 256]");
};
constexpr int kTreeMaxReq = 128;     // requests per CTA (rows per request >= 1)
constexpr int kPrologueThreads = 256;  // warps 0-7 run the prologue's shared-memory phases

struct TreeParams {
  int batch, hq, hkv, group, nodes;
  int max_pages, physical_pages;
  int rows_req;         // nodes * group
  int req_per_block;    // requests sharing one row tile (R)
  int tiles_per_block;  // row tiles per request block
  int blocks;           // ceil(batch / R)
  int splits;           // CTAs of a cluster along the keys (gridDim.z)
  int early_trigger;    // the grid is one wave: let the next kernel be scheduled at once
  const __half* q;      // [B, N, Hq, D]
  const int* pages;
  const int* lengths;
  const int* parent;
  void* out;            // [B, N, Hq, D] FP32 or FP16
  float scale_log2;
  unsigned* err;
  unsigned token;       // this launch's abort token (s_launch_token)
  // The batch copy-on-write commit fused into the launch (commit_tasks > 0):
  // its tasks (commit_batch_task) run on warps 12-15 once their own roles are
  // done, spread over the grid's CTAs. The commit writes only bytes no
  // verified row depends on (fresh pages, and slots at or past every reading
  // request's length: the copy-on-write plan's contract), so it needs no
  // ordering against the verification.
  int commit_tasks, nclones, nentries;
  // (with a device-made plan: nclones / nentries are the plan arrays'
  // capacities and plan_counts[0..2] = clones, entries, planner status; a
  // nonzero status commits nothing)
  const int* plan_counts;
  __half* cache_k;
  __half* cache_v;
  const __half* draft_k;
  const __half* draft_v;
  const int* clone_src;
  const int* clone_dst;
  const int* entry_request;
  const int* entry_node;
  const int* entry_page;
  const int* entry_slot;
  // The planner run inside this launch (plan_inline; one-wave grids only):
  // one extra cluster (blockIdx.x == plan_item) does no verification; its
  // first CTA makes the plan with all its threads and publishes
  // plan.counts[3] = 1, which the commit warps of every other CTA wait for.
  // Each of those CTAs and the planner then count themselves in
  // plan.counts[4]; the last one resets both words to zero, so the next
  // launch (a replayed graph included) starts from an unpublished flag.
  int plan_inline;
  int plan_item;
  CowPlanParams plan;
};

// DUAL: one CTA runs two consecutive 128-row tiles of a request block over
// the same key tiles (softmax warpgroup g owns row tile g), so each K/V tile
// copied into shared memory feeds twice the MMAs: half the L2 -> SM traffic
// per FLOP, for grids of several waves whose blocks span two row tiles.
template <int D, bool PREC, bool DUAL = false>
struct TreeGeom {
  static constexpr int KB = D / 64;                        // 64-wide swizzle blocks
  static constexpr int kRT = DUAL ? 2 : 1;                 // row tiles per CTA
  static constexpr int kKStages = DUAL ? kTreeKStages - 1 : kTreeKStages;
  static constexpr int kVStages = DUAL ? kTreeVStages - 1 : kTreeVStages;
  static constexpr int kHalfTile = KB * kTreeTile * 128;    // K or V of one tile
  static constexpr int kKOff = 0;
  static constexpr int kVOff = kKOff + kKStages * kHalfTile;
  // Q (the A operand of S = Q K^T): 128 rows per row tile, K-major, 128-byte
  // swizzle, [KB][128 rows][128 B] like the K tiles; row tile g at g * kQTile.
  static constexpr int kQOff = kVOff + kVStages * kHalfTile;
  static constexpr int kQTile = KB * kTreeRows * 128;
  static constexpr int kQBytes = kRT * kQTile;
  static constexpr int kBarOff = kQOff + kQBytes;
  static constexpr int kSBufs = 4;  // S/P buffers in TMEM (unit u uses u % 4)
  static constexpr int kNumBars = 2 * kKStages + 2 * kVStages + 3 * kSBufs + 2 + 1 + 1 + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  // misc: tmem base (4) + nruns (4) + run tables 6 x kTreeMaxReq ints
  static constexpr int kRunOff = kMiscOff + 16;
  static constexpr int kORowOff = kRunOff + 6 * kTreeMaxReq * 4;  // [kRT*128] output row of each tile row
  static constexpr int kMlXOff = kORowOff + kRT * kTreeRows * 4;  // [2][128][2] each group's (m, l)
  static constexpr int kCommitOff = kMlXOff + 2 * kTreeRows * 8;  // CommitScratch
  static constexpr int kParOff = kCommitOff + ((int(sizeof(CommitScratch)) + 15) & ~15);
  // Epilogue (after the main loop, reusing the K/V rings): this CTA's output
  // rows at kStageOff, each D FP32 values and a 16-byte trailer holding the
  // row's (m, l) for the cluster merge; for a cluster split, kSlotRows
  // received rows [source rank][row] at kKOff (a DUAL CTA is never split).
  // The odd number of 16-byte units per row spreads a warp's row-per-thread
  // writes over all banks.
  static constexpr int kRowBytes = D * 4 + 16;
  static constexpr int kSlotRows = 136;  // >= csize * ceil(128 / csize), csize <= 8
  static constexpr int kStageOff = DUAL ? kKOff : kKOff + kSlotRows * kRowBytes;
  static_assert(kStageOff + kRT * kTreeRows * kRowBytes <= kQOff,
                "cluster merge buffers must fit in the K/V rings");
  // parent rows (anc_rows ints, 16-byte padded) then ancestor sets (32 B each)
  __host__ __device__ static size_t anc_offset(int anc_rows) { return size_t(kParOff) + ((size_t(anc_rows) * 4 + 15) & ~size_t(15)); }
  static size_t smem_bytes(int anc_rows) { return 1024 + anc_offset(anc_rows) + size_t(anc_rows) * 32; }
  // TMEM columns: four S/P buffers at 0, 64, 128, 192, O of group g at
  // 256 + 128 g (= 512).
  static constexpr uint32_t kTmemO = 256;
  static constexpr uint32_t kTmemCols = 512;
};

template <int D, bool PREC, bool OUT_HALF, bool DUAL = false>
__global__ void __launch_bounds__(kTreeThreads, 1)
    tree_mma_kernel(const __grid_constant__ TreeParams p, const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap vmap,
                    const __grid_constant__ CUtensorMap dkmap,
                    const __grid_constant__ CUtensorMap dvmap) {
  using G = TreeGeom<D, PREC, DUAL>;
  constexpr int KB = G::KB;
  constexpr float kNegInf = -INFINITY;
  constexpr uint32_t kIdescS = umma_idesc_f16(kTreeRows, kTreeTile, false, false);
  constexpr uint32_t kIdescPV = umma_idesc_f16(kTreeRows, D, false, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::kBarOff);
  uint64_t* k_full = bars;                          // [kKStages]
  uint64_t* k_empty = k_full + G::kKStages;
  uint64_t* v_full = k_empty + G::kKStages;         // [kVStages]
  uint64_t* v_empty = v_full + G::kVStages;
  uint64_t* s_full = v_empty + G::kVStages;         // [3] per S/P buffer
  // P written, per S/P buffer (not per softmax group: a group may finish its
  // next tile before the PV issuer looks, and a barrier two phases ahead of
  // its waiter reads as not yet complete; per buffer, the next arrival needs
  // S(i + 3), hence PV(i), hence the waiter's pass).
  uint64_t* p_full = s_full + G::kSBufs;       // [kSBufs]
  uint64_t* pv_done = p_full + G::kSBufs;      // [2] per softmax group (O rescale)
  uint64_t* mma_done = pv_done + 2;            // [1] the S issuer's last MMA
  uint64_t* s_free = mma_done + 1;             // [3] PV done reading S/P buffer b
  uint64_t* pv_fin = s_free + G::kSBufs;       // [1] the PV issuer's last MMA
  uint64_t* anc_ready = pv_fin + 1;            // [1] the ancestor sets are written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + G::kMiscOff);
  int* nruns_s = reinterpret_cast<int*>(smem + G::kMiscOff + 4);
  int* run_first = reinterpret_cast<int*>(smem + G::kRunOff);  // first local request
  int* run_end = run_first + kTreeMaxReq;                       // one past the last
  int* run_tiles = run_end + kTreeMaxReq;                       // prefix tiles
  int* req_same = run_tiles + kTreeMaxReq;                      // scratch flags
  int* run_len = req_same + kTreeMaxReq;                        // prefix length
  int* mismatch = req_same;                                     // first differing page
  int* len_s = run_len + kTreeMaxReq;                           // raw lengths
  int* par_s = reinterpret_cast<int*>(smem + G::kParOff);       // parent rows
  uint32_t* anc = reinterpret_cast<uint32_t*>(
      smem + G::anc_offset(p.req_per_block * p.nodes));           // [req][node][8]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tid = threadIdx.x;
  if (p.plan_inline && int(blockIdx.x) == p.plan_item) {
    // ------------------------------------------------------- the planner
    // The extra cluster: its first CTA plans the batch commit and publishes
    // the plan to the grid; the others have nothing to do.
    if (blockIdx.z == 0) {
      if (tid == 0) s_launch_token = p.token;
      grid_dependency_wait();  // the plan's inputs and state are visible
      cow_plan_run<kTreeThreads>(p.plan, tid, [] { __syncthreads(); },
                                 reinterpret_cast<int*>(smem));
      __threadfence();
      __syncthreads();
      if (tid == 0) {
        st_release_gpu(p.plan.counts + 3, 1);
        plan_flag_arrive(p.plan.counts, (int(gridDim.x) - 1) * int(gridDim.z) + 1);
      }
    }
    return;
  }

  // ---- work unit
  const int item = blockIdx.x;
  // first row tile of this CTA inside the block (DUAL: group g runs trow + g)
  const int trow = (item % p.tiles_per_block) * G::kRT;
  const int bk = item / p.tiles_per_block;
  const int blk = bk % p.blocks;
  const int kvh = bk / p.blocks;
  const int split = blockIdx.z;
  const int b0 = blk * p.req_per_block;
  const int nreq = min(p.req_per_block, p.batch - b0);
  const int npad = (p.nodes + 15) & ~15;              // draft slots per request
  // Set-up that reads no input runs before the wait for the preceding kernel
  // (a programmatic dependent launch may start while that kernel finishes):
  // barriers, the TMEM allocation, the tensor-map prefetch.
  if (tid == 0) {
    s_launch_token = p.token;  // (read by the bounded waits, after the set-up barrier)
    for (int s = 0; s < G::kKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < G::kVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < G::kSBufs; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 1);
      mbar_init(&p_full[s], 4);
    }
    mbar_init(pv_fin, 1);
    mbar_init(anc_ready, 2);  // warps 13 and 15
    for (int s = 0; s < 2; ++s) mbar_init(&pv_done[s], 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, G::kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  if ((warp == 8 || warp == 10) && lane == 0) {
    prefetch_tmap(warp == 8 ? &kmap : &vmap);
    prefetch_tmap(warp == 8 ? &dkmap : &dvmap);
  }
  // TMA producers: warps 8 and 12 copy K, 10 and 14 copy V; warps 8 / 10
  // take the even tiles, 12 / 14 the odd ones (the issue rate of paged boxes
  // is bounded per issuing warp).
  const bool producer = warp == 8 || warp == 10 || warp == 12 || warp == 14;
  const int psub = warp >= 12 ? 1 : 0;  // tile parity of a producer warp
  const bool v_warp = warp == 10 || warp == 14;
  // The barriers and the TMEM allocation are visible to every warp before any
  // input is read, so the producers can issue copies before the prologue's
  // shared-memory phases (still no input read: this may overlap the
  // preceding kernel).
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  // A one-wave grid lets the next kernel of the stream be scheduled now: its
  // CTAs take free SMs, run their set-up and wait there for this grid.
  if (p.early_trigger) grid_launch_dependents();
  grid_dependency_wait();  // inputs written by the preceding kernel are visible

  // ---- prologue. Every global load of the prologue (lengths, parent rows,
  // page-row comparisons, query rows, the producer's speculative page ids) is
  // issued before any of their results is used, so the CTA pays one memory
  // round trip before its first K/V copy.
  const int cap = p.max_pages * kPageSize;
  const int ndraft_tiles = (nreq * npad + kTreeTile - 1) / kTreeTile;
  const int npar = nreq * p.nodes;              // <= 256: R * nodes (host)
  const int ncmp = (nreq - 1) * p.max_pages;    // page-row comparisons
  // Phases 1 and 2 run on the softmax warps (0-7, kPrologueThreads) behind a
  // named barrier; the other warps join only at the barrier that ends the
  // prologue, so the producers' early copies hold nobody up.
  constexpr int kPT = kPrologueThreads;
  const bool pro = tid < kPT;
  const int ld_len = pro && tid < nreq ? __ldg(p.lengths + b0 + tid) : 0;
  const int ld_par = pro && tid < npar ? __ldg(p.parent + size_t(b0) * p.nodes + tid) : 0;
  int cmp_a[4], cmp_b[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int w = tid + k * kPT;
    cmp_a[k] = cmp_b[k] = 0;
    if (pro && w < ncmp) {
      const int i = 1 + w / p.max_pages, j = w % p.max_pages;
      cmp_a[k] = __ldg(p.pages + size_t(b0 + i) * p.max_pages + j);
      cmp_b[k] = __ldg(p.pages + size_t(b0 + i - 1) * p.max_pages + j);
    }
  }
  // Query row r of row tile g (thread 128 g + r of warps 0-3, and 4-7 for a
  // DUAL CTA) into registers.
  uint32_t qv[D / 2];
  if (warp < 4 * G::kRT) {
    const int br = trow * kTreeRows + tid;
    const bool ok = br < nreq * p.rows_req;
    const int rq = ok ? br / p.rows_req : 0, node = ok ? (br % p.rows_req) / p.group : 0;
    const int hh = ok ? br % p.group : 0;
    const uint4* src = reinterpret_cast<const uint4*>(
        p.q + ((size_t(b0 + rq) * p.nodes + node) * p.hq + size_t(kvh) * p.group + hh) * D);
#pragma unroll
    for (int k = 0; k < D / 8; ++k) {
      const uint4 v = ok ? __ldg(src + k) : make_uint4(0u, 0u, 0u, 0u);
      qv[4 * k + 0] = v.x;
      qv[4 * k + 1] = v.y;
      qv[4 * k + 2] = v.z;
      qv[4 * k + 3] = v.w;
    }
  }
  // Producer: page ids of tiles 0..15 of this CTA's key range, speculating
  // that the block is one run of request b0's prefix spanning the whole page
  // table (the common shared-prefix case); the guess is checked after phase 2.
  // Under the guess the CTA's key range is known now, so each producer issues
  // its first prefix tiles (one pass through its ring, no stage to free) at
  // once, before the shared-memory phases: their copies land while those run.
  // The producers end the prologue only once these copies have landed. If
  // the guess fails, they refill the same stages, every consumer of those
  // stages then waiting for one phase more (k_phase / v_phase below). Pages
  // past request b0's length are left out (id -1: the TMA fills zeros),
  // exactly as the checked path masks them.
  const int spec_t0 = (cap + kTreeTile - 1) / kTreeTile;
  // The guessed range's first tile and its count of prefix tiles (a function
  // of the launch parameters only, recomputed where needed).
  auto spec_range = [&](int& v0s) -> int {
    const int tot = spec_t0 + ndraft_tiles;
    const int per = (tot + p.splits - 1) / p.splits;
    v0s = min(tot, split * per);
    const int nt = min(tot, v0s + per) - v0s;
    return max(0, min(nt, spec_t0 - v0s));
  };
  int cur_ids = -1, next_ids = -1;
  if (producer) {
    int spec_v0 = 0;
    const int spec_pre = spec_range(spec_v0);
    const int nspec_k = min(spec_pre, G::kKStages);  // local tiles [0, nspec) speculated
    const int nspec_v = min(spec_pre, G::kVStages);
    // (the ids are loaded with the length, not after it: one round trip)
    const int len_raw = __ldg(p.lengths + b0);
    auto spec_pg = [&](int i) -> int {  // page of this lane in this warp's i-th tile
      const int v = spec_v0 + psub + 2 * i;
      const int pg = v * 4 + (lane & 3);
      return v < spec_t0 && pg < p.max_pages ? pg : -1;
    };
    const int pg_cur = spec_pg(lane >> 2), pg_next = spec_pg(8 + (lane >> 2));
    cur_ids = pg_cur >= 0 ? __ldg(p.pages + size_t(b0) * p.max_pages + pg_cur) : -1;
    next_ids = pg_next >= 0 ? __ldg(p.pages + size_t(b0) * p.max_pages + pg_next) : -1;
    const int len0 = min(max(len_raw, 0), cap);
    if (pg_cur * kPageSize >= len0) cur_ids = -1;  // past request b0's length
    if (pg_next * kPageSize >= len0) next_ids = -1;
    const int nspec = v_warp ? nspec_v : nspec_k;
    for (int jj = 0, i = psub; i < nspec; ++jj, i += 2) {  // local tile i -> stage i
      const int page_id = __shfl_sync(0xffffffffu, cur_ids, (jj & 7) * 4 + min(lane / KB, 3));
      if (!v_warp && lane < 4 * KB && lane % KB == 0 &&
          (page_id >= p.physical_pages || page_id < -1))
        atomicOr(p.err, kErrPageRange);
      uint64_t* full = (v_warp ? v_full : k_full) + i;
      if (lane == 0) mbar_arrive_expect_tx(full, uint32_t(G::kHalfTile));
      __syncwarp();
      if (lane < 4 * KB) {
        uint8_t* dst = smem + (v_warp ? G::kVOff : G::kKOff) + i * G::kHalfTile +
                       (lane % KB) * (kTreeTile * 128) + (lane / KB) * 2048;
        tma_load_4d(dst, v_warp ? &vmap : &kmap, full, (lane % KB) * 64, kvh, 0, page_id);
      }
      __syncwarp();
    }
  }
  const uint32_t lane_addr = uint32_t((warp & 3) * 32) << 16;  // this warp's TMEM lanes
  if (pro) {
  for (int i = tid; i < nreq; i += kPT) mismatch[i] = 0x7fffffff;
  named_barrier_sync(3, kPT);

  // Phase 1: the loaded values into shared memory.
  for (int i = tid; i < nreq; i += kPT)
    len_s[i] = i == tid ? ld_len : __ldg(p.lengths + b0 + i);
  for (int e = tid; e < npar; e += kPT)
    par_s[e] = e == tid ? ld_par : __ldg(p.parent + size_t(b0) * p.nodes + e);
  // First page where request i's row differs from request i-1's.
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int w = tid + k * kPT;
    if (w < ncmp && cmp_a[k] != cmp_b[k]) atomicMin(&mismatch[1 + w / p.max_pages], w % p.max_pages);
  }
  for (int w = tid + 4 * kPT; w < ncmp; w += kPT) {  // very wide tables only
    const int i = 1 + w / p.max_pages, j = w % p.max_pages;
    if (__ldg(p.pages + size_t(b0 + i) * p.max_pages + j) !=
        __ldg(p.pages + size_t(b0 + i - 1) * p.max_pages + j))
      atomicMin(&mismatch[i], j);
  }
  if (warp < 4 * G::kRT) {  // query rows -> shared memory (the A operand of S = Q K^T)
    // K-major with the 128-byte swizzle the MMA descriptor expects: 16-byte
    // chunk c of a 64-dim block's row r at (c ^ (r & 7)) * 16.
    const int qt = tid / kTreeRows, qr = tid % kTreeRows;
    const uint32_t qrow = smem_u32(smem + G::kQOff) + uint32_t(qt * G::kQTile + qr * 128);
#pragma unroll
    for (int k = 0; k < D / 8; ++k)
      st_shared_v4(qrow + (k / 8) * (kTreeRows * 128) + (((k & 7) ^ (qr & 7)) << 4),
                   qv[4 * k + 0], qv[4 * k + 1], qv[4 * k + 2], qv[4 * k + 3]);
    fence_proxy_async_smem();  // the rows -> the MMA's reads
  }
  named_barrier_sync(3, kPT);

  // Phase 2: runs of identical requests (the ancestor sets, needed only by
  // the draft-token tiles at the end of the key range, are written later by
  // warps 13 and 15 while the first tiles run).
  if (tid == 0) {
    int k = -1, prev_len = 0;
    for (int i = 0; i < nreq; ++i) {
      int len = len_s[i];
      if (len < 0 || len > cap) atomicOr(p.err, kErrLength);
      len = min(max(len, 0), cap);
      const bool same = i > 0 && len == prev_len &&
                        mismatch[i] >= (len + kPageSize - 1) / kPageSize;
      if (!same) {
        ++k;
        run_first[k] = i;
        run_len[k] = len;
        run_tiles[k] = (len + kTreeTile - 1) / kTreeTile;
      }
      run_end[k] = i + 1;
      prev_len = len;
    }
    *nruns_s = k + 1;
  }
  }  // pro
  if (producer) {
    // The speculative copies land before the prologue ends: no consumer can
    // then wait on a speculated stage before its first phase is complete (a
    // parity wait cannot tell a failed guess's refill, the phase it wants,
    // from the speculative phase before it).
    int v0s = 0;
    const int nspec = min(spec_range(v0s), v_warp ? G::kVStages : G::kKStages);
    bool landed = true;
    for (int i = psub; i < nspec; i += 2)
      landed = mbar_wait((v_warp ? v_full : k_full) + i, 0) && landed;
    if (!__all_sync(0xffffffffu, landed) && lane == 0) atomicOr(p.err, kErrTimeout);
  }
  tc_fence_before();
  __syncthreads();  // the end of the prologue
  tc_fence_after();
  const int nruns = *nruns_s;
  // The speculation held when the block is one run covering the whole table
  // width: then the CTA's key range is the one the producers guessed. When it
  // failed, stages [0, nspec) took one speculative fill nobody consumes: a
  // wait on such a stage's full barrier looks one phase further.
  const bool spec_ok = nruns == 1 && run_tiles[0] == spec_t0;
  int spec_v0_unused = 0;
  const int spec_pre = spec_range(spec_v0_unused);
  const int nspec_k = min(spec_pre, G::kKStages), nspec_v = min(spec_pre, G::kVStages);
  const int xk = spec_ok ? 0 : nspec_k, xv = spec_ok ? 0 : nspec_v;  // stages one phase ahead
  auto k_phase = [xk](int i) -> uint32_t {
    return uint32_t((i / G::kKStages) + ((i % G::kKStages) < xk ? 1 : 0)) & 1u;
  };
  auto v_phase = [xv](int i) -> uint32_t {
    return uint32_t((i / G::kVStages) + ((i % G::kVStages) < xv ? 1 : 0)) & 1u;
  };

  // ---- this CTA's slice of the key tiles: all runs' prefix tiles, then drafts
  int total = 0;
  for (int k = 0; k < nruns; ++k) total += run_tiles[k];
  total += ndraft_tiles;
  const int per = (total + p.splits - 1) / p.splits;
  const int v0 = min(total, split * per);
  const int ntiles = min(total, v0 + per) - v0;

  // Tile cursor: (run, tile in run) for prefix tiles, draft index after.
  auto start_cursor = [&](int v, int& run, int& t) {
    run = 0;
    t = v;
    while (run < nruns && t >= run_tiles[run]) {
      t -= run_tiles[run];
      ++run;
    }
  };

  const uint32_t k_addr = smem_u32(smem + G::kKOff);
  const uint32_t v_addr = smem_u32(smem + G::kVOff);

  const bool to_cluster = p.splits > 1;
  const int csize = p.splits;
  const uint32_t rank = to_cluster ? cluster_ctarank() : 0u;
  const int valid_rows = min(kTreeRows, nreq * p.rows_req - trow * kTreeRows);
  // Rows owned by each CTA of the cluster in the merge: the tile's valid
  // rows spread over all its CTAs (a 28-row tile split 8 ways: 4 rows each,
  // not 16 rows on two CTAs and none on six).
  const int rpk = (max(valid_rows, 1) + csize - 1) / csize;
  auto out_ptr = [&](int row) -> size_t {
    const int br = trow * kTreeRows + row;
    const int rq = br / p.rows_req, node = (br % p.rows_req) / p.group, hh = br % p.group;
    return ((size_t(b0 + rq) * p.nodes + node) * p.hq + size_t(kvh) * p.group + hh) * D;
  };
  auto store_out4 = [&](size_t base, float a, float b, float c, float d) {
    if constexpr (OUT_HALF) {
      uint2 v;
      v.x = pack_half2(a, b);
      v.y = pack_half2(c, d);
      *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p.out) + base) = v;
    } else {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + base) = make_float4(a, b, c, d);
    }
  };
  int* orow = reinterpret_cast<int*>(smem + G::kORowOff);
  // Rows of this tile owned by this CTA in the cluster merge.
  const int own_rows = to_cluster ? max(0, min(rpk, valid_rows - int(rank) * rpk)) : 0;
  // The cluster merge's last step, shared by all 512 threads: wait for the
  // peers' rows, sum each owned row's slots in rank order and store it.
  // The owners' sums run on the softmax warps (tid < 256); warps 8-15 only
  // take part in the cluster barrier.
  auto merge_owned_rows = [&]() {
    const uint32_t stage = smem_u32(smem + G::kStageOff);
    const int row0 = int(rank) * rpk;
    for (int task = tid; task < own_rows * (D / 4); task += 256) {
      const int rl = task / (D / 4), chunk = task % (D / 4);
      const int row = row0 + rl;
      // this row in every rank's staging area, through the cluster window
      const uint32_t here = stage + uint32_t(row * G::kRowBytes);
      // Every rank's (m, l) and piece of the row, all loads in flight at once.
      float2 ml[8];
      float4 v[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c < csize) {
          const uint32_t there = map_to_rank(here, uint32_t(c));
          ml[c] = ld_cluster_f32x2(there + D * 4);
          v[c] = ld_cluster_f32x4(there + chunk * 16);
        }
      }
      float M = kNegInf;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        if (c < csize) M = fmaxf(M, ml[c].x);
      // Weight of rank c: exp2(m_c - M) / L (0 for a rank without keys).
      float L = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c < csize) {
          ml[c].x = ml[c].x != kNegInf ? fast_exp2(ml[c].x - M) : 0.f;
          L += ml[c].x * ml[c].y;
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);  // rank order: deterministic
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c < csize) {
          const float wgt = ml[c].x * inv;
          acc.x += wgt * v[c].x;
          acc.y += wgt * v[c].y;
          acc.z += wgt * v[c].z;
          acc.w += wgt * v[c].w;
        }
      }
      store_out4(size_t(orow[row]) * D + chunk * 4, acc.x, acc.y, acc.z, acc.w);
    }
    // This CTA's reads of its peers' rows are done; no CTA leaves while its
    // staged rows may still be read.
    cluster_arrive_relaxed();
    cluster_wait();
  };

  // Warps 8-15 (producers, MMA issuers, two idle warps) give up registers to
  // the softmax warpgroups. The two paths never rejoin (this one returns after
  // its share of the epilogue), so each is compiled to its own budget.
  if (warp >= 8) {
  regs_decrease<TreeRegs<D>::kOther>();
  if (producer) {
    // ------------------------------------------------------------ producers
    // warps 8 / 12: K, warps 10 / 14: V; tiles of parity psub
    constexpr int per_part = 4 * KB;  // boxes per tile
    const int nspec = v_warp ? nspec_v : nspec_k;  // (landed before the prologue ended)
    if (ntiles > psub) {
      int run, t;
      start_cursor(v0 + psub, run, t);
      auto step = [&]() {  // the cursor to the next tile
        ++t;
        while (run < nruns && t >= run_tiles[run]) {  // empty runs have no tiles
          t -= run_tiles[run];
          ++run;
        }
      };
      // Lane l holds the page id of page (l & 3) of this warp's tile
      // (batch*8 + l/4), i.e. tile psub + 2 (batch*8 + l/4) of the CTA; the
      // next batch is loaded while this one is issued. The prologue's
      // speculative ids stand when the block is one run of request b0.
      auto load_ids = [&](int batch_first) -> int {
        const int i = psub + 2 * (batch_first + (lane >> 2));
        if (i >= ntiles) return -1;
        int rr, tt;
        start_cursor(v0 + i, rr, tt);
        if (rr >= nruns) return -1;
        const int pg = tt * 4 + (lane & 3);
        if (pg * kPageSize >= run_len[rr]) return -1;
        return __ldg(p.pages + size_t(b0 + run_first[rr]) * p.max_pages + pg);
      };
      if (nruns == 1 && run_tiles[0] == spec_t0) {
        // The speculation held (one run, as many prefix tiles as the table
        // width, hence the same key range): mask the pages past the length.
        auto mask = [&](int id, int first) -> int {
          const int pg = (v0 + psub + 2 * (first + (lane >> 2))) * 4 + (lane & 3);
          return pg * kPageSize >= run_len[0] ? -1 : id;
        };
        cur_ids = mask(cur_ids, 0);
        next_ids = mask(next_ids, 8);
      } else {
        cur_ids = load_ids(0);
        next_ids = load_ids(8);
      }
      // K or V of tile i into its ring; lane 0 posts the expected bytes, then
      // every box is issued by its own lane.
      auto issue = [&](int i, bool is_prefix, int page_id) -> bool {
        const int nst = v_warp ? G::kVStages : G::kKStages;
        const int st = i % nst;
        uint64_t* full = (v_warp ? v_full : k_full) + st;
        if (i >= nst) {
          const bool ok = mbar_wait((v_warp ? v_empty : k_empty) + st, ((i / nst) - 1) & 1);
          if (!__all_sync(0xffffffffu, ok)) return false;
        }
        if (lane == 0) mbar_arrive_expect_tx(full, uint32_t(G::kHalfTile));
        __syncwarp();
        if (lane < per_part) {
          const int j = lane / KB;   // page of the tile
          const int kb = lane % KB;  // 64-dim block
          uint8_t* dst = smem + (v_warp ? G::kVOff : G::kKOff) + st * G::kHalfTile +
                         kb * (kTreeTile * 128) + j * 2048;
          if (is_prefix) {
            tma_load_4d(dst, v_warp ? &vmap : &kmap, full, kb * 64, kvh, 0, page_id);
          } else {
            const int slot = (t * 4 + j) * 16;  // draft slot of this box
            const int rq = slot / npad, nb = slot % npad;
            const int b = rq < nreq ? b0 + rq : p.batch;  // past the block: zeros
            tma_load_4d(dst, v_warp ? &dvmap : &dkmap, full, kb * 64, kvh, nb, b);
          }
        }
        __syncwarp();
        return true;
      };
      for (int j = 0, i = psub; i < ntiles; ++j, i += 2) {
        if (j > 0 && (j & 7) == 0) {
          cur_ids = next_ids;
          next_ids = load_ids(j + 8);
        }
        if (spec_ok && i < nspec) {  // issued before the prologue's phases
          step();
          step();
          continue;
        }
        const bool is_prefix = run < nruns;
        // the page id of this lane's box
        const int page_id = __shfl_sync(0xffffffffu, cur_ids, (j & 7) * 4 + min(lane / KB, 3));
        if (!v_warp && is_prefix && lane < 4 * KB && lane % KB == 0 &&
            (page_id >= p.physical_pages || page_id < -1))
          atomicOr(p.err, kErrPageRange);
        if (!issue(i, is_prefix, page_id)) {
          if (lane == 0) atomicOr(p.err, kErrTimeout);
          break;
        }
        step();
        step();
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ S issuer
    // The whole warp runs the loop (waits, descriptor arithmetic on
    // warp-uniform values) and one elected lane issues each MMA and commit:
    // 1-3 % faster on config 5a than the same loop run by lane 0 alone.
    if (ntiles > 0) {
      bool ok = true;
      // Descriptors for Q and K stage 0; the start-address field (bits 0-13,
      // address >> 4) takes byte offsets >> 4 directly, shared memory being
      // below 256 KB.
      const uint64_t qdesc0 = umma_desc_sw128(smem_u32(smem + G::kQOff), 16, 1024);
      const uint64_t kdesc0 = umma_desc_sw128(k_addr, 16, 1024);
      // Unit u: key tile i = u / kRT against row tile g = u % kRT.
      for (int u = 0; u < ntiles * G::kRT; ++u) {
        const int i = DUAL ? (u >> 1) : u;
        const int g = DUAL ? (u & 1) : 0;
        const int kst = i % G::kKStages;
        const int sb = u % G::kSBufs;
        // S/P buffer sb was last used by unit u-4: its PV must have read P.
        ok = __all_sync(0xffffffffu, (u < G::kSBufs ||
                                      mbar_wait(&s_free[sb], ((u - G::kSBufs) / G::kSBufs) & 1)) &&
                                         (g != 0 || mbar_wait(&k_full[kst], k_phase(i))));
        if (!ok) break;
        tc_fence_after();
        const uint64_t kdesc = kdesc0 + uint64_t((kst * G::kHalfTile) >> 4);
        const uint64_t qdesc = qdesc0 + uint64_t((g * G::kQTile) >> 4);
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const int kb = ks >> 2, kin = ks & 3;
          const uint64_t adesc = qdesc + uint64_t((kb * (kTreeRows * 128) + kin * 32) >> 4);
          const uint64_t bdesc = kdesc + uint64_t((kb * (kTreeTile * 128) + kin * 32) >> 4);
          if (elect_one()) umma_f16(tbase + uint32_t(sb) * 64, adesc, bdesc, kIdescS, ks > 0 ? 1u : 0u);
        }
        if (elect_one()) {
          umma_commit(&s_full[sb]);
          // K stage free once every row tile's S is computed
          if (g == G::kRT - 1) umma_commit(&k_empty[kst]);
        }
        __syncwarp();
      }
      if (!ok && lane == 0) atomicOr(p.err, kErrTimeout);
      if (elect_one()) umma_commit(mma_done);
      __syncwarp();
      if (!__all_sync(0xffffffffu, mbar_wait(mma_done, 0)) && lane == 0) atomicOr(p.err, kErrTimeout);
    }
  } else if (warp == 11) {
    // ------------------------------------------------------------ PV issuer
    // (whole warp, one elected lane issuing, as for S)
    if (ntiles > 0) {
      bool ok = true;
      const uint64_t vdesc0 = umma_desc_sw128(v_addr, kTreeTile * 128, 1024);
      for (int u = 0; u < ntiles * G::kRT; ++u) {
        const int i = DUAL ? (u >> 1) : u;
        const int g = DUAL ? (u & 1) : 0;
        const int vst = i % G::kVStages;
        const int buf = DUAL ? g : (i & 1);  // the O accumulator (and pv_done) of this unit
        const int sb = u % G::kSBufs;
        ok = __all_sync(0xffffffffu, mbar_wait(&p_full[sb], (u / G::kSBufs) & 1) &&
                                         (g != 0 || mbar_wait(&v_full[vst], v_phase(i))));
        if (!ok) break;
        tc_fence_after();
        const uint64_t vdesc = vdesc0 + uint64_t((vst * G::kHalfTile) >> 4);
        const uint32_t tP = tbase + uint32_t(sb) * 64;                // P hi (+32: lo)
        const uint32_t tO = tbase + G::kTmemO + uint32_t(buf) * 128;  // group buf's O
#pragma unroll
        for (int kk = 0; kk < kTreeTile / 16; ++kk) {
          // V: MN-major (dims contiguous); 16 keys = two 8-key groups 1024 B apart;
          // the second 64-dim block sits kTreeTile*128 bytes further. P: 16 keys
          // = 8 TMEM columns of FP16 pairs.
          const uint64_t bdesc = vdesc + uint64_t((kk * 2048) >> 4);
          // (an accumulator's first tile overwrites it)
          const uint32_t acc = (i >= (DUAL ? 1 : 2) || kk > 0) ? 1u : 0u;
          if (elect_one()) {
            umma_f16_ts(tO, tP + kk * 8, bdesc, kIdescPV, acc);
            if (PREC) umma_f16_ts(tO, tP + 32 + kk * 8, bdesc, kIdescPV, 1u);
          }
        }
        if (elect_one()) {
          umma_commit(&pv_done[buf]);
          if (g == G::kRT - 1) umma_commit(&v_empty[vst]);
          umma_commit(&s_free[sb]);
        }
        __syncwarp();
      }
      if (!ok && lane == 0) atomicOr(p.err, kErrTimeout);
      if (elect_one()) umma_commit(pv_fin);
      __syncwarp();
      if (!__all_sync(0xffffffffu, mbar_wait(pv_fin, 0)) && lane == 0) atomicOr(p.err, kErrTimeout);
    }
  }
  else if (warp == 13 || warp == 15) {
    // ------------------------------------------------------- ancestor sets
    // Bit n' of entry (request, node n) is set when n' is n or one of its
    // ancestors; chains leaving [0, nodes) or longer than `nodes` (a cycle)
    // stop and set BC_ERR_PARENT.
    for (int e = (warp == 15 ? 32 : 0) + lane; e < nreq * p.nodes; e += 64) {
      const int rq = e / p.nodes, n = e % p.nodes;
      uint32_t* row = anc + size_t(e) * 8;
#pragma unroll
      for (int w = 0; w < 8; ++w) row[w] = 0u;
      const int* par = par_s + rq * p.nodes;
      int cur = n, steps = 0;
      while (cur >= 0) {
        if (cur >= p.nodes || steps >= p.nodes) {
          atomicOr(p.err, kErrParent);
          break;
        }
        row[cur >> 5] |= 1u << (cur & 31);
        cur = par[cur];
        ++steps;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(anc_ready);
  }
  if (p.commit_tasks > 0 && warp >= 12) {
    // ------------------------------------------------------- fused commit
    // Warps 12-15 (both idle by now: the odd-tile producers have issued
    // their last copies, the ancestor sets are written) take the CTA's share
    // of the batch commit's tasks.
    int nclones = p.nclones, nentries = p.nentries;
    bool plan_ready = true;
    if (p.plan_inline) {
      CommitScratch& flag_sc = *reinterpret_cast<CommitScratch*>(smem + G::kCommitOff);
      // (the grid is one wave: the planning CTA is resident and progresses)
      if (tid == 384) {
        flag_sc.skip = wait_flag_gpu(p.plan.counts + 3, 1) ? 1u : 0u;
        plan_flag_arrive(p.plan.counts, (int(gridDim.x) - 1) * int(gridDim.z) + 1);
      }
      named_barrier_sync(4, 128);
      plan_ready = flag_sc.skip != 0u;
      named_barrier_sync(4, 128);  // (the scratch is reused by the tasks)
      if (!plan_ready && tid == 384) atomicOr(p.err, kErrTimeout);
    }
    if (p.plan_counts) {  // a plan made on the device (by this launch or the preceding one)
      const bool ok = plan_ready && p.plan_counts[2] == 0;
      nclones = ok ? min(max(p.plan_counts[0], 0), p.nclones) : 0;
      nentries = ok ? min(max(p.plan_counts[1], 0), p.nentries) : 0;
    }
    CommitScratch& sc = *reinterpret_cast<CommitScratch*>(smem + G::kCommitOff);
    const int cols = int(gridDim.x) - (p.plan_inline ? 1 : 0);  // (not the planner's cluster)
    const int ncta = cols * int(gridDim.z);
    const int row_halves = p.hkv * D;
    const int tasks = 8 * nclones + nentries;
    for (int task = int(blockIdx.x) + cols * int(blockIdx.z); task < tasks; task += ncta)
      commit_batch_task<128>(task, tid - 384, [] { named_barrier_sync(4, 128); }, sc, row_halves,
                             p.batch, p.nodes, p.physical_pages, p.draft_k, p.draft_v, p.cache_k,
                             p.cache_v, p.clone_src, p.clone_dst, nclones, p.entry_request,
                             p.entry_node, p.entry_page, p.entry_slot, nentries, p.err);
  }
  // ---- epilogue of warps 8-15: the barriers of the softmax warps' epilogue,
  // the TMEM release, and a share of the owners' sums.
  grid_launch_dependents();
  if (to_cluster) cluster_sync_all();
  tc_fence_before();
  named_barrier_sync(1, kTreeThreads);  // every TMEM read is done
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tbase, G::kTmemCols);
  }
  if (to_cluster) {  // the softmax warps' cluster barrier after their sums
    cluster_arrive_relaxed();
    cluster_wait();
  }
  return;
  }

  // ------------------------------------------------------------ softmax rows
  regs_increase<TreeRegs<D>::kSoftmax>();
  float m_ref = kNegInf, l_sum = 0.f;
  const int wg = warp >> 2;                 // softmax group (warps 0-7)
  const int r = (warp & 3) * 32 + lane;     // row of the tile = TMEM lane
  // DUAL: group wg owns row tile trow + wg and takes every key tile; else the
  // groups share the row tile and take alternate key tiles.
  const int brow = (trow + (DUAL ? wg : 0)) * kTreeRows + r;
  const bool row_valid = warp < 8 && brow < nreq * p.rows_req;
  const int my_req = row_valid ? brow / p.rows_req : -1;
  const int my_node = row_valid ? (brow % p.rows_req) / p.group : 0;
  const uint32_t o_col = G::kTmemO + uint32_t(wg & 1) * 128;  // this group's O in TMEM
  bool softmax_ok = true;
  const int i0 = DUAL ? 0 : wg, di = DUAL ? 1 : 2;  // this group's key tiles
  if (warp < 8 && ntiles > i0) {
    int run, t;
    start_cursor(v0 + i0, run, t);
    const uint32_t* my_anc = anc + (size_t(max(my_req, 0)) * p.nodes + my_node) * 8;
    bool anc_seen = false;
    for (int i = i0; i < ntiles; i += di) {
      const int buf = DUAL ? wg : (i & 1);   // this group's O accumulator
      const int u = DUAL ? 2 * i + wg : i;   // the S/P unit
      const int sb = u % G::kSBufs;          // its S/P buffer
      if (!mbar_wait(&s_full[sb], (u / G::kSBufs) & 1)) {
        softmax_ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[64];
      {
        uint32_t (&s0)[32] = *reinterpret_cast<uint32_t (*)[32]>(&s[0]);
        uint32_t (&s1)[32] = *reinterpret_cast<uint32_t (*)[32]>(&s[32]);
        tmem_ld32(tbase + lane_addr + sb * 64, s0);
        tmem_ld32(tbase + lane_addr + sb * 64 + 32, s1);
        tmem_ld_wait();
        tmem_bind32(s0);
        tmem_bind32(s1);
      }
      // Masking: prefix keys of this row's run below the run length; draft
      // slots of this row's request that are ancestors-or-self of its node.
      const bool is_prefix = run < nruns;
      int valid_keys = 0;  // prefix: keys of this tile below the length
      bool in_run = false;
      if (is_prefix) {
        valid_keys = min(kTreeTile, run_len[run] - t * kTreeTile);
        // Rows past the block's last request (zero queries, never stored)
        // are masked like that request's rows: the warp holding the block's
        // last rows then takes one softmax path instead of diverging.
        const int mreq = row_valid ? my_req : nreq - 1;
        in_run = mreq >= run_first[run] && mreq < run_end[run];
      }
      // x[c] holds the raw score (masked keys: -inf); the scale (> 0) is
      // applied after the max and inside the exponent's FMA.
      float x[64];
      if (is_prefix && in_run && valid_keys == kTreeTile) {
#pragma unroll
        for (int c = 0; c < 64; ++c) x[c] = __uint_as_float(s[c]);  // full tile: no mask
      } else if (is_prefix) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          x[c] = (in_run && c < valid_keys) ? __uint_as_float(s[c]) : kNegInf;
      } else {
        if (!anc_seen) {  // (one phase only: the first draft tile waits)
          if (!mbar_wait(anc_ready, 0)) {
            softmax_ok = false;
            break;
          }
          anc_seen = true;
        }
        const int slot0 = t * kTreeTile;
#pragma unroll
        for (int c = 0; c < 64; c += 16) {
          const int slot = slot0 + c;
          const int rq = slot / npad, nb = slot % npad;
          uint32_t bits = 0;
          if (row_valid && rq == my_req) bits = (my_anc[nb >> 5] >> (nb & 31)) & 0xffffu;
#pragma unroll
          for (int e = 0; e < 16; ++e)
            x[c + e] = ((bits >> e) & 1u) ? __uint_as_float(s[c + e]) : kNegInf;
        }
      }
      float mx;
      {  // 8 independent partial maxima of three-input max instructions
        float m8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float a = fmax3(x[k], x[k + 8], x[k + 16]);
          const float b = fmax3(a, x[k + 24], x[k + 32]);
          const float c = fmax3(b, x[k + 40], x[k + 48]);
          m8[k] = fmaxf(c, x[k + 56]);
        }
        mx = fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), fmaxf(m8[6], m8[7]));
        mx *= p.scale_log2;  // -inf stays -inf
      }
      // Lazy max: move the reference only when the max grows by > 8 (log2).
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_ref + 8.f) {
        alpha = fast_exp2(m_ref - mx);  // 0 when m_ref is -inf
        rescale = m_ref != kNegInf;
        m_ref = mx;
        l_sum *= alpha;
      }
      const float mb = m_ref == kNegInf ? 0.f : m_ref;
      // P over S's own TMEM columns: hi at +0, lo at +32 (FP16 pairs), in
      // two halves of 32 keys to bound the live registers.
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t ph[16], pl[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int c = half * 32 + e;
          const float p0 = fast_exp2(fmaf(x[c], p.scale_log2, -mb));
          const float p1 = fast_exp2(fmaf(x[c + 1], p.scale_log2, -mb));
          ls[(e >> 1) & 3] += p0 + p1;
          if (PREC) {
            // hi = p rounded to FP16; lo = p - hi, exact in FP32 (hi is p
            // rounded to fewer bits), then rounded to FP16: P = hi + lo keeps
            // about 22 bits. (Fewer instructions than a Veltkamp split in
            // FP32: the softmax is issue-bound.)
            split_half2(p0, p1, ph[e / 2], pl[e / 2]);
          } else {
            ph[e / 2] = pack_half2(p0, p1);
          }
        }
        tmem_st16(tbase + lane_addr + uint32_t(sb) * 64 + half * 16, ph);
        if (PREC) tmem_st16(tbase + lane_addr + uint32_t(sb) * 64 + 32 + half * 16, pl);
      }
      l_sum += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // Keys past a prefix run's end may hold anything: zero their V rows so
      // that 0 * V stays 0 in the PV product. (DUAL: group 0 does it; the
      // other group's PV of this tile is issued after group 0's.)
      if (is_prefix && valid_keys < kTreeTile && (!DUAL || wg == 0)) {
        // (the V tile may still be in flight: wait for it before writing)
        const int vst = i % G::kVStages;
        if (!mbar_wait(&v_full[vst], v_phase(i))) {
          softmax_ok = false;
          break;
        }
        const uint32_t vbase = v_addr + vst * G::kHalfTile;
        const int rows_bad = kTreeTile - valid_keys;
        for (int c = r; c < rows_bad * KB * 8; c += 128) {
          const int key = valid_keys + c / (KB * 8);
          const int rem = c % (KB * 8);
          const int kb = rem >> 3, ch = rem & 7;
          st_shared_v4(vbase + kb * (kTreeTile * 128) + key * 128 + (ch << 4), 0u, 0u, 0u, 0u);
        }
        fence_proxy_async_smem();
      }
      // O rescale (whole warp when any of its rows needs it), once this
      // group's previous PV (tile i - di) has completed. (Writing P needs no
      // wait: this unit's S was issued only after the PV that last read this
      // S/P buffer had completed.)
      if (__any_sync(0xffffffffu, rescale)) {
        if (i >= i0 + di && !mbar_wait(&pv_done[buf], ((i - i0 - di) / di) & 1)) {
          softmax_ok = false;
          break;
        }
        tc_fence_after();
        const float f = rescale ? alpha : 1.f;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          uint32_t o[32];
          tmem_ld32(tbase + lane_addr + o_col + c, o);
          tmem_ld_wait();
          tmem_bind32(o);
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st32(tbase + lane_addr + o_col + c, o);
        }
      }
      tmem_st_wait();  // P (and a rescaled O) are in TMEM before the MMA reads them
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sb]);
      t += di;  // (non-DUAL: the other group takes the tile in between)
      while (run < nruns && t >= run_tiles[run]) {  // empty runs have no tiles
        t -= run_tiles[run];
        ++run;
      }
    }
    if (!softmax_ok && lane == 0) atomicOr(p.err, kErrTimeout);
  }

  // ------------------------------------------------------------ epilogue
  // The next kernel of the stream may be scheduled (it waits for this grid).
  grid_launch_dependents();
  if constexpr (DUAL) {
    // Each group holds its own rows' final (m, l) and O (a DUAL CTA is never
    // split): normalise, stage the rows, then coalesced stores by both
    // groups. The staging rows reuse the K/V rings, idle once every PV is done.
    bool ok = ntiles > 0 && softmax_ok;
    if (ok && !mbar_wait(pv_fin, 0)) {
      ok = false;
      if (lane == 0) atomicOr(p.err, kErrTimeout);
    }
    const float inv = (ok && m_ref != kNegInf && l_sum > 0.f) ? 1.f / l_sum : 0.f;
    const int q = wg * kTreeRows + r;  // staged row (output row of tile trow + wg)
    uint8_t* srow = smem + G::kStageOff + q * G::kRowBytes;
    if (brow < nreq * p.rows_req) orow[q] = int(out_ptr(q) / D);
    tc_fence_after();
    // The TMEM reads are warp-collective; whether they run depends only on
    // ntiles (uniform across the CTA).
    const bool read = ntiles > 0;
#pragma unroll
    for (int h = 0; h < D / 32; h += 2) {
      uint32_t oa[32], ob[32];
      if (read) {
        tmem_ld32(tbase + lane_addr + G::kTmemO + uint32_t(wg) * 128 + 32 * h, oa);
        tmem_ld32(tbase + lane_addr + G::kTmemO + uint32_t(wg) * 128 + 32 * (h + 1), ob);
        tmem_ld_wait();
        tmem_bind32(oa);
        tmem_bind32(ob);
      }
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        const float4 va = read ? make_float4(inv * __uint_as_float(oa[e]), inv * __uint_as_float(oa[e + 1]),
                                             inv * __uint_as_float(oa[e + 2]), inv * __uint_as_float(oa[e + 3]))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        const float4 vb = read ? make_float4(inv * __uint_as_float(ob[e]), inv * __uint_as_float(ob[e + 1]),
                                             inv * __uint_as_float(ob[e + 2]), inv * __uint_as_float(ob[e + 3]))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(srow + (32 * h + e) * 4) = va;
        *reinterpret_cast<float4*>(srow + (32 * (h + 1) + e) * 4) = vb;
      }
    }
    named_barrier_sync(2, 256);
    const int rows_all = nreq * p.rows_req - trow * kTreeRows;  // valid rows from tile trow on
    for (int task = tid; task < 2 * kTreeRows * (D / 4); task += 256) {
      const int row = task / (D / 4), chunk = task % (D / 4);
      if (row >= rows_all) break;  // rows past the block's end (row grows with task)
      const float4 v = *reinterpret_cast<const float4*>(smem + G::kStageOff +
                                                        row * G::kRowBytes + chunk * 16);
      store_out4(size_t(orow[row]) * D + chunk * 4, v.x, v.y, v.z, v.w);
    }
    tc_fence_before();
    named_barrier_sync(1, kTreeThreads);  // every TMEM read is done (warp 9 frees TMEM)
    return;
  }
  // Wait for the last PV; the two groups exchange their per-row (m, l)
  // through shared memory, so every softmax thread knows its row's merged
  // state; warps w and w+4 share TMEM lanes (rows) and each moves one half of
  // the row's D columns into the staging rows (the K/V rings are idle now).
  float* ml_x = reinterpret_cast<float*>(smem + G::kMlXOff);  // [group][row][m, l]
  constexpr int kHalfD = D / 2;
  const int col0 = wg * kHalfD;  // this thread's columns of O
  {
    // Every PV has completed once the PV issuer's final commit lands: a
    // single-phase barrier (a group's own pv_done may still be two phases
    // behind its last tile here, which its parity cannot tell apart).
    const bool have = ntiles > wg && softmax_ok;
    bool ok = have;
    if (have && !mbar_wait(pv_fin, 0)) {
      ok = false;
      if (lane == 0) atomicOr(p.err, kErrTimeout);
    }
    ml_x[(wg * kTreeRows + r) * 2 + 0] = ok ? m_ref : kNegInf;
    ml_x[(wg * kTreeRows + r) * 2 + 1] = ok ? l_sum : 0.f;
  }
  named_barrier_sync(2, 256);
  const float m0 = ml_x[r * 2 + 0], l0 = ml_x[r * 2 + 1];
  const float m1 = ml_x[(kTreeRows + r) * 2 + 0], l1 = ml_x[(kTreeRows + r) * 2 + 1];
  const float mm = fmaxf(m0, m1);
  // A group contributes only if its max is finite (it saw a valid key).
  const bool use0 = m0 != kNegInf, use1 = m1 != kNegInf;
  float w0 = use0 ? fast_exp2(m0 - mm) : 0.f;
  float w1 = use1 ? fast_exp2(m1 - mm) : 0.f;
  const float lsum = w0 * l0 + w1 * l1;
  uint8_t* srow = smem + G::kStageOff + r * G::kRowBytes;
  if (to_cluster) {
    // Unnormalised rows travel with their (m, l): the owner weighs them.
    if (wg == 0) *reinterpret_cast<float4*>(srow + D * 4) = make_float4(mm, lsum, 0.f, 0.f);
  } else {
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    w0 *= inv;
    w1 *= inv;
  }
  if (wg == 0 && r < valid_rows) orow[r] = int(out_ptr(r) / D);
  // O from TMEM: both groups' accumulators for this thread's columns, one
  // wait for all four loads. The reads are warp-collective: they depend only
  // on whether the group processed any tile at all (uniform across the warp).
  tc_fence_after();
  {
    const bool read0 = ntiles > 0, read1 = ntiles > 1;
    uint32_t oa[kHalfD / 32][32], ob[kHalfD / 32][32];
#pragma unroll
    for (int h = 0; h < kHalfD / 32; ++h) {
      if (read0) tmem_ld32(tbase + lane_addr + G::kTmemO + col0 + 32 * h, oa[h]);
      if (read1) tmem_ld32(tbase + lane_addr + G::kTmemO + 128 + col0 + 32 * h, ob[h]);
    }
    tmem_ld_wait();
#pragma unroll
    for (int h = 0; h < kHalfD / 32; ++h) {
      if (read0) tmem_bind32(oa[h]);
      if (read1) tmem_bind32(ob[h]);
    }
    const float u0 = (read0 && use0) ? w0 : 0.f, u1 = (read1 && use1) ? w1 : 0.f;
#pragma unroll
    for (int h = 0; h < kHalfD / 32; ++h) {
#pragma unroll
      for (int e = 0; e < 32; e += 4) {
        float4 v;
        v.x = (read0 ? u0 * __uint_as_float(oa[h][e + 0]) : 0.f) + (read1 ? u1 * __uint_as_float(ob[h][e + 0]) : 0.f);
        v.y = (read0 ? u0 * __uint_as_float(oa[h][e + 1]) : 0.f) + (read1 ? u1 * __uint_as_float(ob[h][e + 1]) : 0.f);
        v.z = (read0 ? u0 * __uint_as_float(oa[h][e + 2]) : 0.f) + (read1 ? u1 * __uint_as_float(ob[h][e + 2]) : 0.f);
        v.w = (read0 ? u0 * __uint_as_float(oa[h][e + 3]) : 0.f) + (read1 ? u1 * __uint_as_float(ob[h][e + 3]) : 0.f);
        *reinterpret_cast<float4*>(srow + (col0 + 32 * h + e) * 4) = v;
      }
    }
  }
  if (to_cluster) {
    cluster_sync_all();  // every CTA's rows are staged (and readable by its peers)
  } else {
    // Coalesced stores: consecutive threads write consecutive 16-byte
    // pieces of a row (a thread per row would touch a line per store).
    named_barrier_sync(2, 256);
    for (int task = tid; task < valid_rows * (D / 4); task += 256) {
      const int row = task / (D / 4), chunk = task % (D / 4);
      const float4 v = *reinterpret_cast<const float4*>(smem + G::kStageOff +
                                                        row * G::kRowBytes + chunk * 16);
      store_out4(size_t(orow[row]) * D + chunk * 4, v.x, v.y, v.z, v.w);
    }
  }
  tc_fence_before();
  named_barrier_sync(1, kTreeThreads);  // every TMEM read is done (warp 9 frees TMEM)
  if (to_cluster) merge_owned_rows();
}

}  // namespace bc
