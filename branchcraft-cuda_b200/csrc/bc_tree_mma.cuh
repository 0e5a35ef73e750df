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
// output uses P = hi + lo and two MMAs) to shared memory, O += P V (UMMA
// 128xDx16, V as an MN-major operand) accumulating in TMEM.
//
// Warp roles (320 threads): two softmax warpgroups (warps 0-3 and 4-7) take
// alternate key tiles, each with its own online-softmax state and its own O
// accumulator in TMEM (thread (w & 3)*32 + lane owns row = TMEM lane of that
// index); they are merged in the epilogue. Warp 8 is the TMA producer (K/V
// pages of the page table, draft K/V), warp 9 the TMEM allocator and the
// single-thread MMA issuer. K/V tiles stream through a 3-stage ring; S/P
// buffer g belongs to group g, so both groups' softmax overlap each other and
// the MMAs of their neighbouring tiles.
//
// The running max is kept lazily: O and l are rescaled only when a row's max
// grows by more than 2^8 (rare after the first tile), with probabilities up
// to 2^8 — the final O / l is unchanged.
//
// Splits of the key range across the CTAs of a cluster are merged through
// distributed shared memory, as in bc_attn.cuh.
#pragma once

#include "bc_attn.cuh"

namespace bc {

constexpr int kTreeRows = 128;
constexpr int kTreeTile = 64;        // keys per tile = 4 pages
constexpr int kTreeStages = 3;
constexpr int kTreeThreads = 320;   // 8 softmax warps, producer, MMA issuer
constexpr int kTreeMaxReq = 128;     // requests per CTA (rows per request >= 1)

struct TreeParams {
  int batch, hq, hkv, group, nodes;
  int max_pages, physical_pages;
  int rows_req;         // nodes * group
  int req_per_block;    // requests sharing one row tile (R)
  int tiles_per_block;  // row tiles per request block
  int blocks;           // ceil(batch / R)
  int splits;           // CTAs of a cluster along the keys (gridDim.z)
  const __half* q;      // [B, N, Hq, D]
  const int* pages;
  const int* lengths;
  const int* parent;
  void* out;            // [B, N, Hq, D] FP32 or FP16
  float scale_log2;
  unsigned* err;
};

template <int D, bool PREC>
struct TreeGeom {
  static constexpr int KB = D / 64;                        // 64-wide swizzle blocks
  static constexpr int kQBytes = KB * kTreeRows * 128;      // [KB][128 rows][128 B]
  static constexpr int kHalfTile = KB * kTreeTile * 128;    // K or V of one tile
  static constexpr int kStageBytes = 2 * kHalfTile;
  static constexpr int kPBytes = kTreeRows * kTreeTile * 2;  // one FP16 P tile
  static constexpr int kPBufBytes = (PREC ? 2 : 1) * kPBytes;
  static constexpr int kQOff = 0;
  static constexpr int kKVOff = kQOff + kQBytes;
  static constexpr int kPOff = kKVOff + kTreeStages * kStageBytes;
  static constexpr int kBarOff = kPOff + 2 * kPBufBytes;
  static constexpr int kNumBars = 3 * kTreeStages + 8 + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  // misc: tmem base (4) + nruns (4) + run tables 6 x kTreeMaxReq ints
  static constexpr int kRunOff = kMiscOff + 16;
  static constexpr int kWg1Off = kRunOff + 6 * kTreeMaxReq * 4;  // [128][2] second group's (m, l)
  static constexpr int kParOff = kWg1Off + kTreeRows * 8;
  static constexpr int kOStride = D + 4;
  static_assert(kTreeRows * kOStride * 4 + kTreeRows * 8 <= kTreeStages * kStageBytes,
                "epilogue buffers must fit in the K/V ring");
  // parent rows (anc_rows ints, 16-byte padded) then ancestor sets (32 B each)
  __host__ __device__ static size_t anc_offset(int anc_rows) { return size_t(kParOff) + ((size_t(anc_rows) * 4 + 15) & ~size_t(15)); }
  static size_t smem_bytes(int anc_rows) { return 1024 + anc_offset(anc_rows) + size_t(anc_rows) * 32; }
  static constexpr uint32_t kTmemCols = 512;  // S/P: 2 x 64, O: 2 x D (<= 128 each)
};

template <int D, bool PREC, bool OUT_HALF>
__global__ void __launch_bounds__(kTreeThreads, 1)
    tree_mma_kernel(const __grid_constant__ TreeParams p, const __grid_constant__ CUtensorMap kmap,
                    const __grid_constant__ CUtensorMap vmap,
                    const __grid_constant__ CUtensorMap dkmap,
                    const __grid_constant__ CUtensorMap dvmap) {
  using G = TreeGeom<D, PREC>;
  constexpr int KB = G::KB;
  constexpr float kNegInf = -INFINITY;
  constexpr uint32_t kIdescS = umma_idesc_f16(kTreeRows, kTreeTile, false, false);
  constexpr uint32_t kIdescPV = umma_idesc_f16(kTreeRows, D, false, true);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::kBarOff);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = bars + kTreeStages;
  uint64_t* s_full = bars + 2 * kTreeStages;   // [2]
  uint64_t* p_full = s_full + 2;               // [2]
  uint64_t* pv_done = p_full + 2;              // [2]
  uint64_t* mma_done = pv_done + 2;            // [1]
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

  // ---- work unit
  const int item = blockIdx.x;
  const int trow = item % p.tiles_per_block;          // row tile inside the block
  const int bk = item / p.tiles_per_block;
  const int blk = bk % p.blocks;
  const int kvh = bk / p.blocks;
  const int split = blockIdx.z;
  const int b0 = blk * p.req_per_block;
  const int nreq = min(p.req_per_block, p.batch - b0);
  const int npad = (p.nodes + 15) & ~15;              // draft slots per request

  // ---- prologue. Every global load of the prologue is issued in one phase
  // (lengths, parent rows, page-row comparisons, query rows, and the
  // producer's speculative page ids for a single shared prefix), so the CTA
  // pays one memory round trip before its first K/V copy.
  const int cap = p.max_pages * kPageSize;
  const int ndraft_tiles = (nreq * npad + kTreeTile - 1) / kTreeTile;
  if (tid == 0) {
    for (int s = 0; s < kTreeStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 4);
      mbar_init(&pv_done[s], 1);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, G::kTmemCols);
    tmem_relinquish();
  }
  for (int i = tid; i < nreq; i += kTreeThreads) mismatch[i] = 0x7fffffff;
  __syncthreads();

  // Phase 1: loads only.
  for (int i = tid; i < nreq; i += kTreeThreads) len_s[i] = __ldg(p.lengths + b0 + i);
  for (int e = tid; e < nreq * p.nodes; e += kTreeThreads)
    par_s[e] = __ldg(p.parent + size_t(b0) * p.nodes + e);
  // First page where request i's row differs from request i-1's.
  for (int w0 = tid; w0 < (nreq - 1) * p.max_pages; w0 += 4 * kTreeThreads) {
    int a[4], bb[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int w = w0 + k * kTreeThreads;
      a[k] = bb[k] = 0;
      if (w < (nreq - 1) * p.max_pages) {
        const int i = 1 + w / p.max_pages, j = w % p.max_pages;
        a[k] = __ldg(p.pages + size_t(b0 + i) * p.max_pages + j);
        bb[k] = __ldg(p.pages + size_t(b0 + i - 1) * p.max_pages + j);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int w = w0 + k * kTreeThreads;
      if (w < (nreq - 1) * p.max_pages && a[k] != bb[k])
        atomicMin(&mismatch[1 + w / p.max_pages], w % p.max_pages);
    }
  }
  {  // query rows -> shared memory (K-major, 128-byte swizzle); all loads of
     // a thread are issued before its stores.
    constexpr int kChunks = kTreeRows * (D / 8);
    constexpr int kPer = (kChunks + kTreeThreads - 1) / kTreeThreads;
    uint4 v[kPer];
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int c = tid + k * kTreeThreads;
      v[k] = make_uint4(0u, 0u, 0u, 0u);
      if (c < kChunks) {
        const int r = c / (D / 8), chunk = c % (D / 8);
        const int br = trow * kTreeRows + r;
        if (br < nreq * p.rows_req) {
          const int rq = br / p.rows_req, node = (br % p.rows_req) / p.group, hh = br % p.group;
          v[k] = __ldg(reinterpret_cast<const uint4*>(
              p.q + ((size_t(b0 + rq) * p.nodes + node) * p.hq + size_t(kvh) * p.group + hh) * D +
              chunk * 8));
        }
      }
    }
    uint8_t* qs = smem + G::kQOff;
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int c = tid + k * kTreeThreads;
      if (c < kChunks) {
        const int r = c / (D / 8), chunk = c % (D / 8);
        const int blkq = chunk >> 3, cc = chunk & 7;
        *reinterpret_cast<uint4*>(qs + blkq * (kTreeRows * 128) + r * 128 + ((cc ^ (r & 7)) << 4)) =
            v[k];
      }
    }
    fence_proxy_async_smem();
  }
  // Producer: speculative page ids of tiles 0..15 of this CTA's range under
  // the assumption that all requests of the block share request b0's prefix.
  int spec_len0 = 0, spec_v0 = 0, cur_ids = -1, next_ids = -1;
  if (warp == 8) {
    spec_len0 = min(max(__ldg(p.lengths + b0), 0), cap);
    const int t0 = (spec_len0 + kTreeTile - 1) / kTreeTile;
    const int tot = t0 + ndraft_tiles;
    const int per0 = (tot + p.splits - 1) / p.splits;
    spec_v0 = min(tot, split * per0);
    auto spec_id = [&](int i) -> int {
      const int v = spec_v0 + i;
      if (v >= t0) return -1;
      const int pg = v * 4 + (lane & 3);
      if (pg * kPageSize >= spec_len0) return -1;
      return __ldg(p.pages + size_t(b0) * p.max_pages + pg);
    };
    cur_ids = spec_id(lane >> 2);
    next_ids = spec_id(8 + (lane >> 2));
  }
  tc_fence_before();
  __syncthreads();

  // Phase 2: shared memory only — ancestor sets and runs of identical requests.
  for (int e = tid; e < nreq * p.nodes; e += kTreeThreads) {
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
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  const int nruns = *nruns_s;

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

  const uint32_t q_addr = smem_u32(smem + G::kQOff);
  const uint32_t kv_addr = smem_u32(smem + G::kKVOff);
  const uint32_t p_addr = smem_u32(smem + G::kPOff);

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (ntiles > 0) {
      int run, t;
      start_cursor(v0, run, t);
      if (lane == 0) {
        prefetch_tmap(&kmap);
        prefetch_tmap(&vmap);
      }
      // Lane l holds the page id of page (l & 3) of tile (batch*8 + l/4); the
      // next batch is loaded while this one is issued. The prologue's
      // speculative ids stand when the block is one run of request b0.
      auto load_ids = [&](int batch_first) -> int {
        const int i = batch_first + (lane >> 2);
        if (i >= ntiles) return -1;
        int rr, tt;
        start_cursor(v0 + i, rr, tt);
        if (rr >= nruns) return -1;
        const int pg = tt * 4 + (lane & 3);
        if (pg * kPageSize >= run_len[rr]) return -1;
        return __ldg(p.pages + size_t(b0 + run_first[rr]) * p.max_pages + pg);
      };
      if (!(nruns == 1 && spec_v0 == v0)) {
        cur_ids = load_ids(0);
        next_ids = load_ids(8);
      }
      for (int i = 0; i < ntiles; ++i) {
        const int stage = i % kTreeStages;
        if (i >= kTreeStages) {
          const bool ok = mbar_wait(&kv_empty[stage], ((i / kTreeStages) - 1) & 1);
          if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicOr(p.err, kErrTimeout);
            break;
          }
        }
        if (i > 0 && (i & 7) == 0) {
          cur_ids = next_ids;
          next_ids = load_ids(i + 8);
        }
        const bool is_prefix = run < nruns;
        int ids[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) ids[j] = __shfl_sync(0xffffffffu, cur_ids, (i & 7) * 4 + j);
        if (lane == 0 && is_prefix)
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (ids[j] >= p.physical_pages || ids[j] < -1) atomicOr(p.err, kErrPageRange);
        // Lane 0 posts the expected bytes, then every box of the tile is
        // issued by its own lane: a single issuing thread caps the copy rate
        // of the CTA well below what the tensor cores consume.
        uint8_t* kdst = smem + G::kKVOff + stage * G::kStageBytes;
        if (lane == 0) mbar_arrive_expect_tx(&kv_full[stage], uint32_t(G::kStageBytes));
        __syncwarp();
        if (lane < 4 * KB * 2) {
          const int j = lane / (KB * 2);         // page of the tile
          const int kb = (lane >> 1) % KB;       // 64-dim half
          const bool is_v = lane & 1;
          uint8_t* dst = kdst + (is_v ? G::kHalfTile : 0) + kb * (kTreeTile * 128) + j * 2048;
          if (is_prefix) {
            tma_load_4d(dst, is_v ? &vmap : &kmap, &kv_full[stage], kb * 64, kvh, 0, ids[j]);
          } else {
            const int slot = (t * 4 + j) * 16;  // draft slot of this box
            const int rq = slot / npad, nb = slot % npad;
            const int b = rq < nreq ? b0 + rq : p.batch;  // past the block: zeros
            tma_load_4d(dst, is_v ? &dvmap : &dkmap, &kv_full[stage], kb * 64, kvh, nb, b);
          }
        }
        __syncwarp();
        ++t;
        while (run < nruns && t >= run_tiles[run]) {  // empty runs have no tiles
          t -= run_tiles[run];
          ++run;
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    if (ntiles > 0 && lane == 0) {
      bool ok = true;
      const uint32_t tS[2] = {tbase, tbase + 64};
      auto issue_pv = [&](int i) {
        const int stage = i % kTreeStages;
        const int buf = i & 1;
        if (!mbar_wait(&p_full[buf], (i >> 1) & 1)) return false;
        tc_fence_after();
        const uint32_t vbase = kv_addr + stage * G::kStageBytes + G::kHalfTile;
        const uint32_t pbase = p_addr + buf * G::kPBufBytes;
        const uint32_t tO = tbase + 128 + buf * 128;  // group buf's accumulator
#pragma unroll
        for (int kk = 0; kk < kTreeTile / 16; ++kk) {
          // V: MN-major (dims contiguous); 16 keys = two 8-key groups 1024 B apart;
          // the second 64-dim block sits kTreeTile*128 bytes further.
          const uint64_t bdesc = umma_desc_sw128(vbase + kk * 2048, kTreeTile * 128, 1024);
          const uint64_t adesc = umma_desc_sw128(pbase + kk * 32, 16, 1024);
          umma_f16(tO, adesc, bdesc, kIdescPV, (i >= 2 || kk > 0) ? 1u : 0u);
          if (PREC) {
            const uint64_t ldesc = umma_desc_sw128(pbase + G::kPBytes + kk * 32, 16, 1024);
            umma_f16(tO, ldesc, bdesc, kIdescPV, 1u);
          }
        }
        umma_commit(&pv_done[buf]);
        umma_commit(&kv_empty[stage]);
        return true;
      };
      for (int i = 0; i < ntiles && ok; ++i) {
        const int stage = i % kTreeStages;
        if (!mbar_wait(&kv_full[stage], (i / kTreeStages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kbase = kv_addr + stage * G::kStageBytes;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const int kb = ks >> 2, kin = ks & 3;
          const uint64_t adesc = umma_desc_sw128(q_addr + kb * (kTreeRows * 128) + kin * 32, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(kbase + kb * (kTreeTile * 128) + kin * 32, 16, 1024);
          umma_f16(tS[i & 1], adesc, bdesc, kIdescS, ks > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[i & 1]);
        if (i > 0) ok = issue_pv(i - 1);
      }
      if (ok) ok = issue_pv(ntiles - 1);
      if (!ok) atomicOr(p.err, kErrTimeout);
      umma_commit(mma_done);
      if (!mbar_wait(mma_done, 0)) atomicOr(p.err, kErrTimeout);
    }
  }

  // ------------------------------------------------------------ softmax rows
  float m_ref = kNegInf, l_sum = 0.f;
  const int wg = warp >> 2;                 // softmax group (warps 0-7)
  const int r = (warp & 3) * 32 + lane;     // row of the tile = TMEM lane
  const int brow = trow * kTreeRows + r;
  const bool row_valid = warp < 8 && brow < nreq * p.rows_req;
  const int my_req = row_valid ? brow / p.rows_req : -1;
  const int my_node = row_valid ? (brow % p.rows_req) / p.group : 0;
  const uint32_t lane_addr = uint32_t((warp & 3) * 32) << 16;
  const uint32_t o_col = 128 + uint32_t(wg & 1) * 128;  // this group's O in TMEM
  bool softmax_ok = true;
  if (warp < 8 && ntiles > wg) {
    int run, t;
    start_cursor(v0 + wg, run, t);
    const uint32_t* my_anc = anc + (size_t(max(my_req, 0)) * p.nodes + my_node) * 8;
    for (int i = wg; i < ntiles; i += 2) {
      const int buf = i & 1;
      if (!mbar_wait(&s_full[buf], (i >> 1) & 1)) {
        softmax_ok = false;
        break;
      }
      tc_fence_after();
      uint32_t s[64];
      {
        uint32_t (&s0)[32] = *reinterpret_cast<uint32_t (*)[32]>(&s[0]);
        uint32_t (&s1)[32] = *reinterpret_cast<uint32_t (*)[32]>(&s[32]);
        tmem_ld32(tbase + lane_addr + buf * 64, s0);
        tmem_ld32(tbase + lane_addr + buf * 64 + 32, s1);
        tmem_ld_wait();
      }
      // Masking: prefix keys of this row's run below the run length; draft
      // slots of this row's request that are ancestors-or-self of its node.
      const bool is_prefix = run < nruns;
      int valid_keys = 0;  // prefix: keys of this tile below the length
      bool in_run = false;
      if (is_prefix) {
        valid_keys = min(kTreeTile, run_len[run] - t * kTreeTile);
        in_run = row_valid && my_req >= run_first[run] && my_req < run_end[run];
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
      {  // tree reduction: 8 independent partial maxima
        float m8[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) m8[k] = x[k];
#pragma unroll
        for (int c = 8; c < 64; ++c) m8[c & 7] = fmaxf(m8[c & 7], x[c]);
        mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                   fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
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
      // P tile buffer `buf` is free once PV of tile i-2 is done.
      if (i >= 2 && !mbar_wait(&pv_done[buf], ((i - 2) >> 1) & 1)) {
        softmax_ok = false;
        break;
      }
      uint8_t* prow = smem + G::kPOff + buf * G::kPBufBytes + r * 128;
      float ls[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 64; c += 8) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const float p0 = fast_exp2(fmaf(x[c + e], p.scale_log2, -mb));
          const float p1 = fast_exp2(fmaf(x[c + e + 1], p.scale_log2, -mb));
          ls[(e >> 1) & 3] += p0 + p1;
          if (PREC) {
            // Veltkamp split: h = p rounded to 11 significant bits (exact in
            // FP16 for p >= 2^-14), q = p - h exactly; FP32 FMA-pipe work
            // instead of FP16 round trips.
            // (_rn intrinsics: never contracted into FMAs.)
            const float t0 = __fmul_rn(p0, 8193.f), t1 = __fmul_rn(p1, 8193.f);
            const float h0 = __fsub_rn(t0, __fsub_rn(t0, p0));
            const float h1 = __fsub_rn(t1, __fsub_rn(t1, p1));
            hi[e / 2] = pack_half2(h0, h1);
            lo[e / 2] = pack_half2(__fsub_rn(p0, h0), __fsub_rn(p1, h1));
          } else {
            hi[e / 2] = pack_half2(p0, p1);
          }
        }
        const int chunk = c >> 3;
        uint8_t* a = prow + ((chunk ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(a) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        if (PREC) *reinterpret_cast<uint4*>(a + G::kPBytes) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
      }
      l_sum += (ls[0] + ls[1]) + (ls[2] + ls[3]);
      // Keys past a prefix run's end may hold anything: zero their V rows so
      // that 0 * V stays 0 in the PV product.
      if (is_prefix && valid_keys < kTreeTile) {
        const int stage = i % kTreeStages;
        const uint32_t vbase = kv_addr + stage * G::kStageBytes + G::kHalfTile;
        const int rows_bad = kTreeTile - valid_keys;
        for (int c = r; c < rows_bad * KB * 8; c += 128) {
          const int key = valid_keys + c / (KB * 8);
          const int rem = c % (KB * 8);
          const int kb = rem >> 3, ch = rem & 7;
          st_shared_v4(vbase + kb * (kTreeTile * 128) + key * 128 + (ch << 4), 0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();
      // O rescale (whole warp when any of its rows needs it). This group's
      // previous PV (tile i-2) is complete: it was waited for above.
      if (__any_sync(0xffffffffu, rescale)) {
        tc_fence_after();
        const float f = rescale ? alpha : 1.f;
#pragma unroll
        for (int c = 0; c < D; c += 32) {
          uint32_t o[32];
          tmem_ld32(tbase + lane_addr + o_col + c, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * f);
          tmem_st32(tbase + lane_addr + o_col + c, o);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[buf]);
      t += 2;  // the other group takes the tile in between
      while (run < nruns && t >= run_tiles[run]) {  // empty runs have no tiles
        t -= run_tiles[run];
        ++run;
      }
    }
    if (!softmax_ok && lane == 0) atomicOr(p.err, kErrTimeout);
  }

  // ------------------------------------------------------------ epilogue
  // Wait for the last PV, then each row thread reads its O row.
  const bool to_cluster = p.splits > 1;
  using TG = TreeGeom<D, PREC>;
  float* fo = reinterpret_cast<float*>(smem + G::kKVOff);          // [128][D+4]
  float* fml = fo + kTreeRows * TG::kOStride;                       // [128][2]
  auto out_ptr = [&](int row) -> size_t {
    const int br = trow * kTreeRows + row;
    const int rq = br / p.rows_req, node = (br % p.rows_req) / p.group, hh = br % p.group;
    return ((size_t(b0 + rq) * p.nodes + node) * p.hq + size_t(kvh) * p.group + hh) * D;
  };
  // Group 1 hands its (m, l) to group 0 through shared memory; group 0 merges
  // the two O accumulators row by row.
  float* wg1_ml = reinterpret_cast<float*>(smem + G::kWg1Off);
  bool have = false;
  if (warp < 8) {
    have = ntiles > wg && softmax_ok;
    const int last = have ? wg + 2 * ((ntiles - 1 - wg) / 2) : 0;
    if (have && !mbar_wait(&pv_done[last & 1], (last >> 1) & 1)) {
      have = false;
      if (lane == 0) atomicOr(p.err, kErrTimeout);
    }
    if (wg == 1) {
      wg1_ml[r * 2 + 0] = have ? m_ref : kNegInf;
      wg1_ml[r * 2 + 1] = have ? l_sum : 0.f;
    }
    named_barrier_sync(2, 256);
  }
  if (warp < 4) {
    tc_fence_after();
    const float m1 = wg1_ml[r * 2 + 0], l1 = wg1_ml[r * 2 + 1];
    const float m0 = have ? m_ref : kNegInf, l0 = have ? l_sum : 0.f;
    const float mm = fmaxf(m0, m1);
    // Per row: a group contributes only if its max is finite. The TMEM reads
    // themselves are warp-collective, so they depend only on whether the
    // group processed any tile at all (uniform across the warp).
    const bool use0 = m0 != kNegInf, use1 = m1 != kNegInf;
    const float w0 = use0 ? fast_exp2(m0 - mm) : 0.f;
    const float w1 = use1 ? fast_exp2(m1 - mm) : 0.f;
    const float lsum = w0 * l0 + w1 * l1;
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    const bool read0 = ntiles > 0, read1 = ntiles > 1;
#pragma unroll 1
    for (int c = 0; c < D; c += 32) {
      uint32_t o[32], o1[32];
      if (read0) tmem_ld32(tbase + lane_addr + 128 + c, o);
      if (read1) tmem_ld32(tbase + lane_addr + 256 + c, o1);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const float a = (read0 && use0) ? w0 * __uint_as_float(o[e]) : 0.f;
        const float b = (read1 && use1) ? w1 * __uint_as_float(o1[e]) : 0.f;
        o[e] = __float_as_uint(a + b);
      }
      if (to_cluster) {
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4*>(fo + r * TG::kOStride + c + e) =
              make_float4(__uint_as_float(o[e]), __uint_as_float(o[e + 1]),
                          __uint_as_float(o[e + 2]), __uint_as_float(o[e + 3]));
      } else if (row_valid) {
        const size_t base = out_ptr(r) + c;
        if constexpr (OUT_HALF) {
          __half* dst = reinterpret_cast<__half*>(p.out) + base;
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 v;
            v.x = pack_half2(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv);
            v.y = pack_half2(__uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
            v.z = pack_half2(__uint_as_float(o[e + 4]) * inv, __uint_as_float(o[e + 5]) * inv);
            v.w = pack_half2(__uint_as_float(o[e + 6]) * inv, __uint_as_float(o[e + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + e) = v;
          }
        } else {
          float* dst = reinterpret_cast<float*>(p.out) + base;
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            *reinterpret_cast<float4*>(dst + e) =
                make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                            __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
        }
      }
    }
    if (to_cluster) {
      fml[r * 2 + 0] = mm;
      fml[r * 2 + 1] = lsum;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tbase, G::kTmemCols);
  }

  if (to_cluster) {
    // Merge the key splits of this row tile across the cluster (DSMEM).
    __syncwarp();
    cluster_sync_all();
    const uint32_t rank = cluster_ctarank();
    const int csize = p.splits;
    const uint32_t fo_addr = smem_u32(fo), fml_addr = smem_u32(fml);
    // Only rows that exist are merged: tasks cover valid_rows x D/4 quads.
    const int valid_rows = min(kTreeRows, nreq * p.rows_req - trow * kTreeRows);
    const int quads = valid_rows * (D / 4);
    for (int task = int(rank) * kTreeThreads + tid; task < quads;
         task += csize * kTreeThreads) {
      const int row = task / (D / 4), d4 = (task % (D / 4)) * 4;
      float mc[8], lc[8];
      float4 oc[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c < csize) {
          const float2 ml = ld_cluster_f32x2(map_to_rank(fml_addr + row * 8, c));
          mc[c] = ml.x;
          lc[c] = ml.y;
          oc[c] = ld_cluster_f32x4(map_to_rank(fo_addr + (row * TG::kOStride + d4) * 4, c));
        }
      }
      float mmax = kNegInf;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        if (c < csize) mmax = fmaxf(mmax, mc[c]);
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      float lsum = 0.f;
      if (mmax != kNegInf) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          if (c < csize) {
            const float wt = fast_exp2(mc[c] - mmax);
            lsum += wt * lc[c];
            acc.x += wt * oc[c].x;
            acc.y += wt * oc[c].y;
            acc.z += wt * oc[c].z;
            acc.w += wt * oc[c].w;
          }
        }
      }
      const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
      const size_t base = out_ptr(row) + d4;
      if constexpr (OUT_HALF) {
        uint2 v;
        v.x = pack_half2(acc.x * inv, acc.y * inv);
        v.y = pack_half2(acc.z * inv, acc.w * inv);
        *reinterpret_cast<uint2*>(reinterpret_cast<__half*>(p.out) + base) = v;
      } else {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + base) =
            make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
      }
    }
    cluster_sync_all();
  }
}

}  // namespace bc
