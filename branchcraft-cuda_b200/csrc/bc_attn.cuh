// The sm_100a decode kernel for every single-query read of the paged KV cache:
//   * paged GQA decode      (reference src/paged_gqa.cu:16-74),
//   * packed-cache decode   (reference src/packed_decode.cu:16-61).
// (Tree verification, whose rows are dense enough for tcgen05, lives in
// bc_tree_mma.cuh.)
//
// Work unit (one CTA): one request, one KV head, up to 8*RT query rows (the
// q-heads of the GQA group that share that KV head) and one contiguous range of
// the request's pages.
//
// Data path per CTA (160 threads):
//   warp 4      TMA producer: for each stage of 4 pages it issues 4-D tiled
//               bulk-tensor loads (one 16-token x 64-dim box per K or V half
//               page, 128-byte swizzle) straight from the page table into a
//               3-stage shared-memory ring, completing on an mbarrier.
//   warps 0..3  consumers, arranged as RT row tiles x (4/RT) page groups. Per
//               16-token page: S^T = K Q^T with mma.sync m16n8k16 (FP16 in,
//               FP32 accumulate; K fragments by ldmatrix from the swizzled
//               tile, Q fragments resident in registers), masking, an FP32
//               online softmax in the log2 domain, then O^T += V^T P^T with P
//               split into FP16 hi + lo halves (two MMAs) so the probabilities
//               keep ~22 bits, i.e. the PV product is FP32-accurate.
// End of CTA: the page groups' (m, l, O) states are merged in shared memory;
// the CTA result is then either normalised and stored, written as a split
// partial to global scratch, or merged across the CTAs of a thread-block
// cluster through distributed shared memory (no scratch, no second launch).
//
// Numerics follow the reference: FP32 accumulation, scale 1/sqrt(D) (or the
// caller's), empty sequences produce zeros.
#pragma once

#include <cmath>

#include "bc_device.cuh"

namespace bc {

constexpr int kPageSize = 16;
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kPagesPerStage = 4;
constexpr int kStages = 3;

enum SplitMode : int { kSplitNone = 0, kSplitCluster = 1, kSplitGlobal = 2 };

struct AttnParams {
  int batch, hq, hkv, group;
  int max_pages, physical_pages;
  int rows;        // query rows per (request, KV head) = group
  int row_chunks;  // CTAs along the rows: ceil(rows / (8 * RT))
  int splits;      // CTAs along the virtual page range (gridDim.z)
  int split_mode;  // SplitMode
  int emit_partial;  // cluster/none mode: store (m, l, acc) per row instead of output
  int slot_major;    // K/V maps are (D, 16, Hkv, P) instead of (D, Hkv, 16, P)
  const __half* q;
  const int* pages;
  const int* lengths;
  void* out;
  float* partial_a;
  float* partial_ml;
  float scale_log2;  // softmax scale * log2(e)
  unsigned* err;
  unsigned token;    // this launch's abort token (s_launch_token)
};

template <int D>
struct AttnGeom {
  static constexpr int kPageBytes = kPageSize * D * 2;  // K or V of one head, one page
  static constexpr int kStageBytes = kPagesPerStage * 2 * kPageBytes;
  static constexpr int kPipeBytes = kStages * kStageBytes;
  static constexpr int kOStride = D + 4;  // padded FP32 row of the merge buffers
  static constexpr int kMergeBytes =
      (kConsumerWarps * 8 * kOStride + kConsumerWarps * 8 * 2 + 32 * kOStride + 32 * 2) * 4;
  static_assert(kMergeBytes <= kPipeBytes, "merge buffers must fit in the pipeline ring");
  static constexpr int kBarrierOffset = kPipeBytes;
  static constexpr size_t kSmemBytes = 1024 + size_t(kPipeBytes) + 2 * kStages * 8;
};

__device__ __forceinline__ float shfl_xor_max(float x, int m) {
  return fmaxf(x, __shfl_xor_sync(0xffffffffu, x, m));
}

template <int D, int RT, bool OUT_HALF>
__global__ void __launch_bounds__(kThreads, 2)
    attn_kernel(const __grid_constant__ AttnParams p, const __grid_constant__ CUtensorMap kmap,
                const __grid_constant__ CUtensorMap vmap) {
  using G = AttnGeom<D>;
  constexpr int PG = kConsumerWarps / RT;  // page groups
  constexpr int ROWS = 8 * RT;             // query rows per CTA
  constexpr int NT = D / 16;               // QK k-steps == PV m-tiles
  constexpr int KB = D / 64;               // 64-wide swizzled boxes per row
  constexpr int PAGE = G::kPageBytes;
  constexpr int STAGE = G::kStageBytes;
  constexpr int OS = G::kOStride;
  constexpr float kNegInf = -INFINITY;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::kBarrierOffset);
  uint64_t* empty = full + kStages;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // ---- work unit
  const int item = blockIdx.x;
  const int rc = item % p.row_chunks;
  const int bk = item / p.row_chunks;
  const int b = bk % p.batch;
  const int kvh = bk / p.batch;
  const int split = blockIdx.z;

  // Barriers need no input: set them up before waiting for the preceding
  // kernel (a programmatic dependent launch may start while it finishes).
  if (threadIdx.x == 0) {
    s_launch_token = p.token;  // (read by the bounded waits, after the set-up barrier)
#pragma unroll
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumerWarps);
    }
    fence_mbar_init();
  }
  grid_dependency_wait();

  int len = p.lengths[b];
  const int cap = p.max_pages * kPageSize;
  if (len < 0 || len > cap) {
    if (threadIdx.x == 0) atomicOr(p.err, kErrLength);
    len = len < 0 ? 0 : cap;
  }
  const int npref = (len + kPageSize - 1) / kPageSize;
  const int nv = npref;
  const int per = (nv + p.splits - 1) / p.splits;
  const int vbeg = min(nv, split * per);
  const int vend = min(nv, vbeg + per);
  const int nstages = (vend - vbeg + kPagesPerStage - 1) / kPagesPerStage;

  __syncthreads();

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------------ producer
    // The whole warp walks the stages; lane 0 issues the copies. Page ids are
    // read 32 at a time with one coalesced load per lane, one group ahead, so
    // the page-table latency never sits between two stages.
    if (nstages > 0) {
      if (lane == 0) {
        prefetch_tmap(&kmap);
        prefetch_tmap(&vmap);
      }
      const size_t prow = size_t(b) * p.max_pages;
      auto load_id = [&](int v) -> int {
        return (v < vend && v < npref) ? __ldg(p.pages + prow + v) : 0;
      };
      int cur_ids = load_id(vbeg + lane);
      int next_ids = load_id(vbeg + 32 + lane);
      int group = 0;
      for (int i = 0; i < nstages; ++i) {
        const int slot = i % kStages;
        if (i >= kStages) {
          const bool ok = mbar_wait(&empty[slot], ((i / kStages) - 1) & 1);
          if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) atomicOr(p.err, kErrTimeout);
            break;
          }
        }
        const int v0 = vbeg + i * kPagesPerStage;
        if (v0 - vbeg >= 32 * (group + 1)) {
          ++group;
          cur_ids = next_ids;
          next_ids = load_id(vbeg + 32 * (group + 1) + lane);
        }
        const int np = min(kPagesPerStage, vend - v0);
        const int off = v0 - vbeg - 32 * group;
        int ids[kPagesPerStage];
#pragma unroll
        for (int j = 0; j < kPagesPerStage; ++j) ids[j] = __shfl_sync(0xffffffffu, cur_ids, off + j);
        // Lane 0 posts the expected bytes; then each box of the stage is
        // issued by its own lane (one issuing thread caps the copy rate).
        uint8_t* st = smem + slot * STAGE;
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], uint32_t(np * 2 * PAGE));
        __syncwarp();
        if (lane < kPagesPerStage * KB * 2) {
          const int j = lane / (KB * 2);
          const int kb = (lane >> 1) % KB;
          const bool is_v = lane & 1;
          if (j < np) {
            const int phys = ids[j];
            // Out-of-pool ids read as zeros (TMA out-of-bounds fill).
            if (!is_v && kb == 0 && (phys < 0 || phys >= p.physical_pages))
              atomicOr(p.err, kErrPageRange);
            const int c1 = p.slot_major ? 0 : kvh, c2 = p.slot_major ? kvh : 0;
            uint8_t* dst = st + j * 2 * PAGE + (is_v ? PAGE : 0) + kb * 2048;
            tma_load_4d(dst, is_v ? &vmap : &kmap, &full[slot], kb * 64, c1, c2, phys);
          }
        }
        __syncwarp();
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    const int rt = warp % RT;
    const int pg = warp / RT;
    const int g = lane >> 2;
    const int tq = lane & 3;

    // Q^T fragments (B operand): query row g of this warp's 8-row tile.
    uint32_t qf[NT][2];
    {
      const int r = rc * ROWS + rt * 8 + g;
      if (r < p.rows) {
        const __half* qp = p.q + (size_t(b) * p.hq + size_t(kvh) * p.group + r) * D;
#pragma unroll
        for (int ks = 0; ks < NT; ++ks) {
          qf[ks][0] = *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 2 * tq);
          qf[ks][1] = *reinterpret_cast<const uint32_t*>(qp + ks * 16 + 2 * tq + 8);
        }
      } else {
#pragma unroll
        for (int ks = 0; ks < NT; ++ks) qf[ks][0] = qf[ks][1] = 0u;
      }
    }
    // This lane's two rows (columns of S^T): r0 and r0 + 1.
    const int r0 = rc * ROWS + rt * 8 + 2 * tq;
    const bool rv0 = r0 < p.rows, rv1 = r0 + 1 < p.rows;

    float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;
    float o[NT][4];
#pragma unroll
    for (int mt = 0; mt < NT; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.f;

    // Lane-constant parts of the ldmatrix addresses (128-byte swizzle: the
    // 16-byte chunk c of row t sits at chunk c ^ (t & 7)).
    const int tk = (lane & 7) + ((lane >> 3) & 1) * 8;
    const int ck = lane >> 4;
    const int tv = (lane & 7) + (lane >> 4) * 8;
    const int cv = (lane >> 3) & 1;

    for (int i = 0; i < nstages; ++i) {
      const int slot = i % kStages;
      if (!mbar_wait(&full[slot], (i / kStages) & 1)) {
        if (lane == 0) atomicOr(p.err, kErrTimeout);
        break;
      }
      uint8_t* st = smem + slot * STAGE;
#pragma unroll 1
      for (int j = pg; j < kPagesPerStage; j += PG) {
        const int v = vbeg + i * kPagesPerStage + j;
        if (v >= vend) break;
        const uint32_t kbase = smem_u32(st + j * 2 * PAGE);
        const uint32_t vbase = kbase + PAGE;

        // S^T[16 tokens x 8 rows] = K Q^T
        float s[4] = {0.f, 0.f, 0.f, 0.f}, s2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < NT; ++ks) {
          const int c = 2 * ks + ck;
          uint32_t a[4];
          ldsm_x4(kbase + (c >> 3) * 2048 + tk * 128 + (((c & 7) ^ (tk & 7)) << 4), a);
          if (ks & 1)
            mma_16816(s2, a, qf[ks][0], qf[ks][1]);
          else
            mma_16816(s, a, qf[ks][0], qf[ks][1]);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) s[c] += s2[c];

        // Validity of (token g | g+8) x (row r0 | r0+1).
        const int vcount = min(kPageSize, len - v * kPageSize);
        const bool t0 = g < vcount, t1 = g + 8 < vcount;
        const bool va = t0 && rv0, vb = t0 && rv1, vc = t1 && rv0, vd = t1 && rv1;
        const float x0 = va ? s[0] * p.scale_log2 : kNegInf;
        const float x1 = vb ? s[1] * p.scale_log2 : kNegInf;
        const float x2 = vc ? s[2] * p.scale_log2 : kNegInf;
        const float x3 = vd ? s[3] * p.scale_log2 : kNegInf;

        // Online softmax (log2 domain); l stays a per-lane partial sum.
        float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
        mx0 = shfl_xor_max(mx0, 4);
        mx1 = shfl_xor_max(mx1, 4);
        mx0 = shfl_xor_max(mx0, 8);
        mx1 = shfl_xor_max(mx1, 8);
        mx0 = shfl_xor_max(mx0, 16);
        mx1 = shfl_xor_max(mx1, 16);
        const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
        const float base0 = mn0 == kNegInf ? 0.f : mn0;
        const float base1 = mn1 == kNegInf ? 0.f : mn1;
        const float al0 = fast_exp2(m0 - base0), al1 = fast_exp2(m1 - base1);
        const float p0 = fast_exp2(x0 - base0), p1 = fast_exp2(x1 - base1);
        const float p2 = fast_exp2(x2 - base0), p3 = fast_exp2(x3 - base1);
        m0 = mn0;
        m1 = mn1;
        l0 = l0 * al0 + (p0 + p2);
        l1 = l1 * al1 + (p1 + p3);
#pragma unroll
        for (int mt = 0; mt < NT; ++mt) {
          o[mt][0] *= al0;
          o[mt][1] *= al1;
          o[mt][2] *= al0;
          o[mt][3] *= al1;
        }

        // P^T fragments (B operand) as FP16 hi + lo, transposed in registers.
        uint32_t h0, q0, h1, q1;
        split_half2(p0, p1, h0, q0);  // tokens g     x rows (r0, r0+1)
        split_half2(p2, p3, h1, q1);  // tokens g + 8 x rows (r0, r0+1)
        const uint32_t bh0 = movmatrix_trans(h0), bh1 = movmatrix_trans(h1);
        const uint32_t bl0 = movmatrix_trans(q0), bl1 = movmatrix_trans(q1);

        // Slots past the sequence end may hold anything: zero their V.
        const bool partial = vcount < kPageSize;
        uint32_t vm_lo = 0xffffffffu, vm_hi = 0xffffffffu;
        if (partial) {
          vm_lo = (2 * tq < vcount ? 0x0000ffffu : 0u) | (2 * tq + 1 < vcount ? 0xffff0000u : 0u);
          vm_hi = (2 * tq + 8 < vcount ? 0x0000ffffu : 0u) |
                  (2 * tq + 9 < vcount ? 0xffff0000u : 0u);
        }
        // O^T[D x 8 rows] += V^T P^T
#pragma unroll
        for (int mt = 0; mt < NT; ++mt) {
          const int c = 2 * mt + cv;
          uint32_t a[4];
          ldsm_x4_trans(vbase + (c >> 3) * 2048 + tv * 128 + (((c & 7) ^ (tv & 7)) << 4), a);
          if (partial) {
            a[0] &= vm_lo;
            a[1] &= vm_lo;
            a[2] &= vm_hi;
            a[3] &= vm_hi;
          }
          mma_16816(o[mt], a, bh0, bh1);
          mma_16816(o[mt], a, bl0, bl1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    // Full l per row: sum the per-lane partials over the 8 lanes of a column.
#pragma unroll
    for (int m = 4; m <= 16; m <<= 1) {
      l0 += __shfl_xor_sync(0xffffffffu, l0, m);
      l1 += __shfl_xor_sync(0xffffffffu, l1, m);
    }

    // Every consumer is done with the ring: reuse it for the merge buffers.
    named_barrier_sync(1, kConsumerWarps * 32);
    float* mo = reinterpret_cast<float*>(smem);     // [warp][8][OS]
    float* mml = mo + kConsumerWarps * 8 * OS;       // [warp][8][2]
    float* wo = mo + warp * 8 * OS;
#pragma unroll
    for (int mt = 0; mt < NT; ++mt) {
      wo[(2 * tq) * OS + mt * 16 + g] = o[mt][0];
      wo[(2 * tq + 1) * OS + mt * 16 + g] = o[mt][1];
      wo[(2 * tq) * OS + mt * 16 + g + 8] = o[mt][2];
      wo[(2 * tq + 1) * OS + mt * 16 + g + 8] = o[mt][3];
    }
    if (g == 0) {
      mml[(warp * 8 + 2 * tq) * 2 + 0] = m0;
      mml[(warp * 8 + 2 * tq) * 2 + 1] = l0;
      mml[(warp * 8 + 2 * tq + 1) * 2 + 0] = m1;
      mml[(warp * 8 + 2 * tq + 1) * 2 + 1] = l1;
    }
    named_barrier_sync(1, kConsumerWarps * 32);
  }

  // ---- merge the page groups of this CTA, then finish by split mode
  grid_launch_dependents();  // the merge kernel may be scheduled (it waits for this grid)
  float* mo = reinterpret_cast<float*>(smem);
  float* mml = mo + kConsumerWarps * 8 * OS;
  float* fo = mml + kConsumerWarps * 8 * 2;  // [ROWS][OS] CTA result
  float* fml = fo + 32 * OS;                  // [ROWS][2]   (m log2, l)
  const int tid = threadIdx.x;
  const bool to_cluster = p.split_mode == kSplitCluster;
  const float ln2 = 0.69314718055994531f;

  auto out_index = [&](int r, int d) -> size_t {
    return (size_t(b) * p.hq + size_t(kvh) * p.group + r) * D + d;
  };
  auto store_out = [&](int r, int d, float value) {
    const size_t idx = out_index(r, d);
    if constexpr (OUT_HALF)
      reinterpret_cast<__half*>(p.out)[idx] = __float2half_rn(value);
    else
      reinterpret_cast<float*>(p.out)[idx] = value;
  };
  // Writes one finished row state (natural-log m) as a partial, or the output.
  auto finish = [&](int rl, int d, float m, float l, float acc) {
    const int r = rc * ROWS + rl;
    if (r >= p.rows) return;
    if (p.split_mode == kSplitGlobal || p.emit_partial) {
      const size_t slot_row =
          (p.split_mode == kSplitGlobal ? (size_t(split) * p.batch + b) : size_t(b)) * p.hq +
          size_t(kvh) * p.group + r;
      p.partial_a[slot_row * D + d] = acc;
      if (d == 0) {
        p.partial_ml[slot_row * 2 + 0] = m == kNegInf ? kNegInf : m * ln2;
        p.partial_ml[slot_row * 2 + 1] = l;
      }
    } else {
      store_out(r, d, l > 0.f ? acc / l : 0.f);
    }
  };

  if (tid < kConsumerWarps * 32) {
    for (int e = tid; e < ROWS * D; e += kConsumerWarps * 32) {
      const int rl = e / D, d = e % D;
      const int rtl = rl >> 3, rr = rl & 7;
      float mmax = kNegInf;
#pragma unroll
      for (int q = 0; q < PG; ++q) mmax = fmaxf(mmax, mml[((rtl + RT * q) * 8 + rr) * 2]);
      float acc = 0.f, lsum = 0.f;
      if (mmax != kNegInf) {
#pragma unroll
        for (int q = 0; q < PG; ++q) {
          const int w = rtl + RT * q;
          const float wt = fast_exp2(mml[(w * 8 + rr) * 2] - mmax);
          acc += wt * mo[(w * 8 + rr) * OS + d];
          lsum += wt * mml[(w * 8 + rr) * 2 + 1];
        }
      }
      if (to_cluster) {
        fo[rl * OS + d] = acc;
        if (d == 0) {
          fml[rl * 2 + 0] = mmax;
          fml[rl * 2 + 1] = lsum;
        }
      } else {
        finish(rl, d, mmax, lsum, acc);
      }
    }
  }

  if (to_cluster) {
    __syncwarp();
    // All CTAs of the cluster (the splits of this work unit) hold their result
    // in shared memory. Each thread of the cluster merges 4 consecutive
    // elements of one row: it first issues every remote load it needs (m and
    // l of each CTA, one float4 of accumulators per CTA) and only then
    // combines, so the distributed-shared-memory latency is paid once.
    cluster_sync_all();
    const uint32_t rank = cluster_ctarank();
    const int csize = p.splits;
    const uint32_t fo_addr = smem_u32(fo), fml_addr = smem_u32(fml);
    constexpr int kQuads = ROWS * D / 4;
    for (int task = int(rank) * kThreads + tid; task < kQuads; task += csize * kThreads) {
      const int rl = task / (D / 4), d4 = (task % (D / 4)) * 4;
      if (rc * ROWS + rl >= p.rows) continue;
      float mc[8], lc[8];
      float4 oc[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        if (c < csize) {
          const float2 ml = ld_cluster_f32x2(map_to_rank(fml_addr + rl * 8, c));
          mc[c] = ml.x;
          lc[c] = ml.y;
          oc[c] = ld_cluster_f32x4(map_to_rank(fo_addr + (rl * OS + d4) * 4, c));
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
      finish(rl, d4 + 0, mmax, lsum, acc.x);
      finish(rl, d4 + 1, mmax, lsum, acc.y);
      finish(rl, d4 + 2, mmax, lsum, acc.z);
      finish(rl, d4 + 3, mmax, lsum, acc.w);
    }
    cluster_sync_all();  // keep this CTA's shared memory alive for its readers
  }
}

// FP32 merge of global split partials (reference src/paged_gqa.cu:76-106):
// one warp per row; partial m is in natural-log units. Partial p lives in
// block p / per_block at block_stride floats times that block index past
// pml and pa (block_stride 0: one block, the reference scratch layout); a
// context split across GPUs gathers one block per rank, each rank's
// (m, l) pairs followed by its accumulators in one buffer.
// TO_PARTIAL: instead of the normalised row, store the merged state itself —
// (M, L) at out_ml[row] and the unnormalised accumulator at out[row], every
// partial weighted by exp(m_p - M) — one partial per row for a later merge
// (all-empty rows: M = -inf, L = 0, accumulator 0).
template <int D, bool TO_PARTIAL = false>
__global__ void __launch_bounds__(128)
    merge_kernel(int rows, int splits, int per_block, long long block_stride,
                 const float* __restrict__ pml, const float* __restrict__ pa,
                 float* __restrict__ out, float* __restrict__ out_ml) {
  constexpr int R = D / 32;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + (threadIdx.x >> 5);
  grid_dependency_wait();  // the partials of the preceding kernel are visible
  if (row >= rows) return;
  auto at = [&](int s, size_t width) -> size_t {  // offset of partial s's row
    const int blk = s / per_block, sb = s % per_block;
    return size_t(blk) * size_t(block_stride) + (size_t(sb) * rows + row) * width;
  };
  float mmax = -INFINITY;
  for (int s = 0; s < splits; ++s) mmax = fmaxf(mmax, pml[at(s, 2)]);
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  float* o = out + size_t(row) * D;
  if (mmax == -INFINITY) {
#pragma unroll
    for (int r = 0; r < R; ++r) o[r * 32 + lane] = 0.f;
    if (TO_PARTIAL && lane == 0) {
      out_ml[size_t(row) * 2] = -INFINITY;
      out_ml[size_t(row) * 2 + 1] = 0.f;
    }
    return;
  }
  float denom = 0.f;
  for (int s = 0; s < splits; ++s) {
    const size_t ml = at(s, 2), a = at(s, D);
    const float w = __expf(pml[ml] - mmax);
    denom += w * pml[ml + 1];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] += w * pa[a + r * 32 + lane];
  }
  if constexpr (TO_PARTIAL) {
#pragma unroll
    for (int r = 0; r < R; ++r) o[r * 32 + lane] = acc[r];
    if (lane == 0) {
      out_ml[size_t(row) * 2] = mmax;
      out_ml[size_t(row) * 2 + 1] = denom;
    }
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) o[r * 32 + lane] = acc[r] / denom;
  }
}

}  // namespace bc
