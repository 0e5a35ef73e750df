// Host side of libbranchcraft.so: argument validation (the reference's rules,
// src/paged_gqa.cu:122-132, src/tree_attention.cu:93-122,
// src/packed_decode.cu:64-82), TMA tensor-map encoding, launch-shape choice and
// the extern "C" entry points declared in include/branchcraft.h.
//
// The library is stateless with respect to its callers: it allocates nothing,
// launches only on the stream it is given and keeps just per-device caches of
// immutable facts (SM count, the error-word address, which kernels had their
// shared-memory limit raised).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "bc_attn.cuh"
#include "bc_commit.cuh"
#include "bc_cow_plan.cuh"
#include "bc_exchange.cuh"
#include "bc_tree_mma.cuh"
#include "branchcraft.h"

static_assert(bc::kCowPlanMaxNodes == BC_MAX_NODES, "the planner's node cap is the API's");

namespace bc {

// Per-device error word (BC_ERR_* bits), set by kernels with atomicOr.
__device__ unsigned g_error_word;

namespace {

constexpr int kMaxDevices = 64;
constexpr float kLog2e = 1.4426950408889634f;

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
  return dev;
}

unsigned* error_word(int dev) {
  static std::atomic<unsigned*> cache[kMaxDevices];
  static std::mutex mu;
  unsigned* p = cache[dev].load(std::memory_order_acquire);
  if (p) return p;
  std::lock_guard<std::mutex> lock(mu);
  p = cache[dev].load(std::memory_order_relaxed);
  if (!p) {
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_error_word) != cudaSuccess)
      return nullptr;
    cache[dev].store(p, std::memory_order_release);
  }
  return p;
}

// A fresh abort token for each launch (never 0: 0 disables the abort check).
unsigned next_launch_token() {
  static std::atomic<unsigned> counter{0};
  unsigned t = counter.fetch_add(1, std::memory_order_relaxed) + 1;
  if (t == 0) t = counter.fetch_add(1, std::memory_order_relaxed) + 1;
  return t;
}

int sm_count(int dev) {
  static std::atomic<int> cache[kMaxDevices];
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1)
    n = 148;
  cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

// ------------------------------------------------------------ tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<EncodeTiledFn>(nullptr);
    return reinterpret_cast<EncodeTiledFn>(f);
  }();
  return fn;
}

// FP16 4-D map with a 64-element inner box and 128-byte swizzle.
bool encode_map(CUtensorMap* map, const void* base, const uint64_t dims[4],
                const uint64_t strides_bytes[3], const uint32_t box[4]) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  if (reinterpret_cast<uintptr_t>(base) % 16) return false;
  for (int i = 0; i < 3; ++i)
    if (strides_bytes[i] % 16 || strides_bytes[i] >= (uint64_t(1) << 40)) return false;
  cuuint64_t gdim[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t gstr[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t bdim[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), gdim, gstr, bdim,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// K or V of a paged cache viewed as 4-D (D, heads, 16 slots, pages) — or
// (D, 16 slots, heads, pages) when the slot stride is the smaller one — with
// strides given in elements.
bool encode_cache_map(CUtensorMap* map, const void* base, int dim, int heads, int pages,
                      long long head_stride, long long slot_stride, long long block_stride,
                      bool* slot_major) {
  *slot_major = slot_stride < head_stride;
  const uint64_t dims[4] = {uint64_t(dim), uint64_t(*slot_major ? 16 : heads),
                            uint64_t(*slot_major ? heads : 16), uint64_t(pages)};
  const uint64_t st[3] = {uint64_t(*slot_major ? slot_stride : head_stride) * 2,
                          uint64_t(*slot_major ? head_stride : slot_stride) * 2,
                          uint64_t(block_stride) * 2};
  const uint32_t box[4] = {64, uint32_t(*slot_major ? 16 : 1), uint32_t(*slot_major ? 1 : 16), 1};
  return encode_map(map, base, dims, st, box);
}

// Draft K or V [batch, nodes, heads, D] as 4-D (D, heads, nodes, batch).
bool encode_draft_map(CUtensorMap* map, const void* base, int dim, int heads, int nodes,
                      int batch) {
  const uint64_t dims[4] = {uint64_t(dim), uint64_t(heads), uint64_t(nodes), uint64_t(batch)};
  const uint64_t st[3] = {uint64_t(dim) * 2, uint64_t(heads) * dim * 2,
                          uint64_t(nodes) * heads * dim * 2};
  const uint32_t box[4] = {64, 1, 16, 1};
  return encode_map(map, base, dims, st, box);
}

// ---------------------------------------------------------------- launches
// FP32 merge of split partials, a programmatic dependent of the kernel that
// wrote them.
cudaError_t launch_merge(int dim, int rows, int splits, const float* pml, const float* pa,
                         float* out, cudaStream_t stream, int per_block = 0,
                         long long block_stride = 0, float* out_ml = nullptr) {
  if (per_block <= 0) per_block = splits;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((rows + 3) / 4), 1, 1);
  cfg.blockDim = dim3(128, 1, 1);
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (out_ml)  // merged state, not the normalised rows
    return dim == 64 ? cudaLaunchKernelEx(&cfg, merge_kernel<64, true>, rows, splits, per_block,
                                          block_stride, pml, pa, out, out_ml)
                     : cudaLaunchKernelEx(&cfg, merge_kernel<128, true>, rows, splits, per_block,
                                          block_stride, pml, pa, out, out_ml);
  return dim == 64 ? cudaLaunchKernelEx(&cfg, merge_kernel<64>, rows, splits, per_block,
                                        block_stride, pml, pa, out, out_ml)
                   : cudaLaunchKernelEx(&cfg, merge_kernel<128>, rows, splits, per_block,
                                        block_stride, pml, pa, out, out_ml);
}

template <int D, int RT, bool OUT_HALF>
cudaError_t launch_attn_t(const AttnParams& p, const CUtensorMap* maps, int items, int cluster,
                          cudaStream_t stream) {
  auto kern = attn_kernel<D, RT, OUT_HALF>;
  const size_t smem = AttnGeom<D>::kSmemBytes;
  static std::atomic<uint64_t> configured{0};
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  if (!(configured.load(std::memory_order_relaxed) & (uint64_t(1) << dev))) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
    configured.fetch_or(uint64_t(1) << dev);
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(items), 1, unsigned(p.splits));
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // Programmatic dependent launch: scheduled while the preceding kernel
  // finishes, waiting for it before the first input read.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cluster > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = unsigned(cluster);
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kern, p, maps[0], maps[1]);
}

template <int D, bool OUT_HALF>
cudaError_t launch_attn_rt(int rt, const AttnParams& p, const CUtensorMap* maps, int items,
                           int cluster, cudaStream_t stream) {
  switch (rt) {
    case 1: return launch_attn_t<D, 1, OUT_HALF>(p, maps, items, cluster, stream);
    case 2: return launch_attn_t<D, 2, OUT_HALF>(p, maps, items, cluster, stream);
    default: return launch_attn_t<D, 4, OUT_HALF>(p, maps, items, cluster, stream);
  }
}

cudaError_t launch_attn(int dim, int rt, bool out_half, const AttnParams& p,
                        const CUtensorMap* maps, int items, int cluster, cudaStream_t stream) {
  if (dim == 64)
    return out_half ? launch_attn_rt<64, true>(rt, p, maps, items, cluster, stream)
                    : launch_attn_rt<64, false>(rt, p, maps, items, cluster, stream);
  return out_half ? launch_attn_rt<128, true>(rt, p, maps, items, cluster, stream)
                  : launch_attn_rt<128, false>(rt, p, maps, items, cluster, stream);
}

// Row tiling: RT 8-row tiles per CTA (1, 2 or 4) and the CTAs along the rows.
void row_tiling(int rows, int* rt, int* row_chunks) {
  *rt = rows <= 8 ? 1 : rows <= 16 ? 2 : 4;
  *row_chunks = (rows + 8 * *rt - 1) / (8 * *rt);
}

// Cluster split for one launch: split only to fill the GPU (two CTAs per SM),
// keep at least 8 pages per CTA, and never exceed 8 CTAs (the portable cluster
// size). Splitting large ragged batches for balance loses: a cluster needs all
// of its CTAs free at once inside one GPC, which leaves SMs idle.
int auto_cluster(long long items, int max_virtual_pages, int sms) {
  int c = 1;
  while (c < 8 && items * c < 2LL * sms) c *= 2;
  while (c > 1 && (max_virtual_pages + c - 1) / c < 8) c /= 2;
  return c;
}

bool basic_shape_ok(const bc_shape* s) {
  return s && s->batch >= 1 && s->query_heads >= 1 && s->kv_heads >= 1 &&
         s->query_heads % s->kv_heads == 0 && (s->dim == 64 || s->dim == 128) &&
         s->max_pages >= 1 && s->physical_pages >= 1;
}

AttnParams base_params(const bc_shape* s, unsigned* err) {
  AttnParams p = {};
  p.batch = s->batch;
  p.hq = s->query_heads;
  p.hkv = s->kv_heads;
  p.group = s->query_heads / s->kv_heads;
  p.max_pages = s->max_pages;
  p.physical_pages = s->physical_pages;
  p.rows = p.group;
  p.err = err;
  p.token = next_launch_token();
  return p;
}

// Paged decode core shared by bc_decode / bc_paged_decode / partial variants.
// mode: kSplitNone / kSplitCluster / kSplitGlobal; emit_partial stores one
// (m, l, acc) partial per (request, q-head).
cudaError_t paged_decode_core(const bc_shape* s, const void* q, const void* k, const void* v,
                              const int* pages, const int* lengths, void* out, bool out_half,
                              float scale, int splits, int mode, bool emit_partial,
                              float* partial_a, float* partial_ml, bool slot_major_hint,
                              const CUtensorMap* kv_maps, cudaStream_t stream) {
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  unsigned* err = error_word(dev);
  if (!err) return cudaErrorInvalidDevice;
  AttnParams p = base_params(s, err);
  int rt = 1;
  row_tiling(p.rows, &rt, &p.row_chunks);
  p.splits = splits;
  p.split_mode = mode;
  p.emit_partial = emit_partial ? 1 : 0;
  p.slot_major = slot_major_hint ? 1 : 0;
  p.q = static_cast<const __half*>(q);
  p.pages = pages;
  p.lengths = lengths;
  p.out = out;
  p.partial_a = partial_a;
  p.partial_ml = partial_ml;
  p.scale_log2 = scale * kLog2e;
  CUtensorMap maps[2];
  if (kv_maps) {
    maps[0] = kv_maps[0];
    maps[1] = kv_maps[1];
  } else {
    bool sm = false;
    const long long hs = s->dim, ss = (long long)s->kv_heads * s->dim, bs = 16 * ss;
    if (!encode_cache_map(&maps[0], k, s->dim, s->kv_heads, s->physical_pages, hs, ss, bs, &sm) ||
        !encode_cache_map(&maps[1], v, s->dim, s->kv_heads, s->physical_pages, hs, ss, bs, &sm))
      return cudaErrorInvalidValue;
    p.slot_major = sm ? 1 : 0;
  }
  const long long items = (long long)s->kv_heads * s->batch * p.row_chunks;
  if (items > 0x7fffffffLL) return cudaErrorInvalidValue;
  const int cluster = mode == kSplitCluster ? splits : 1;
  cudaError_t e = launch_attn(s->dim, rt, out_half, p, maps, int(items), cluster, stream);
  if (e != cudaSuccess || mode != kSplitGlobal || emit_partial) return e;
  const int rows = s->batch * s->query_heads;
  return launch_merge(s->dim, rows, splits, partial_ml, partial_a, static_cast<float*>(out),
                      stream);
}

int pick_mode(int splits) { return splits <= 1 ? kSplitNone : splits <= 8 ? kSplitCluster : kSplitGlobal; }

template <int D, bool PREC, bool OUT_HALF, bool DUAL = false>
cudaError_t configure_tree_kernel(int dev) {
  static std::atomic<uint64_t> configured{0};
  if (configured.load(std::memory_order_relaxed) & (uint64_t(1) << dev)) return cudaSuccess;
  // The kernel's register split (setmaxnreg) hands out exactly the launch
  // budget of kTreeLaunchRegs per thread; with fewer registers at launch its
  // increase could never be granted, so such a build is refused here.
  cudaFuncAttributes fa;
  cudaError_t e = cudaFuncGetAttributes(&fa, tree_mma_kernel<D, PREC, OUT_HALF, DUAL>);
  if (e != cudaSuccess) return e;
  if (fa.numRegs != kTreeLaunchRegs) return cudaErrorInvalidDeviceFunction;
  const size_t most = TreeGeom<D, PREC, DUAL>::smem_bytes(BC_MAX_NODES);
  e = cudaFuncSetAttribute(tree_mma_kernel<D, PREC, OUT_HALF, DUAL>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, int(most));
  if (e != cudaSuccess) return e;
  configured.fetch_or(uint64_t(1) << dev);
  return cudaSuccess;
}

// How many clusters of `c` CTAs of this kernel can be resident at once (one
// CTA per SM at this shared-memory size); cached per device and size.
template <int D, bool PREC, bool OUT_HALF>
int tree_max_clusters(int dev, int c) {
  static std::atomic<int> cache[kMaxDevices][9];
  const int slot = c;  // 1..8
  int n = cache[dev][slot].load(std::memory_order_relaxed);
  if (n > 0) return n;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, unsigned(c));
  cfg.blockDim = dim3(kTreeThreads, 1, 1);
  cfg.dynamicSmemBytes = TreeGeom<D, PREC>::smem_bytes(BC_MAX_NODES);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = unsigned(c);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (configure_tree_kernel<D, PREC, OUT_HALF>(dev) != cudaSuccess ||
      cudaOccupancyMaxActiveClusters(&n, tree_mma_kernel<D, PREC, OUT_HALF>, &cfg) !=
          cudaSuccess ||
      n < 1) {
    cudaGetLastError();
    n = sm_count(dev) / c;
  }
  cache[dev][slot].store(n, std::memory_order_relaxed);
  return n;
}

// Cluster split along the keys: the largest size (any of 1..8) whose CTAs fit
// on the SMs in one wave of resident clusters, with at least two key tiles per
// CTA. A small batch needs every SM it can get: each CTA's copy rate, not the
// memory, bounds it.
template <int D, bool PREC, bool OUT_HALF>
int tree_splits(int dev, long long items, int tiles) {
  const int sms = sm_count(dev);
  int c = int(std::min<long long>(8, std::max<long long>(1, sms / std::max<long long>(items, 1))));
  while (c > 1 && (items > tree_max_clusters<D, PREC, OUT_HALF>(dev, c) || (tiles + c - 1) / c < 2))
    --c;
  return c;
}

// The planner as its own single-CTA launch (a programmatic dependent).
cudaError_t launch_cow_plan(const CowPlanParams& p, cudaStream_t stream) {
  const size_t smem = cow_plan_smem_bytes(p.batch);
  static std::atomic<uint64_t> configured{0};
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  if (!(configured.load(std::memory_order_relaxed) & (uint64_t(1) << dev))) {
    const cudaError_t e = cudaFuncSetAttribute(
        cow_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
        int(cow_plan_smem_bytes(kCowPlanMaxBatch)));
    if (e != cudaSuccess) return e;
    configured.fetch_or(uint64_t(1) << dev);
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(1, 1, 1);
  cfg.blockDim = dim3(kCowPlanThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, cow_plan_kernel, p);
}

template <int D, bool PREC, bool OUT_HALF, bool DUAL>
cudaError_t launch_tree_t(TreeParams& p, const CUtensorMap* maps, int items, int tiles,
                          size_t smem, cudaStream_t stream) {
  auto kern = tree_mma_kernel<D, PREC, OUT_HALF, DUAL>;
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  cudaError_t e = configure_tree_kernel<D, PREC, OUT_HALF, DUAL>(dev);
  if (e != cudaSuccess) return e;
  // A DUAL grid has several waves by construction: never split.
  p.splits = DUAL ? 1 : tree_splits<D, PREC, OUT_HALF>(dev, items, tiles);
  // One CTA per SM: a cluster split fits one wave by construction, an
  // unsplit grid when it has no more CTAs than SMs.
  p.early_trigger = (p.splits > 1 || items <= sm_count(dev)) ? 1 : 0;
  int grid_items = items;
  if (p.plan_inline == 2) {
    // A device plan was asked for: made by one extra cluster of this launch
    // when the grid, that cluster included, is one wave (every CTA resident:
    // the verification CTAs can wait for the planner), else by the planner
    // launch, which this one then follows as a programmatic dependent.
    const bool wave = !DUAL && (p.splits > 1
                                    ? items + 1 <= tree_max_clusters<D, PREC, OUT_HALF>(dev, p.splits)
                                    : items + 1 <= sm_count(dev));
    if (wave && cow_plan_smem_bytes(p.plan.batch) + 1024 <= smem) {
      p.plan_inline = 1;
      p.plan_item = items;
      grid_items = items + 1;
    } else {
      p.plan_inline = 0;
      const cudaError_t e2 = launch_cow_plan(p.plan, stream);
      if (e2 != cudaSuccess) return e2;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid_items), 1, unsigned(p.splits));
  cfg.blockDim = dim3(kTreeThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  // Programmatic dependent launch: the CTAs may be scheduled while the
  // preceding kernel finishes; they wait for it before their first load.
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (p.splits > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = 1;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = unsigned(p.splits);
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, kern, p, maps[0], maps[1], maps[2], maps[3]);
}

// Tree verification on tcgen05. Requests are grouped R to a 128-row tile
// (R = 128 / (nodes * group)); a group whose page tables match shares each
// K/V tile of the prefix. FP32 output accumulates P as FP16 hi + lo (FP32-exact
// products); FP16 output uses one FP16 P, matching its own rounding.
// The batch commit fused into a tree launch (bc_tree_verify_commit).
struct FusedCommit {
  const int *clone_src, *clone_dst, *entry_request, *entry_node, *entry_page, *entry_slot;
  int nclones, nentries;         // counts, or the capacities of a device-made plan
  const int* plan_counts;        // device-made plan: [clones, entries, status]
  const CowPlanParams* plan;     // the plan to make first (bc_tree_step)
};

cudaError_t tree_core(const bc_shape* s, const void* draft_q, const void* prefix_k,
                      const void* prefix_v, const int* pages, const int* lengths,
                      const void* draft_k, const void* draft_v, const int* parent, void* out,
                      bool out_half, int nodes, cudaStream_t stream,
                      const FusedCommit* commit = nullptr) {
  if (!basic_shape_ok(s) || nodes < 1 || nodes > BC_MAX_NODES || !prefix_k || !prefix_v ||
      !pages || !lengths || !draft_q || !draft_k || !draft_v || !parent || !out)
    return cudaErrorInvalidValue;
  if (commit) {
    const FusedCommit& c = *commit;
    if (c.nclones < 0 || c.nclones > 256 || c.nentries < 0 ||
        (c.nclones > 0 && (!c.clone_src || !c.clone_dst)) ||
        (c.nentries > 0 && (!c.entry_request || !c.entry_node || !c.entry_page || !c.entry_slot)) ||
        ((reinterpret_cast<uintptr_t>(prefix_k) | reinterpret_cast<uintptr_t>(prefix_v) |
          reinterpret_cast<uintptr_t>(draft_k) | reinterpret_cast<uintptr_t>(draft_v)) % 16))
      return cudaErrorInvalidValue;
  }
  if ((reinterpret_cast<uintptr_t>(draft_q) | reinterpret_cast<uintptr_t>(out)) % 16)
    return cudaErrorInvalidValue;
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  unsigned* err = error_word(dev);
  if (!err) return cudaErrorInvalidDevice;
  TreeParams p = {};
  p.batch = s->batch;
  p.hq = s->query_heads;
  p.hkv = s->kv_heads;
  p.group = s->query_heads / s->kv_heads;
  p.nodes = nodes;
  p.max_pages = s->max_pages;
  p.physical_pages = s->physical_pages;
  p.rows_req = nodes * p.group;
  int R = p.rows_req >= kTreeRows ? 1 : kTreeRows / p.rows_req;
  R = std::min(R, std::min(s->batch, kTreeMaxReq));
  p.req_per_block = R;
  p.tiles_per_block = (R * p.rows_req + kTreeRows - 1) / kTreeRows;
  p.blocks = (s->batch + R - 1) / R;
  long long items = (long long)s->kv_heads * p.blocks * p.tiles_per_block;
  // Blocks of an even number of row tiles, in a grid of at least two waves
  // even after pairing: one CTA runs two row tiles over each K/V tile (half
  // the copies per FLOP). Small grids keep one row tile per CTA and split
  // the keys instead.
  const bool dual = p.tiles_per_block % 2 == 0 && items / 2 >= 2LL * sm_count(dev);
  if (dual) {
    p.tiles_per_block /= 2;
    items /= 2;
  }
  if (items > 0x7fffffffLL) return cudaErrorInvalidValue;
  // Key tiles of one CTA before splitting: prefix tiles plus draft tiles.
  const int npad = (nodes + 15) & ~15;
  const int tiles = (s->max_pages * kPageSize + kTreeTile - 1) / kTreeTile +
                    (R * npad + kTreeTile - 1) / kTreeTile;
  p.q = static_cast<const __half*>(draft_q);
  p.pages = pages;
  p.lengths = lengths;
  p.parent = parent;
  p.out = out;
  p.scale_log2 = kLog2e / std::sqrt(float(s->dim));
  p.err = err;
  p.token = next_launch_token();
  if (commit) {
    p.nclones = commit->nclones;
    p.nentries = commit->nentries;
    p.commit_tasks = 8 * commit->nclones + commit->nentries;
    p.plan_counts = commit->plan_counts;
    if (commit->plan) {
      p.plan = *commit->plan;
      p.plan_inline = 2;  // (launch_tree_t decides: inside this launch or before it)
    }
    p.cache_k = static_cast<__half*>(const_cast<void*>(prefix_k));
    p.cache_v = static_cast<__half*>(const_cast<void*>(prefix_v));
    p.draft_k = static_cast<const __half*>(draft_k);
    p.draft_v = static_cast<const __half*>(draft_v);
    p.clone_src = commit->clone_src;
    p.clone_dst = commit->clone_dst;
    p.entry_request = commit->entry_request;
    p.entry_node = commit->entry_node;
    p.entry_page = commit->entry_page;
    p.entry_slot = commit->entry_slot;
  }
  CUtensorMap maps[4];
  bool sm = false;
  const long long hs = s->dim, ss = (long long)s->kv_heads * s->dim, bs = 16 * ss;
  if (!encode_cache_map(&maps[0], prefix_k, s->dim, s->kv_heads, s->physical_pages, hs, ss, bs,
                        &sm) ||
      !encode_cache_map(&maps[1], prefix_v, s->dim, s->kv_heads, s->physical_pages, hs, ss, bs,
                        &sm) ||
      !encode_draft_map(&maps[2], draft_k, s->dim, s->kv_heads, nodes, s->batch) ||
      !encode_draft_map(&maps[3], draft_v, s->dim, s->kv_heads, nodes, s->batch))
    return cudaErrorInvalidValue;
  const int anc_rows = R * nodes;
  const int it = int(items);
  if (s->dim == 64) {
    if (dual)
      return out_half ? launch_tree_t<64, false, true, true>(p, maps, it, tiles, TreeGeom<64, false, true>::smem_bytes(anc_rows), stream)
                      : launch_tree_t<64, true, false, true>(p, maps, it, tiles, TreeGeom<64, true, true>::smem_bytes(anc_rows), stream);
    return out_half ? launch_tree_t<64, false, true, false>(p, maps, it, tiles, TreeGeom<64, false>::smem_bytes(anc_rows), stream)
                    : launch_tree_t<64, true, false, false>(p, maps, it, tiles, TreeGeom<64, true>::smem_bytes(anc_rows), stream);
  }
  if (dual)
    return out_half ? launch_tree_t<128, false, true, true>(p, maps, it, tiles, TreeGeom<128, false, true>::smem_bytes(anc_rows), stream)
                    : launch_tree_t<128, true, false, true>(p, maps, it, tiles, TreeGeom<128, true, true>::smem_bytes(anc_rows), stream);
  return out_half ? launch_tree_t<128, false, true, false>(p, maps, it, tiles, TreeGeom<128, false>::smem_bytes(anc_rows), stream)
                  : launch_tree_t<128, true, false, false>(p, maps, it, tiles, TreeGeom<128, true>::smem_bytes(anc_rows), stream);
}

// Self-test of the bounded waits: every CTA waits on an mbarrier that no
// one arrives at, with a short limit. The first wait to give up records the
// launch's abort token; the CTAs of later waves then give up at their first
// check. `smem` bytes of dynamic shared memory per CTA control how many CTAs
// share an SM (hence the waves).
__global__ void __launch_bounds__(32) selftest_wait_kernel(unsigned long long limit_ns,
                                                           unsigned token, unsigned* err) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    s_launch_token = token;
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (!__all_sync(0xffffffffu, mbar_wait(&bar, 0, limit_ns)) && threadIdx.x == 0)
    atomicOr(err, kErrTimeout);
}

}  // namespace
}  // namespace bc

using namespace bc;

extern "C" {

int bc_decode(const bc_shape* s, const void* q, const void* k, const void* v, const int* pages,
              const int* lengths, float* output, float* partial_a, float* partial_ml, int splits,
              void* stream) {
  if (!basic_shape_ok(s) || splits < 1 || splits > BC_MAX_SPLITS || !q || !k || !v || !pages ||
      !lengths || !output || (splits > 1 && (!partial_a || !partial_ml)))
    return cudaErrorInvalidValue;
  return paged_decode_core(s, q, k, v, pages, lengths, output, false,
                           1.0f / std::sqrt(float(s->dim)), splits, pick_mode(splits), false,
                           partial_a, partial_ml, false, nullptr,
                           static_cast<cudaStream_t>(stream));
}

int bc_auto_splits(const bc_shape* s, int max_length, int sm_count_arg) {
  if (!s || max_length < 512) return 1;
  const int groups = s->kv_heads > 0 ? s->kv_heads : 1;
  const int g = s->kv_heads > 0 ? s->query_heads / s->kv_heads : 1;
  int rt = 1, chunks = 1;
  row_tiling(g < 1 ? 1 : g, &rt, &chunks);
  const long long base = (long long)(s->batch > 0 ? s->batch : 1) * groups * chunks;
  // As many splits as make one wave of CTAs (two resident per SM): a second,
  // partial wave costs more than the longer key range of fewer splits. Any
  // count works (the merge takes 1..64); each split keeps >= 256 keys.
  const long long wave = 2LL * (sm_count_arg > 0 ? sm_count_arg : 148);
  long long splits = std::max(1LL, std::min<long long>(BC_MAX_SPLITS, wave / base));
  splits = std::min<long long>(splits, std::max(1, max_length / 256));
  return int(splits);
}

int bc_paged_decode(const bc_shape* s, const void* q, const void* k, const void* v,
                    const int* pages, const int* lengths, float* output, int splits,
                    void* stream) {
  if (!basic_shape_ok(s) || splits > 8 || !q || !k || !v || !pages || !lengths || !output)
    return cudaErrorInvalidValue;
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  if (splits <= 0) {
    int rt = 1, chunks = 1;
    row_tiling(s->query_heads / s->kv_heads, &rt, &chunks);
    splits = auto_cluster((long long)s->batch * s->kv_heads * chunks, s->max_pages, sm_count(dev));
  }
  return paged_decode_core(s, q, k, v, pages, lengths, output, false,
                           1.0f / std::sqrt(float(s->dim)), splits, pick_mode(splits), false,
                           nullptr, nullptr, false, nullptr, static_cast<cudaStream_t>(stream));
}

int bc_paged_decode_partial(const bc_shape* s, const void* q, const void* k, const void* v,
                            const int* pages, const int* lengths, float* partial_ml,
                            float* partial_a, int splits, void* stream) {
  if (!basic_shape_ok(s) || splits > BC_MAX_SPLITS || !q || !k || !v || !pages || !lengths ||
      !partial_ml || !partial_a)
    return cudaErrorInvalidValue;
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  if (splits <= 0) {
    int rt = 1, chunks = 1;
    row_tiling(s->query_heads / s->kv_heads, &rt, &chunks);
    splits = auto_cluster((long long)s->batch * s->kv_heads * chunks, s->max_pages, sm_count(dev));
  }
  // 1..8: merged inside a cluster, one partial per row. Above 8: every split
  // stores its own partial (global mode with the merge kernel left out).
  const int mode = splits <= 1 ? kSplitNone : splits <= 8 ? kSplitCluster : kSplitGlobal;
  return paged_decode_core(s, q, k, v, pages, lengths, nullptr, false,
                           1.0f / std::sqrt(float(s->dim)), splits, mode, true, partial_a,
                           partial_ml, false, nullptr, static_cast<cudaStream_t>(stream));
}

int bc_tree_verify(const bc_shape* s, const void* draft_q, const void* prefix_k,
                   const void* prefix_v, const int* pages, const int* lengths,
                   const void* draft_k, const void* draft_v, const int* parent, float* output,
                   int nodes, void* stream) {
  return tree_core(s, draft_q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent,
                   output, false, nodes, static_cast<cudaStream_t>(stream));
}

int bc_tree_verify_f16(const bc_shape* s, const void* draft_q, const void* prefix_k,
                       const void* prefix_v, const int* pages, const int* lengths,
                       const void* draft_k, const void* draft_v, const int* parent,
                       void* output_f16, int nodes, void* stream) {
  return tree_core(s, draft_q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent,
                   output_f16, true, nodes, static_cast<cudaStream_t>(stream));
}

int bc_tree_verify_commit(const bc_shape* s, const void* draft_q, void* cache_k, void* cache_v,
                          const int* pages, const int* lengths, const void* draft_k,
                          const void* draft_v, const int* parent, void* output, int output_f16,
                          int nodes, const int* clone_src, const int* clone_dst, int nclones,
                          const int* entry_request, const int* entry_node,
                          const int* entry_page, const int* entry_slot, int nentries,
                          void* stream) {
  const FusedCommit c{clone_src, clone_dst, entry_request, entry_node, entry_page, entry_slot,
                      nclones, nentries, nullptr, nullptr};
  return tree_core(s, draft_q, cache_k, cache_v, pages, lengths, draft_k, draft_v, parent,
                   output, output_f16 != 0, nodes, static_cast<cudaStream_t>(stream), &c);
}

int bc_cow_plan(int batch, int nodes, int physical_pages, const int* pages_in,
                int max_pages_in, const int* lengths_in, const int* path_len,
                const int* path_nodes, const int* refcount_in, const int* free_stack_in,
                const int* free_count_in, int* refcount, int* free_stack, int* free_count,
                int* pages_out, int max_pages_out, int* lengths_out, int* clone_src,
                int* clone_dst, int* entry_request, int* entry_node, int* entry_page,
                int* entry_slot, int* counts, void* stream) {
  if (batch < 1 || batch > kCowPlanMaxBatch || nodes < 1 || nodes > BC_MAX_NODES ||
      physical_pages < 1 || max_pages_in < 1 || max_pages_out < 1 ||
      !pages_in || !lengths_in || !path_len || !path_nodes || !refcount_in || !free_stack_in ||
      !free_count_in || !refcount || !free_stack || !free_count || !pages_out || !lengths_out || !clone_src || !clone_dst || !entry_request ||
      !entry_node || !entry_page || !entry_slot || !counts ||
      (long long)batch * nodes > 0x7fffffffLL || (long long)batch * max_pages_out > 0x7fffffffLL)
    return cudaErrorInvalidValue;
  const CowPlanParams p{batch, nodes, physical_pages, max_pages_in, max_pages_out, pages_in,
                        lengths_in, path_len, path_nodes, refcount_in, free_stack_in,
                        free_count_in, refcount, free_stack, free_count, pages_out,
                        lengths_out, clone_src, clone_dst, entry_request, entry_node,
                        entry_page, entry_slot, counts};
  return launch_cow_plan(p, static_cast<cudaStream_t>(stream));
}

int bc_tree_step(const bc_shape* s, const void* draft_q, void* cache_k, void* cache_v,
                 const int* pages, const int* lengths, const void* draft_k, const void* draft_v,
                 const int* parent, void* output, int output_f16, int nodes, const int* path_len,
                 const int* path_nodes, const int* refcount_in, const int* free_stack_in,
                 const int* free_count_in, int* refcount, int* free_stack, int* free_count,
                 int* pages_out, int max_pages_out, int* lengths_out, int* clone_src,
                 int* clone_dst, int* entry_request, int* entry_node, int* entry_page,
                 int* entry_slot, int* counts, void* stream) {
  if (!basic_shape_ok(s) || s->batch > kCowPlanMaxBatch || nodes < 1 || nodes > BC_MAX_NODES ||
      max_pages_out < 1 || !path_len || !path_nodes ||
      !refcount_in || !free_stack_in || !free_count_in || !refcount || !free_stack ||
      !free_count || !pages_out || !lengths_out || !clone_src || !clone_dst || !entry_request ||
      !entry_node || !entry_page || !entry_slot || !counts)
    return cudaErrorInvalidValue;
  const CowPlanParams plan{s->batch, nodes, s->physical_pages, s->max_pages, max_pages_out,
                           pages, lengths, path_len, path_nodes, refcount_in, free_stack_in,
                           free_count_in, refcount, free_stack, free_count, pages_out,
                           lengths_out, clone_src, clone_dst, entry_request, entry_node,
                           entry_page, entry_slot, counts};
  const FusedCommit c{clone_src, clone_dst, entry_request, entry_node, entry_page, entry_slot,
                      s->batch, s->batch * nodes, counts, &plan};
  return tree_core(s, draft_q, cache_k, cache_v, pages, lengths, draft_k, draft_v, parent,
                   output, output_f16 != 0, nodes, static_cast<cudaStream_t>(stream), &c);
}

int bc_packed_decode_kv(const bc_shape* s, const void* q, const void* packed_kv,
                        const int* pages, const int* lengths, void* output,
                        long long block_stride, long long head_stride, long long slot_stride,
                        long long kv_offset, float scale, int splits, void* stream) {
  if (!basic_shape_ok(s) || !q || !packed_kv || !pages || !lengths || !output ||
      block_stride < 1 || head_stride < 1 || slot_stride < 1 || !(scale > 0.f) || splits > 8)
    return cudaErrorInvalidValue;
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  CUtensorMap maps[2];
  bool sm = false;
  const __half* kbase = static_cast<const __half*>(packed_kv);
  if (!encode_cache_map(&maps[0], kbase, s->dim, s->kv_heads, s->physical_pages, head_stride,
                        slot_stride, block_stride, &sm) ||
      !encode_cache_map(&maps[1], kbase + kv_offset, s->dim, s->kv_heads, s->physical_pages,
                        head_stride, slot_stride, block_stride, &sm))
    return cudaErrorInvalidValue;
  if (splits <= 0) {
    int rt = 1, chunks = 1;
    row_tiling(s->query_heads / s->kv_heads, &rt, &chunks);
    splits = auto_cluster((long long)s->batch * s->kv_heads * chunks, s->max_pages, sm_count(dev));
  }
  return paged_decode_core(s, q, nullptr, nullptr, pages, lengths, output, true, scale, splits,
                           splits > 1 ? kSplitCluster : kSplitNone, false, nullptr, nullptr, sm,
                           maps, static_cast<cudaStream_t>(stream));
}

int bc_packed_decode(const bc_shape* s, const void* q, const void* packed_kv, const int* pages,
                     const int* lengths, void* output, long long block_stride,
                     long long head_stride, long long slot_stride, float scale, void* stream) {
  if (!s) return cudaErrorInvalidValue;
  return bc_packed_decode_kv(s, q, packed_kv, pages, lengths, output, block_stride, head_stride,
                             slot_stride, s->dim, scale, 0, stream);
}

int bc_commit_path(const bc_shape* s, const void* draft_k, const void* draft_v, void* cache_k,
                   void* cache_v, const int* path_nodes, const int* dest_pages,
                   const int* dest_slots, int request, int nodes, int accepted, void* stream) {
  if (!s || !draft_k || !draft_v || !cache_k || !cache_v || !path_nodes || !dest_pages ||
      !dest_slots || request < 0 || request >= s->batch || nodes < 1 || accepted < 1 ||
      accepted > nodes || s->kv_heads < 1 || (s->dim != 64 && s->dim != 128))
    return cudaErrorInvalidValue;
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  unsigned* err = error_word(dev);
  if (!err) return cudaErrorInvalidDevice;
  const int row = s->kv_heads * s->dim;
  const bool vec = ((reinterpret_cast<uintptr_t>(draft_k) | reinterpret_cast<uintptr_t>(draft_v) |
                     reinterpret_cast<uintptr_t>(cache_k) | reinterpret_cast<uintptr_t>(cache_v)) %
                    16) == 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int physical = s->physical_pages > 0 ? s->physical_pages : 0x7fffffff;
  if (vec)
    commit_kernel<true><<<accepted, 256, 0, st>>>(
        row, s->batch, nodes, physical, static_cast<const __half*>(draft_k),
        static_cast<const __half*>(draft_v), static_cast<__half*>(cache_k),
        static_cast<__half*>(cache_v), nullptr, path_nodes, dest_pages, dest_slots, request, err);
  else
    commit_kernel<false><<<accepted, 256, 0, st>>>(
        row, s->batch, nodes, physical, static_cast<const __half*>(draft_k),
        static_cast<const __half*>(draft_v), static_cast<__half*>(cache_k),
        static_cast<__half*>(cache_v), nullptr, path_nodes, dest_pages, dest_slots, request, err);
  return cudaGetLastError();
}

int bc_commit_batch(const bc_shape* s, int nodes, const void* draft_k, const void* draft_v,
                    void* cache_k, void* cache_v, const int* clone_src, const int* clone_dst,
                    int nclones, const int* entry_request, const int* entry_node,
                    const int* entry_page, const int* entry_slot, int nentries, void* stream) {
  if (!s || !draft_k || !draft_v || !cache_k || !cache_v || nodes < 1 || nclones < 0 ||
      nentries < 0 || s->kv_heads < 1 || (s->dim != 64 && s->dim != 128) ||
      s->physical_pages < 1 || s->batch < 1 || (nclones > 0 && (!clone_src || !clone_dst)) ||
      (nentries > 0 && (!entry_request || !entry_node || !entry_page || !entry_slot)))
    return cudaErrorInvalidValue;
  const uintptr_t mis = (reinterpret_cast<uintptr_t>(draft_k) | reinterpret_cast<uintptr_t>(draft_v) |
                         reinterpret_cast<uintptr_t>(cache_k) | reinterpret_cast<uintptr_t>(cache_v)) %
                        16;
  if (mis) return cudaErrorInvalidValue;
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  unsigned* err = error_word(dev);
  if (!err) return cudaErrorInvalidDevice;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int row = s->kv_heads * s->dim;
  // Programmatic dependent launches: scheduled while the kernel before them
  // finishes, waiting for it before the first read.
  cudaLaunchAttribute pdl[1];
  pdl[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  pdl[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(256, 1, 1);
  cfg.stream = st;
  cfg.attrs = pdl;
  cfg.numAttrs = 1;
  if (nclones + nentries == 0) return cudaSuccess;
  if (nclones <= 256) {  // one launch (each entry CTA lists at most 256 clones)
    cfg.gridDim = dim3(unsigned(8 * nclones + nentries), 1, 1);
    return cudaLaunchKernelEx(&cfg, commit_batch_kernel, row, s->batch, nodes, s->physical_pages,
                              static_cast<const __half*>(draft_k),
                              static_cast<const __half*>(draft_v), static_cast<__half*>(cache_k),
                              static_cast<__half*>(cache_v), clone_src, clone_dst, nclones,
                              entry_request, entry_node, entry_page, entry_slot, nentries, err);
  }
  // Larger batches: every clone, then every row commit.
  if (nclones > 0) {
    cfg.gridDim = dim3(4, unsigned(nclones), 2);
    cudaError_t e = cudaLaunchKernelEx(&cfg, clone_kernel, 16 * row, s->physical_pages,
                                       static_cast<__half*>(cache_k),
                                       static_cast<__half*>(cache_v), clone_src, clone_dst, err);
    if (e != cudaSuccess) return e;
  }
  if (nentries > 0) {
    cfg.gridDim = dim3(unsigned(nentries), 1, 1);
    return cudaLaunchKernelEx(&cfg, commit_kernel<true>, row, s->batch, nodes,
                              s->physical_pages, static_cast<const __half*>(draft_k),
                              static_cast<const __half*>(draft_v), static_cast<__half*>(cache_k),
                              static_cast<__half*>(cache_v), entry_request, entry_node,
                              entry_page, entry_slot, 0, err);
  }
  return cudaSuccess;
}

int bc_merge_partials(int splits, int rows, int dim, const float* partial_ml,
                      const float* partial_a, float* out, void* stream) {
  if (splits < 1 || rows < 1 || (dim != 64 && dim != 128) || !partial_ml || !partial_a || !out)
    return cudaErrorInvalidValue;
  return launch_merge(dim, rows, splits, partial_ml, partial_a, out,
                      static_cast<cudaStream_t>(stream));
}

int bc_merge_to_partial(int splits, int rows, int dim, const float* partial_ml,
                        const float* partial_a, float* out_ml, float* out_a, void* stream) {
  if (splits < 1 || rows < 1 || (dim != 64 && dim != 128) || !partial_ml || !partial_a ||
      !out_ml || !out_a)
    return cudaErrorInvalidValue;
  return launch_merge(dim, rows, splits, partial_ml, partial_a, out_a,
                      static_cast<cudaStream_t>(stream), 0, 0, out_ml);
}

size_t bc_exchange_bytes(int world, int rows, int dim) {
  if (world < 1 || world > BC_MAX_EXCHANGE_RANKS || rows < 1 || (dim != 64 && dim != 128))
    return 0;
  return dim == 64 ? Exch<64>::bytes(world, rows) : Exch<128>::bytes(world, rows);
}

int bc_exchange_create(int world, int rows, int dim, void** buffer, void* ipc_handle) {
  const size_t n = bc_exchange_bytes(world, rows, dim);
  if (n == 0 || !buffer || !ipc_handle) return cudaErrorInvalidValue;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, n);
  if (e != cudaSuccess) return e;
  // zero flags: no epoch (>= 1) is published yet
  e = cudaMemset(p, 0, n);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return e;
  }
  *buffer = p;
  return cudaSuccess;
}

int bc_exchange_open(const void* ipc_handle, void** peer_buffer) {
  if (!ipc_handle || !peer_buffer) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, ipc_handle, sizeof(h));
  return cudaIpcOpenMemHandle(peer_buffer, h, cudaIpcMemLazyEnablePeerAccess);
}

int bc_exchange_close(void* peer_buffer) {
  return peer_buffer ? cudaIpcCloseMemHandle(peer_buffer) : cudaErrorInvalidValue;
}

int bc_exchange_destroy(void* buffer) { return buffer ? cudaFree(buffer) : cudaErrorInvalidValue; }

int bc_merge_exchange(int world, int rank, unsigned epoch, int splits, int rows, int dim,
                      const float* partial_ml, const float* partial_a, float* const* peer_buffers,
                      float* out, void* stream) {
  if (world < 1 || world > BC_MAX_EXCHANGE_RANKS || rank < 0 || rank >= world || epoch == 0 ||
      splits < 1 || rows < 1 || (dim != 64 && dim != 128) || !partial_ml || !partial_a ||
      !peer_buffers || !out)
    return cudaErrorInvalidValue;
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  unsigned* err = error_word(dev);
  if (!err) return cudaErrorInvalidDevice;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned((rows + kExchRowsPerBlock - 1) / kExchRowsPerBlock), 1, 1);
  cfg.blockDim = dim3(32 * kExchRowsPerBlock, 1, 1);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const unsigned token = next_launch_token();
  return dim == 64
             ? cudaLaunchKernelEx(&cfg, exchange_merge_kernel<64>, world, rank, epoch, splits, rows,
                                  partial_ml, partial_a, peer_buffers, out, token, err)
             : cudaLaunchKernelEx(&cfg, exchange_merge_kernel<128>, world, rank, epoch, splits,
                                  rows, partial_ml, partial_a, peer_buffers, out, token, err);
}

int bc_merge_gathered(int world, int splits, int rows, int dim, const float* gathered,
                      float* out, void* stream) {
  if (world < 1 || splits < 1 || rows < 1 || (dim != 64 && dim != 128) || !gathered || !out ||
      (long long)world * splits > 0x7fffffffLL)
    return cudaErrorInvalidValue;
  // rank r's block: splits*rows (m, l) pairs, then splits*rows*dim accumulators
  const long long ml_floats = (long long)splits * rows * 2;
  const long long block = ml_floats + (long long)splits * rows * dim;
  return launch_merge(dim, rows, world * splits, gathered, gathered + ml_floats, out,
                      static_cast<cudaStream_t>(stream), splits, block);
}

// ---------------------------------------------------------------------------
// Allocation-free decode: split partials in a library-owned device array.
// ---------------------------------------------------------------------------
}  // extern "C"

namespace {

// The array is a device symbol: host code must use its device address, which
// cudaGetSymbolAddress returns for the device that is current at the call.
static __device__ __align__(256) float bc_static_decode_scratch[BC_STATIC_SCRATCH_FLOATS];

// The array's device address on `dev` (current), looked up once per device.
// A failed look-up returns its own error code and clears it from the
// runtime's last-error slot, so the caller's next cudaGetLastError() does not
// report it a second time.
cudaError_t static_scratch_address(int dev, float** out) {
  static std::atomic<float*> cache[kMaxDevices];
  static std::mutex mu;
  float* p = cache[dev].load(std::memory_order_acquire);
  if (!p) {
    std::lock_guard<std::mutex> lock(mu);
    p = cache[dev].load(std::memory_order_relaxed);
    if (!p) {
      void* addr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&addr, bc_static_decode_scratch);
      if (e != cudaSuccess || !addr) {
        cudaGetLastError();
        return e != cudaSuccess ? e : cudaErrorInvalidDevice;
      }
      p = static_cast<float*>(addr);
      cache[dev].store(p, std::memory_order_release);
    }
  }
  *out = p;
  return cudaSuccess;
}

}  // namespace

extern "C" {

int bc_decode_static_scratch(const bc_shape* s, const void* q, const void* k, const void* v,
                             const int* pages, const int* lengths, float* output, int splits,
                             void* stream) {
  if (!basic_shape_ok(s) || splits < 1 || splits > BC_MAX_SPLITS || !q || !k || !v || !pages ||
      !lengths || !output)
    return cudaErrorInvalidValue;
  const long long rows = (long long)s->batch * s->query_heads;
  const long long need = (long long)splits * rows * (s->dim + 2);
  if (need > BC_STATIC_SCRATCH_FLOATS) return cudaErrorInvalidValue;  // beyond the fixed array
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  float* scratch = nullptr;
  const cudaError_t e = static_scratch_address(dev, &scratch);
  if (e != cudaSuccess) return e;
  float* partial_a = scratch;                                  // splits * rows * dim
  float* partial_ml = scratch + (long long)splits * rows * s->dim;  // splits * rows * 2
  return paged_decode_core(s, q, k, v, pages, lengths, output, false,
                           1.0f / std::sqrt(float(s->dim)), splits,
                           splits > 1 ? kSplitGlobal : kSplitNone, false, partial_a, partial_ml,
                           false, nullptr, static_cast<cudaStream_t>(stream));
}

int bc_selftest_bounded_wait(int ctas, int smem_bytes, unsigned limit_us, void* stream) {
  if (ctas < 1 || smem_bytes < 0 || smem_bytes > 200 * 1024 || limit_us < 1 ||
      limit_us > 2000000u)
    return cudaErrorInvalidValue;
  const int dev = current_device();
  if (dev < 0) return cudaErrorInvalidDevice;
  unsigned* err = error_word(dev);
  if (!err) return cudaErrorInvalidDevice;
  cudaError_t e = cudaFuncSetAttribute(selftest_wait_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return e;
  selftest_wait_kernel<<<ctas, 32, size_t(smem_bytes), static_cast<cudaStream_t>(stream)>>>(
      (unsigned long long)limit_us * 1000ull, next_launch_token(), err);
  return cudaGetLastError();
}

unsigned bc_last_device_error(int reset) {
  const int dev = current_device();
  if (dev < 0) return 0xffffffffu;
  if (cudaDeviceSynchronize() != cudaSuccess) return 0xffffffffu;
  unsigned word = 0;
  if (cudaMemcpyFromSymbol(&word, g_error_word, sizeof(word)) != cudaSuccess) return 0xffffffffu;
  if (reset) {
    // (the abort token too: a captured graph keeps its launches' tokens, so
    // a replay after a timeout would otherwise find itself aborted)
    const unsigned zero = 0;
    if (cudaMemcpyToSymbol(g_error_word, &zero, sizeof(zero)) != cudaSuccess ||
        cudaMemcpyToSymbol(g_abort_token, &zero, sizeof(zero)) != cudaSuccess)
      return 0xffffffffu;
  }
  return word;
}

const char* bc_version(void) { return "branchcraft-b200 0.1.0 (sm_100a)"; }

}  // extern "C"
