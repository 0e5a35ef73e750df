// CPU oracle for the branchcraft attention hot path.
//
// TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is
// compared against. Only the pytest suite, the smoke check and the CPU-baseline
// leg of bench.py may load it; the product library never links or calls it.
//
// Every function restates an algorithm of the reference implementation
// (Haaziq386/branchcraft-cuda) in plain C++ with double accumulation:
//   bco_decode        <- src/main.cu:81-113    (cpu_reference)
//   bco_tree          <- src/main.cu:204-240   (cpu_tree_reference)
//   bco_packed_decode <- tests/test_torch_ops.py:77-88 (FP32 softmax, then FP16)
//   bco_commit        <- src/tree_attention.cu:73-89 (commit_kernel semantics)
//   bco_merge         <- src/paged_gqa.cu:76-106 (FP32 (m, l, o) merge)
//   bco_ref_fixture / bco_ref_tree_fixture
//                     <- src/main.cu:48-79 and :145-179 (seeded fixture
//                        generators; they use the C++ standard library's
//                        mt19937, shuffle and normal_distribution exactly as
//                        the reference does, so the same seed gives the same
//                        bytes on the same standard library)
//
// FP16 values travel as raw uint16 bit patterns; conversion is IEEE binary16
// with round-to-nearest-even (the same rounding as CUDA's __float2half).
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <random>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

constexpr int kPage = 16;

inline uint32_t f2u(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float u2f(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

// binary16 -> binary32 (exact).
inline float h2f(uint16_t h) {
  const uint32_t sign = uint32_t(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t man = h & 0x3ffu;
  if (exp == 0x1f) return u2f(sign | 0x7f800000u | (man << 13));  // inf / nan
  if (exp != 0) return u2f(sign | ((exp + 112u) << 23) | (man << 13));
  if (man == 0) return u2f(sign);
  // subnormal: value = man * 2^-24
  int e = -1;
  do { ++e; man <<= 1; } while ((man & 0x400u) == 0);
  return u2f(sign | ((112u - uint32_t(e)) << 23) | ((man & 0x3ffu) << 13));
}

// binary32 -> binary16, round to nearest, ties to even.
inline uint16_t f2h(float f) {
  const uint32_t u = f2u(f);
  const uint16_t sign = uint16_t((u >> 16) & 0x8000u);
  const uint32_t a = u & 0x7fffffffu;
  if (a >= 0x7f800000u)  // inf or nan (keep a quiet payload bit for nan)
    return sign | (a > 0x7f800000u ? uint16_t(0x7e00u | ((a >> 13) & 0x3ffu)) : 0x7c00u);
  if (a >= 0x477ff000u) return sign | 0x7c00u;  // rounds to >= 65520 -> inf
  if (a >= 0x38800000u) {                       // normal half range
    const uint32_t mant = a & 0x7fffffu;
    uint32_t h = ((a >> 23) - 112u) << 10 | (mant >> 13);
    const uint32_t rest = mant & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (h & 1u))) ++h;
    return sign | uint16_t(h);
  }
  if (a < 0x33000000u) return sign;  // below half of the smallest subnormal
  // subnormal half: value = round(x * 2^24)
  const uint32_t e = a >> 23;               // 102..112
  const uint32_t mant = (a & 0x7fffffu) | 0x800000u;
  const uint32_t shift = 126u - e;          // 14..24
  uint32_t h = mant >> shift;
  const uint32_t rest = mant & ((1u << shift) - 1u);
  const uint32_t halfway = 1u << (shift - 1u);
  if (rest > halfway || (rest == halfway && (h & 1u))) ++h;
  return sign | uint16_t(h);
}

// h2f of every binary16 pattern, built once: the attention loops convert
// each K/V element through this table (same values as h2f, no branches).
const float* h2f_table() {
  static const std::vector<float> table = [] {
    std::vector<float> t(65536);
    for (uint32_t h = 0; h < 65536; ++h) t[h] = h2f(uint16_t(h));
    return t;
  }();
  return table.data();
}

inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

void set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}

}  // namespace

extern "C" {

struct BcoShape {
  int batch, query_heads, kv_heads, dim, max_pages, physical_pages;
};

float bco_h2f(uint16_t h) { return h2f(h); }
uint16_t bco_f2h(float f) { return f2h(f); }

void bco_h2f_array(const uint16_t* in, float* out, long long n) {
  for (long long i = 0; i < n; ++i) out[i] = h2f(in[i]);
}
void bco_f2h_array(const float* in, uint16_t* out, long long n) {
  for (long long i = 0; i < n; ++i) out[i] = f2h(in[i]);
}

// ---------------------------------------------------------------------------
// Fixture generators (reference src/main.cu:48-79 and :145-179).
// ---------------------------------------------------------------------------

// Sizes of make_fixture's output: max_pages = max(1, ceil(max_len/16)),
// physical_pages = sum(ceil(len/16)) + 7.
int bco_ref_fixture_shape(int batch, const int* lengths, int* max_pages,
                          int* physical_pages) {
  int max_len = 0, used = 0;
  for (int b = 0; b < batch; ++b) {
    if (lengths[b] < 0) return -1;
    max_len = std::max(max_len, lengths[b]);
    used += ceil_div(lengths[b], kPage);
  }
  *max_pages = std::max(1, ceil_div(max_len, kPage));
  *physical_pages = used + 7;
  return 0;
}

// Fills q [B,Hq,D], k/v [P,16,Hkv,D], pages [B,max_pages] exactly as the
// reference fixture does: shuffled page ids, then N(0, 0.5) draws for q, k, v
// in that order from one mt19937 stream.
int bco_ref_fixture(int batch, int hq, int hkv, int dim, const int* lengths,
                    uint32_t seed, uint16_t* q, uint16_t* k, uint16_t* v,
                    int* pages) {
  int max_pages = 0, physical = 0;
  if (bco_ref_fixture_shape(batch, lengths, &max_pages, &physical)) return -1;
  std::fill(pages, pages + size_t(batch) * max_pages, -1);
  std::mt19937 gen(seed);
  std::vector<int> ids(physical);
  std::iota(ids.begin(), ids.end(), 0);
  std::shuffle(ids.begin(), ids.end(), gen);
  int cursor = 0;
  for (int b = 0; b < batch; ++b)
    for (int p = 0; p < ceil_div(lengths[b], kPage); ++p)
      pages[b * max_pages + p] = ids[cursor++];
  std::normal_distribution<float> dist(0.f, 0.5f);
  const size_t nq = size_t(batch) * hq * dim;
  const size_t nkv = size_t(physical) * kPage * hkv * dim;
  for (size_t i = 0; i < nq; ++i) q[i] = f2h(dist(gen));
  for (size_t i = 0; i < nkv; ++i) k[i] = f2h(dist(gen));
  for (size_t i = 0; i < nkv; ++i) v[i] = f2h(dist(gen));
  return 0;
}

// Tree fixture (src/main.cu:145-179): the prefix is a one-request fixture with
// Hq=32, Hkv=8 whose pages and query are shared by every request; the physical
// pool grows by 2 pages per request (zero-filled) and the page table by 2
// columns. Draft q/k/v come from a second stream seeded seed+99; parents form
// a binary tree (n-1)/2.
// Shapes: out_shape = {batch, 32, 8, dim, max_pages, physical_pages}.
int bco_ref_tree_fixture_shape(int batch, int prefix_len, BcoShape* out_shape) {
  int mp = 0, phys = 0;
  if (bco_ref_fixture_shape(1, &prefix_len, &mp, &phys)) return -1;
  *out_shape = BcoShape{batch, 32, 8, 0, mp + 2, phys + batch * 2};
  return 0;
}

int bco_ref_tree_fixture(int batch, int prefix_len, int nodes, int dim,
                         uint32_t seed, uint16_t* q, uint16_t* k, uint16_t* v,
                         int* pages, int* lengths, uint16_t* draft_q,
                         uint16_t* draft_k, uint16_t* draft_v, int* parent) {
  if (nodes < 1) return -1;
  int mp = 0, phys = 0;
  bco_ref_fixture_shape(1, &prefix_len, &mp, &phys);
  const size_t base_q = size_t(32) * dim;
  const size_t base_kv = size_t(phys) * kPage * 8 * dim;
  std::vector<uint16_t> bq(base_q), bk(base_kv), bv(base_kv);
  std::vector<int> bpages(mp);
  bco_ref_fixture(1, 32, 8, dim, &prefix_len, seed, bq.data(), bk.data(),
                  bv.data(), bpages.data());
  const int max_pages = mp + 2, physical = phys + batch * 2;
  std::fill(pages, pages + size_t(batch) * max_pages, -1);
  for (int b = 0; b < batch; ++b) {
    lengths[b] = prefix_len;
    for (int p = 0; p < ceil_div(prefix_len, kPage); ++p)
      pages[b * max_pages + p] = bpages[p];
    std::copy(bq.begin(), bq.end(), q + size_t(b) * base_q);
  }
  const size_t full_kv = size_t(physical) * kPage * 8 * dim;
  std::copy(bk.begin(), bk.end(), k);
  std::copy(bv.begin(), bv.end(), v);
  std::fill(k + base_kv, k + full_kv, uint16_t(0));
  std::fill(v + base_kv, v + full_kv, uint16_t(0));
  std::mt19937 gen(seed + 99);
  std::normal_distribution<float> dist(0.f, .5f);
  const size_t ndq = size_t(batch) * nodes * 32 * dim;
  const size_t ndkv = size_t(batch) * nodes * 8 * dim;
  for (size_t i = 0; i < ndq; ++i) draft_q[i] = f2h(dist(gen));
  for (size_t i = 0; i < ndkv; ++i) draft_k[i] = f2h(dist(gen));
  for (size_t i = 0; i < ndkv; ++i) draft_v[i] = f2h(dist(gen));
  for (int b = 0; b < batch; ++b)
    for (int n = 0; n < nodes; ++n) parent[b * nodes + n] = n == 0 ? -1 : (n - 1) / 2;
  return 0;
}

// ---------------------------------------------------------------------------
// Attention oracles.
// ---------------------------------------------------------------------------

// Paged GQA decode, src/main.cu:81-113: double dot products, the scaled score
// stored as float, exp in double of (float score - float max), output
// accumulated in float and divided by the double denominator only when it is
// non-zero (empty sequences give zeros).
void bco_decode(const BcoShape* shape, const uint16_t* q, const uint16_t* k,
                const uint16_t* v, const int* pages, const int* lengths,
                float* out, int threads) {
  const BcoShape s = *shape;
  set_threads(threads);
  const float* hf = h2f_table();
  const int group = s.query_heads / s.kv_heads;
  const double root = std::sqrt(double(s.dim));
#pragma omp parallel for schedule(dynamic, 1)
  for (int row = 0; row < s.batch * s.query_heads; ++row) {
    const int b = row / s.query_heads, h = row % s.query_heads;
    const int kvh = h / group;
    const size_t qbase = size_t(row) * s.dim;
    const int len = lengths[b];
    std::vector<float> scores(std::max(len, 0));
    std::vector<float> qf(s.dim);
    for (int d = 0; d < s.dim; ++d) qf[d] = h2f(q[qbase + d]);
    float* o = out + qbase;
    for (int d = 0; d < s.dim; ++d) o[d] = 0.f;
    float max_score = -INFINITY;
    for (int t = 0; t < len; ++t) {
      const long long phys = pages[size_t(b) * s.max_pages + t / kPage];
      const size_t base = ((size_t(phys) * kPage + t % kPage) * s.kv_heads + kvh) * s.dim;
      double dot = 0;
      for (int d = 0; d < s.dim; ++d) dot += double(qf[d]) * hf[k[base + d]];
      scores[t] = float(dot / root);
      max_score = std::max(max_score, scores[t]);
    }
    double denom = 0;
    for (int t = 0; t < len; ++t) {
      const double p = std::exp(double(scores[t] - max_score));
      denom += p;
      const long long phys = pages[size_t(b) * s.max_pages + t / kPage];
      const size_t base = ((size_t(phys) * kPage + t % kPage) * s.kv_heads + kvh) * s.dim;
      for (int d = 0; d < s.dim; ++d) o[d] += float(p * hf[v[base + d]]);
    }
    if (denom != 0)
      for (int d = 0; d < s.dim; ++d) o[d] /= float(denom);
  }
}

// Tree verify, src/main.cu:204-240: for each (request, node, q-head) the keys
// are the request's prefix tokens followed by the node's ancestor chain walked
// leaf to root (the node itself first). Scores stay in double.
// Any negative parent ends a chain (as in the reference). Returns 0, or -1
// if a chain leaves [0, nodes) or is longer than `nodes` (a cycle, on which
// the reference would loop forever).
int bco_tree(const BcoShape* shape, int nodes, const uint16_t* draft_q,
             const uint16_t* k, const uint16_t* v, const int* pages,
             const int* lengths, const uint16_t* draft_k,
             const uint16_t* draft_v, const int* parent, float* out,
             int threads) {
  const BcoShape s = *shape;
  for (int b = 0; b < s.batch; ++b)
    for (int n = 0; n < nodes; ++n) {
      int cur = n, steps = 0;
      while (cur >= 0) {
        if (cur >= nodes || steps >= nodes) return -1;
        cur = parent[b * nodes + cur];
        ++steps;
      }
    }
  set_threads(threads);
  const float* hf = h2f_table();
  const int group = s.query_heads / s.kv_heads;
  const double root = std::sqrt(double(s.dim));
  const int rows = s.batch * nodes * s.query_heads;
#pragma omp parallel for schedule(dynamic, 1)
  for (int row = 0; row < rows; ++row) {
    const int h = row % s.query_heads;
    const int node = (row / s.query_heads) % nodes;
    const int b = row / (s.query_heads * nodes);
    const int kvh = h / group;
    const size_t qbase = size_t(row) * s.dim;
    std::vector<float> qf(s.dim);
    for (int d = 0; d < s.dim; ++d) qf[d] = h2f(draft_q[qbase + d]);
    struct Tok { size_t base; bool draft; };
    std::vector<Tok> toks;
    for (int t = 0; t < lengths[b]; ++t) {
      const long long phys = pages[size_t(b) * s.max_pages + t / kPage];
      toks.push_back({((size_t(phys) * kPage + t % kPage) * s.kv_heads + kvh) * s.dim, false});
    }
    for (int cur = node; cur >= 0; cur = parent[b * nodes + cur])
      toks.push_back({((size_t(b) * nodes + cur) * s.kv_heads + kvh) * s.dim, true});
    std::vector<double> sc(toks.size());
    double mx = -INFINITY;
    for (size_t t = 0; t < toks.size(); ++t) {
      const uint16_t* kk = toks[t].draft ? draft_k : k;
      double dot = 0;
      for (int d = 0; d < s.dim; ++d) dot += double(qf[d]) * hf[kk[toks[t].base + d]];
      sc[t] = dot / root;
      mx = std::max(mx, sc[t]);
    }
    float* o = out + qbase;
    for (int d = 0; d < s.dim; ++d) o[d] = 0.f;
    double denom = 0;
    for (size_t t = 0; t < toks.size(); ++t) {
      const double p = std::exp(sc[t] - mx);
      denom += p;
      const uint16_t* vv = toks[t].draft ? draft_v : v;
      for (int d = 0; d < s.dim; ++d) o[d] += float(p * hf[vv[toks[t].base + d]]);
    }
    for (int d = 0; d < s.dim; ++d) o[d] /= float(denom);
  }
  return 0;
}

// Packed-cache decode (tests/test_torch_ops.py:77-88, src/packed_decode.cu):
// K of (page, kv-head, slot) starts at page*block_stride + kvh*head_stride +
// slot*slot_stride elements and V at kv_offset elements after it (the
// reference fixes kv_offset = D). Softmax in double with the caller's scale;
// the FP32 result is rounded once to FP16. Empty sequences give zeros.
void bco_packed_decode(const BcoShape* shape, const uint16_t* q,
                       const uint16_t* cache, const int* pages,
                       const int* lengths, long long block_stride,
                       long long head_stride, long long slot_stride,
                       long long kv_offset, float scale, uint16_t* out,
                       float* out_f32, int threads) {
  const BcoShape s = *shape;
  set_threads(threads);
  const float* hf = h2f_table();
  const int group = s.query_heads / s.kv_heads;
#pragma omp parallel for schedule(dynamic, 1)
  for (int row = 0; row < s.batch * s.query_heads; ++row) {
    const int b = row / s.query_heads, h = row % s.query_heads;
    const int kvh = h / group;
    const size_t qbase = size_t(row) * s.dim;
    const int len = lengths[b];
    std::vector<double> sc(std::max(len, 0));
    std::vector<double> acc(s.dim, 0.0);
    std::vector<float> qf(s.dim);
    for (int d = 0; d < s.dim; ++d) qf[d] = h2f(q[qbase + d]);
    double mx = -INFINITY;
    for (int t = 0; t < len; ++t) {
      const long long phys = pages[size_t(b) * s.max_pages + t / kPage];
      const long long off = phys * block_stride + kvh * head_stride + (t % kPage) * slot_stride;
      double dot = 0;
      for (int d = 0; d < s.dim; ++d) dot += double(qf[d]) * hf[cache[off + d]];
      sc[t] = dot * double(scale);
      mx = std::max(mx, sc[t]);
    }
    double denom = 0;
    for (int t = 0; t < len; ++t) {
      const double p = std::exp(sc[t] - mx);
      denom += p;
      const long long phys = pages[size_t(b) * s.max_pages + t / kPage];
      const long long off = phys * block_stride + kvh * head_stride + (t % kPage) * slot_stride + kv_offset;
      for (int d = 0; d < s.dim; ++d) acc[d] += p * hf[cache[off + d]];
    }
    for (int d = 0; d < s.dim; ++d) {
      const float r = denom > 0 ? float(acc[d] / denom) : 0.f;
      if (out) out[qbase + d] = f2h(r);
      if (out_f32) out_f32[qbase + d] = r;
    }
  }
}

// commit_path (src/tree_attention.cu:73-89): for i < accepted,
// cache[dest_pages[i], dest_slots[i], :, :] = draft[request, path_nodes[i], :, :]
// for K and V, applied in path order. Returns -1 on an out-of-range index.
int bco_commit(int kv_heads, int dim, int physical_pages, int nodes,
               const uint16_t* draft_k, const uint16_t* draft_v,
               uint16_t* cache_k, uint16_t* cache_v, const int* path_nodes,
               const int* dest_pages, const int* dest_slots, int request,
               int accepted) {
  const size_t elems = size_t(kv_heads) * dim;
  for (int i = 0; i < accepted; ++i) {
    const int node = path_nodes[i], page = dest_pages[i], slot = dest_slots[i];
    if (node < 0 || node >= nodes || page < 0 || page >= physical_pages ||
        slot < 0 || slot >= kPage)
      return -1;
    const size_t src = (size_t(request) * nodes + node) * elems;
    const size_t dst = (size_t(page) * kPage + slot) * elems;
    std::copy(draft_k + src, draft_k + src + elems, cache_k + dst);
    std::copy(draft_v + src, draft_v + src + elems, cache_v + dst);
  }
  return 0;
}

// FP32 merge of split partial states (src/paged_gqa.cu:76-106).
// partial_ml[(part*rows + r)*2 + {0,1}] = (m, l); partial_a[(part*rows + r)*D].
// All-empty rows (every m = -inf) give zeros.
void bco_merge(int splits, int rows, int dim, const float* partial_ml,
               const float* partial_a, float* out) {
  for (int r = 0; r < rows; ++r) {
    double mx = -INFINITY;
    for (int p = 0; p < splits; ++p) mx = std::max(mx, double(partial_ml[(size_t(p) * rows + r) * 2]));
    float* o = out + size_t(r) * dim;
    if (mx == -INFINITY) { std::fill(o, o + dim, 0.f); continue; }
    double denom = 0;
    std::vector<double> acc(dim, 0.0);
    for (int p = 0; p < splits; ++p) {
      const size_t row = size_t(p) * rows + r;
      const double w = std::exp(double(partial_ml[row * 2]) - mx);
      denom += w * partial_ml[row * 2 + 1];
      for (int d = 0; d < dim; ++d) acc[d] += w * partial_a[row * dim + d];
    }
    for (int d = 0; d < dim; ++d) o[d] = float(acc[d] / denom);
  }
}

int bco_max_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
