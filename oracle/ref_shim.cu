// TEST INFRASTRUCTURE ONLY: a C-ABI shim over the reference implementation,
// compiled from the reference's own, unmodified sources: its src/main.cu is
// included below with `main` renamed, and its src/paged_gqa.cu,
// src/tree_attention.cu and src/packed_decode.cu are compiled beside this file
// for sm_100a by oracle/Makefile into oracle/_ref/libbcref.so.
//
// It exposes the reference's CPU oracle and fixture generators (used to pin
// oracle/bc_oracle.cpp and to make the golden fixtures under tests/golden/)
// and the reference's own GPU launchers built for sm_100a (the "reference
// compiled for B200" comparison arm). Nothing in the product links it.
#define main branchcraft_reference_cli_main
#include "main.cu"  // the reference's src/main.cu, found through -I
#undef main

#include <cstring>

extern "C" {

struct BcrShape {
  int batch, query_heads, kv_heads, dim, max_pages, physical_pages;
};

}  // extern "C"

namespace {

Shape to_shape(const BcrShape& s) {
  return Shape{s.batch, s.query_heads, s.kv_heads, s.dim, s.max_pages, s.physical_pages};
}

void put_half(std::vector<half>& dst, const uint16_t* src, size_t n) {
  dst.resize(n);
  std::memcpy(dst.data(), src, n * sizeof(uint16_t));
}

void get_half(uint16_t* dst, const std::vector<half>& src) {
  std::memcpy(dst, src.data(), src.size() * sizeof(uint16_t));
}

Fixture fixture_from(const BcrShape& s, const uint16_t* q, const uint16_t* k,
                     const uint16_t* v, const int* pages, const int* lengths) {
  Fixture f;
  f.shape = to_shape(s);
  put_half(f.q, q, size_t(s.batch) * s.query_heads * s.dim);
  const size_t kv = size_t(s.physical_pages) * kPageSize * s.kv_heads * s.dim;
  put_half(f.k, k, kv);
  put_half(f.v, v, kv);
  f.pages.assign(pages, pages + size_t(s.batch) * s.max_pages);
  f.lengths.assign(lengths, lengths + s.batch);
  return f;
}

}  // namespace

extern "C" {

// make_fixture (src/main.cu:48-79): first call with null arrays to get sizes.
int bcr_make_fixture(int batch, int hq, int hkv, int dim, const int* lengths,
                     uint32_t seed, BcrShape* shape, uint16_t* q, uint16_t* k,
                     uint16_t* v, int* pages) {
  try {
    Fixture f = make_fixture(batch, hq, hkv, dim,
                             std::vector<int>(lengths, lengths + batch), seed);
    const Shape& s = f.shape;
    *shape = BcrShape{s.batch, s.query_heads, s.kv_heads, s.dim, s.max_pages, s.physical_pages};
    if (q) get_half(q, f.q);
    if (k) get_half(k, f.k);
    if (v) get_half(v, f.v);
    if (pages) std::memcpy(pages, f.pages.data(), f.pages.size() * sizeof(int));
    return 0;
  } catch (...) {
    return -1;
  }
}

// cpu_reference (src/main.cu:81-113).
int bcr_cpu_reference(const BcrShape* s, const uint16_t* q, const uint16_t* k,
                      const uint16_t* v, const int* pages, const int* lengths,
                      float* out) {
  Fixture f = fixture_from(*s, q, k, v, pages, lengths);
  const std::vector<float> r = cpu_reference(f);
  std::memcpy(out, r.data(), r.size() * sizeof(float));
  return 0;
}

// make_tree_fixture (src/main.cu:145-179): call with null arrays for sizes.
int bcr_make_tree_fixture(int batch, int prefix_len, int nodes, int dim,
                          uint32_t seed, BcrShape* shape, uint16_t* q,
                          uint16_t* k, uint16_t* v, int* pages, int* lengths,
                          uint16_t* draft_q, uint16_t* draft_k,
                          uint16_t* draft_v, int* parent) {
  try {
    TreeFixture t = make_tree_fixture(batch, prefix_len, nodes, dim, seed);
    const Shape& s = t.prefix.shape;
    *shape = BcrShape{s.batch, s.query_heads, s.kv_heads, s.dim, s.max_pages, s.physical_pages};
    if (q) get_half(q, t.prefix.q);
    if (k) get_half(k, t.prefix.k);
    if (v) get_half(v, t.prefix.v);
    if (pages) std::memcpy(pages, t.prefix.pages.data(), t.prefix.pages.size() * sizeof(int));
    if (lengths) std::memcpy(lengths, t.prefix.lengths.data(), t.prefix.lengths.size() * sizeof(int));
    if (draft_q) get_half(draft_q, t.draft_q);
    if (draft_k) get_half(draft_k, t.draft_k);
    if (draft_v) get_half(draft_v, t.draft_v);
    if (parent) std::memcpy(parent, t.parent.data(), t.parent.size() * sizeof(int));
    return 0;
  } catch (...) {
    return -1;
  }
}

// cpu_tree_reference (src/main.cu:204-240).
int bcr_cpu_tree_reference(const BcrShape* s, int nodes, const uint16_t* draft_q,
                           const uint16_t* k, const uint16_t* v,
                           const int* pages, const int* lengths,
                           const uint16_t* draft_k, const uint16_t* draft_v,
                           const int* parent, float* out) {
  TreeFixture t;
  t.nodes = nodes;
  t.prefix = fixture_from(*s, draft_q, k, v, pages, lengths);  // q unused
  const size_t nq = size_t(s->batch) * nodes * s->query_heads * s->dim;
  const size_t nkv = size_t(s->batch) * nodes * s->kv_heads * s->dim;
  put_half(t.draft_q, draft_q, nq);
  put_half(t.draft_k, draft_k, nkv);
  put_half(t.draft_v, draft_v, nkv);
  t.parent.assign(parent, parent + size_t(s->batch) * nodes);
  const std::vector<float> r = cpu_tree_reference(t);
  std::memcpy(out, r.data(), r.size() * sizeof(float));
  return 0;
}

// The reference's GPU launchers (device pointers), built for sm_100a.
int bcr_gpu_decode(const BcrShape* s, const void* q, const void* k, const void* v,
                   const int* pages, const int* lengths, float* out,
                   float* partial_a, float* partial_ml, int splits, void* stream) {
  Inputs in{static_cast<const half*>(q), static_cast<const half*>(k),
            static_cast<const half*>(v), pages, lengths, out};
  return int(branchcraft::decode(to_shape(*s), in, Scratch{partial_a, partial_ml},
                                 splits, static_cast<cudaStream_t>(stream)));
}

int bcr_gpu_auto_splits(const BcrShape* s, int max_length, int sm_count) {
  return branchcraft::auto_splits(to_shape(*s), max_length, sm_count);
}

int bcr_gpu_tree_verify(const BcrShape* s, int nodes, const void* draft_q,
                        const void* k, const void* v, const int* pages,
                        const int* lengths, const void* draft_k,
                        const void* draft_v, const int* parent, float* out,
                        void* stream) {
  Inputs prefix{nullptr, static_cast<const half*>(k), static_cast<const half*>(v),
                pages, lengths, nullptr};
  branchcraft::TreeInputs in{prefix, static_cast<const half*>(draft_q),
                             static_cast<const half*>(draft_k),
                             static_cast<const half*>(draft_v), parent, out};
  return int(branchcraft::tree_verify(to_shape(*s), in, nodes,
                                      static_cast<cudaStream_t>(stream)));
}

int bcr_gpu_commit_path(const BcrShape* s, const void* draft_k, const void* draft_v,
                        void* cache_k, void* cache_v, const int* path_nodes,
                        const int* dest_pages, const int* dest_slots,
                        int request, int nodes, int accepted, void* stream) {
  return int(branchcraft::commit_path(
      to_shape(*s), static_cast<const half*>(draft_k), static_cast<const half*>(draft_v),
      static_cast<half*>(cache_k), static_cast<half*>(cache_v), path_nodes,
      dest_pages, dest_slots, request, nodes, accepted,
      static_cast<cudaStream_t>(stream)));
}

int bcr_gpu_packed_decode(const BcrShape* s, const void* q, const void* packed_kv,
                          const int* pages, const int* lengths, void* output,
                          long long block_stride, long long head_stride,
                          long long slot_stride, float scale, void* stream) {
  return int(branchcraft::packed_decode(
      to_shape(*s), static_cast<const half*>(q), static_cast<const half*>(packed_kv),
      pages, lengths, static_cast<half*>(output), block_stride, head_stride,
      slot_stride, scale, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
