// `branchcraft test | bench | tree-bench [--quick] [--output FILE]` — the
// reference's standalone driver (src/main.cu:527-553) rebuilt on this
// library's C++ API (include/branchcraft.hpp), with the same modes, seeds,
// tolerances and CSV columns.
//
// Test infrastructure: `test` compares the GPU against the CPU oracle
// (oracle/bc_oracle.cpp, linked in as the checker); `bench` and `tree-bench`
// compare GPU paths with each other (split vs single, tree vs expanded cache),
// as the reference does.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <iterator>
#include <numeric>
#include <stdexcept>
#include <string>
#include <vector>

#include "branchcraft.hpp"

extern "C" {
struct BcoShape {
  int batch, query_heads, kv_heads, dim, max_pages, physical_pages;
};
int bco_ref_fixture_shape(int batch, const int* lengths, int* max_pages, int* physical_pages);
int bco_ref_fixture(int batch, int hq, int hkv, int dim, const int* lengths, uint32_t seed,
                    uint16_t* q, uint16_t* k, uint16_t* v, int* pages);
int bco_ref_tree_fixture_shape(int batch, int prefix_len, BcoShape* out_shape);
int bco_ref_tree_fixture(int batch, int prefix_len, int nodes, int dim, uint32_t seed,
                         uint16_t* q, uint16_t* k, uint16_t* v, int* pages, int* lengths,
                         uint16_t* draft_q, uint16_t* draft_k, uint16_t* draft_v, int* parent);
void bco_decode(const BcoShape* shape, const uint16_t* q, const uint16_t* k, const uint16_t* v,
                const int* pages, const int* lengths, float* out, int threads);
int bco_tree(const BcoShape* shape, int nodes, const uint16_t* draft_q, const uint16_t* k,
             const uint16_t* v, const int* pages, const int* lengths, const uint16_t* draft_k,
             const uint16_t* draft_v, const int* parent, float* out, int threads);
}

using branchcraft::kPageSize;
using branchcraft::Shape;

#define CHECK(call)                                                                          \
  do {                                                                                       \
    cudaError_t e_ = (call);                                                                 \
    if (e_ != cudaSuccess)                                                                   \
      throw std::runtime_error(std::string(#call) + ": " + cudaGetErrorString(e_));          \
  } while (0)

template <typename T>
struct Dev {
  T* ptr = nullptr;
  size_t count = 0;
  Dev() = default;
  explicit Dev(size_t n) : count(n) { CHECK(cudaMalloc(&ptr, std::max<size_t>(1, n) * sizeof(T))); }
  Dev(const Dev&) = delete;
  Dev& operator=(const Dev&) = delete;
  ~Dev() {
    if (ptr) cudaFree(ptr);
  }
  void up(const std::vector<T>& v) {
    if (v.size() != count) throw std::runtime_error("upload size mismatch");
    CHECK(cudaMemcpy(ptr, v.data(), count * sizeof(T), cudaMemcpyHostToDevice));
  }
  std::vector<T> down() const {
    std::vector<T> v(count);
    CHECK(cudaMemcpy(v.data(), ptr, count * sizeof(T), cudaMemcpyDeviceToHost));
    return v;
  }
};

struct Fixture {
  Shape shape;
  std::vector<uint16_t> q, k, v;
  std::vector<int> pages, lengths;
};

Fixture make_fixture(int batch, int hq, int hkv, int dim, std::vector<int> lengths,
                     uint32_t seed = 17) {
  int mp = 0, phys = 0;
  if (bco_ref_fixture_shape(batch, lengths.data(), &mp, &phys))
    throw std::runtime_error("negative length");
  Fixture f{{batch, hq, hkv, dim, mp, phys}};
  f.lengths = lengths;
  f.q.resize(size_t(batch) * hq * dim);
  f.k.resize(size_t(phys) * kPageSize * hkv * dim);
  f.v.resize(f.k.size());
  f.pages.resize(size_t(batch) * mp);
  bco_ref_fixture(batch, hq, hkv, dim, lengths.data(), seed, f.q.data(), f.k.data(), f.v.data(),
                  f.pages.data());
  return f;
}

BcoShape to_oracle(const Shape& s) {
  return {s.batch, s.query_heads, s.kv_heads, s.dim, s.max_pages, s.physical_pages};
}

std::vector<float> cpu_decode(const Fixture& f) {
  std::vector<float> out(size_t(f.shape.batch) * f.shape.query_heads * f.shape.dim);
  const BcoShape s = to_oracle(f.shape);
  bco_decode(&s, f.q.data(), f.k.data(), f.v.data(), f.pages.data(), f.lengths.data(), out.data(),
             0);
  return out;
}

struct GpuFixture {
  Dev<uint16_t> q, k, v;
  Dev<int> pages, lengths;
  Dev<float> output, partial_a, partial_ml;
  Shape shape;
  explicit GpuFixture(const Fixture& f)
      : q(f.q.size()), k(f.k.size()), v(f.v.size()), pages(f.pages.size()),
        lengths(f.lengths.size()),
        output(size_t(f.shape.batch) * f.shape.query_heads * f.shape.dim),
        partial_a(64 * output.count),
        partial_ml(64 * size_t(f.shape.batch) * f.shape.query_heads * 2), shape(f.shape) {
    q.up(f.q);
    k.up(f.k);
    v.up(f.v);
    pages.up(f.pages);
    lengths.up(f.lengths);
  }
  branchcraft::Inputs inputs() {
    return {reinterpret_cast<const half*>(q.ptr), reinterpret_cast<const half*>(k.ptr),
            reinterpret_cast<const half*>(v.ptr), pages.ptr, lengths.ptr, output.ptr};
  }
  branchcraft::Scratch scratch() { return {partial_a.ptr, partial_ml.ptr}; }
  void run(int splits) {
    CHECK(branchcraft::decode(shape, inputs(), scratch(), splits));
    CHECK(cudaDeviceSynchronize());
  }
};

struct TreeFixture {
  Fixture prefix;
  int nodes = 0;
  std::vector<uint16_t> draft_q, draft_k, draft_v;
  std::vector<int> parent;
};

TreeFixture make_tree_fixture(int batch, int prefix_len, int nodes, int dim, uint32_t seed = 31) {
  BcoShape s{};
  bco_ref_tree_fixture_shape(batch, prefix_len, &s);
  TreeFixture t;
  t.nodes = nodes;
  t.prefix.shape = {batch, 32, 8, dim, s.max_pages, s.physical_pages};
  t.prefix.q.resize(size_t(batch) * 32 * dim);
  t.prefix.k.resize(size_t(s.physical_pages) * kPageSize * 8 * dim);
  t.prefix.v.resize(t.prefix.k.size());
  t.prefix.pages.resize(size_t(batch) * s.max_pages);
  t.prefix.lengths.resize(batch);
  t.draft_q.resize(size_t(batch) * nodes * 32 * dim);
  t.draft_k.resize(size_t(batch) * nodes * 8 * dim);
  t.draft_v.resize(t.draft_k.size());
  t.parent.resize(size_t(batch) * nodes);
  if (bco_ref_tree_fixture(batch, prefix_len, nodes, dim, seed, t.prefix.q.data(),
                           t.prefix.k.data(), t.prefix.v.data(), t.prefix.pages.data(),
                           t.prefix.lengths.data(), t.draft_q.data(), t.draft_k.data(),
                           t.draft_v.data(), t.parent.data()))
    throw std::runtime_error("bad tree fixture");
  return t;
}

std::vector<float> cpu_tree(const TreeFixture& t) {
  std::vector<float> out(t.draft_q.size());
  const BcoShape s = to_oracle(t.prefix.shape);
  if (bco_tree(&s, t.nodes, t.draft_q.data(), t.prefix.k.data(), t.prefix.v.data(),
               t.prefix.pages.data(), t.prefix.lengths.data(), t.draft_k.data(), t.draft_v.data(),
               t.parent.data(), out.data(), 0))
    throw std::runtime_error("bad parent pointers");
  return out;
}

struct TreeGpu {
  GpuFixture prefix;
  Dev<uint16_t> draft_q, draft_k, draft_v;
  Dev<int> parent;
  Dev<float> output;
  int nodes;
  explicit TreeGpu(const TreeFixture& f)
      : prefix(f.prefix), draft_q(f.draft_q.size()), draft_k(f.draft_k.size()),
        draft_v(f.draft_v.size()), parent(f.parent.size()), output(f.draft_q.size()),
        nodes(f.nodes) {
    draft_q.up(f.draft_q);
    draft_k.up(f.draft_k);
    draft_v.up(f.draft_v);
    parent.up(f.parent);
  }
  branchcraft::TreeInputs inputs() {
    return {prefix.inputs(), reinterpret_cast<const half*>(draft_q.ptr),
            reinterpret_cast<const half*>(draft_k.ptr), reinterpret_cast<const half*>(draft_v.ptr),
            parent.ptr, output.ptr};
  }
  void run() {
    CHECK(branchcraft::tree_verify(prefix.shape, inputs(), nodes));
    CHECK(cudaDeviceSynchronize());
  }
};

// The comparison the CLI gates on: the largest elementwise |a - b|, where a
// pair with a non-finite member counts as an infinite difference (so a NaN or
// an overflow can never pass a tolerance).
float max_abs_error(const std::vector<float>& a, const std::vector<float>& b) {
  if (a.size() != b.size()) throw std::runtime_error("comparison size mismatch");
  const auto gap = [](float x, float y) {
    return std::isfinite(x) && std::isfinite(y) ? std::fabs(x - y) : INFINITY;
  };
  const auto larger = [](float x, float y) { return x < y ? y : x; };
  return std::transform_reduce(a.begin(), a.end(), b.begin(), 0.0f, larger, gap);
}

void check_device_errors() {
  const unsigned word = bc_last_device_error(1);
  if (word) throw std::runtime_error("device error word " + std::to_string(word));
}

void run_tests() {
  struct Case {
    int b, hq, hkv, d;
    std::vector<int> lens;
  };
  const std::vector<Case> cases = {
      {1, 8, 2, 64, {0}},          {1, 8, 2, 64, {1}},
      {1, 8, 2, 64, {16}},         {1, 8, 2, 64, {17}},
      {3, 10, 2, 64, {0, 37, 91}}, {3, 12, 3, 128, {7, 128, 257}},
      {2, 32, 8, 128, {513, 3}},
  };
  int checks = 0;
  for (const auto& c : cases) {
    Fixture f = make_fixture(c.b, c.hq, c.hkv, c.d, c.lens);
    const auto expected = cpu_decode(f);
    GpuFixture gpu(f);
    for (int splits : {1, 2, 4, 8, 16, 64}) {
      gpu.run(splits);
      const float error = max_abs_error(expected, gpu.output.down());
      if (error > 3e-4f)
        throw std::runtime_error("FAIL B=" + std::to_string(c.b) + " D=" + std::to_string(c.d) +
                                 " splits=" + std::to_string(splits) +
                                 " max_abs_error=" + std::to_string(error));
      ++checks;
    }
  }
  Fixture f = make_fixture(1, 8, 2, 64, {17});
  GpuFixture gpu(f);
  Shape bad = f.shape;
  bad.dim = 96;
  if (branchcraft::decode(bad, gpu.inputs(), gpu.scratch(), 1) != cudaErrorInvalidValue ||
      branchcraft::decode(f.shape, gpu.inputs(), {nullptr, nullptr}, 2) != cudaErrorInvalidValue)
    throw std::runtime_error("invalid API arguments were accepted");
  check_device_errors();
  std::cout << "PASS " << checks << " CPU-oracle checks across empty, page-boundary,"
            << " ragged, GQA, D64/D128, and split-KV cases.\n";
}

void run_tree_tests() {
  int checks = 0;
  for (const auto& spec : std::vector<std::pair<int, int>>{{0, 64}, {17, 64}, {257, 128}}) {
    TreeFixture f = make_tree_fixture(2, spec.first, 7, spec.second);
    TreeGpu gpu(f);
    gpu.run();
    const float error = max_abs_error(cpu_tree(f), gpu.output.down());
    if (error > 3e-4f)
      throw std::runtime_error("tree CPU-oracle mismatch, max error=" + std::to_string(error));
    ++checks;
  }
  // Shared partial final page: clone it, commit path {0,1,3} to slots 1..3,
  // check accepted == tree output of node 3, sibling untouched, rollback exact.
  TreeFixture f = make_tree_fixture(2, 17, 7, 128, 49);
  TreeGpu gpu(f);
  gpu.run();
  const auto tree_out = gpu.output.down();
  gpu.prefix.run(1);
  const auto before = gpu.prefix.output.down();
  const int new_page = f.prefix.shape.physical_pages - 1;
  const int old_page = f.prefix.pages[1];
  const size_t page_elems = size_t(kPageSize) * f.prefix.shape.kv_heads * f.prefix.shape.dim;
  CHECK(cudaMemcpy(gpu.prefix.k.ptr + size_t(new_page) * page_elems,
                   gpu.prefix.k.ptr + size_t(old_page) * page_elems, page_elems * 2,
                   cudaMemcpyDeviceToDevice));
  CHECK(cudaMemcpy(gpu.prefix.v.ptr + size_t(new_page) * page_elems,
                   gpu.prefix.v.ptr + size_t(old_page) * page_elems, page_elems * 2,
                   cudaMemcpyDeviceToDevice));
  Dev<int> path(3), dest_pages(3), dest_slots(3);
  path.up({0, 1, 3});
  dest_pages.up({new_page, new_page, new_page});
  dest_slots.up({1, 2, 3});
  CHECK(branchcraft::commit_path(f.prefix.shape, reinterpret_cast<const half*>(gpu.draft_k.ptr),
                                 reinterpret_cast<const half*>(gpu.draft_v.ptr),
                                 reinterpret_cast<half*>(gpu.prefix.k.ptr),
                                 reinterpret_cast<half*>(gpu.prefix.v.ptr), path.ptr,
                                 dest_pages.ptr, dest_slots.ptr, 0, f.nodes, 3));
  CHECK(cudaDeviceSynchronize());
  auto committed_pages = f.prefix.pages;
  auto committed_lengths = f.prefix.lengths;
  committed_pages[1] = new_page;
  committed_lengths[0] += 3;
  gpu.prefix.pages.up(committed_pages);
  gpu.prefix.lengths.up(committed_lengths);
  const size_t query_elems = size_t(f.prefix.shape.query_heads) * f.prefix.shape.dim;
  CHECK(cudaMemcpy(gpu.prefix.q.ptr, gpu.draft_q.ptr + 3 * query_elems, query_elems * 2,
                   cudaMemcpyDeviceToDevice));
  gpu.prefix.run(1);
  const auto after = gpu.prefix.output.down();
  float accepted_error = 0, sibling_error = 0;
  for (size_t i = 0; i < query_elems; ++i) {
    accepted_error = std::max(accepted_error, std::fabs(after[i] - tree_out[3 * query_elems + i]));
    sibling_error =
        std::max(sibling_error, std::fabs(after[query_elems + i] - before[query_elems + i]));
  }
  if (accepted_error > 3e-4f || sibling_error > 1e-7f)
    throw std::runtime_error("commit changed accepted path or shared sibling");
  gpu.prefix.pages.up(f.prefix.pages);
  gpu.prefix.lengths.up(f.prefix.lengths);
  gpu.prefix.q.up(f.prefix.q);
  gpu.prefix.run(1);
  if (max_abs_error(before, gpu.prefix.output.down()) > 1e-7f)
    throw std::runtime_error("rollback failed");
  check_device_errors();
  std::cout << "PASS " << checks << " tree CPU-oracle cases plus shared-page"
            << " commit, sibling isolation, and rollback.\n";
}

template <typename F>
double median_us(F&& launch, int repeats = 20) {
  cudaEvent_t start, stop;
  CHECK(cudaEventCreate(&start));
  CHECK(cudaEventCreate(&stop));
  for (int i = 0; i < 5; ++i) CHECK(launch());
  CHECK(cudaDeviceSynchronize());
  std::vector<double> times;
  for (int trial = 0; trial < 7; ++trial) {
    CHECK(cudaEventRecord(start));
    for (int i = 0; i < repeats; ++i) CHECK(launch());
    CHECK(cudaEventRecord(stop));
    CHECK(cudaEventSynchronize(stop));
    float ms = 0;
    CHECK(cudaEventElapsedTime(&ms, start, stop));
    times.push_back(double(ms) * 1000.0 / repeats);
  }
  CHECK(cudaEventDestroy(start));
  CHECK(cudaEventDestroy(stop));
  std::sort(times.begin(), times.end());
  return times[times.size() / 2];
}

// Each (request, node) materialised as its own paged sequence: the prefix
// followed by its root-to-node chain (reference src/main.cu:375-423).
Fixture make_expanded_fixture(const TreeFixture& tree) {
  const Shape ps = tree.prefix.shape;
  const int sequences = ps.batch * tree.nodes;
  int max_len = 0, total_pages = 0;
  std::vector<int> lengths(sequences);
  std::vector<std::vector<int>> paths(sequences);
  for (int b = 0; b < ps.batch; ++b)
    for (int node = 0; node < tree.nodes; ++node) {
      const int seq = b * tree.nodes + node;
      for (int cur = node; cur >= 0; cur = tree.parent[b * tree.nodes + cur])
        paths[seq].push_back(cur);
      std::reverse(paths[seq].begin(), paths[seq].end());
      lengths[seq] = tree.prefix.lengths[b] + int(paths[seq].size());
      max_len = std::max(max_len, lengths[seq]);
      total_pages += (lengths[seq] + kPageSize - 1) / kPageSize;
    }
  const int max_pages = (max_len + kPageSize - 1) / kPageSize;
  Fixture flat{{sequences, ps.query_heads, ps.kv_heads, ps.dim, max_pages, total_pages + 7}};
  flat.lengths = lengths;
  flat.pages.assign(size_t(sequences) * max_pages, -1);
  flat.q = tree.draft_q;
  const size_t token_elems = size_t(ps.kv_heads) * ps.dim;
  flat.k.assign(size_t(flat.shape.physical_pages) * kPageSize * token_elems, 0);
  flat.v.assign(flat.k.size(), 0);
  // Sequences take consecutive physical pages in order; each token's K/V row
  // comes either from the shared prefix (through the request's page table) or
  // from the draft rows of its path node.
  struct Source {
    const std::vector<uint16_t>* k;
    const std::vector<uint16_t>* v;
    size_t row;  // element offset of the token's row
  };
  int page_cursor = 0;
  for (int seq = 0; seq < sequences; ++seq) {
    const int b = seq / tree.nodes;
    const int prefix_len = tree.prefix.lengths[b];
    std::vector<Source> rows;
    rows.reserve(lengths[seq]);
    for (int t = 0; t < prefix_len; ++t) {
      const int page = tree.prefix.pages[size_t(b) * ps.max_pages + t / kPageSize];
      rows.push_back({&tree.prefix.k, &tree.prefix.v,
                      (size_t(page) * kPageSize + t % kPageSize) * token_elems});
    }
    for (int node : paths[seq])
      rows.push_back({&tree.draft_k, &tree.draft_v,
                      (size_t(b) * tree.nodes + node) * token_elems});
    int* table = flat.pages.data() + size_t(seq) * max_pages;
    for (size_t first = 0; first < rows.size(); first += kPageSize) {
      const int page = page_cursor++;
      table[first / kPageSize] = page;
      const size_t count = std::min<size_t>(kPageSize, rows.size() - first);
      for (size_t slot = 0; slot < count; ++slot) {
        const Source& src = rows[first + slot];
        const size_t dst = (size_t(page) * kPageSize + slot) * token_elems;
        std::copy_n(src.k->begin() + src.row, token_elems, flat.k.begin() + dst);
        std::copy_n(src.v->begin() + src.row, token_elems, flat.v.begin() + dst);
      }
    }
  }
  return flat;
}

std::string gpu_name(int* major, int* minor) {
  cudaDeviceProp prop{};
  CHECK(cudaGetDeviceProperties(&prop, 0));
  *major = prop.major;
  *minor = prop.minor;
  return prop.name;
}

void run_tree_bench(const std::string& output_path, bool quick) {
  int major = 0, minor = 0;
  const std::string name = gpu_name(&major, &minor);
  std::ofstream out(output_path);
  if (!out) throw std::runtime_error("cannot open output: " + output_path);
  out << "gpu,sm,cuda_runtime,requests,tree_nodes,prefix_tokens,query_heads,"
         "kv_heads,head_dim,page_size,tree_us,expanded_us,latency_ratio,"
         "max_abs_diff,shared_kv_mib,expanded_kv_mib,memory_saving_pct\n";
  const auto batches = quick ? std::vector<int>{1, 4} : std::vector<int>{1, 4, 8};
  const auto contexts = quick ? std::vector<int>{256, 1024} : std::vector<int>{256, 1024, 2048};
  for (int b : batches)
    for (int context : contexts) {
      TreeFixture f = make_tree_fixture(b, context, 7, 128, 91 + b + context);
      Fixture expanded = make_expanded_fixture(f);
      TreeGpu tree(f);
      GpuFixture flat(expanded);
      tree.run();
      flat.run(1);
      const float diff = max_abs_error(tree.output.down(), flat.output.down());
      if (diff > 3e-4f) throw std::runtime_error("expanded-cache output mismatch");
      const double tree_us = median_us(
          [&] { return branchcraft::tree_verify(tree.prefix.shape, tree.inputs(), tree.nodes); });
      const double expanded_us = median_us(
          [&] { return branchcraft::decode(flat.shape, flat.inputs(), flat.scratch(), 1); });
      const double bytes_per_token = double(f.prefix.shape.kv_heads) * f.prefix.shape.dim * 2 * 2;
      const double shared_tokens =
          double((context + kPageSize - 1) / kPageSize * kPageSize) + b * f.nodes;
      int expanded_slots = 0;
      for (int len : expanded.lengths) expanded_slots += (len + kPageSize - 1) / kPageSize * kPageSize;
      const double shared_mib = shared_tokens * bytes_per_token / (1024. * 1024.);
      const double expanded_mib = expanded_slots * bytes_per_token / (1024. * 1024.);
      out << '"' << name << '"' << ',' << major << '.' << minor << ',' << CUDART_VERSION << ','
          << b << ",7," << context << ",32,8,128,16," << std::fixed << std::setprecision(3)
          << tree_us << ',' << expanded_us << ',' << expanded_us / tree_us << ','
          << std::scientific << std::setprecision(8) << diff << std::fixed << std::setprecision(3)
          << ',' << shared_mib << ',' << expanded_mib << ','
          << 100. * (1. - shared_mib / expanded_mib) << '\n';
      out.flush();
      std::cout << "tree B=" << b << " S=" << context << " tree=" << tree_us
                << "us expanded=" << expanded_us << "us ratio=" << expanded_us / tree_us
                << "x KV saved=" << 100. * (1. - shared_mib / expanded_mib) << "%\n";
    }
  check_device_errors();
  std::cout << "Wrote " << output_path << '\n';
}

void run_bench(const std::string& output_path, bool quick) {
  int major = 0, minor = 0;
  const std::string name = gpu_name(&major, &minor);
  int sms = 0;
  CHECK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0));
  std::ofstream out(output_path);
  if (!out) throw std::runtime_error("cannot open output: " + output_path);
  out << "gpu,sm,cuda_runtime,batch,query_heads,kv_heads,head_dim,context,"
         "page_size,splits,single_us,split_us,speedup,max_abs_diff,kv_mib\n";
  const std::vector<int> batches = quick ? std::vector<int>{1, 8} : std::vector<int>{1, 4, 16, 32};
  const std::vector<int> contexts =
      quick ? std::vector<int>{256, 2048} : std::vector<int>{256, 1024, 4096, 8192};
  for (int b : batches)
    for (int context : contexts) {
      std::vector<int> lengths(b);
      for (int i = 0; i < b; ++i) lengths[i] = context - (i % 4) * context / 8;
      Fixture f = make_fixture(b, 32, 8, 128, lengths, 17 + b + context);
      GpuFixture gpu(f);
      const int splits = branchcraft::auto_splits(f.shape, context, sms);
      gpu.run(1);
      const auto baseline_out = gpu.output.down();
      gpu.run(splits);
      const float diff = max_abs_error(baseline_out, gpu.output.down());
      if (diff > 3e-4f) throw std::runtime_error("benchmark split output mismatch");
      const double single = median_us(
          [&] { return branchcraft::decode(gpu.shape, gpu.inputs(), gpu.scratch(), 1); });
      const double split =
          splits == 1 ? single
                      : median_us([&] {
                          return branchcraft::decode(gpu.shape, gpu.inputs(), gpu.scratch(),
                                                     splits);
                        });
      const double kv_mib = double(f.k.size() + f.v.size()) * 2 / (1024. * 1024.);
      out << '"' << name << '"' << ',' << major << '.' << minor << ',' << CUDART_VERSION << ','
          << b << ",32,8,128," << context << ',' << kPageSize << ',' << splits << ','
          << std::fixed << std::setprecision(3) << single << ',' << split << ','
          << single / split << ',' << std::scientific << std::setprecision(8) << diff
          << std::fixed << std::setprecision(3) << ',' << kv_mib << '\n';
      out.flush();
      std::cout << "B=" << b << " S=" << context << " split=" << splits << " single=" << single
                << "us chosen=" << split << "us speedup=" << single / split << "x diff=" << diff
                << '\n';
    }
  check_device_errors();
  std::cout << "Wrote " << output_path << '\n';
}

namespace {

// Options of the bench modes: `--quick` and `--output FILE`, in any order.
struct BenchOptions {
  bool quick = false;
  std::string output;
};

BenchOptions parse_bench_options(const std::vector<std::string>& args, std::string output) {
  BenchOptions opt;
  opt.output = std::move(output);
  for (auto it = args.begin(); it != args.end(); ++it) {
    if (*it == "--quick") {
      opt.quick = true;
    } else if (*it == "--output" && std::next(it) != args.end()) {
      opt.output = *++it;
    } else {
      throw std::runtime_error("unknown or incomplete argument: " + *it);
    }
  }
  return opt;
}

}  // namespace

// The reference's command line (src/main.cu:527-553): `test`, `bench` and
// `tree-bench`, exit code 2 with the usage line when no mode is given, 1 on
// any failure.
int main(int argc, char** argv) {
  const std::vector<std::string> args(argv + std::min(argc, 1), argv + argc);
  if (args.empty()) {
    std::cerr << "Usage: branchcraft test | bench | tree-bench [--quick] [--output FILE]\n";
    return 2;
  }
  const std::vector<std::string> rest(args.begin() + 1, args.end());
  try {
    if (args[0] == "test") {
      run_tests();
      run_tree_tests();
    } else if (args[0] == "bench") {
      const BenchOptions opt = parse_bench_options(rest, "decode_results.csv");
      run_bench(opt.output, opt.quick);
    } else if (args[0] == "tree-bench") {
      const BenchOptions opt = parse_bench_options(rest, "tree_results.csv");
      run_tree_bench(opt.output, opt.quick);
    } else {
      throw std::runtime_error("unknown mode: " + args[0]);
    }
  } catch (const std::exception& e) {
    std::cerr << "ERROR: " << e.what() << '\n';
    return 1;
  }
  return 0;
}
