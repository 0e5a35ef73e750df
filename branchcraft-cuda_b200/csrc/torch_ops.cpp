// PyTorch dispatcher binding: TORCH_LIBRARY(branchcraft) with the reference's
// three schemas (bindings/torch_ops.cpp:144-148) and the same argument checks
// (bindings/torch_ops.cpp:11-140), plus the ops the reference lacks:
//   paged_decode          paged GQA decode, FP32 out (optional split count)
//   tree_verify_out       tree verify into a preallocated FP32 or FP16 output
//   packed_decode_kv_out  decode from separate K / V views of one packed cache
//                         (vLLM's [num_blocks, 2, 16, Hkv, D]: k = cache[:, 0])
//   commit_batch_         a whole batch of copy-on-write commits
// Every op calls the C ABI (branchcraft.h) on the current CUDA stream.
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <torch/library.h>

#include "branchcraft.h"

namespace {

void check_cuda_contiguous(const at::Tensor& t, const char* name, at::ScalarType dtype) {
  TORCH_CHECK(t.is_cuda(), name, " must be CUDA");
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.scalar_type() == dtype, name, " has wrong dtype");
}

void check_launch(int err, const char* op) {
  TORCH_CHECK(err == 0, op, ": ", cudaGetErrorString(static_cast<cudaError_t>(err)));
}

void* stream() { return at::cuda::getCurrentCUDAStream().stream(); }

void check_tree(const at::Tensor& q, const at::Tensor& prefix_k, const at::Tensor& prefix_v,
                const at::Tensor& pages, const at::Tensor& lengths, const at::Tensor& draft_k,
                const at::Tensor& draft_v, const at::Tensor& parent) {
  check_cuda_contiguous(q, "q", at::kHalf);
  check_cuda_contiguous(prefix_k, "prefix_k", at::kHalf);
  check_cuda_contiguous(prefix_v, "prefix_v", at::kHalf);
  check_cuda_contiguous(draft_k, "draft_k", at::kHalf);
  check_cuda_contiguous(draft_v, "draft_v", at::kHalf);
  check_cuda_contiguous(pages, "pages", at::kInt);
  check_cuda_contiguous(lengths, "lengths", at::kInt);
  check_cuda_contiguous(parent, "parent", at::kInt);
  TORCH_CHECK(q.dim() == 4 && prefix_k.dim() == 4 && prefix_v.dim() == 4 && draft_k.dim() == 4 &&
                  draft_v.dim() == 4 && pages.dim() == 2 && lengths.dim() == 1 &&
                  parent.dim() == 2,
              "invalid tree tensor rank");
  const int64_t b = q.size(0), nodes = q.size(1), hq = q.size(2), d = q.size(3);
  const int64_t hkv = prefix_k.size(2);
  TORCH_CHECK(b > 0 && nodes > 0 && nodes <= BC_MAX_NODES && hq > 0 && hkv > 0 && hq % hkv == 0 &&
                  (d == 64 || d == 128),
              "unsupported tree shape");
  TORCH_CHECK(prefix_k.size(1) == BC_PAGE_SIZE && prefix_k.size(3) == d &&
                  prefix_v.sizes() == prefix_k.sizes(),
              "prefix K/V shape mismatch");
  TORCH_CHECK(draft_k.sizes() == at::IntArrayRef({b, nodes, hkv, d}) &&
                  draft_v.sizes() == draft_k.sizes(),
              "draft K/V shape mismatch");
  TORCH_CHECK(pages.size(0) == b && lengths.size(0) == b &&
                  parent.sizes() == at::IntArrayRef({b, nodes}),
              "tree metadata shape mismatch");
  TORCH_CHECK(q.device() == prefix_k.device() && q.device() == prefix_v.device() &&
                  q.device() == draft_k.device() && q.device() == draft_v.device() &&
                  q.device() == pages.device() && q.device() == lengths.device() &&
                  q.device() == parent.device(),
              "all tensors must share a device");
}

int launch_tree(const at::Tensor& q, const at::Tensor& prefix_k, const at::Tensor& prefix_v,
                const at::Tensor& pages, const at::Tensor& lengths, const at::Tensor& draft_k,
                const at::Tensor& draft_v, const at::Tensor& parent, at::Tensor& output) {
  const bc_shape s{int(q.size(0)), int(q.size(2)), int(prefix_k.size(2)), int(q.size(3)),
                   int(pages.size(1)), int(prefix_k.size(0))};
  const int nodes = int(q.size(1));
  if (output.scalar_type() == at::kHalf)
    return bc_tree_verify_f16(&s, q.data_ptr(), prefix_k.data_ptr(), prefix_v.data_ptr(),
                              pages.data_ptr<int>(), lengths.data_ptr<int>(), draft_k.data_ptr(),
                              draft_v.data_ptr(), parent.data_ptr<int>(), output.data_ptr(),
                              nodes, stream());
  return bc_tree_verify(&s, q.data_ptr(), prefix_k.data_ptr(), prefix_v.data_ptr(),
                        pages.data_ptr<int>(), lengths.data_ptr<int>(), draft_k.data_ptr(),
                        draft_v.data_ptr(), parent.data_ptr<int>(), output.data_ptr<float>(),
                        nodes, stream());
}

at::Tensor tree_verify_cuda(const at::Tensor& q, const at::Tensor& prefix_k,
                            const at::Tensor& prefix_v, const at::Tensor& pages,
                            const at::Tensor& lengths, const at::Tensor& draft_k,
                            const at::Tensor& draft_v, const at::Tensor& parent) {
  check_tree(q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent);
  auto output = at::empty(q.sizes(), q.options().dtype(at::kFloat));
  check_launch(launch_tree(q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent, output),
               "tree_verify");
  return output;
}

at::Tensor& tree_verify_out_cuda(const at::Tensor& q, const at::Tensor& prefix_k,
                                 const at::Tensor& prefix_v, const at::Tensor& pages,
                                 const at::Tensor& lengths, const at::Tensor& draft_k,
                                 const at::Tensor& draft_v, const at::Tensor& parent,
                                 at::Tensor& output) {
  check_tree(q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent);
  TORCH_CHECK(output.is_cuda() && output.is_contiguous() && output.sizes() == q.sizes() &&
                  (output.scalar_type() == at::kFloat || output.scalar_type() == at::kHalf) &&
                  output.device() == q.device(),
              "output must be a contiguous CUDA FP32/FP16 tensor shaped like q");
  check_launch(launch_tree(q, prefix_k, prefix_v, pages, lengths, draft_k, draft_v, parent, output),
               "tree_verify_out");
  return output;
}

void check_packed_common(const at::Tensor& q, const at::Tensor& pages, const at::Tensor& lengths,
                         const at::Tensor& output) {
  check_cuda_contiguous(q, "q", at::kHalf);
  check_cuda_contiguous(pages, "pages", at::kInt);
  check_cuda_contiguous(lengths, "lengths", at::kInt);
  check_cuda_contiguous(output, "output", at::kHalf);
  TORCH_CHECK(q.dim() == 3 && pages.dim() == 2 && lengths.dim() == 1,
              "invalid packed decode tensor rank");
}

at::Tensor& packed_decode_out_cuda(const at::Tensor& q, const at::Tensor& packed_kv,
                                   const at::Tensor& pages, const at::Tensor& lengths,
                                   at::Tensor& output, double scale) {
  check_packed_common(q, pages, lengths, output);
  TORCH_CHECK(packed_kv.is_cuda() && packed_kv.scalar_type() == at::kHalf &&
                  packed_kv.dim() == 4 && packed_kv.stride(3) == 1,
              "packed_kv must be a CUDA FP16 tensor with contiguous content dim");
  const int64_t b = q.size(0), hq = q.size(1), d = q.size(2);
  const int64_t hkv = packed_kv.size(1);
  TORCH_CHECK(b > 0 && hq > 0 && hkv > 0 && hq % hkv == 0 && (d == 64 || d == 128),
              "unsupported packed decode shape");
  TORCH_CHECK(packed_kv.size(2) == BC_PAGE_SIZE && packed_kv.size(3) == 2 * d,
              "packed KV shape mismatch");
  TORCH_CHECK(pages.size(0) == b && lengths.size(0) == b && output.numel() == q.numel(),
              "packed decode metadata/output mismatch");
  TORCH_CHECK(q.device() == packed_kv.device() && q.device() == pages.device() &&
                  q.device() == lengths.device() && q.device() == output.device(),
              "all tensors must share a device");
  const bc_shape s{int(b), int(hq), int(hkv), int(d), int(pages.size(1)), int(packed_kv.size(0))};
  check_launch(bc_packed_decode(&s, q.data_ptr(), packed_kv.data_ptr(), pages.data_ptr<int>(),
                                lengths.data_ptr<int>(), output.data_ptr(), packed_kv.stride(0),
                                packed_kv.stride(1), packed_kv.stride(2), float(scale), stream()),
               "packed_decode_out");
  return output;
}

at::Tensor& packed_decode_kv_out_cuda(const at::Tensor& q, const at::Tensor& k_cache,
                                      const at::Tensor& v_cache, const at::Tensor& pages,
                                      const at::Tensor& lengths, at::Tensor& output, double scale,
                                      int64_t splits) {
  check_packed_common(q, pages, lengths, output);
  TORCH_CHECK(k_cache.is_cuda() && v_cache.is_cuda() && k_cache.scalar_type() == at::kHalf &&
                  v_cache.scalar_type() == at::kHalf && k_cache.dim() == 4 &&
                  v_cache.sizes() == k_cache.sizes() && k_cache.strides() == v_cache.strides() &&
                  k_cache.stride(3) == 1,
              "k_cache / v_cache must be FP16 CUDA views [P, Hkv, 16, D] with equal strides "
              "and a contiguous last dim");
  const int64_t b = q.size(0), hq = q.size(1), d = q.size(2);
  const int64_t hkv = k_cache.size(1);
  TORCH_CHECK(b > 0 && hq > 0 && hkv > 0 && hq % hkv == 0 && (d == 64 || d == 128),
              "unsupported packed decode shape");
  TORCH_CHECK(k_cache.size(2) == BC_PAGE_SIZE && k_cache.size(3) == d, "KV view shape mismatch");
  TORCH_CHECK(pages.size(0) == b && lengths.size(0) == b && output.numel() == q.numel(),
              "packed decode metadata/output mismatch");
  TORCH_CHECK(splits >= 0 && splits <= 8, "splits must be 0 (auto) or 1..8");
  const auto* kb = static_cast<const at::Half*>(k_cache.data_ptr());
  const auto* vb = static_cast<const at::Half*>(v_cache.data_ptr());
  const bc_shape s{int(b), int(hq), int(hkv), int(d), int(pages.size(1)), int(k_cache.size(0))};
  check_launch(bc_packed_decode_kv(&s, q.data_ptr(), kb, pages.data_ptr<int>(),
                                   lengths.data_ptr<int>(), output.data_ptr(), k_cache.stride(0),
                                   k_cache.stride(1), k_cache.stride(2), (long long)(vb - kb),
                                   float(scale), int(splits), stream()),
               "packed_decode_kv_out");
  return output;
}

at::Tensor paged_decode_cuda(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                             const at::Tensor& pages, const at::Tensor& lengths, int64_t splits) {
  check_cuda_contiguous(q, "q", at::kHalf);
  check_cuda_contiguous(k, "k", at::kHalf);
  check_cuda_contiguous(v, "v", at::kHalf);
  check_cuda_contiguous(pages, "pages", at::kInt);
  check_cuda_contiguous(lengths, "lengths", at::kInt);
  TORCH_CHECK(q.dim() == 3 && k.dim() == 4 && v.sizes() == k.sizes() && pages.dim() == 2 &&
                  lengths.dim() == 1,
              "invalid paged decode tensor rank");
  const int64_t b = q.size(0), hq = q.size(1), d = q.size(2), hkv = k.size(2);
  TORCH_CHECK(k.size(1) == BC_PAGE_SIZE && k.size(3) == d && hkv > 0 && hq % hkv == 0 &&
                  (d == 64 || d == 128) && pages.size(0) == b && lengths.size(0) == b,
              "paged decode shape mismatch");
  TORCH_CHECK(q.device() == k.device() && q.device() == v.device() &&
                  q.device() == pages.device() && q.device() == lengths.device(),
              "all tensors must share a device");
  TORCH_CHECK(splits >= 0 && splits <= BC_MAX_SPLITS, "splits must be 0 (auto) or 1..64");
  auto output = at::empty(q.sizes(), q.options().dtype(at::kFloat));
  const bc_shape s{int(b), int(hq), int(hkv), int(d), int(pages.size(1)), int(k.size(0))};
  if (splits > 8) {
    auto pa = at::empty({splits * b * hq * d}, q.options().dtype(at::kFloat));
    auto pml = at::empty({splits * b * hq * 2}, q.options().dtype(at::kFloat));
    check_launch(bc_decode(&s, q.data_ptr(), k.data_ptr(), v.data_ptr(), pages.data_ptr<int>(),
                           lengths.data_ptr<int>(), output.data_ptr<float>(),
                           pa.data_ptr<float>(), pml.data_ptr<float>(), int(splits), stream()),
                 "paged_decode");
  } else {
    check_launch(bc_paged_decode(&s, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                 pages.data_ptr<int>(), lengths.data_ptr<int>(),
                                 output.data_ptr<float>(), int(splits), stream()),
                 "paged_decode");
  }
  return output;
}

void commit_path_cuda(at::Tensor& cache_k, at::Tensor& cache_v, const at::Tensor& draft_k,
                      const at::Tensor& draft_v, const at::Tensor& path_nodes,
                      const at::Tensor& dest_pages, const at::Tensor& dest_slots,
                      int64_t request) {
  check_cuda_contiguous(cache_k, "cache_k", at::kHalf);
  check_cuda_contiguous(cache_v, "cache_v", at::kHalf);
  check_cuda_contiguous(draft_k, "draft_k", at::kHalf);
  check_cuda_contiguous(draft_v, "draft_v", at::kHalf);
  check_cuda_contiguous(path_nodes, "path_nodes", at::kInt);
  check_cuda_contiguous(dest_pages, "dest_pages", at::kInt);
  check_cuda_contiguous(dest_slots, "dest_slots", at::kInt);
  TORCH_CHECK(cache_k.dim() == 4 && cache_v.sizes() == cache_k.sizes() && draft_k.dim() == 4 &&
                  draft_v.sizes() == draft_k.sizes() && path_nodes.dim() == 1 &&
                  dest_pages.sizes() == path_nodes.sizes() &&
                  dest_slots.sizes() == path_nodes.sizes(),
              "commit tensor shape mismatch");
  const int64_t b = draft_k.size(0), nodes = draft_k.size(1), hkv = draft_k.size(2),
                d = draft_k.size(3);
  TORCH_CHECK(request >= 0 && request < b && path_nodes.numel() > 0 &&
                  path_nodes.numel() <= nodes && cache_k.size(1) == BC_PAGE_SIZE &&
                  cache_k.size(2) == hkv && cache_k.size(3) == d,
              "invalid commit destination");
  TORCH_CHECK(cache_k.device() == draft_k.device() && cache_k.device() == cache_v.device() &&
                  cache_k.device() == draft_v.device() &&
                  cache_k.device() == path_nodes.device() &&
                  cache_k.device() == dest_pages.device() &&
                  cache_k.device() == dest_slots.device(),
              "all tensors must share a device");
  const bc_shape s{int(b), int(hkv), int(hkv), int(d), 1, int(cache_k.size(0))};
  check_launch(bc_commit_path(&s, draft_k.data_ptr(), draft_v.data_ptr(), cache_k.data_ptr(),
                              cache_v.data_ptr(), path_nodes.data_ptr<int>(),
                              dest_pages.data_ptr<int>(), dest_slots.data_ptr<int>(),
                              int(request), int(nodes), int(path_nodes.numel()), stream()),
               "commit_path_");
}

void commit_batch_cuda(at::Tensor& cache_k, at::Tensor& cache_v, const at::Tensor& draft_k,
                       const at::Tensor& draft_v, const at::Tensor& clone_src,
                       const at::Tensor& clone_dst, const at::Tensor& entry_request,
                       const at::Tensor& entry_node, const at::Tensor& entry_page,
                       const at::Tensor& entry_slot) {
  check_cuda_contiguous(cache_k, "cache_k", at::kHalf);
  check_cuda_contiguous(cache_v, "cache_v", at::kHalf);
  check_cuda_contiguous(draft_k, "draft_k", at::kHalf);
  check_cuda_contiguous(draft_v, "draft_v", at::kHalf);
  for (const at::Tensor* t : {&clone_src, &clone_dst, &entry_request, &entry_node, &entry_page,
                              &entry_slot})
    check_cuda_contiguous(*t, "commit plan", at::kInt);
  TORCH_CHECK(cache_k.dim() == 4 && cache_v.sizes() == cache_k.sizes() && draft_k.dim() == 4 &&
                  draft_v.sizes() == draft_k.sizes() && clone_src.sizes() == clone_dst.sizes() &&
                  entry_node.sizes() == entry_request.sizes() &&
                  entry_page.sizes() == entry_request.sizes() &&
                  entry_slot.sizes() == entry_request.sizes(),
              "commit_batch_ tensor shape mismatch");
  const int64_t hkv = draft_k.size(2), d = draft_k.size(3);
  TORCH_CHECK(cache_k.size(1) == BC_PAGE_SIZE && cache_k.size(2) == hkv && cache_k.size(3) == d,
              "cache / draft head shape mismatch");
  const bc_shape s{int(draft_k.size(0)), int(hkv), int(hkv), int(d), 1, int(cache_k.size(0))};
  check_launch(bc_commit_batch(&s, int(draft_k.size(1)), draft_k.data_ptr(), draft_v.data_ptr(),
                               cache_k.data_ptr(), cache_v.data_ptr(),
                               clone_src.data_ptr<int>(), clone_dst.data_ptr<int>(),
                               int(clone_src.numel()), entry_request.data_ptr<int>(),
                               entry_node.data_ptr<int>(), entry_page.data_ptr<int>(),
                               entry_slot.data_ptr<int>(), int(entry_node.numel()), stream()),
               "commit_batch_");
}

}  // namespace

TORCH_LIBRARY(branchcraft, m) {
  m.def("tree_verify(Tensor q, Tensor prefix_k, Tensor prefix_v, Tensor pages, Tensor lengths, "
        "Tensor draft_k, Tensor draft_v, Tensor parent) -> Tensor");
  m.def("packed_decode_out(Tensor q, Tensor packed_kv, Tensor pages, Tensor lengths, "
        "Tensor(a!) output, float scale) -> Tensor(a!)");
  m.def("commit_path_(Tensor(a!) cache_k, Tensor(b!) cache_v, Tensor draft_k, Tensor draft_v, "
        "Tensor path_nodes, Tensor dest_pages, Tensor dest_slots, int request) -> ()");
  m.def("paged_decode(Tensor q, Tensor k, Tensor v, Tensor pages, Tensor lengths, "
        "int splits=0) -> Tensor");
  m.def("tree_verify_out(Tensor q, Tensor prefix_k, Tensor prefix_v, Tensor pages, "
        "Tensor lengths, Tensor draft_k, Tensor draft_v, Tensor parent, Tensor(a!) output) "
        "-> Tensor(a!)");
  m.def("packed_decode_kv_out(Tensor q, Tensor k_cache, Tensor v_cache, Tensor pages, "
        "Tensor lengths, Tensor(a!) output, float scale, int splits=0) -> Tensor(a!)");
  m.def("commit_batch_(Tensor(a!) cache_k, Tensor(b!) cache_v, Tensor draft_k, Tensor draft_v, "
        "Tensor clone_src, Tensor clone_dst, Tensor entry_request, Tensor entry_node, "
        "Tensor entry_page, Tensor entry_slot) -> ()");
}

TORCH_LIBRARY_IMPL(branchcraft, CUDA, m) {
  m.impl("tree_verify", tree_verify_cuda);
  m.impl("packed_decode_out", packed_decode_out_cuda);
  m.impl("commit_path_", commit_path_cuda);
  m.impl("paged_decode", paged_decode_cuda);
  m.impl("tree_verify_out", tree_verify_out_cuda);
  m.impl("packed_decode_kv_out", packed_decode_kv_out_cuda);
  m.impl("commit_batch_", commit_batch_cuda);
}
