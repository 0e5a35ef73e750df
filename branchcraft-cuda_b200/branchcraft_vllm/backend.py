"""vLLM V1 attention backend: one-token decode on the Branchcraft packed-KV
kernels, everything else on vLLM's Triton implementation.

Mirrors the reference's python/branchcraft_vllm/backend.py:20-96 (same class
names, same guard, same trace lines) and adds the cache layout the installed
vLLM allocates. Two cache layouts take the fast path:

* ``[num_blocks, Hkv, 16, 2*D]`` (logical), K in ``[..., :D]`` and V in
  ``[..., D:]`` of each token row: the layout the reference's guard accepts
  (backend.py:62-63), decoded by ``torch.ops.branchcraft.packed_decode_out``.
* ``[num_blocks, 2, 16, Hkv, D]``: what ``TritonAttentionBackend.
  get_kv_cache_shape`` returns for block size 16 in vLLM 0.22. K and V are
  the two planes of dim 1; ``packed_decode_kv_out`` reads them through
  ``[num_blocks, Hkv, 16, D]`` views (no copy) with the K->V offset taken
  from the two views' addresses. The reference cannot express this layout.

Prefill, sliding windows, ALiBi, sinks, soft-capping, quantized or
non-FP16 caches, block sizes other than 16 and cascade attention all fall
back to ``TritonAttentionImpl.forward`` unchanged.
"""

import os

import torch

import branchcraft_torch  # noqa: F401  registers torch.ops.branchcraft
from vllm.v1.attention.backend import AttentionType
from vllm.v1.attention.backends.triton_attn import TritonAttentionBackend, TritonAttentionImpl

PAGE = 16

# Fast-path kinds returned by BranchcraftImpl._decode_layout.
INTERLEAVED = "packed_decode_out"
PLANES = "packed_decode_kv_out"


class BranchcraftBackend(TritonAttentionBackend):
    """vLLM resolves the backend by name through AttentionBackendEnum; the
    implementation class is what differs (reference backend.py:20-29)."""

    @staticmethod
    def get_name() -> str:
        return "CUSTOM"

    @staticmethod
    def get_impl_cls() -> type["BranchcraftImpl"]:
        return BranchcraftImpl


def _int32_contiguous(t) -> bool:
    return t.dtype == torch.int32 and t.is_contiguous()


class BranchcraftImpl(TritonAttentionImpl):
    _reported_fast_path = False
    _reported_prefill_fallback = False

    def _cache_layout(self, kv_cache):
        """INTERLEAVED, PLANES or None for this cache's shape and strides."""
        d = self.head_size
        if kv_cache.dim() == 4:
            if kv_cache.shape[2] == PAGE and kv_cache.shape[3] == 2 * d and kv_cache.stride(3) == 1:
                return INTERLEAVED
            return None
        if kv_cache.dim() == 5:
            if (kv_cache.shape[1] == 2 and kv_cache.shape[2] == PAGE
                    and kv_cache.shape[3] == self.num_kv_heads and kv_cache.shape[4] == d
                    and kv_cache.stride(4) == 1):
                return PLANES
        return None

    def _decode_layout(self, query, kv_cache, metadata, output, output_scale,
                       output_block_scale):
        """The fast-path kind for this call, or None to fall back.

        The conditions are the reference guard's (backend.py:36-71). vLLM
        0.22's metadata has no `causal` or `rswa_window` field (its Triton
        path is always causal, with no ragged window), so absent fields read
        as causal / no window; a per-token-head quantized cache falls back.
        """
        if metadata is None:
            return None
        n = metadata.num_actual_tokens
        if not (
            n > 0
            and metadata.max_query_len == 1
            and metadata.query_start_loc.numel() == n + 1
            and getattr(metadata, "causal", True)
            and not metadata.use_cascade
            and getattr(metadata, "mm_prefix_range_tensor", None) is None
            and getattr(metadata, "rswa_window", None) is None
            and self.attn_type == AttentionType.DECODER
            and tuple(self.sliding_window) == (-1, -1)
            and self.alibi_slopes is None
            and self.sinks is None
            and not self.logits_soft_cap
            and self.kv_cache_dtype in ("auto", "float16")
            and not getattr(self, "_is_per_token_head_quant", False)
            and getattr(self, "chunk_lookback", -1) == -1
            and query.dtype == torch.float16
            and kv_cache.dtype == torch.float16
            and output.dtype == torch.float16
            and query.is_contiguous()
            and output.is_contiguous()
            and self.head_size in (64, 128)
            and output_scale is None
            and output_block_scale is None
            and _int32_contiguous(metadata.block_table)
            and _int32_contiguous(metadata.seq_lens)
        ):
            return None
        return self._cache_layout(kv_cache)

    def _can_decode(self, query, kv_cache, metadata, output, output_scale,
                    output_block_scale):
        return self._decode_layout(query, kv_cache, metadata, output, output_scale,
                                   output_block_scale) is not None

    def forward(self, layer, query, key, value, kv_cache, attn_metadata, output,
                output_scale=None, output_block_scale=None):
        kind = self._decode_layout(query, kv_cache, attn_metadata, output, output_scale,
                                   output_block_scale)
        if kind is not None:
            n = attn_metadata.num_actual_tokens
            if os.getenv("BRANCHCRAFT_TRACE") and not type(self)._reported_fast_path:
                print(f"BRANCHCRAFT_FAST_PATH {kind}", flush=True)
                type(self)._reported_fast_path = True
            out = output[:n].view(n, self.num_heads, self.head_size)
            pages = attn_metadata.block_table[:n]
            lengths = attn_metadata.seq_lens[:n]
            if kind == INTERLEAVED:
                torch.ops.branchcraft.packed_decode_out(query[:n], kv_cache, pages, lengths, out,
                                                        self.scale)
            else:
                k_view = kv_cache[:, 0].transpose(1, 2)
                v_view = kv_cache[:, 1].transpose(1, 2)
                torch.ops.branchcraft.packed_decode_kv_out(query[:n], k_view, v_view, pages,
                                                           lengths, out, self.scale, 0)
            return output
        if (os.getenv("BRANCHCRAFT_TRACE") and attn_metadata is not None
                and attn_metadata.max_query_len > 1
                and not type(self)._reported_prefill_fallback):
            print("BRANCHCRAFT_PREFILL_FALLBACK TritonAttentionImpl", flush=True)
            type(self)._reported_prefill_fallback = True
        return super().forward(layer, query, key, value, kv_cache, attn_metadata, output,
                               output_scale, output_block_scale)
