"""The torch binding without a GPU: the extension loads, registers the
reference's three schemas verbatim (bindings/torch_ops.cpp:144-148) plus the
added ops, and every fake (meta) kernel gives the right output under
FakeTensorMode, so torch.compile can trace the ops."""
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import branchcraft_torch  # noqa: F401

REFERENCE_SCHEMAS = {
    "tree_verify": "branchcraft::tree_verify(Tensor q, Tensor prefix_k, Tensor prefix_v, "
                   "Tensor pages, Tensor lengths, Tensor draft_k, Tensor draft_v, "
                   "Tensor parent) -> Tensor",
    "packed_decode_out": "branchcraft::packed_decode_out(Tensor q, Tensor packed_kv, "
                         "Tensor pages, Tensor lengths, Tensor(a!) output, float scale) "
                         "-> Tensor(a!)",
    "commit_path_": "branchcraft::commit_path_(Tensor(a!) cache_k, Tensor(b!) cache_v, "
                    "Tensor draft_k, Tensor draft_v, Tensor path_nodes, Tensor dest_pages, "
                    "Tensor dest_slots, int request) -> ()",
}


def test_reference_schemas_verbatim():
    for name, schema in REFERENCE_SCHEMAS.items():
        assert str(getattr(torch.ops.branchcraft, name).default._schema) == schema


def test_added_ops_registered():
    for name in ("paged_decode", "tree_verify_out", "packed_decode_kv_out", "commit_batch_"):
        assert getattr(torch.ops.branchcraft, name).default is not None


def test_fake_kernels():
    with FakeTensorMode():
        q = torch.empty(2, 7, 32, 128, dtype=torch.float16)
        pk = torch.empty(40, 16, 8, 128, dtype=torch.float16)
        pages = torch.empty(2, 3, dtype=torch.int32)
        lengths = torch.empty(2, dtype=torch.int32)
        dk = torch.empty(2, 7, 8, 128, dtype=torch.float16)
        par = torch.empty(2, 7, dtype=torch.int32)
        out = torch.ops.branchcraft.tree_verify(q, pk, pk, pages, lengths, dk, dk, par)
        assert out.shape == q.shape and out.dtype == torch.float32
        q3 = torch.empty(2, 32, 128, dtype=torch.float16)
        dec = torch.ops.branchcraft.paged_decode(q3, pk, pk, pages, lengths)
        assert dec.shape == q3.shape and dec.dtype == torch.float32
        o16 = torch.empty(2, 32, 128, dtype=torch.float16)
        packed = torch.empty(40, 8, 16, 256, dtype=torch.float16)
        assert torch.ops.branchcraft.packed_decode_out(q3, packed, pages, lengths, o16,
                                                       0.1) is not None


def test_cpu_tensors_are_rejected_loudly():
    """No CPU fallback: the ops only have CUDA kernels."""
    q = torch.zeros(1, 1, 4, 64, dtype=torch.float16)
    pk = torch.zeros(1, 16, 2, 64, dtype=torch.float16)
    i = torch.zeros(1, 1, dtype=torch.int32)
    try:
        torch.ops.branchcraft.tree_verify(q, pk, pk, i, i[0], pk[:, :1].reshape(1, 1, 2, 64),
                                          pk[:, :1].reshape(1, 1, 2, 64), i)
    except (RuntimeError, NotImplementedError):
        return
    raise AssertionError("a CPU tensor was accepted")
