"""vLLM general-plugin hook: registers BranchcraftBackend as the CUSTOM
attention backend (reference python/branchcraft_vllm/plugin.py:4-13)."""


def register():
    from vllm.v1.attention.backends.registry import AttentionBackendEnum, register_backend

    register_backend(AttentionBackendEnum.CUSTOM, "branchcraft_vllm.backend.BranchcraftBackend")
