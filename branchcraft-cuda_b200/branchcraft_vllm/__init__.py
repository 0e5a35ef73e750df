"""Opt-in vLLM V1 attention backend over the Branchcraft packed decode.

Select it with attention_backend='CUSTOM' once `plugin.register()` has run
(vLLM calls it through the `vllm.general_plugins` entry point). Mirrors the
reference's python/branchcraft_vllm package (__init__.py:1, plugin.py:4-13,
backend.py:20-96).
"""
