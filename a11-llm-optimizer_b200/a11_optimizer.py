"""``a11_optimizer``: the module name of the reference's pybind extension
(src/bindings/python_bindings.cpp:23-143), answered by this library.

Code written against the reference's binding imports this module and finds
the speculative-decoding classes and constants it used, under the same names:

* ``SpecConfig``, ``TreeNode``, ``SpecDiagnostics``, ``SpeculativeTreeVerifier``,
  ``SPEC_K`` (python_bindings.cpp:27, 78-143): acceptance decisions run on the GPU
  through the C ABI (``a11spec.verifier``);
* ``KVCacheConfig``, ``PagedKVCacheManager``, ``BLOCK_TOKENS``,
  ``KV_CACHE_VRAM_GB`` (python_bindings.cpp:28-29, 46-76): the block-table semantics
  of the reference's paged KV cache over one page pool per K and V
  (``a11spec.kv_pages``).

The binding's ``NvmeAsyncLoader`` (python_bindings.cpp:34-41, NVMe weight streaming) belongs to the
reference's weight-paging subsystem, which this library does not cover, so the
name is absent here.
"""
from a11spec.kv_pages import KV_CACHE_VRAM_GB, KVCacheConfig, PagedKVCacheManager
from a11spec.verifier import (BLOCK_TOKENS, SPEC_K, SpecConfig, SpecDiagnostics, SpeculativeTreeVerifier,
                              TreeNode)

__all__ = ["BLOCK_TOKENS", "KV_CACHE_VRAM_GB", "KVCacheConfig", "PagedKVCacheManager", "SPEC_K",
           "SpecConfig", "SpecDiagnostics", "SpeculativeTreeVerifier", "TreeNode"]
