"""B200-native (sm_100a) paged attention for akshajravi/llm-inference-server.

The reference's attention seam with ``ATTENTION=cuda``:

* ``paged_attention_cuda`` — drop-in for ``paged_attention_gather``
  (inference_server/core/attention.py:92-187): split-K decode + combine and a generic
  ragged kernel on the GPU, no CPU fallback.
* ``reshape_and_cache`` — fused K+V append (inference_server/core/paged_executor.py:116-125).
* ``StepMetadata`` — the step's ragged metadata planned once on the host and uploaded
  with a single copy (inference_server/core/paged_executor.py:211-263).

``executor.CudaPagedExecutor`` is the reference's ``PagedExecutor`` on this path
(imported on demand: it needs ``transformers``).

The directory name is not a Python identifier; the package is imported under the name
``llm_inference_server_b200`` (see ``__graft_entry__.import_package``).
"""

from __future__ import annotations

from .attention import paged_attention, paged_attention_cuda, read_device_error
from .kv_cache import HostBlocks, KVPool, allocate_pool, copy_blocks, reshape_and_cache
from .metadata import StepMetadata, attach, attached, prefill_tile_tokens

__all__ = [
    "paged_attention",
    "paged_attention_cuda",
    "read_device_error",
    "reshape_and_cache",
    "allocate_pool",
    "KVPool",
    "HostBlocks",
    "copy_blocks",
    "StepMetadata",
    "attach",
    "attached",
    "prefill_tile_tokens",
]
