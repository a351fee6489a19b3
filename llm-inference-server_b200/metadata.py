"""Per-step ragged-batch metadata: planned once on the host, uploaded with ONE copy.

The reference rebuilds its step metadata with six ``torch.tensor(..., device=dev)``
copies (inference_server/core/paged_executor.py:253-262) and then re-validates it in
every layer with host-syncing reductions (inference_server/core/attention.py:202-219,
125, 162-163).  Here the C++ planner (``pa_plan_step``) validates the batch once with the
reference's error messages, and packs the int32 block table, lengths, prefix sums,
per-token ``seq_idx``/``q_pos`` (attention_triton.py:129-150), new-token slot mapping
(block_table.py:143-159) and the split-K work list into one buffer.  Every layer's
attention and KV append then reads that single device copy.
"""

from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _lib


def _as_i64(x) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach().to("cpu")
        return np.ascontiguousarray(x.numpy(), dtype=np.int64)
    return np.ascontiguousarray(np.asarray(x, dtype=np.int64))


_SM_COUNT: dict[int, int] = {}

def prefill_tile_rows(head_dim: int = 128) -> int:
    """(token, query-head) rows of one tensor-core prefill tile at this head_dim, as the
    loaded library's kernels are built (256 for the CTA-pair kernel at head_dim 128)."""
    return int(_lib.lib().pa_prefill_tile_rows(int(head_dim)))


def prefill_tile_tokens(num_heads: int, num_kv_heads: int, head_dim: int = 128) -> int:
    """Query tokens per prefill tile (the kernel's rows / G heads per KV head), or 0 when
    the group size has no tensor-core prefill instantiation (the generic kernel runs)."""
    if num_kv_heads <= 0 or num_heads % num_kv_heads:
        return 0
    g = num_heads // num_kv_heads
    return prefill_tile_rows(head_dim) // g if g in (1, 2, 4, 8) else 0


def sm_count(device: torch.device | None) -> int:
    """Streaming multiprocessors of the device the step runs on (148 on B200)."""
    if device is None or device.type != "cuda":
        return 148
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SM_COUNT:
        _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SM_COUNT[idx]


class StepMetadata:
    """One step's plan plus its packed metadata, on the host and (after ``upload``) on
    the device.  Immutable once built; shared by every layer of the step."""

    def __init__(self, plan: _lib.StepPlan, host: np.ndarray, pool_num_blocks: int):
        self.plan = plan
        self.host = host                      # int32 [plan.words]
        self.pool_num_blocks = int(pool_num_blocks)
        self.device_buffer: torch.Tensor | None = None

    # ------------------------------------------------------------------ planning
    @classmethod
    def plan_host(cls, context_lens, query_lens, block_tables, *, num_tokens: int, pool_num_blocks: int,
                  block_size: int, num_kv_heads: int, sm: int = 148, prefill_tile_tokens: int = 0,
                  pinned: bool = False) -> "StepMetadata":
        """Validate and pack on the host (no device work).  Raises ValueError with the
        reference's messages on a contract violation."""
        lib = _lib.lib()
        ctx = _as_i64(context_lens)
        ql = _as_i64(query_lens)
        bt = _as_i64(block_tables)
        if bt.ndim != 2:
            raise ValueError("block_tables must be [batch, max_blocks]")
        b = ctx.shape[0]
        if ctx.shape != (bt.shape[0],) or ql.shape != (bt.shape[0],):
            raise ValueError("context_lens and query_lens must be [batch] to match block_tables")
        plan = _lib.StepPlan()
        args = (ctx.ctypes.data, ql.ctypes.data, b, bt.ctypes.data, bt.shape[1], bt.shape[1], int(num_tokens),
                int(pool_num_blocks), int(block_size), int(num_kv_heads), int(sm), int(prefill_tile_tokens))
        _lib.check(lib.pa_plan_step(*args, None, 0, ctypes.byref(plan)))
        words = max(int(plan.words), 1)
        if pinned:
            host_t = torch.empty(words, dtype=torch.int32, pin_memory=True)
            host = host_t.numpy()
        else:
            host_t = None
            host = np.empty(words, dtype=np.int32)
        _lib.check(lib.pa_plan_step(*args, host.ctypes.data, words, ctypes.byref(plan)))
        meta = cls(plan, host, pool_num_blocks)
        meta._host_tensor = host_t
        return meta

    @classmethod
    def plan_decode_padded(cls, context_lens, block_tables, *, pool_num_blocks: int, block_size: int,
                           num_kv_heads: int, split_blocks: int, width: int, items: int, combine: int,
                           host: np.ndarray | None = None) -> "StepMetadata":
        """An all-decode step planned to a fixed shape (a CUDA-graph bucket): split size
        ``split_blocks``, tables ``width`` wide, ``items`` decode work items and ``combine``
        combine entries (the unused ones are null entries the kernels skip).  Writes into
        ``host`` when given (a graph's pinned buffer).  Raises ValueError("bucket: ...")
        when the step does not fit."""
        lib = _lib.lib()
        ctx = _as_i64(context_lens)
        bt = _as_i64(block_tables)
        if bt.ndim != 2 or ctx.shape != (bt.shape[0],):
            raise ValueError("block_tables must be [batch, max_blocks] and context_lens [batch]")
        plan = _lib.StepPlan()
        args = (ctx.ctypes.data, ctx.shape[0], bt.ctypes.data, bt.shape[1], bt.shape[1], int(pool_num_blocks),
                int(block_size), int(num_kv_heads), int(split_blocks), int(width), int(items), int(combine))
        _lib.check(lib.pa_plan_decode_padded(*args, None, 0, ctypes.byref(plan)))
        words = max(int(plan.words), 1)
        if host is None:
            host = np.empty(words, dtype=np.int32)
        elif host.size < words:
            raise ValueError(f"host buffer holds {host.size} words, the plan needs {words}")
        _lib.check(lib.pa_plan_decode_padded(*args, host.ctypes.data, host.size, ctypes.byref(plan)))
        return cls(plan, host, pool_num_blocks)

    @classmethod
    def build(cls, context_lens, query_lens, block_tables, *, num_tokens: int, pool_num_blocks: int,
              block_size: int, num_kv_heads: int, device, prefill_tile_tokens: int = 0) -> "StepMetadata":
        """Plan on the host and upload to ``device`` with one asynchronous copy."""
        device = torch.device(device)
        meta = cls.plan_host(context_lens, query_lens, block_tables, num_tokens=num_tokens,
                             pool_num_blocks=pool_num_blocks, block_size=block_size, num_kv_heads=num_kv_heads,
                             sm=sm_count(device), prefill_tile_tokens=prefill_tile_tokens,
                             pinned=device.type == "cuda")
        meta.upload(device)
        return meta

    def upload(self, device) -> "StepMetadata":
        host_t = getattr(self, "_host_tensor", None)
        if host_t is None:
            host_t = torch.from_numpy(self.host)
        dev = torch.empty(host_t.shape, dtype=torch.int32, device=device)
        dev.copy_(host_t, non_blocking=True)
        self.device_buffer = dev
        return self

    # ------------------------------------------------------------------ views
    def _view(self, off: int, n: int, on_device: bool = True):
        if on_device:
            return self.device_buffer[off:off + n]
        return self.host[off:off + n]

    @property
    def num_tokens(self) -> int:
        return int(self.plan.num_tokens)

    def slot_mapping(self, on_device: bool = True):
        return self._view(self.plan.off_slot_mapping, self.plan.num_tokens, on_device)

    def seq_idx(self, on_device: bool = True):
        return self._view(self.plan.off_seq_idx, self.plan.num_tokens, on_device)

    def q_pos(self, on_device: bool = True):
        return self._view(self.plan.off_q_pos, self.plan.num_tokens, on_device)

    def cu_query_lens(self, on_device: bool = True):
        return self._view(self.plan.off_cu_query_lens, self.plan.num_seqs + 1, on_device)

    def block_tables(self, on_device: bool = True):
        b, w = self.plan.num_seqs, self.plan.table_width
        v = self._view(self.plan.off_block_tables, b * w, on_device)
        return v.reshape(b, w)

    def decode_items(self):
        return self.host[self.plan.off_decode_items:self.plan.off_decode_items + 4 * self.plan.num_decode_items
                         ].reshape(-1, 4)

    def matches(self, num_tokens: int, block_size: int, pool_num_blocks: int) -> bool:
        return (self.plan.num_tokens == num_tokens and self.plan.block_size == block_size
                and self.pool_num_blocks == pool_num_blocks)


def attach(block_tables: torch.Tensor, meta: StepMetadata) -> torch.Tensor:
    """Let a step's metadata ride on its block-table tensor.

    The attention seam keeps the gather path's exact seven-parameter signature
    (inference_server/core/attention.py:73-81, arity pinned by
    tests/test_paged_attention.py:197-204), so the executor hands the already-planned
    metadata over as an attribute of the ``block_tables`` argument it passes anyway.
    """
    block_tables._pa_step = meta
    return block_tables


def attached(block_tables: torch.Tensor) -> StepMetadata | None:
    return getattr(block_tables, "_pa_step", None)
