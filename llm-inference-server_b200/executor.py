"""The reference's paged executor on the CUDA path.

Mirror of ``PagedExecutor`` (inference_server/core/paged_executor.py:162-295) with the
same contract — ``execute(seqs) -> one greedy token per sequence``, ``num_cached``
advanced here and nowhere else, the HuggingFace model reused untouched through its two
seams — and the three hot-path changes:

* ``_pack`` (paged_executor.py:211-263) plans the step once on the host
  (``StepMetadata``: validation, int32 block tables, lengths, prefix sums, per-token
  positions, the new tokens' slots, the split-K work list) and uploads it with one copy;
  the reference makes six ``torch.tensor(..., device=dev)`` copies and computes each
  sequence's slots over its whole context (``table.slots(after)``, O(context) Python).
  Position ids are the planned ``q_pos`` (the reference's ``range(num_cached, after)``).
* ``PagedCache.update`` (paged_executor.py:116-125) writes K and V with one fused
  append launch at the planned slots instead of two ``index_copy_`` calls.
* The registered attention function (paged_executor.py:134-156) calls
  ``paged_attention_cuda``; the step's metadata rides on its ``block_tables`` argument,
  so no layer synchronises with the host.

Sequences and pools are duck-typed exactly as the reference uses them: a sequence has
``next_input_ids``, ``num_cached``, ``is_prefilling`` and a ``block_table`` with
``blocks``, ``block_size``, ``capacity`` and ``ensure_private(logical, copy)``
(inference_server/core/sequence.py, core/block_table.py); a pool has per-layer ``k`` /
``v`` lists of ``[num_blocks, block_size, Hkv, D]`` tensors (core/kv_pool.py:106-125).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
from transformers import AttentionInterface, Cache

from .attention import paged_attention_cuda
from .kv_cache import copy_blocks, reshape_and_cache
from .metadata import StepMetadata, attach, prefill_tile_tokens

#: Name under which the CUDA attention is registered with transformers while a paged
#: forward runs (prefixed so it cannot collide with transformers' own entries).
ATTN_IMPL = "llm_inference_server_b200_paged"


@dataclass(frozen=True)
class StepContext:
    """Everything one forward pass needs, built once per step (paged_executor.py:83-95)."""

    meta: StepMetadata
    block_tables: torch.Tensor   # device int64 [B, W] carrying `meta`
    context_lens: torch.Tensor   # device [B]
    query_lens: torch.Tensor     # device [B]
    pool: object


class PagedCache(Cache):
    """A `Cache` whose only job is to intercept `update` and write into the pool with the
    fused append (paged_executor.py:98-131)."""

    def __init__(self, ctx: StepContext) -> None:
        super().__init__(layers=[])
        self.ctx = ctx

    def update(self, key_states, value_states, layer_idx: int, *args, **kwargs):
        # [1, Hkv, T, D] -> [T, Hkv, D]: strided views, the kernel takes the strides.
        k = key_states[0].transpose(0, 1)
        v = value_states[0].transpose(0, 1)
        pool = self.ctx.pool
        reshape_and_cache(k, v, pool.k[layer_idx], pool.v[layer_idx], self.ctx.meta.slot_mapping())
        return key_states, value_states

    def get_seq_length(self, layer_idx: int = 0) -> int:
        raise RuntimeError("the paged executor passes explicit position_ids; the pool has no single length")

    def get_mask_sizes(self, query_length: int, layer_idx: int = 0):
        raise RuntimeError("no mask is built for the paged kernel; create_causal_mask should have early-exited")


def paged_attention_forward(module, query, key, value, attention_mask, scaling=None, **kwargs):
    """transformers' attention-interface signature: [1, H, T, D] in, ([1, T, H, D], None)
    out.  `key`/`value` are ignored on purpose: the kernel reads the new tokens back out
    of the pool with the old ones, through the block table (paged_executor.py:134-156)."""
    ctx: StepContext = kwargs["paged_ctx"]
    if scaling is None:
        scaling = query.shape[-1] ** -0.5
    q = query[0].transpose(0, 1)                                  # [T, H, D], strided
    out = paged_attention_cuda(q, ctx.pool.k[module.layer_idx], ctx.pool.v[module.layer_idx], ctx.block_tables,
                               ctx.context_lens, ctx.query_lens, scaling)
    return out.unsqueeze(0), None


AttentionInterface.register(ATTN_IMPL, paged_attention_forward)


class CudaPagedExecutor:
    """One forward pass over the pool, no policy.  Drop-in for the reference's
    ``PagedExecutor`` with ``ATTENTION=cuda``."""

    #: Batch and table-width buckets of the captured decode passes (``decode_graphs``).
    GRAPH_BATCHES = (1, 2, 4, 8, 16, 32, 64, 128, 256, 512)

    def __init__(self, model, tokenizer, pool, device=None, decode_graphs: bool = False) -> None:
        self.model = model
        self.tokenizer = tokenizer
        self.pool = pool
        #: Run all-decode passes as captured CUDA graphs of the whole model forward
        #: (graphs.ModelDecodeGraph), one per (batch bucket, width bucket), built on
        #: first use; other passes run eagerly.
        self.decode_graphs = bool(decode_graphs)
        self._graphs: dict = {}
        self.device = torch.device(device) if device is not None else pool.k[0].device
        if self.device.type != "cuda":
            raise NotImplementedError(f"ATTENTION=cuda: the paged executor needs a CUDA device, got {self.device}")
        self.num_blocks, self.block_size, self.num_kv_heads, head_dim = pool.k[0].shape
        cfg = model.config
        heads = getattr(cfg, "num_attention_heads", None) or cfg.n_head
        self.tile_tokens = prefill_tile_tokens(heads, self.num_kv_heads, head_dim)

    @torch.inference_mode()
    def execute(self, seqs) -> list[int]:
        """Advance every sequence by one token; returns the greedy token ids
        (paged_executor.py:172-203).  Mixed prefill/decode batches also run correctly."""
        if not seqs:
            return []
        if self.decode_graphs and len(seqs) <= self.GRAPH_BATCHES[-1] and all(
                len(s.next_input_ids) == 1 for s in seqs):
            return self._execute_graph(seqs)
        input_ids, position_ids, ctx = self._pack(seqs)
        logits = self._forward(input_ids, position_ids, ctx)
        for s in seqs:
            s.num_cached += len(s.next_input_ids)
        ends = ctx.meta.cu_query_lens()[1:].long()
        return logits[0, ends - 1, :].argmax(-1).tolist()

    def _execute_graph(self, seqs) -> list[int]:
        """An all-decode pass through a captured graph: rows padded to the batch bucket
        by repeating the last sequence, tables to a power-of-two width bucket."""
        from .graphs import ModelDecodeGraph

        bs = self.block_size
        ctx_lens, rows, ids = [], [], []
        for i, s in enumerate(seqs):
            table = s.block_table
            assert table is not None, f"{getattr(s, 'seq_id', i)} reached the paged executor without a block table"
            after = s.num_cached + 1
            assert table.capacity >= after, (
                f"{getattr(s, 'seq_id', i)}: block table holds {table.capacity} slots, pass needs {after} — "
                "the scheduler must call ensure_capacity before execute")
            table.ensure_private((after - 1) // bs, self._copy_block)   # paged_executor.py:234-241
            ctx_lens.append(after)
            rows.append(table.blocks)
            ids.append(s.next_input_ids[0])
        b = len(seqs)
        bp = next(x for x in self.GRAPH_BATCHES if x >= b)
        need = max(len(r) for r in rows)
        width = 8
        while width < need:
            width *= 2
        tables = np.zeros((bp, width), dtype=np.int64)
        for i in range(bp):
            r = rows[min(i, b - 1)]
            tables[i, :len(r)] = r
        ctx = np.asarray(ctx_lens + [ctx_lens[-1]] * (bp - b), dtype=np.int64)
        g = self._graphs.get((bp, width))
        if g is None:
            g = self._graphs[(bp, width)] = ModelDecodeGraph(self, bp, width)
        g.set_step(ctx, tables, ids + [ids[-1]] * (bp - b))
        tokens = g.run()
        for s in seqs:
            s.num_cached += 1
        return tokens[:b].tolist()

    def reset(self) -> None:
        """Nothing survives between steps (paged_executor.py:205-208)."""

    # ------------------------------------------------------------------ packing
    def _pack(self, seqs):
        bs = self.block_size
        ids: list[int] = []
        q_lens = np.empty(len(seqs), dtype=np.int64)
        c_lens = np.empty(len(seqs), dtype=np.int64)
        rows = []
        for i, s in enumerate(seqs):
            new = s.next_input_ids
            table = s.block_table
            assert table is not None, f"{getattr(s, 'seq_id', i)} reached the paged executor without a block table"
            after = s.num_cached + len(new)
            assert table.capacity >= after, (
                f"{getattr(s, 'seq_id', i)}: block table holds {table.capacity} slots, pass needs {after} — "
                "the scheduler must call ensure_capacity before execute")
            # Copy-on-write guard of paged_executor.py:234-241 (a refcount read per
            # written block; a copy only under partial-block sharing).
            for logical in range(s.num_cached // bs, (after - 1) // bs + 1):
                table.ensure_private(logical, self._copy_block)
            ids.extend(new)
            q_lens[i] = len(new)
            c_lens[i] = after
            rows.append(table.blocks)
        width = max(len(r) for r in rows)
        tables = np.zeros((len(seqs), width), dtype=np.int64)
        for i, r in enumerate(rows):
            tables[i, :len(r)] = r
        meta = StepMetadata.build(c_lens, q_lens, tables, num_tokens=len(ids), pool_num_blocks=self.num_blocks,
                                  block_size=bs, num_kv_heads=self.num_kv_heads, device=self.device,
                                  prefill_tile_tokens=self.tile_tokens)
        dev = self.device
        block_tables = attach(torch.empty(len(seqs), meta.plan.table_width, dtype=torch.long, device=dev), meta)
        buf = meta.device_buffer
        ctx_lens = buf[meta.plan.off_context_lens:meta.plan.off_context_lens + len(seqs)]
        query_lens = buf[meta.plan.off_query_lens:meta.plan.off_query_lens + len(seqs)]
        ctx = StepContext(meta=meta, block_tables=block_tables, context_lens=ctx_lens, query_lens=query_lens,
                          pool=self.pool)
        input_ids = torch.tensor([ids], dtype=torch.long).pin_memory().to(dev, non_blocking=True)
        position_ids = meta.q_pos().unsqueeze(0)          # ctx_i - q_i + t, int32, already on the device
        return input_ids, position_ids, ctx

    def _copy_block(self, src: int, dst: int) -> None:
        """Move one block's K/V, every layer, for ``BlockTable.ensure_private``
        (paged_executor.py:265-270): one block-copy launch for all layers."""
        copy_blocks(self.pool.k, self.pool.v, [(src, dst)])

    # ------------------------------------------------------------------ forward
    def _forward(self, input_ids, position_ids, ctx: StepContext):
        """Run the shared model with attention swapped for the paged kernel for exactly
        this call (paged_executor.py:273-295)."""
        config = self.model.config
        previous = config._attn_implementation
        config._attn_implementation = ATTN_IMPL
        try:
            out = self.model(input_ids=input_ids, position_ids=position_ids, past_key_values=PagedCache(ctx),
                             use_cache=True, paged_ctx=ctx)
        finally:
            config._attn_implementation = previous
        return out.logits
