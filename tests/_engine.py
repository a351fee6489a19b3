"""A minimal continuous-batching driver for executor tests.

Stand-ins with exactly the attributes the executor reads from the reference's
`Sequence`, `BlockTable` and `BlockAllocator` (inference_server/core/sequence.py:134-161,
core/block_table.py:61-159, core/block_allocator.py:65-90), and `OracleExecutor`: the
reference executor's algorithm (paged_executor.py:162-295) with the CPU oracle doing the
KV append and the gather-path attention, the HF model running on the same device as the
CUDA arm so only the attention path differs between the two.
"""

from __future__ import annotations

import numpy as np
import torch
from transformers import AttentionInterface, Cache

from oracle import paged_attention_oracle as oracle

ORACLE_ATTN = "oracle_paged_gather_for_tests"


class Allocator:
    def __init__(self, num_blocks: int):
        self.free = list(range(num_blocks))[::-1]          # LIFO like the reference's free list

    def allocate(self) -> int:
        if not self.free:
            raise MemoryError("pool exhausted")
        return self.free.pop()


class Table:
    def __init__(self, alloc: Allocator, block_size: int):
        self.alloc, self.block_size, self.blocks = alloc, block_size, []

    @property
    def capacity(self) -> int:
        return len(self.blocks) * self.block_size

    def ensure_capacity(self, num_tokens: int) -> None:
        while self.capacity < num_tokens:
            self.blocks.append(self.alloc.allocate())

    def ensure_private(self, logical, copy=None):
        return None                                         # no sharing in these tests


class Seq:
    def __init__(self, prompt: list[int]):
        self.prompt_token_ids = list(prompt)
        self.output_token_ids: list[int] = []
        self.num_cached = 0
        self.block_table: Table | None = None

    @property
    def next_input_ids(self) -> list[int]:
        return (self.prompt_token_ids + self.output_token_ids)[self.num_cached:]

    @property
    def is_prefilling(self) -> bool:
        return self.num_cached == 0 or len(self.next_input_ids) > 1


def generate(executor, prompts, steps: int, num_blocks: int, block_size: int = 16, join_at: dict | None = None):
    """Greedy decode: step 0 prefills the first prompts; prompts listed in `join_at`
    ({step: [prompt index...]}) join later, so their prefill runs beside decodes."""
    alloc = Allocator(num_blocks)
    join_at = join_at or {}
    late = {i for idxs in join_at.values() for i in idxs}
    seqs = [Seq(p) for p in prompts]
    for s in seqs:
        s.block_table = Table(alloc, block_size)
    active = [s for i, s in enumerate(seqs) if i not in late]
    for step in range(steps):
        active += [seqs[i] for i in join_at.get(step, [])]
        for s in active:
            s.block_table.ensure_capacity(s.num_cached + len(s.next_input_ids))
        toks = executor.execute(active)
        for s, t in zip(active, toks):
            s.output_token_ids.append(int(t))
    return [s.output_token_ids for s in seqs]


class _OracleCache(Cache):
    def __init__(self, ex, ctx):
        super().__init__(layers=[])
        self.ex, self.ctx = ex, ctx

    def update(self, key_states, value_states, layer_idx, *args, **kwargs):
        k = key_states[0].transpose(0, 1).float().cpu().numpy()
        v = value_states[0].transpose(0, 1).float().cpu().numpy()
        self.ex.k[layer_idx] = oracle.kv_append(self.ex.k[layer_idx], self.ctx["write_slots"], k)
        self.ex.v[layer_idx] = oracle.kv_append(self.ex.v[layer_idx], self.ctx["write_slots"], v)
        return key_states, value_states

    def get_seq_length(self, layer_idx: int = 0) -> int:
        raise RuntimeError("explicit position_ids are passed")


def _oracle_attention(module, query, key, value, attention_mask, scaling=None, **kwargs):
    ctx = kwargs["oracle_ctx"]
    ex = ctx["ex"]
    if scaling is None:
        scaling = query.shape[-1] ** -0.5
    q = query[0].transpose(0, 1).float().cpu().numpy()
    out = oracle.paged_attention_gather(q, ex.k[module.layer_idx], ex.v[module.layer_idx], ctx["block_tables"],
                                        ctx["context_lens"], ctx["query_lens"], scaling, ex.dtype)
    return torch.from_numpy(out).to(device=query.device, dtype=query.dtype).unsqueeze(0), None


AttentionInterface.register(ORACLE_ATTN, _oracle_attention)


class OracleExecutor:
    """The reference's executor algorithm with the oracle as attention and KV append."""

    def __init__(self, model, num_layers, num_blocks, block_size, kv_heads, head_dim, dtype: str = "f32"):
        shape = (num_blocks, block_size, kv_heads, head_dim)
        self.k = [np.zeros(shape, np.float32) for _ in range(num_layers)]
        self.v = [np.zeros(shape, np.float32) for _ in range(num_layers)]
        self.model, self.block_size, self.dtype = model, block_size, dtype
        self.device = next(model.parameters()).device

    @torch.inference_mode()
    def execute(self, seqs) -> list[int]:
        packed = oracle.pack_step([(list(s.block_table.blocks), s.num_cached, len(s.next_input_ids)) for s in seqs],
                                  self.block_size)
        ids = [t for s in seqs for t in s.next_input_ids]
        ctx = dict(packed, ex=self)
        input_ids = torch.tensor([ids], dtype=torch.long, device=self.device)
        position_ids = torch.from_numpy(packed["position_ids"])[None].to(self.device)
        cfg = self.model.config
        prev = cfg._attn_implementation
        cfg._attn_implementation = ORACLE_ATTN
        try:
            logits = self.model(input_ids=input_ids, position_ids=position_ids, past_key_values=_OracleCache(self, ctx),
                                use_cache=True, oracle_ctx=ctx).logits
        finally:
            cfg._attn_implementation = prev
        for s in seqs:
            s.num_cached += len(s.next_input_ids)
        ends = torch.from_numpy(packed["ends"]).to(self.device)
        self.last_logits = logits[0, ends - 1, :].float()
        return self.last_logits.argmax(-1).tolist()
