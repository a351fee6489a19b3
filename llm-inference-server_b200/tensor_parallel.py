"""KV-head tensor parallelism for the large-GQA configurations (Llama-3-70B shape: 64
query heads, 8 KV heads).

Rank r of a tensor-parallel group of size tp holds KV heads ``[r*Hkv/tp, (r+1)*Hkv/tp)``
and the ``Hq/tp`` query heads that read them, so its KV pool is
``[num_blocks, 16, Hkv/tp, D]`` and every rank shares the same block tables (each rank
runs the same deterministic scheduler on the same requests).  Per layer a rank appends its
heads' new K/V, runs paged attention over its heads, multiplies by its row slice of the
output projection, and one all-reduce (NCCL over NVLink on GPUs) sums the partial
projections.  The reference has no multi-GPU path (its design notes name it a non-goal);
the arithmetic here is the single-device layer's, split by heads.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def kv_head_shard(num_heads: int, num_kv_heads: int, rank: int, world: int) -> tuple[slice, slice]:
    """(query-head slice, KV-head slice) owned by ``rank``.  KV heads split evenly; each
    KV head keeps its whole GQA group of query heads on the same rank."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a group of {world}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads cannot be split across {world} ranks")
    if num_heads % num_kv_heads:
        raise ValueError(f"{num_heads} query heads not divisible by {num_kv_heads} kv heads")
    kv = num_kv_heads // world
    group = num_heads // num_kv_heads
    return slice(rank * kv * group, (rank + 1) * kv * group), slice(rank * kv, (rank + 1) * kv)


def o_proj_shard(weight: torch.Tensor, num_heads: int, head_dim: int, rank: int, world: int,
                 num_kv_heads: int) -> torch.Tensor:
    """Rows of the output projection this rank multiplies, as an ``[in, out]`` matrix.

    ``weight`` is a ``torch.nn.Linear`` weight ``[d_model_out, num_heads * head_dim]``; the
    rank's query heads select a contiguous block of its input columns."""
    qs, _ = kv_head_shard(num_heads, num_kv_heads, rank, world)
    cols = slice(qs.start * head_dim, qs.stop * head_dim)
    return weight[:, cols].t().contiguous()


@dataclass
class KVHeadParallelAttention:
    """One layer's attention hot path on one tensor-parallel rank.

    ``attention`` and ``append`` default to the sm_100a kernels (``paged_attention_cuda``,
    ``reshape_and_cache``); they are parameters so the host logic — sharding, the o_proj
    split and the collective — can be exercised with other implementations of the same
    signatures."""

    w_o: torch.Tensor                 # [Hq_local * D, d_model]
    group: object = None              # torch.distributed process group (None = default)
    attention: object = None
    append: object = None

    def __post_init__(self):
        if self.attention is None:
            from .attention import paged_attention_cuda

            self.attention = paged_attention_cuda
        if self.append is None:
            from .kv_cache import reshape_and_cache

            self.append = reshape_and_cache

    def __call__(self, q, k_new, v_new, k_pool, v_pool, block_tables, context_lens, query_lens, scale,
                 slot_mapping) -> torch.Tensor:
        """q ``[T, Hq/tp, D]``, new K/V ``[T, Hkv/tp, D]`` -> the all-reduced o_proj output
        ``[T, d_model]`` (identical on every rank)."""
        self.append(k_new, v_new, k_pool, v_pool, slot_mapping)
        attn = self.attention(q, k_pool, v_pool, block_tables, context_lens, query_lens, scale)
        partial = attn.reshape(attn.shape[0], -1).to(self.w_o.dtype) @ self.w_o
        if dist.is_available() and dist.is_initialized():
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
        return partial
