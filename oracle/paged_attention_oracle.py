"""CPU oracle for the paged-attention hot path.  TEST INFRASTRUCTURE ONLY.

This module is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` may import it.  The CUDA path in ``llm-inference-server_b200/`` never
calls it and has no CPU fallback.

It restates, in numpy, the algorithm of the reference's PyTorch gather path and the
integer arithmetic around it.  Every function cites the reference file:line it follows
(paths relative to the akshajravi/llm-inference-server project root):

  check                  inference_server/core/attention.py:202-219   (_check)
  expand_kv_heads        inference_server/core/attention.py:190-199   (_expand_kv_heads)
  paged_attention_gather inference_server/core/attention.py:92-127    (dispatch decode/ragged)
  _decode_batched        inference_server/core/attention.py:130-153
  _ragged_loop           inference_server/core/attention.py:156-187
  paged_attention_mirror inference_server/core/attention_triton.py:309-384
                         (paged_attention_reference: the Triton kernel's per-(token,
                         head) block loop and online softmax, the secondary oracle)
  token_map              inference_server/core/attention_triton.py:129-150 (_token_map)
  slots                  inference_server/core/block_table.py:143-159 (BlockTable.slots)
  pack_step              inference_server/core/paged_executor.py:211-263 (_pack)
  kv_append              inference_server/core/paged_executor.py:116-125 (_PagedCache.update)
  swap_out               inference_server/core/kv_pool.py:142-166 (PagedKVPool.swap_out)
  swap_in                inference_server/core/kv_pool.py:168-182 (PagedKVPool.swap_in)
  copy_block             inference_server/core/paged_executor.py:265-270 (_copy_block)

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference itself (imported
from its source tree in the development container) on seeded inputs and commits its
outputs under ``tests/golden/``; ``tests/test_oracle_golden.py`` checks this module
against every one of those vectors, including the reference test-suite's own
known-answer ``_token_map`` case.

Precision emulation.  Inputs are float32 arrays holding values exactly representable
in the storage dtype (``"f32"``, ``"f16"`` or ``"bf16"``).  For half dtypes the
reference's torch ops round at the same places this code does: ``q @ k^T`` rounds to
the storage dtype, ``* scale`` rounds again, softmax runs in float32
(``softmax(dtype=float32)``), probabilities are cast to the V dtype, and ``probs @ v``
rounds its float32-accumulated result to the storage dtype (attention.py:145-153,
176-185).
"""

from __future__ import annotations

import numpy as np

DTYPES = ("f32", "f16", "bf16")


# ------------------------------------------------------------------ dtype emulation
def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to the storage dtype, returned as float32.

    The reference narrows at two points: the probabilities, ``softmax(..., dtype=float32)
    .to(v.dtype)`` (inference_server/core/attention.py:152 and :184), and every tensor op
    whose inputs are half precision (its matmuls return the input dtype).  bf16 uses
    round-to-nearest-even on the float32 bit pattern (the IEEE rule torch applies when it
    narrows float32 to bfloat16); f16 goes through numpy's half type.
    """
    x = np.asarray(x, dtype=np.float32)
    if dtype == "f32":
        return x
    if dtype == "f16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        u = x.view(np.uint32).astype(np.uint64)
        bias = ((u >> 16) & 1) + 0x7FFF
        r = ((u + bias) & 0xFFFF0000).astype(np.uint32)
        out = r.view(np.float32)
        return np.where(np.isnan(x), x, out).astype(np.float32)
    raise ValueError(f"unknown dtype {dtype!r}")


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """The upper 16 bits of float32 values that are exact bf16 numbers (the storage form
    of the reference's bfloat16 tensors, compared bit for bit in the golden fixtures)."""
    return (np.asarray(x, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits: np.ndarray) -> np.ndarray:
    """float32 values of stored bf16 bit patterns (the inverse of :func:`bf16_bits`)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------ contract
def check(query_shape, pool_shape, block_tables, context_lens, query_lens) -> None:
    """The ragged-batch contract (attention.py:202-219); same ValueError texts."""
    if len(query_shape) != 3:
        raise ValueError(f"query must be [num_tokens, heads, dim], got {tuple(query_shape)}")
    if len(pool_shape) != 4:
        raise ValueError(f"k_pool must be [blocks, block_size, kv_heads, dim], got {tuple(pool_shape)}")
    block_tables = np.asarray(block_tables)
    context_lens = np.asarray(context_lens, dtype=np.int64)
    query_lens = np.asarray(query_lens, dtype=np.int64)
    batch = block_tables.shape[0]
    if context_lens.shape != (batch,) or query_lens.shape != (batch,):
        raise ValueError("context_lens and query_lens must be [batch] to match block_tables")
    if int(query_lens.sum()) != query_shape[0]:
        raise ValueError(f"query_lens sum to {int(query_lens.sum())} but query has {query_shape[0]} tokens")
    if bool((query_lens > context_lens).any()):
        raise ValueError("query_len exceeds context_len — the query tokens must be counted in the context")
    block_size = pool_shape[1]
    need = -(-context_lens // block_size)
    if bool((need > block_tables.shape[1]).any()):
        raise ValueError("a sequence's context needs more blocks than its block_tables row holds")


def expand_kv_heads(kv: np.ndarray, num_heads: int) -> np.ndarray:
    """repeat_interleave of each KV head over its query group (attention.py:190-199)."""
    kv_heads = kv.shape[-2]
    if kv_heads == num_heads:
        return kv
    if num_heads % kv_heads:
        raise ValueError(f"{num_heads} query heads not divisible by {kv_heads} kv heads")
    return np.repeat(kv, num_heads // kv_heads, axis=-2)


def _softmax_f32(scores: np.ndarray) -> np.ndarray:
    """Row softmax in float32, the reference's ``torch.softmax(scores, dim=-1,
    dtype=torch.float32)`` (inference_server/core/attention.py:152, :184); rows masked to
    -inf contribute exact zeros."""
    m = scores.max(axis=-1, keepdims=True)
    e = np.exp(scores - m, dtype=np.float32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)


# ------------------------------------------------------------------ attention
def paged_attention_gather(query, k_pool, v_pool, block_tables, context_lens, query_lens,
                           scale: float, dtype: str = "f32") -> np.ndarray:
    """Causal paged attention over a ragged batch (attention.py:92-127).

    query [T, Hq, D], pools [NB, BS, Hkv, D] (float32 arrays holding ``dtype`` values),
    block_tables [B, W] int, context_lens / query_lens [B] int -> [T, Hq, D] float32
    holding ``dtype`` values.  Token t of sequence i sits at logical position
    ``ctx_i - q_i + t`` and attends to keys ``0 .. that`` (attention.py:44-53, 116-119).
    """
    query = np.asarray(query, dtype=np.float32)
    k_pool = np.asarray(k_pool, dtype=np.float32)
    v_pool = np.asarray(v_pool, dtype=np.float32)
    block_tables = np.asarray(block_tables, dtype=np.int64)
    context_lens = np.asarray(context_lens, dtype=np.int64)
    query_lens = np.asarray(query_lens, dtype=np.int64)
    check(query.shape, k_pool.shape, block_tables, context_lens, query_lens)
    if query.shape[0] == 0:
        return np.empty((0, query.shape[1], query.shape[2]), dtype=np.float32)
    if bool((query_lens == 1).all()):
        return _decode_batched(query, k_pool, v_pool, block_tables, context_lens, scale, dtype)
    return _ragged_loop(query, k_pool, v_pool, block_tables, context_lens, query_lens, scale, dtype)


def _decode_batched(query, k_pool, v_pool, block_tables, context_lens, scale, dtype):
    """All-decode batch: one padded gather for every sequence (attention.py:130-153)."""
    batch, num_heads, head_dim = query.shape
    block_size = k_pool.shape[1]
    max_ctx = int(context_lens.max())
    max_blocks = -(-max_ctx // block_size)
    tables = block_tables[:, :max_blocks]
    k = k_pool[tables].reshape(batch, max_blocks * block_size, *k_pool.shape[2:])[:, :max_ctx]
    v = v_pool[tables].reshape(batch, max_blocks * block_size, *v_pool.shape[2:])[:, :max_ctx]
    k = expand_kv_heads(k, num_heads).transpose(0, 2, 1, 3)          # [B, H, ctx, D]
    v = expand_kv_heads(v, num_heads).transpose(0, 2, 1, 3)
    q = query[:, :, None, :]                                          # [B, H, 1, D]
    scores = round_to(np.matmul(q, k.transpose(0, 1, 3, 2)), dtype)   # [B, H, 1, ctx]
    scores = round_to(scores * np.float32(scale), dtype)
    valid = np.arange(max_ctx)[None, :] < context_lens[:, None]
    scores = np.where(valid[:, None, None, :], scores, np.float32(-np.inf))
    probs = round_to(_softmax_f32(scores), dtype)
    return round_to(np.matmul(probs, v), dtype)[:, :, 0, :]


def _ragged_loop(query, k_pool, v_pool, block_tables, context_lens, query_lens, scale, dtype):
    """Prefill / partial / mixed batch: one sequence at a time (attention.py:156-187)."""
    num_heads = query.shape[1]
    block_size = k_pool.shape[1]
    out = np.empty_like(query)
    start = 0
    for i in range(block_tables.shape[0]):
        q_len = int(query_lens[i])
        ctx = int(context_lens[i])
        if q_len == 0:
            continue
        nblocks = -(-ctx // block_size)
        blocks = block_tables[i, :nblocks]
        k = k_pool[blocks].reshape(-1, *k_pool.shape[2:])[:ctx]       # [ctx, Hkv, D]
        v = v_pool[blocks].reshape(-1, *v_pool.shape[2:])[:ctx]
        k = expand_kv_heads(k, num_heads).transpose(1, 0, 2)          # [H, ctx, D]
        v = expand_kv_heads(v, num_heads).transpose(1, 0, 2)
        q = query[start:start + q_len].transpose(1, 0, 2)             # [H, q_len, D]
        scores = round_to(np.matmul(q, k.transpose(0, 2, 1)), dtype)
        scores = round_to(scores * np.float32(scale), dtype)
        q_pos = np.arange(ctx - q_len, ctx)
        k_pos = np.arange(ctx)
        causal = k_pos[None, :] <= q_pos[:, None]
        scores = np.where(causal[None], scores, np.float32(-np.inf))
        probs = round_to(_softmax_f32(scores), dtype)
        out[start:start + q_len] = round_to(np.matmul(probs, v), dtype).transpose(1, 0, 2)
        start += q_len
    return out


def paged_attention_mirror(query, k_pool, v_pool, block_tables, context_lens, query_lens,
                           scale: float, dtype: str = "f32") -> np.ndarray:
    """The online-softmax order of the reference's Triton kernel, as its PyTorch mirror
    states it (attention_triton.py:309-384): for every (token, head), q is scaled in
    float32 before the dot products; the keys ``0 .. q_pos`` are walked one pool block at
    a time (block ``b`` of the sequence's row, keys past ``q_pos`` masked to -inf);
    per block ``m_new = max(m, max s)``, ``alpha = exp(m - m_new)``, ``p = exp(s - m_new)``,
    ``l = alpha*l + sum p``, ``acc = alpha*acc + p.v``; the output is ``acc / l`` rounded
    once to the storage dtype.  Everything runs in float32 (the mirror's ``.float()``);
    heads are vectorised here, the mirror loops over them."""
    query = np.asarray(query, dtype=np.float32)
    k_pool = np.asarray(k_pool, dtype=np.float32)
    v_pool = np.asarray(v_pool, dtype=np.float32)
    block_tables = np.asarray(block_tables, dtype=np.int64)
    check(query.shape, k_pool.shape, block_tables, context_lens, query_lens)
    num_tokens, num_heads, head_dim = query.shape
    block_size, num_kv_heads = k_pool.shape[1], k_pool.shape[2]
    group = num_heads // num_kv_heads
    out = np.empty_like(query)
    if num_tokens == 0:
        return out
    seq_idx, q_pos, _ = token_map(context_lens, query_lens)
    kv_of_head = np.arange(num_heads) // group
    offs = np.arange(block_size)
    for tok in range(num_tokens):
        seq, pos = int(seq_idx[tok]), int(q_pos[tok])
        n_keys = pos + 1
        q = query[tok] * np.float32(scale)                              # [H, D]
        m = np.full(num_heads, -np.inf, dtype=np.float32)
        l = np.zeros(num_heads, dtype=np.float32)
        acc = np.zeros((num_heads, head_dim), dtype=np.float32)
        for blk in range(-(-n_keys // block_size)):
            phys = int(block_tables[seq, blk])
            valid = blk * block_size + offs < n_keys                    # [BS]
            k = k_pool[phys][:, kv_of_head, :]                          # [BS, H, D]
            v = v_pool[phys][:, kv_of_head, :]
            k = np.where(valid[:, None, None], k, np.float32(0))
            v = np.where(valid[:, None, None], v, np.float32(0))
            s = np.einsum("bhd,hd->hb", k, q, dtype=np.float32)          # [H, BS]
            s = np.where(valid[None, :], s, np.float32(-np.inf))
            m_new = np.maximum(m, s.max(axis=1))
            alpha = np.exp(m - m_new, dtype=np.float32)
            p = np.exp(s - m_new[:, None], dtype=np.float32)
            l = alpha * l + p.sum(axis=1, dtype=np.float32)
            acc = alpha[:, None] * acc + np.einsum("hb,bhd->hd", p, v, dtype=np.float32)
            m = m_new
        out[tok] = round_to(acc / l[:, None], dtype)
    return out


# ------------------------------------------------------------------ integer metadata
def token_map(context_lens, query_lens):
    """(seq_idx, q_pos, cu_query_lens) per packed token (attention_triton.py:129-150)."""
    context_lens = np.asarray(context_lens, dtype=np.int64)
    query_lens = np.asarray(query_lens, dtype=np.int64)
    batch = query_lens.shape[0]
    cu = np.zeros(batch + 1, dtype=np.int64)
    cu[1:] = np.cumsum(query_lens)
    seq_idx = np.repeat(np.arange(batch, dtype=np.int64), query_lens)
    tok = np.arange(int(cu[-1]), dtype=np.int64)
    q_pos = context_lens[seq_idx] - query_lens[seq_idx] + (tok - cu[seq_idx])
    return seq_idx, q_pos, cu


def slots(blocks, block_size: int, num_tokens: int) -> np.ndarray:
    """Flat slot ``block*block_size + offset`` of positions 0..num_tokens-1
    (block_table.py:143-159); IndexError past capacity like the reference."""
    blocks = np.asarray(blocks, dtype=np.int64)
    if num_tokens > blocks.shape[0] * block_size:
        raise IndexError(f"{num_tokens} tokens requested, capacity is {blocks.shape[0] * block_size}")
    p = np.arange(num_tokens, dtype=np.int64)
    return blocks[p // block_size] * block_size + (p % block_size)


def pack_step(seqs, block_size: int):
    """Per-step metadata of the paged executor (paged_executor.py:211-263).

    ``seqs`` is a list of ``(blocks, num_cached, num_new)``.  Returns a dict with the
    reference's tensors as int64 arrays: ``write_slots`` (new tokens only),
    ``block_tables`` (0-padded to the widest row), ``context_lens`` (after the pass),
    ``query_lens``, ``ends`` (cumsum of query_lens) and ``position_ids``.
    """
    write_slots, positions, q_lens, c_lens, tables = [], [], [], [], []
    for blocks, num_cached, num_new in seqs:
        after = num_cached + num_new
        if len(blocks) * block_size < after:
            raise ValueError(f"block table holds {len(blocks) * block_size} slots, pass needs {after}")
        positions.extend(range(num_cached, after))
        write_slots.extend(slots(blocks, block_size, after)[num_cached:].tolist())
        q_lens.append(num_new)
        c_lens.append(after)
        tables.append(list(blocks))
    width = max(len(t) for t in tables)
    padded = [t + [0] * (width - len(t)) for t in tables]
    return {
        "write_slots": np.asarray(write_slots, dtype=np.int64),
        "block_tables": np.asarray(padded, dtype=np.int64),
        "context_lens": np.asarray(c_lens, dtype=np.int64),
        "query_lens": np.asarray(q_lens, dtype=np.int64),
        "ends": np.cumsum(np.asarray(q_lens, dtype=np.int64)),
        "position_ids": np.asarray(positions, dtype=np.int64),
    }


def kv_append(pool: np.ndarray, write_slots, new: np.ndarray) -> np.ndarray:
    """Scatter new K (or V) rows into the pool at flat slots (paged_executor.py:116-125).

    pool [NB, BS, Hkv, D] and new [T, Hkv, D] of any numpy dtype (the copy is bitwise);
    returns the updated pool (a copy, the input is not modified).
    """
    out = np.array(pool, copy=True)
    flat = out.reshape(-1, *out.shape[2:])
    flat[np.asarray(write_slots, dtype=np.int64)] = new
    return out


def swap_out(k_layers: np.ndarray, v_layers: np.ndarray, blocks) -> tuple[np.ndarray, np.ndarray]:
    """Per-layer ``index_select(0, blocks)`` of K and V (kv_pool.py:142-166).

    k_layers / v_layers [L, NB, BS, Hkv, D] (any dtype, bitwise); returns the host copies
    [L, n, BS, Hkv, D] for K and V.
    """
    idx = np.asarray(blocks, dtype=np.int64)
    return np.array(k_layers[:, idx], copy=True), np.array(v_layers[:, idx], copy=True)


def swap_in(k_layers: np.ndarray, v_layers: np.ndarray, host_k: np.ndarray, host_v: np.ndarray,
            blocks) -> tuple[np.ndarray, np.ndarray]:
    """Per-layer ``index_copy_(0, blocks, host)`` (kv_pool.py:168-182), with its length
    check; returns the updated pools (copies)."""
    if len(blocks) != host_k.shape[1]:
        raise ValueError(f"swap_in: {host_k.shape[1]} host blocks into {len(blocks)} device blocks")
    k, v = np.array(k_layers, copy=True), np.array(v_layers, copy=True)
    idx = np.asarray(blocks, dtype=np.int64)
    k[:, idx] = host_k
    v[:, idx] = host_v
    return k, v


def copy_block(k_layers: np.ndarray, v_layers: np.ndarray, pairs) -> tuple[np.ndarray, np.ndarray]:
    """``layer[dst].copy_(layer[src])`` for every layer, K then V, pair by pair in order
    (paged_executor.py:265-270); returns the updated pools (copies)."""
    k, v = np.array(k_layers, copy=True), np.array(v_layers, copy=True)
    for src, dst in pairs:
        k[:, dst] = k[:, src]
        v[:, dst] = v[:, src]
    return k, v
