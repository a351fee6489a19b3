"""Seeded ragged batches for the parity tests (the layout of the reference tests'
`_build`: N(0,1) pools, blocks from a seeded permutation, 0-padded block tables)."""

from __future__ import annotations

import numpy as np
import torch


def lognormal_contexts(batch: int, median: float, sigma: float, lo: int, hi: int, seed: int = 0) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return np.clip(np.exp(rng.normal(np.log(median), sigma, size=batch)), lo, hi).astype(np.int64)


def ragged_batch(lengths, *, bs: int, d: int, heads: int, kv_heads: int, dtype=torch.float32, seed: int = 0,
                 spare_blocks: int = 3):
    """lengths: list of (context_len, query_len).  Returns CPU tensors
    (query, k_pool, v_pool, block_tables, context_lens, query_lens)."""
    g = torch.Generator().manual_seed(seed)
    need = [-(-c // bs) for c, _ in lengths]
    nb = sum(need) + spare_blocks
    k_pool = torch.randn(nb, bs, kv_heads, d, generator=g).to(dtype)
    v_pool = torch.randn(nb, bs, kv_heads, d, generator=g).to(dtype)
    perm = torch.randperm(nb, generator=g)
    width = max(need) if need else 1
    tables = torch.zeros(len(lengths), width, dtype=torch.long)
    off = 0
    for i, n in enumerate(need):
        tables[i, :n] = perm[off:off + n]
        off += n
    t = sum(q for _, q in lengths)
    query = torch.randn(t, heads, d, generator=g).to(dtype)
    return (query, k_pool, v_pool, tables, torch.tensor([c for c, _ in lengths], dtype=torch.long),
            torch.tensor([q for _, q in lengths], dtype=torch.long))


def subset_rows(lengths, picks):
    """Token rows of the picked sequences in the packed order."""
    starts = np.concatenate([[0], np.cumsum([q for _, q in lengths])])
    return np.concatenate([np.arange(starts[i], starts[i + 1]) for i in picks])


def ragged_batch_device(lengths, *, bs: int, d: int, heads: int, kv_heads: int, dtype, device, seed: int = 0):
    """Like `ragged_batch`, with the (large) pools and queries drawn on the device."""
    g = torch.Generator(device=device).manual_seed(seed)
    need = [-(-c // bs) for c, _ in lengths]
    nb = sum(need) + 3
    k_pool = torch.randn(nb, bs, kv_heads, d, generator=g, device=device, dtype=torch.float32).to(dtype)
    v_pool = torch.randn(nb, bs, kv_heads, d, generator=g, device=device, dtype=torch.float32).to(dtype)
    perm = torch.randperm(nb, generator=torch.Generator().manual_seed(seed))
    tables = torch.zeros(len(lengths), max(need), dtype=torch.long)
    off = 0
    for i, n in enumerate(need):
        tables[i, :n] = perm[off:off + n]
        off += n
    t = sum(q for _, q in lengths)
    query = torch.randn(t, heads, d, generator=g, device=device, dtype=torch.float32).to(dtype)
    return (query, k_pool, v_pool, tables, torch.tensor([c for c, _ in lengths], dtype=torch.long),
            torch.tensor([q for _, q in lengths], dtype=torch.long))


def compact_subbatch(query, k_pool, v_pool, tables, ctx, ql, lengths, picks, bs: int):
    """The picked sequences with only their own blocks, as float32 numpy arrays for the
    oracle: (query, k_pool, v_pool, block_tables, context_lens, query_lens)."""
    rows = subset_rows(lengths, picks)
    need = [-(-int(ctx[i]) // bs) for i in picks]
    ids = torch.cat([tables[i, :n] for i, n in zip(picks, need)])
    sub_tables = torch.zeros(len(picks), max(need), dtype=torch.long)
    off = 0
    for j, n in enumerate(need):
        sub_tables[j, :n] = torch.arange(off, off + n)
        off += n
    dev_ids = ids.to(k_pool.device)
    return (query[torch.as_tensor(rows, device=query.device)].float().cpu().numpy(),
            k_pool[dev_ids].float().cpu().numpy(), v_pool[dev_ids].float().cpu().numpy(),
            sub_tables.numpy(), ctx[list(picks)].numpy(), ql[list(picks)].numpy())
