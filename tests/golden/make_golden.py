"""Generate the golden vectors under tests/golden/ by running the reference itself.

Usage (development container only; the reference source tree is not on GPU boxes):

    python tests/golden/make_golden.py --reference <path to llm-inference-server checkout>

What it records, all from the reference's own code on CPU:

* ``attn_<case>.npz``: inputs and the output of ``paged_attention_gather``
  (inference_server/core/attention.py:92-187) for the shapes the reference's test-suite
  uses (tests/test_paged_attention.py, tests/test_paged_attention_triton.py:74-84,
  :118-128, :172-192) plus the serving shapes this project targets (GPT-2 12/12/64 and
  Llama-3 32/8/128, 16/2/128 at block size 16) in fp32, fp16 and bf16.
* ``mirror.npz``: the output of ``paged_attention_reference`` (attention_triton.py:309-384,
  the PyTorch mirror of the Triton kernel's online softmax) on the inputs of a subset of
  the ``attn_<case>`` files (key: the case name).
* ``token_map.npz``: ``_token_map`` (attention_triton.py:129-150), including the
  known-answer case of tests/test_paged_attention_triton.py:140-147.
* ``pack.npz``: ``PagedExecutor._pack`` (paged_executor.py:211-263) over real
  reference ``Sequence``/``BlockTable``/``BlockAllocator`` objects: write slots, block
  tables, context/query lengths, position ids.
* ``kv_append_<dtype>.npz``: pool contents after ``_PagedCache.update``
  (paged_executor.py:116-125).
* ``blocks_<dtype>.npz``: block moves of a 3-layer pool: ``PagedKVPool.swap_out`` /
  ``swap_in`` (kv_pool.py:142-182) and ``PagedExecutor._copy_block``
  (paged_executor.py:265-270).
* ``gpt2_greedy_cpu.npz``: greedy tokens of the reference's own ``PagedExecutor`` with
  the gather path (paged_executor.py:162-295) on CPU, driving a random-init GPT-2 124M
  (``GPT2LMHeadModel(GPT2Config())`` after ``torch.manual_seed(0)``, fp32) over three
  prompts of random token ids for six steps (one prefill, five decodes).

Half-precision tensors are stored as their raw 16-bit patterns (uint16 arrays; the
``dtype`` entry says which format), float32 tensors as float32, so every stored value
is exact.  Inputs are drawn with a
seeded ``torch.Generator`` laid out the way the reference tests' ``_build`` does it:
N(0,1) pools, blocks taken from a seeded permutation (unsorted, non-contiguous),
block tables 0-padded.
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# name -> (lengths, dict(bs, d, heads, kv_heads, num_blocks, dtype, seed))
CASES: dict[str, tuple[list[tuple[int, int]], dict]] = {}


def _case(name, lengths, bs=4, d=8, heads=3, kv_heads=3, num_blocks=64, dtype="f32", seed=0):
    CASES[name] = (lengths, dict(bs=bs, d=d, heads=heads, kv_heads=kv_heads,
                                 num_blocks=num_blocks, dtype=dtype, seed=seed))


# The reference test-suite's shapes (block size 4, 3 heads, head_dim 8).
_case("prefill_on_boundary", [(4, 4), (8, 8), (16, 16)])
_case("prefill_spilling", [(5, 5), (9, 9), (17, 17)])
_case("prefill_partial", [(1, 1), (3, 3), (15, 15)])
_case("prefill_ragged", [(7, 7), (4, 4), (13, 13), (1, 1), (16, 16)])
_case("decode_singles", [(1, 1), (4, 1), (5, 1), (8, 1), (9, 1), (16, 1), (17, 1)])
_case("decode_ragged", [(9, 1), (4, 1), (17, 1), (1, 1), (12, 1), (5, 1)])
_case("mixed", [(6, 1), (10, 10), (4, 1), (9, 5), (16, 16), (13, 1)])
_case("partial_query", [(11, 3), (8, 4), (20, 7)])
for _s in range(3):
    _case(f"padding_hits_block0_s{_s}", [(3, 3), (19, 1), (4, 1)], seed=_s)
_case("gqa_kv1", [(9, 9), (5, 1), (12, 3)], kv_heads=1)
_case("non_pow2_bs6_d12", [(13, 13), (7, 1), (18, 4)], bs=6, d=12)
_case("mixed_f16", [(6, 1), (10, 10), (4, 1), (9, 5), (16, 16), (13, 1)], dtype="f16")
_case("mixed_bf16", [(6, 1), (10, 10), (4, 1), (9, 5), (16, 16), (13, 1)], dtype="bf16")
# Production block size 16.
_case("prod_bs16_d64", [(33, 1), (16, 16), (40, 9)], bs=16, d=64, num_blocks=16)
_case("prod_long_bs16_d64", [(300, 1), (16, 16), (129, 1), (64, 40)], bs=16, d=64, num_blocks=40)
_case("gpt2_decode_f32", [(60, 1), (17, 1), (1, 1), (20, 1)], bs=16, d=64,
      heads=12, kv_heads=12, num_blocks=10)
_case("gpt2_decode_bf16", [(60, 1), (17, 1), (1, 1), (20, 1)], bs=16, d=64,
      heads=12, kv_heads=12, num_blocks=10, dtype="bf16")
_case("llama8b_mixed_bf16", [(40, 1), (16, 1), (33, 33), (20, 7)], bs=16, d=128,
      heads=32, kv_heads=8, num_blocks=12, dtype="bf16")
_case("llama70b_group8_bf16", [(50, 1), (31, 31), (17, 1)], bs=16, d=128,
      heads=16, kv_heads=2, num_blocks=12, dtype="bf16")
_case("llama8b_decode_f16", [(40, 1), (16, 1), (70, 1)], bs=16, d=128,
      heads=32, kv_heads=8, num_blocks=10, dtype="f16")

TORCH_DTYPE = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


# Cases whose inputs also go through the reference's online-softmax mirror.
MIRROR_CASES = ["prefill_ragged", "decode_ragged", "mixed", "partial_query", "padding_hits_block0_s1", "gqa_kv1",
                "non_pow2_bs6_d12", "mixed_bf16", "prod_long_bs16_d64", "llama70b_group8_bf16"]


def build(lengths, bs, d, heads, kv_heads, num_blocks, dtype, seed):
    """Seeded inputs in the layout of the reference tests' `_build`."""
    g = torch.Generator().manual_seed(seed)
    k_pool = torch.randn(num_blocks, bs, kv_heads, d, generator=g)
    v_pool = torch.randn(num_blocks, bs, kv_heads, d, generator=g)
    perm = torch.randperm(num_blocks, generator=g).tolist()
    queries, tables = [], []
    for ctx, q_len in lengths:
        nblocks = -(-ctx // bs)
        blocks, perm = perm[:nblocks], perm[nblocks:]
        queries.append(torch.randn(q_len, heads, d, generator=g))
        tables.append(blocks)
    width = max(len(t) for t in tables)
    block_tables = torch.tensor([t + [0] * (width - len(t)) for t in tables], dtype=torch.long)
    td = TORCH_DTYPE[dtype]
    return (torch.cat(queries).to(td), k_pool.to(td), v_pool.to(td), block_tables,
            torch.tensor([c for c, _ in lengths], dtype=torch.long),
            torch.tensor([q for _, q in lengths], dtype=torch.long))


def _store(t: torch.Tensor, dtype: str) -> np.ndarray:
    if dtype == "f32":
        return t.float().numpy()
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the llm-inference-server checkout")
    ap.add_argument("--only", nargs="*", default=None,
                    help="regenerate only these outputs: attn mirror token_map pack kv_append blocks gpt2_greedy")
    args = ap.parse_args()
    want = set(args.only) if args.only else {"attn", "mirror", "token_map", "pack", "kv_append", "blocks",
                                             "gpt2_greedy"}
    os.environ.setdefault("DEVICE", "cpu")
    sys.path.insert(0, str(Path(args.reference).resolve()))

    from inference_server.core.attention import paged_attention_gather
    from inference_server.core.attention_triton import _token_map
    from inference_server.core.block_allocator import BlockAllocator
    from inference_server.core.block_table import BlockTable
    from inference_server.core.kv_pool import ModelDims, PagedKVPool
    from inference_server.core.paged_executor import PagedExecutor, _PagedCache, _StepContext
    from inference_server.core.sequence import Sequence

    for name, (lengths, kw) in (CASES.items() if "attn" in want else ()):
        q, kp, vp, bt, cl, ql = build(lengths, **kw)
        scale = kw["d"] ** -0.5
        out = paged_attention_gather(q, kp, vp, bt, cl, ql, scale)
        dt = kw["dtype"]
        np.savez_compressed(
            HERE / f"attn_{name}.npz",
            query=_store(q, dt), k_pool=_store(kp, dt), v_pool=_store(vp, dt),
            out=_store(out, dt), block_tables=bt.numpy(), context_lens=cl.numpy(),
            query_lens=ql.numpy(), scale=np.float64(scale), dtype=np.bytes_(dt),
        )

    if "mirror" in want:
        from inference_server.core.attention_triton import paged_attention_reference

        mirror = {}
        for name in MIRROR_CASES:
            lengths, kw = CASES[name]
            q, kp, vp, bt, cl, ql = build(lengths, **kw)
            mirror[name] = _store(paged_attention_reference(q, kp, vp, bt, cl, ql, kw["d"] ** -0.5), kw["dtype"])
        np.savez_compressed(HERE / "mirror.npz", **mirror)

    if "gpt2_greedy" in want:
        _gpt2_greedy(PagedExecutor, PagedKVPool, ModelDims, BlockAllocator, BlockTable, Sequence)
    if "blocks" in want:
        _blocks(PagedExecutor, PagedKVPool, ModelDims)
    if not want & {"token_map", "pack", "kv_append"}:
        return

    # _token_map: the reference test's known answer plus a random ragged batch.
    rng = np.random.default_rng(7)
    c2 = rng.integers(1, 300, size=17)
    q2 = np.minimum(c2, rng.integers(1, 40, size=17))
    tm = {}
    for tag, (c, qq) in {"known": ([6, 10, 4], [1, 3, 4]), "random": (c2.tolist(), q2.tolist())}.items():
        s, p, cu = _token_map(torch.tensor(c), torch.tensor(qq))
        tm.update({f"{tag}_context_lens": np.asarray(c), f"{tag}_query_lens": np.asarray(qq),
                   f"{tag}_seq_idx": s.numpy(), f"{tag}_q_pos": p.numpy(), f"{tag}_cu": cu.numpy()})
    np.savez_compressed(HERE / "token_map.npz", **tm)

    # _pack over real reference sequences: two prefills (one after a prefix hit), decodes.
    bs = 16
    alloc = BlockAllocator(64)
    pool = PagedKVPool(ModelDims(1, 2, 8, torch.float32), num_blocks=64, block_size=bs, device="cpu")
    seqs = []
    specs = [("p0", 37, 0), ("p1", 50, 32), ("d0", 20, 20), ("d1", 16, 16), ("d2", 1, 1), ("d3", 90, 90)]
    for sid, prompt_len, cached in specs:
        s = Sequence(seq_id=sid, prompt_token_ids=list(range(1, prompt_len + 1)), max_tokens=8)
        s.block_table = BlockTable(alloc, bs)
        if cached >= prompt_len:            # a decode: one generated token not yet cached
            s.output_token_ids.append(99)
        s.num_cached = cached
        s.block_table.ensure_capacity(s.num_cached + len(s.next_input_ids))
        seqs.append(s)
    ex = PagedExecutor(model=None, tokenizer=None, pool=pool)
    input_ids, position_ids, ctx, ends = ex._pack(seqs)
    np.savez_compressed(
        HERE / "pack.npz",
        blocks=np.array([np.pad(s.block_table.blocks, (0, 16 - len(s.block_table.blocks)),
                                constant_values=-1) for s in seqs]),
        num_blocks_per_seq=np.array([len(s.block_table.blocks) for s in seqs]),
        num_cached=np.array([s.num_cached for s in seqs]),
        num_new=np.array([len(s.next_input_ids) for s in seqs]),
        write_slots=ctx.write_slots.numpy(), block_tables=ctx.block_tables.numpy(),
        context_lens=ctx.context_lens.numpy(), query_lens=ctx.query_lens.numpy(),
        ends=ends.numpy(), position_ids=position_ids[0].numpy(), input_ids=input_ids[0].numpy(),
        block_size=np.int64(bs),
    )

    # _PagedCache.update: the pool after the scatter, fp32 and bf16.
    for dt in ("f32", "bf16"):
        td = TORCH_DTYPE[dt]
        g = torch.Generator().manual_seed(11)
        heads, dim = 4, 32
        pool = PagedKVPool(ModelDims(2, heads, dim, td), num_blocks=8, block_size=bs, device="cpu")
        for layer in range(2):
            pool.k[layer].copy_(torch.randn(pool.k[layer].shape, generator=g).to(td))
            pool.v[layer].copy_(torch.randn(pool.v[layer].shape, generator=g).to(td))
        k_before = pool.k[1].clone()
        v_before = pool.v[1].clone()
        slots_ = torch.tensor([5, 6, 7, 40, 41, 127, 0, 64, 65, 66, 99], dtype=torch.long)
        t = slots_.numel()
        key = torch.randn(1, heads, t, dim, generator=g).to(td)
        val = torch.randn(1, heads, t, dim, generator=g).to(td)
        sctx = _StepContext(write_slots=slots_, block_tables=torch.zeros(1, 1, dtype=torch.long),
                            context_lens=torch.ones(1, dtype=torch.long),
                            query_lens=torch.ones(1, dtype=torch.long), pool=pool)
        _PagedCache(sctx).update(key, val, 1)
        np.savez_compressed(
            HERE / f"kv_append_{dt}.npz",
            k_before=_store(k_before, dt), v_before=_store(v_before, dt),
            key=_store(key, dt), value=_store(val, dt), write_slots=slots_.numpy(),
            k_after=_store(pool.k[1], dt), v_after=_store(pool.v[1], dt), dtype=np.bytes_(dt),
        )
    print(f"wrote {len(CASES)} attention cases + token_map, pack, kv_append to {HERE}")


def _blocks(PagedExecutor, PagedKVPool, ModelDims) -> None:
    """Swap-out, swap-in and copy-on-write moves of the reference pool (CPU)."""
    for dt in ("f32", "bf16"):
        td = TORCH_DTYPE[dt]
        g = torch.Generator().manual_seed(23)
        pool = PagedKVPool(ModelDims(3, 2, 8, td), num_blocks=16, block_size=4, device="cpu")
        for layer in range(3):
            pool.k[layer].copy_(torch.randn(pool.k[layer].shape, generator=g).to(td))
            pool.v[layer].copy_(torch.randn(pool.v[layer].shape, generator=g).to(td))
        k0 = torch.stack(pool.k).clone()
        v0 = torch.stack(pool.v).clone()
        out_blocks, in_blocks = [5, 2, 11, 7], [0, 9, 3, 14]
        host = pool.swap_out(out_blocks)
        pool.swap_in(host, in_blocks)
        k1, v1 = torch.stack(pool.k).clone(), torch.stack(pool.v).clone()
        ex = PagedExecutor(model=None, tokenizer=None, pool=pool)
        pairs = [(4, 12), (1, 6), (9, 15)]
        for src, dst in pairs:
            ex._copy_block(src, dst)
        np.savez_compressed(
            HERE / f"blocks_{dt}.npz",
            k_before=_store(k0, dt), v_before=_store(v0, dt),
            swap_out_blocks=np.array(out_blocks), host_k=_store(torch.stack(host.k), dt),
            host_v=_store(torch.stack(host.v), dt), swap_in_blocks=np.array(in_blocks),
            k_after_swap_in=_store(k1, dt), v_after_swap_in=_store(v1, dt),
            copy_pairs=np.array(pairs), k_after_copy=_store(torch.stack(pool.k), dt),
            v_after_copy=_store(torch.stack(pool.v), dt), dtype=np.bytes_(dt),
        )


def _gpt2_greedy(PagedExecutor, PagedKVPool, ModelDims, BlockAllocator, BlockTable, Sequence) -> None:
    """Greedy tokens of the reference executor on a seeded random-init GPT-2 (CPU)."""
    from transformers import GPT2Config, GPT2LMHeadModel

    torch.manual_seed(0)
    model = GPT2LMHeadModel(GPT2Config()).eval()
    rng = np.random.default_rng(0)
    prompts = [rng.integers(0, 50257, size=int(rng.integers(16, 257))).tolist() for _ in range(3)]
    nb, steps = 96, 6
    pool = PagedKVPool(ModelDims(12, 12, 64, torch.float32), num_blocks=nb, block_size=16, device="cpu")
    ex = PagedExecutor(model, None, pool)
    alloc = BlockAllocator(nb)
    seqs = [Sequence(seq_id=str(i), prompt_token_ids=p, max_tokens=100) for i, p in enumerate(prompts)]
    for s in seqs:
        s.block_table = BlockTable(alloc, 16)
    for _ in range(steps):
        for s in seqs:
            s.block_table.ensure_capacity(s.num_cached + len(s.next_input_ids))
        for s, tok in zip(seqs, ex.execute(seqs)):
            s.output_token_ids.append(tok)
    lens = np.array([len(p) for p in prompts])
    np.savez_compressed(HERE / "gpt2_greedy_cpu.npz", prompt_lens=lens, prompts=np.concatenate(prompts),
                        tokens=np.array([s.output_token_ids for s in seqs]), num_blocks=np.int64(nb),
                        steps=np.int64(steps))


if __name__ == "__main__":
    main()
