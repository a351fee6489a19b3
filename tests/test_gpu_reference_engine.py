"""The reference's own scheduler policy driving ``ATTENTION=cuda`` on the GPU.

Everything but attention is the unmodified reference from ``baseline/_ref`` (its
``Scheduler``, ``BlockAllocator``, ``BlockTable``, ``PrefixCache``, ``Sequence``,
``PagedKVPool`` and ``PagedExecutor``), with the INTEGRATION.md dispatcher patch applied
to a temporary copy.  Three arms serve the same requests on the same random-init model:

* ``gather``   — the reference's ``PagedExecutor`` with ``ATTENTION=gather`` (its own path);
* ``dispatch`` — the same ``PagedExecutor`` with ``ATTENTION=cuda``: only the dispatcher
  changed, so attention runs in this library's kernels;
* ``executor`` — ``CudaPagedExecutor`` (one-copy step metadata, fused KV append, block
  moves in one launch) in place of ``PagedExecutor``;
* ``executor_graphs`` (config 1 mix and recompute preemption) — the same executor with
  its all-decode passes replayed from captured CUDA graphs of the whole model forward.

The north star's parity target is greedy token ids identical to the gather path for fp32
GPT-2, which every case asserts for all three arms.  ``PagedEngine`` itself cannot be
built here (it loads pretrained weights and a tokenizer by name, and neither exists
offline), so the tests assemble exactly what its constructor assembles
(engine/paged.py:52-82) around a random-init GPT-2 and drive ``Scheduler.step()`` the way
its step loop does.

Cases: BASELINE config 1's request mix at concurrency 32 and 4; a shared system prefix
with ``PREFIX_CACHING=1`` (refcounted shared blocks from the reference's prefix cache); a
partially filled block shared between two sequences so that ``BlockTable.ensure_private``
copies it before the write; and a pool small enough that recompute, then swap,
preemption fire (scheduler.py:267-293).
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

import _reference

pytestmark = pytest.mark.gpu
DEV = "cuda"
VOCAB = 50257


@pytest.fixture(scope="module")
def ref(tmp_path_factory, pkg):
    _reference.require()
    dest = _reference.make_patched_copy(tmp_path_factory.mktemp("ref_engine"))
    mod = _reference.import_patched(dest)
    names = ["config", "core.block_allocator", "core.block_table", "core.kv_pool", "core.paged_executor",
             "core.prefix_cache", "core.scheduler", "core.sequence"]
    return {n.rsplit(".", 1)[-1]: importlib.import_module(f"{mod.__name__}.{n}") for n in names}


@pytest.fixture(scope="module")
def gpt2():
    from transformers import GPT2Config, GPT2LMHeadModel

    torch.manual_seed(0)
    return GPT2LMHeadModel(GPT2Config()).to(DEV).eval()


@pytest.fixture(scope="module")
def cuda_executor(pkg):
    return importlib.import_module(f"{pkg.__name__}.executor").CudaPagedExecutor


@pytest.fixture
def config(ref, monkeypatch):
    C = ref["config"].CONFIG
    monkeypatch.setattr(C, "device", DEV)
    monkeypatch.setattr(C, "block_size", 16)
    monkeypatch.setattr(C, "preemption", "recompute")
    monkeypatch.setattr(C, "max_queue_depth", 1024)
    return C


def config1_requests(n: int, seed: int = 0, max_out: int = 512):
    """BASELINE config 1's mix: prompts of uniform random ids, lengths uniform in
    16..256; output lengths lognormal with median 30 (sigma 0.9), clipped to 1..max_out."""
    rng = np.random.default_rng(seed)
    reqs = []
    for _ in range(n):
        prompt = rng.integers(0, VOCAB, size=int(rng.integers(16, 257))).tolist()
        out = int(np.clip(np.exp(rng.normal(np.log(30.0), 0.9)), 1, max_out))
        reqs.append((prompt, out))
    return reqs


def _make_pool(ref, arm, model, num_blocks, pkg):
    if arm == "executor_kvpool":
        return pkg.KVPool.from_model(model, num_blocks=num_blocks, block_size=16)
    return ref["kv_pool"].PagedKVPool.from_model(model, num_blocks=num_blocks, block_size=16, device=DEV)


def _make_executor(ref, arm, model, pool, config, cuda_executor, monkeypatch):
    if arm == "gather":
        monkeypatch.setattr(config, "attention", "gather")
        return ref["paged_executor"].PagedExecutor(model, None, pool)
    if arm == "dispatch":
        monkeypatch.setattr(config, "attention", "cuda")
        return ref["paged_executor"].PagedExecutor(model, None, pool)
    monkeypatch.setattr(config, "attention", "cuda")
    return cuda_executor(model, None, pool, decode_graphs=arm == "executor_graphs")


def serve(ref, arm, model, requests, *, num_blocks, max_running, config, cuda_executor, monkeypatch, pkg,
          prefix_caching=False, max_steps=20000):
    """Drive the reference Scheduler to completion; returns ({seq_id: tokens}, stats)."""
    monkeypatch.setattr(config, "max_running", max_running)
    monkeypatch.setattr(config, "prefix_caching", prefix_caching)
    pool = _make_pool(ref, arm, model, num_blocks, pkg)
    executor = _make_executor(ref, arm, model, pool, config, cuda_executor, monkeypatch)
    alloc = ref["block_allocator"].BlockAllocator(num_blocks)
    cache = ref["prefix_cache"].PrefixCache(alloc, 16) if prefix_caching else None
    sched = ref["scheduler"].Scheduler(executor, -1, allocator=alloc, pool=pool, prefix_cache=cache)
    seqs = [ref["sequence"].Sequence(seq_id=f"r{i}", prompt_token_ids=list(p), max_tokens=m)
            for i, (p, m) in enumerate(requests)]
    for s in seqs:
        sched.add(s)
    steps = 0
    while sched.has_work:
        sched.step()
        steps += 1
        assert steps < max_steps, "scheduler did not drain"
    torch.cuda.synchronize()
    stats = dict(sched.stats(), steps=steps)
    assert stats["free_blocks"] == num_blocks, stats          # the free list returns to full
    del pool, executor
    torch.cuda.empty_cache()
    return {s.seq_id: list(s.output_token_ids) for s in seqs}, stats


ARMS = ("gather", "dispatch", "executor")


def _all_arms(arms, **kw):
    return {arm: serve(arm=arm, **kw) for arm in arms}


def _assert_identical(results, requests):
    base, _ = results["gather"]
    assert len(base) == len(requests)
    for (p, m), (sid, toks) in zip(requests, sorted(base.items(), key=lambda kv: int(kv[0][1:]))):
        assert len(toks) == m, (sid, len(toks), m)
    for arm, (toks, _) in results.items():
        bad = [sid for sid in base if toks[sid] != base[sid]]
        assert not bad, f"{arm}: {len(bad)} of {len(base)} sequences differ from the gather path, e.g. {bad[:3]}"


@pytest.mark.parametrize("concurrency,n", [(32, 200), (4, 40)])
def test_config1_mix_tokens_identical(ref, gpt2, config, cuda_executor, monkeypatch, pkg, concurrency, n):
    """BASELINE config 1 (GPT-2 fp32, 2048-block pool, greedy, EOS disabled) through the
    reference scheduler; 200 requests at concurrency 32 and the first 40 at
    concurrency 4."""
    reqs = config1_requests(n)
    res = _all_arms(ARMS + ("executor_graphs",), ref=ref, model=gpt2, requests=reqs, num_blocks=2048, max_running=concurrency,
                    config=config, cuda_executor=cuda_executor, monkeypatch=monkeypatch, pkg=pkg)
    _assert_identical(res, reqs)
    assert all(st["preemptions"] == 0 for _, st in res.values())
    assert pkg.read_device_error() == 0


def test_shared_prefix_blocks_tokens_identical(ref, gpt2, config, cuda_executor, monkeypatch, pkg):
    """Config 4's shape on GPT-2 fp32: every request starts with the same 128 random ids
    (8 full blocks) followed by a unique suffix; with PREFIX_CACHING=1 the reference's
    prefix cache hands later requests the shared, refcounted blocks, which the kernels
    read in place."""
    rng = np.random.default_rng(4)
    system = rng.integers(0, VOCAB, size=128).tolist()
    reqs = [(system + rng.integers(0, VOCAB, size=int(rng.integers(32, 257))).tolist(),
             int(np.clip(np.exp(rng.normal(np.log(64.0), 0.9)), 1, 160))) for _ in range(48)]
    res = _all_arms(ARMS, ref=ref, model=gpt2, requests=reqs, num_blocks=2048, max_running=16,
                    config=config, cuda_executor=cuda_executor, monkeypatch=monkeypatch, pkg=pkg,
                    prefix_caching=True)
    _assert_identical(res, reqs)
    for arm, (_, st) in res.items():
        assert st["prefix_hits"] >= 8 * 32, (arm, st)         # most requests adopted the 8 shared blocks


@pytest.mark.parametrize("preemption", ["recompute", "swap"])
def test_preemption_tokens_identical(ref, gpt2, config, cuda_executor, monkeypatch, pkg, preemption):
    """A 40-block pool under 10 requests of up to ~20 blocks each: the reference's
    ``_grow`` preempts the most recently admitted sequence, which is re-prefilled over
    prompt + generated tokens (recompute) or copied to host memory and back (swap).  In
    the swap case the CUDA executor's arm uses this library's pool, whose swaps are one
    gather / scatter launch plus one copy."""
    monkeypatch.setattr(config, "preemption", preemption)
    rng = np.random.default_rng(7)
    reqs = [(rng.integers(0, VOCAB, size=int(rng.integers(60, 161))).tolist(), int(rng.integers(40, 121)))
            for _ in range(10)]
    arms = ARMS + (("executor_kvpool",) if preemption == "swap" else ("executor_graphs",))
    res = _all_arms(arms, ref=ref, model=gpt2, requests=reqs, num_blocks=40, max_running=8,
                    config=config, cuda_executor=cuda_executor, monkeypatch=monkeypatch, pkg=pkg)
    _assert_identical(res, reqs)
    for arm, (_, st) in res.items():
        assert st["preemptions"] > 0, (arm, st)
        if preemption == "swap":
            assert st["swaps"] > 0, (arm, st)


def test_partial_block_share_copies_on_write(ref, gpt2, config, cuda_executor, monkeypatch, pkg):
    """Two sequences share a partially filled block (refcount 2 in the reference's
    allocator).  Each executor's ``_pack`` calls ``BlockTable.ensure_private`` before
    writing into it, which allocates a fresh block and has the executor copy the shared
    block's K/V (every layer) before the write; both sequences then decode.  Tokens
    must match the gather arm and the copy must have happened in every arm."""
    rng = np.random.default_rng(11)
    head = rng.integers(0, VOCAB, size=40).tolist()             # 2 full blocks + 8 tokens
    tail = rng.integers(0, VOCAB, size=20).tolist()
    Seq, Table, Alloc = ref["sequence"].Sequence, ref["block_table"].BlockTable, ref["block_allocator"].BlockAllocator
    results = {}
    for arm in ARMS:
        pool = _make_pool(ref, arm, gpt2, 64, pkg)
        ex = _make_executor(ref, arm, gpt2, pool, config, cuda_executor, monkeypatch)
        alloc = Alloc(64)
        a = Seq(seq_id="a", prompt_token_ids=list(head), max_tokens=32)
        a.block_table = Table(alloc, 16)
        a.block_table.ensure_capacity(40)
        a.append_token(ex.execute([a])[0], -1)
        # b adopts all three of a's blocks, the third holding 8 of 16 slots.
        b = Seq(seq_id="b", prompt_token_ids=head + tail, max_tokens=32)
        b.block_table = Table(alloc, 16)
        b.block_table.adopt(list(a.block_table.blocks), [b"h0", b"h1", b"h2"])
        b.num_cached = 40
        shared = a.block_table.blocks[2]
        assert alloc.refcount(shared) == 2
        b.block_table.ensure_capacity(60)
        b.append_token(ex.execute([b])[0], -1)                  # writes slots 40..59: copy-on-write of block 2
        assert b.block_table.blocks[2] != shared and alloc.refcount(shared) == 1
        for _ in range(12):                                     # both decode; a writes into its own block 2
            for s in (a, b):
                s.block_table.ensure_capacity(s.cached_after_next_pass)
            for s, t in zip((a, b), ex.execute([a, b])):
                s.append_token(t, -1)
        results[arm] = (a.output_token_ids, b.output_token_ids)
        del pool, ex
    assert results["dispatch"] == results["gather"]
    assert results["executor"] == results["gather"]
    assert pkg.read_device_error() == 0
