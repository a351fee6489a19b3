"""Host-side logic and the C ABI, no GPU: the library loads and exports every symbol the
public header declares; the C++ step planner reproduces the reference's integer
metadata and contract errors; the seam keeps the gather path's signature and fails
loudly off-GPU."""

from __future__ import annotations

import inspect
import subprocess

import numpy as np
import pytest
import torch

from _golden import load

REFERENCE_SIGNATURE = ["query", "k_pool", "v_pool", "block_tables", "context_lens", "query_lens", "scale"]


def test_library_exports_every_declared_symbol(pkg):
    lib = pkg._lib.lib()
    declared = pkg._lib.declared_symbols()
    assert len(declared) == 21
    for name in declared:
        assert hasattr(lib, name), name
    dyn = subprocess.run(["nm", "-D", "--defined-only", str(pkg._lib.LIB_PATH)], capture_output=True,
                         text=True).stdout
    for name in declared:
        assert f" T {name}" in dyn, f"{name} is not a dynamic export"


def test_launch_bits_match_the_header(pkg, monkeypatch):
    """Every PA_LAUNCH_* bit the header defines has the same value in the Python binding and
    a name in last_launches(), and the bits are distinct, so the tests that check which
    kernel served a call read the library's own report."""
    import re

    text = pkg._lib.HEADER.read_text()
    bits = {m.group(1): int(m.group(2)) for m in re.finditer(r"^#define (PA_LAUNCH_\w+) (\d+)", text, flags=re.M)}
    assert len(bits) >= 7
    assert len(set(bits.values())) == len(bits) and all(v & (v - 1) == 0 for v in bits.values())
    for name, value in bits.items():
        assert getattr(pkg._lib, name) == value, name

    class _Lib:  # last_launches() reads the mask from the library; feed it every bit at once
        @staticmethod
        def pa_last_launches():
            return sum(bits.values())

    monkeypatch.setattr(pkg._lib, "lib", lambda: _Lib())
    assert len(pkg._lib.last_launches()) == len(bits)


def test_every_entry_point_cites_its_reference_interface_or_has_none(pkg):
    """Each declaration's doc block (the nearest comment opening at column 0 before it)
    names the reference interface it replaces (inference_server/...:line) or says it has
    no counterpart in the reference."""
    import re

    text = pkg._lib.HEADER.read_text()
    blocks = [(m.start(), re.sub(r"\s*\n\s*\*?\s?", " ", m.group(0)))
              for m in re.finditer(r"^/\*.*?\*/", text, flags=re.S | re.M)]
    for name in pkg._lib.declared_symbols():
        decl = re.search(rf"^[\w ]+\**\s*\b{name}\(", text, flags=re.M)
        assert decl, name
        doc = [b for start, b in blocks if start < decl.start()][-1]
        assert re.search(r"inference_server/\S+:\s*\d+|counterpart", doc), (name, doc[:200])


def test_abi_version_and_struct_size(pkg):
    lib = pkg._lib.lib()
    assert lib.pa_abi_version() == pkg._lib.ABI_VERSION
    assert pkg._lib.ctypes.sizeof(pkg._lib.StepPlan) == 14 * 4 + 12 * 8


def _plan(pkg, ctx, ql, tables, num_blocks=64, bs=4, kv_heads=1, sm=148, tile=0):
    return pkg.StepMetadata.plan_host(ctx, ql, np.asarray(tables), num_tokens=int(np.sum(ql)),
                                      pool_num_blocks=num_blocks, block_size=bs, num_kv_heads=kv_heads, sm=sm,
                                      prefill_tile_tokens=tile)


@pytest.mark.parametrize("tag", ["known", "random"])
def test_planner_token_map_matches_reference(pkg, tag):
    """seq_idx / q_pos / cu_query_lens of attention_triton.py:129-150, from the golden."""
    z = load("token_map")
    ctx, ql = z[f"{tag}_context_lens"], z[f"{tag}_query_lens"]
    bs = 16
    width = int(max(-(-c // bs) for c in ctx))
    tables = np.zeros((len(ctx), width), dtype=np.int64)
    m = _plan(pkg, ctx, ql, tables, num_blocks=1, bs=bs)
    np.testing.assert_array_equal(m.seq_idx(False), z[f"{tag}_seq_idx"])
    np.testing.assert_array_equal(m.q_pos(False), z[f"{tag}_q_pos"])
    np.testing.assert_array_equal(m.cu_query_lens(False), z[f"{tag}_cu"])


def test_planner_pack_matches_reference(pkg):
    """write_slots, 0-padded block tables and lengths of the reference's _pack."""
    z = load("pack")
    m = _plan(pkg, z["context_lens"], z["query_lens"], z["block_tables"], num_blocks=64, bs=int(z["block_size"]))
    np.testing.assert_array_equal(m.slot_mapping(False), z["write_slots"])
    w = m.plan.table_width
    np.testing.assert_array_equal(m.block_tables(False), z["block_tables"][:, :w])
    assert m.plan.num_tokens == int(z["ends"][-1])


def test_planner_matches_oracle_on_random_batches(pkg, oracle):
    rng = np.random.default_rng(3)
    for _ in range(20):
        b = int(rng.integers(1, 40))
        bs = int(rng.choice([4, 6, 16]))
        ctx = rng.integers(1, 400, size=b)
        ql = np.where(rng.random(b) < 0.6, 1, np.minimum(ctx, rng.integers(1, 60, size=b)))
        need = -(-ctx // bs)
        nb = int(need.sum()) + 5
        perm = rng.permutation(nb)
        width = int(need.max()) + int(rng.integers(0, 3))
        tables = np.zeros((b, width), dtype=np.int64)
        off = 0
        for i in range(b):
            tables[i, :need[i]] = perm[off:off + need[i]]
            off += need[i]
        m = _plan(pkg, ctx, ql, tables, num_blocks=nb, bs=bs, kv_heads=int(rng.choice([1, 8])),
                  sm=int(rng.choice([8, 148])))
        seqs = [(tables[i, :need[i]].tolist(), int(ctx[i] - ql[i]), int(ql[i])) for i in range(b)]
        ref = oracle.pack_step(seqs, bs)
        np.testing.assert_array_equal(m.slot_mapping(False), ref["write_slots"])
        s, p, cu = oracle.token_map(ctx, ql)
        np.testing.assert_array_equal(m.seq_idx(False), s)
        np.testing.assert_array_equal(m.q_pos(False), p)
        # split-K work list covers every decode block exactly once
        items = m.decode_items()
        sb = m.plan.split_blocks
        covered = {}
        for seq, split, part, ns in items.tolist():
            assert ql[seq] == 1 and ns == -(-need[seq] // sb)
            for blk in range(split * sb, min((split + 1) * sb, need[seq])):
                covered[(seq, blk)] = covered.get((seq, blk), 0) + 1
        expect = {(i, k) for i in range(b) if ql[i] == 1 for k in range(need[i])}
        assert set(covered) == expect and all(v == 1 for v in covered.values())
        parts = sorted(int(x) for x in items[:, 2])
        assert parts == list(range(len(parts)))


def test_planner_contract_errors_use_reference_messages(pkg):
    t = np.zeros((2, 4), dtype=np.int64)
    with pytest.raises(ValueError, match="query_lens sum"):
        pkg.StepMetadata.plan_host([4, 2], [4, 2], t, num_tokens=5, pool_num_blocks=8, block_size=4,
                                   num_kv_heads=1)
    with pytest.raises(ValueError, match="query_len exceeds context_len"):
        _plan(pkg, [3, 2], [4, 2], t)
    with pytest.raises(ValueError, match="needs more blocks than its block_tables row holds"):
        _plan(pkg, [17, 2], [1, 2], t)
    with pytest.raises(ValueError, match="outside the pool"):
        _plan(pkg, [5, 2], [1, 2], np.array([[3, 9], [1, 0]]), num_blocks=8)
    with pytest.raises(ValueError, match="must be \\[batch\\]"):
        _plan(pkg, [5, 2, 1], [1, 2, 1], t)


def test_planner_empty_batch(pkg):
    m = _plan(pkg, np.zeros(0, np.int64), np.zeros(0, np.int64), np.zeros((0, 1), np.int64))
    assert m.plan.num_tokens == 0 and m.plan.num_decode_items == 0


def test_split_size_fills_the_gpu(pkg):
    """At the batch-256 / 4k-context decode shape the split keeps >= 4 CTAs per SM."""
    rng = np.random.default_rng(0)
    ctx = np.clip(np.exp(rng.normal(np.log(4096) - 0.405, 0.9, size=256)), 128, 16384).astype(np.int64)
    need = -(-ctx // 16)
    tables = np.zeros((256, int(need.max())), dtype=np.int64)
    m = _plan(pkg, ctx, np.ones(256, np.int64), tables, num_blocks=1, bs=16, kv_heads=8)
    assert m.plan.num_decode_items * 8 >= 148 * 4
    assert 1 <= m.plan.split_blocks <= 256


def test_padded_decode_plan_keeps_the_real_entries(pkg):
    """A CUDA-graph bucket's plan: the same tables, lengths, slots, work items and
    combines as the ordinary plan at the same split size, padded with null entries, and
    fixed counts and offsets however the contexts move inside the bucket."""
    rng = np.random.default_rng(4)
    ctx = rng.integers(1, 600, size=24).astype(np.int64)
    need = -(-ctx // 16)
    tables = np.zeros((24, 64), dtype=np.int64)
    for i, n in enumerate(need):
        tables[i, :n] = rng.permutation(4000)[:n]
    kw = dict(pool_num_blocks=4000, block_size=16, num_kv_heads=8)
    base = pkg.StepMetadata.plan_host(ctx, np.ones(24, np.int64), tables, num_tokens=24, sm=1, **kw)
    sb = int(base.plan.split_blocks)
    pad = pkg.StepMetadata.plan_decode_padded(ctx, tables, split_blocks=sb, width=64, items=200, combine=30, **kw)
    p, b = pad.plan, base.plan
    assert (p.table_width, p.num_decode_items, p.num_combine_seqs, p.split_blocks) == (64, 200, 30, sb)
    np.testing.assert_array_equal(pad.block_tables(False)[:, :b.table_width], base.block_tables(False))
    assert not pad.block_tables(False)[:, b.table_width:].any()
    np.testing.assert_array_equal(pad.slot_mapping(False), base.slot_mapping(False))
    items = pad.decode_items()
    np.testing.assert_array_equal(items[:b.num_decode_items], base.decode_items())
    assert (items[b.num_decode_items:, 0] == -1).all()
    comb = pad.host[p.off_combine:p.off_combine + 4 * 30].reshape(30, 4)
    np.testing.assert_array_equal(comb[:b.num_combine_seqs],
                                  base.host[b.off_combine:b.off_combine + 4 * b.num_combine_seqs].reshape(-1, 4))
    assert (comb[b.num_combine_seqs:, 0] == -1).all()
    later = pkg.StepMetadata.plan_decode_padded(ctx + 7, tables, split_blocks=sb, width=64, items=200, combine=30, **kw)
    offs = [n for n, _ in pkg._lib.StepPlan._fields_ if n.startswith("off_") or n == "words"]
    assert all(getattr(later.plan, n) == getattr(p, n) for n in offs)
    with pytest.raises(ValueError, match="bucket"):
        pkg.StepMetadata.plan_decode_padded(ctx, tables, split_blocks=sb, width=64, items=4, combine=30, **kw)
    with pytest.raises(ValueError, match="bucket"):
        pkg.StepMetadata.plan_decode_padded(ctx, tables, split_blocks=sb, width=8, items=200, combine=30, **kw)


def test_seam_keeps_the_gather_signature(pkg, oracle):
    """The reference pins the dispatcher and every backend to one parameter list
    (tests/test_paged_attention.py:197-204); the cuda backend keeps it."""
    for fn in (pkg.paged_attention_cuda, pkg.paged_attention):
        assert list(inspect.signature(fn).parameters) == REFERENCE_SIGNATURE
    assert list(inspect.signature(oracle.paged_attention_gather).parameters)[:7] == REFERENCE_SIGNATURE


def test_cuda_path_fails_loudly_off_gpu(pkg, monkeypatch):
    """No silent fallback (attention_triton.py:250-264): CPU tensors raise."""
    q = torch.randn(5, 3, 8)
    pool = torch.randn(8, 4, 3, 8)
    bt = torch.tensor([[0, 1]])
    ctx, ql = torch.tensor([5]), torch.tensor([5])
    with pytest.raises(NotImplementedError, match="ATTENTION=cuda"):
        pkg.paged_attention_cuda(q, pool, pool, bt, ctx, ql, 0.5)
    monkeypatch.setenv("ATTENTION", "cuda")
    with pytest.raises(NotImplementedError, match="CUDA device"):
        pkg.paged_attention(q, pool, pool, bt, ctx, ql, 0.5)
    monkeypatch.setenv("ATTENTION", "cuda-graphs")
    with pytest.raises(ValueError, match="ATTENTION"):
        pkg.paged_attention(q, pool, pool, bt, ctx, ql, 0.5)
    with pytest.raises(NotImplementedError, match="CUDA device"):
        pkg.reshape_and_cache(q[:, :3], q[:, :3], pool, pool, torch.zeros(5, dtype=torch.int32))


def test_executor_graphs_and_fused_oproj_refuse_what_they_cannot_run(pkg):
    """The executor and the decode-step graphs need CUDA pools, the fused o_proj
    collective a 16-bit dtype; each says so before touching a device (no fallback)."""
    import importlib

    executor = importlib.import_module(f"{pkg.__name__}.executor")
    graphs = importlib.import_module(f"{pkg.__name__}.graphs")
    tp = importlib.import_module(f"{pkg.__name__}.tensor_parallel")
    pool = pkg.KVPool(2, 4, 16, 2, 8, torch.float32, "cpu")

    class Model:
        config = type("Config", (), {"num_attention_heads": 4})()

    with pytest.raises(NotImplementedError, match="CUDA device"):
        executor.CudaPagedExecutor(Model(), None, pool)
    with pytest.raises(NotImplementedError, match="CUDA pools"):
        graphs.DecodeStepGraph(pool.k, pool.v, 4, 0.5, 2, 4)
    with pytest.raises(NotImplementedError, match="bf16 or fp16"):
        tp.FusedOProjAllReduce(8, 256, torch.float32)


def test_shape_errors_match_reference(pkg):
    pool = torch.randn(8, 4, 3, 8)
    with pytest.raises(ValueError, match="query must be"):
        pkg.paged_attention_cuda(torch.randn(5, 8), pool, pool, None, None, None, 0.5)
    with pytest.raises(ValueError, match="k_pool must be"):
        pkg.paged_attention_cuda(torch.randn(5, 3, 8), pool[0], pool[0], None, None, None, 0.5)


def test_words_bound_covers_plans(pkg):
    lib = pkg._lib.lib()
    rng = np.random.default_rng(1)
    for _ in range(10):
        b = int(rng.integers(1, 64))
        ctx = rng.integers(1, 3000, size=b)
        ql = np.where(rng.random(b) < 0.5, 1, np.minimum(ctx, 50))
        need = -(-ctx // 16)
        tables = np.zeros((b, int(need.max())), dtype=np.int64)
        m = _plan(pkg, ctx, ql, tables, num_blocks=1, bs=16, kv_heads=8, sm=148, tile=64)
        assert m.plan.words <= lib.pa_plan_words_bound(b, int(ql.sum()), int(need.max()))


def test_multi_gpu_and_block_entry_points_reject_bad_arguments(pkg):
    """The argument checks of the block moves, the peer all-reduce and CUDA IPC run on the
    host before any device work (so they hold without a GPU) and name the problem."""
    import ctypes

    lib = pkg._lib.lib()
    arr = (ctypes.c_void_p * 1)(None)
    err = ctypes.c_int32(0)
    with pytest.raises(ValueError, match="multiple of 16"):
        pkg._lib.check(lib.pa_copy_blocks(arr, arr, 1, 8, 24, None, 1, ctypes.addressof(err), None))
    with pytest.raises(ValueError, match="bad sizes"):
        pkg._lib.check(lib.pa_gather_blocks(arr, arr, -1, 8, 32, None, 1, None, ctypes.addressof(err), None))
    pkg._lib.check(lib.pa_scatter_blocks(arr, arr, 1, 8, 32, None, 0, None, ctypes.addressof(err), None))  # no-op
    bases = (ctypes.c_void_p * 2)(None, None)
    with pytest.raises(ValueError, match="rank 2 of 2"):
        pkg._lib.check(lib.pa_peer_allreduce(bases, 2, 2, 0, 256, 64, 2, 1.0, ctypes.addressof(err), None))
    with pytest.raises(ValueError, match="at most 8"):
        pkg._lib.check(lib.pa_peer_allreduce(bases, 9, 0, 0, 256, 64, 2, 1.0, ctypes.addressof(err), None))
    with pytest.raises(NotImplementedError, match="16-byte vectors"):
        pkg._lib.check(lib.pa_peer_allreduce(bases, 2, 0, 0, 256, 3, 2, 1.0, ctypes.addressof(err), None))
    with pytest.raises(ValueError, match="timeout"):
        pkg._lib.check(lib.pa_peer_allreduce(bases, 2, 0, 0, 256, 64, 2, 0.0, ctypes.addressof(err), None))
    with pytest.raises(ValueError, match="NULL"):
        pkg._lib.check(lib.pa_ipc_export(None, None, None))
    with pytest.raises(ValueError):
        pkg._lib.check(lib.pa_ipc_open(None, 0, None))
    # default plans use the single-CTA kernel's 128-row tiles at every head_dim
    assert pkg.metadata.prefill_tile_rows(128) == lib.pa_prefill_tile_rows(128) == 128
    assert pkg.metadata.prefill_tile_rows(64) == lib.pa_prefill_tile_rows(64) == 128
    assert pkg.metadata.prefill_tile_tokens(32, 8, 128) == 32 and pkg.metadata.prefill_tile_tokens(12, 12, 64) == 128


def test_fused_oproj_allreduce_rejects_bad_arguments(pkg):
    """pa_oproj_allreduce checks shapes, dtypes, alignment and ranks on the host before any
    device work; zero rows is a no-op."""
    import ctypes

    lib = pkg._lib.lib()
    err = ctypes.c_int32(0)
    fake = 1 << 20                      # aligned, never dereferenced by the host checks
    bases = (ctypes.c_void_p * 2)(fake, fake)

    def call(rows=256, k=1024, n=1024, dtype=2, world=2, rank=0, a=fake, a_stride=1024, w=fake, stage=0, out=4096,
             flags=8192, timeout=1.0, b=bases):
        return lib.pa_oproj_allreduce(a, a_stride, rows, k, w, n, dtype, b, world, rank, stage, out, flags, timeout,
                                      ctypes.addressof(err), None)

    with pytest.raises(ValueError, match="rank 2 of 2"):
        pkg._lib.check(call(rank=2))
    with pytest.raises(NotImplementedError, match="bf16 or fp16"):
        pkg._lib.check(call(dtype=0))
    with pytest.raises(NotImplementedError, match="k a multiple of 64"):
        pkg._lib.check(call(k=1000, a_stride=1000))
    with pytest.raises(NotImplementedError, match="n of 256 x 2 ranks"):
        pkg._lib.check(call(n=384))
    with pytest.raises(ValueError, match="row stride"):
        pkg._lib.check(call(a_stride=1020))
    with pytest.raises(ValueError, match="unaligned pointer"):
        pkg._lib.check(call(a=fake + 8))
    with pytest.raises(ValueError, match="offsets"):
        pkg._lib.check(call(out=4100))
    with pytest.raises(ValueError, match="timeout"):
        pkg._lib.check(call(timeout=0.0))
    with pytest.raises(ValueError, match="rank 1 is NULL"):
        pkg._lib.check(call(b=(ctypes.c_void_p * 2)(fake, None)))
    pkg._lib.check(call(rows=0))        # nothing to do, nothing launched
