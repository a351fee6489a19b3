"""Parity of the sm_100a attention path with the reference (golden vectors) and the CPU
oracle, through the C ABI (ctypes) on a real GPU.

Tolerances: fp32 atol = rtol = 1e-5 (the north star's 1e-5 relative; the reference's
own kernel tier allows 1e-4, tests/test_paged_attention_triton.py:165-169), fp16/bf16
2e-2 (tests/test_paged_attention_triton.py:172-178).
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from _batches import compact_subbatch, lognormal_contexts, ragged_batch, ragged_batch_device, subset_rows
from _golden import TOL, attention_cases, load, load_attention

pytestmark = pytest.mark.gpu

DT = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
NAME = {v: k for k, v in DT.items()}
DEV = "cuda"


def _pf(rows: int = 128) -> str:
    """The tcgen05 prefill kernel a plan tiled at `rows` runs: 128-row tiles the persistent
    kernel (the single-CTA kernel under PA_PREFILL_KERNEL=per_tile), 256-row tiles the
    CTA-pair kernel."""
    if rows == 256:
        return "prefill_pair"
    return "prefill_tc" if os.environ.get("PA_PREFILL_KERNEL") == "per_tile" else "prefill_persist"


# (PA_PREFILL_KERNEL value, tile rows) of every tcgen05 prefill kernel
PREFILL_KERNELS = [("persistent", 128), ("per_tile", 128), ("per_tile", 256)]


def _close(got: np.ndarray, ref: np.ndarray, dt: str, what: str = ""):
    np.testing.assert_allclose(got, ref, err_msg=what, **TOL[dt])


def _run(pkg, q, kp, vp, bt, cl, ql, scale):
    out = pkg.paged_attention_cuda(q.to(DEV), kp.to(DEV), vp.to(DEV), bt.to(DEV), cl.to(DEV), ql.to(DEV), scale)
    torch.cuda.synchronize()
    return out


@pytest.mark.parametrize("case", attention_cases())
def test_matches_reference_golden(pkg, case):
    """Every shape the reference's test-suite uses plus the serving shapes, against the
    reference gather path's own outputs."""
    g = load_attention(case)
    td = DT[g["dtype"]]
    q = torch.from_numpy(g["query"]).to(td)
    kp = torch.from_numpy(g["k_pool"]).to(td)
    vp = torch.from_numpy(g["v_pool"]).to(td)
    out = _run(pkg, q, kp, vp, torch.from_numpy(g["block_tables"]), torch.from_numpy(g["context_lens"]),
               torch.from_numpy(g["query_lens"]), g["scale"])
    assert out.dtype == td and tuple(out.shape) == g["out"].shape
    _close(out.float().cpu().numpy(), g["out"], g["dtype"], case)
    assert pkg.read_device_error() == 0


@pytest.mark.parametrize("case", sorted(load("mirror").keys()))
def test_mirror_cuda_matches_online_softmax_mirror(pkg, oracle, case):
    """The secondary oracle: the CUDA kernels against the reference's online-softmax
    order (its Triton kernel's PyTorch mirror, attention_triton.py:309-384, restated in
    the oracle and pinned to the mirror's own outputs) on the mirror's cases."""
    g = load_attention(case)
    td = DT[g["dtype"]]
    q = torch.from_numpy(g["query"]).to(td)
    kp = torch.from_numpy(g["k_pool"]).to(td)
    vp = torch.from_numpy(g["v_pool"]).to(td)
    out = _run(pkg, q, kp, vp, torch.from_numpy(g["block_tables"]), torch.from_numpy(g["context_lens"]),
               torch.from_numpy(g["query_lens"]), g["scale"])
    ref = oracle.paged_attention_mirror(g["query"], g["k_pool"], g["v_pool"], g["block_tables"], g["context_lens"],
                                        g["query_lens"], g["scale"], g["dtype"])
    _close(out.float().cpu().numpy(), ref, g["dtype"], case)
    assert pkg.read_device_error() == 0


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("heads,kv_heads,d", [(12, 12, 64), (32, 8, 128), (64, 8, 128), (16, 8, 64), (8, 1, 128)])
def test_split_k_decode_matches_oracle(pkg, oracle, dtype, heads, kv_heads, d):
    """Long ragged decode batches: many splits per sequence, so the combine pass runs;
    every GQA group the fast kernel instantiates (1, 2, 4, 8)."""
    ctx = lognormal_contexts(24, 700, 0.9, 1, 3000, seed=heads + d)
    lengths = [(int(c), 1) for c in ctx] + [(1, 1), (16, 1), (17, 1)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=d, heads=heads, kv_heads=kv_heads, dtype=DT[dtype])
    out = _run(pkg, q, kp, vp, bt, cl, ql, d ** -0.5)
    ref = oracle.paged_attention_gather(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), bt.numpy(),
                                        cl.numpy(), ql.numpy(), d ** -0.5, dtype)
    _close(out.float().cpu().numpy(), ref, dtype)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_mixed_prefill_and_decode(pkg, oracle, dtype):
    """Decode rows on the split-K kernel and prefill / partial-query rows on the generic
    kernel in one call (tests/test_paged_attention.py:123-135 shapes at block size 16)."""
    lengths = [(300, 1), (16, 16), (129, 1), (64, 40), (90, 90), (33, 3), (1, 1), (700, 1)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=128, heads=32, kv_heads=8, dtype=DT[dtype], seed=5)
    out = _run(pkg, q, kp, vp, bt, cl, ql, 128 ** -0.5)
    ref = oracle.paged_attention_gather(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), bt.numpy(),
                                        cl.numpy(), ql.numpy(), 128 ** -0.5, dtype)
    _close(out.float().cpu().numpy(), ref, dtype)


def test_accepts_non_contiguous_query(pkg):
    """The executor hands over `query[0].transpose(0, 1)` (tests/test_paged_attention_triton.py:209-220)."""
    lengths = [(6, 1), (10, 10), (4, 1), (9, 5), (16, 16), (13, 1), (300, 1)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=64, heads=12, kv_heads=12)
    strided = q.to(DEV).transpose(0, 1).contiguous().transpose(0, 1)
    assert not strided.is_contiguous()
    a = pkg.paged_attention_cuda(strided, kp.to(DEV), vp.to(DEV), bt.to(DEV), cl.to(DEV), ql.to(DEV), 0.125)
    b = pkg.paged_attention_cuda(q.to(DEV), kp.to(DEV), vp.to(DEV), bt.to(DEV), cl.to(DEV), ql.to(DEV), 0.125)
    torch.testing.assert_close(a, b, atol=0, rtol=0)


def test_fast_and_generic_kernels_agree(pkg):
    """A query with non-unit dim stride routes decode rows to the generic kernel; both
    kernels must give the same answer to fp32 rounding."""
    lengths = [(int(c), 1) for c in lognormal_contexts(16, 400, 0.9, 1, 2000, seed=2)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=128, heads=32, kv_heads=8)
    q_dev = q.to(DEV)
    odd = torch.empty(q.shape[0], q.shape[1], q.shape[2] * 2, device=DEV)[:, :, ::2]
    odd.copy_(q_dev)
    assert odd.stride(2) == 2
    fast = pkg.paged_attention_cuda(q_dev, kp.to(DEV), vp.to(DEV), bt.to(DEV), cl.to(DEV), ql.to(DEV), 0.088)
    assert pkg._lib.last_launches() <= {"decode_simt", "combine"}
    slow = pkg.paged_attention_cuda(odd, kp.to(DEV), vp.to(DEV), bt.to(DEV), cl.to(DEV), ql.to(DEV), 0.088)
    assert pkg._lib.last_launches() == {"generic"}
    torch.testing.assert_close(fast, slow, atol=2e-6, rtol=2e-6)


def test_empty_batch(pkg):
    q = torch.empty(0, 3, 8, device=DEV)
    pool = torch.zeros(4, 4, 3, 8, device=DEV)
    zero = torch.zeros(0, dtype=torch.long, device=DEV)
    out = pkg.paged_attention_cuda(q, pool, pool, torch.zeros(0, 1, dtype=torch.long, device=DEV), zero, zero, 0.5)
    assert out.shape == (0, 3, 8)


def test_contract_errors_on_device(pkg):
    q, kp, vp, bt, cl, ql = ragged_batch([(4, 4), (2, 2)], bs=4, d=8, heads=3, kv_heads=3)
    args = [t.to(DEV) for t in (q, kp, vp, bt)]
    with pytest.raises(ValueError, match="query_len exceeds context_len"):
        pkg.paged_attention_cuda(*args, (cl - 1).to(DEV), ql.to(DEV), 0.5)
    with pytest.raises(ValueError, match="query_lens sum"):
        pkg.paged_attention_cuda(args[0][:-1], *args[1:], cl.to(DEV), ql.to(DEV), 0.5)


def test_deterministic_and_batch_order_invariant(pkg):
    """Same inputs -> bitwise-equal outputs; permuting the sequences of a batch permutes
    the outputs bitwise (each sequence's splits depend only on its own length and the
    batch's length multiset)."""
    lengths = [(int(c), 1) for c in lognormal_contexts(64, 1024, 0.9, 16, 8192, seed=9)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=64, heads=12, kv_heads=12, dtype=torch.bfloat16)
    a = _run(pkg, q, kp, vp, bt, cl, ql, 0.125)
    b = _run(pkg, q, kp, vp, bt, cl, ql, 0.125)
    assert torch.equal(a, b)
    perm = torch.randperm(len(lengths), generator=torch.Generator().manual_seed(1))
    c = _run(pkg, q[perm], kp, vp, bt[perm], cl[perm], ql[perm], 0.125)
    assert torch.equal(c, a[perm.to(DEV)])


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_full_size_microbench_config_sampled(pkg, oracle, dtype):
    """BASELINE config 2 at full size (B=256, GPT-2 heads, lognormal median 1024 clipped
    16..8192): the whole batch runs on the GPU; 8 sampled sequences plus the longest are
    re-computed by the oracle (a sequence's output depends only on its own blocks)."""
    ctx = lognormal_contexts(256, 1024, 0.9, 16, 8192, seed=0)
    lengths = [(int(c), 1) for c in ctx]
    batch = ragged_batch_device(lengths, bs=16, d=64, heads=12, kv_heads=12, dtype=DT[dtype], device=DEV)
    q, kp, vp, bt, cl, ql = batch
    out = pkg.paged_attention_cuda(q, kp, vp, bt.to(DEV), cl.to(DEV), ql.to(DEV), 0.125).float().cpu().numpy()
    picks = list(np.random.default_rng(1).choice(256, size=8, replace=False)) + [int(np.argmax(ctx))]
    sub = compact_subbatch(*batch, lengths, picks, 16)
    ref = oracle.paged_attention_gather(*sub, 0.125, dtype)
    _close(out[subset_rows(lengths, picks)], ref, dtype)


def test_full_size_llama8b_decode_sampled(pkg, oracle):
    """BASELINE config 3 decode shape at full size (B=256, 32/8/128 bf16, contexts
    lognormal mean 4096 clipped 128..16384): one layer on the GPU, 4 sequences re-computed
    by the oracle."""
    ctx = lognormal_contexts(256, 4096 * np.exp(-0.405), 0.9, 128, 16384, seed=0)
    lengths = [(int(c), 1) for c in ctx]
    batch = ragged_batch_device(lengths, bs=16, d=128, heads=32, kv_heads=8, dtype=torch.bfloat16, device=DEV)
    q, kp, vp, bt, cl, ql = batch
    out = pkg.paged_attention_cuda(q, kp, vp, bt.to(DEV), cl.to(DEV), ql.to(DEV), 128 ** -0.5)
    out = out.float().cpu().numpy()
    picks = [int(np.argmax(ctx)), int(np.argmin(ctx)), 7, 100]
    sub = compact_subbatch(*batch, lengths, picks, 16)
    ref = oracle.paged_attention_gather(*sub, 128 ** -0.5, "bf16")
    _close(out[subset_rows(lengths, picks)], ref, "bf16")
    assert pkg.read_device_error() == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("heads,kv_heads,d", [(32, 8, 128), (64, 8, 128), (12, 12, 64), (16, 8, 64)])
def test_tensor_pipe_and_simt_decode_agree(pkg, oracle, dtype, heads, kv_heads, d):
    """16-bit decode rows run on the tensor-pipe kernel; a query whose head stride is odd
    cannot be read as 32-bit pairs and routes the same rows to the SIMT decode kernel.
    Both must match the oracle, and each other to the rounding of P to the pool dtype."""
    ctx = lognormal_contexts(20, 600, 0.9, 1, 2500, seed=d + heads)
    lengths = [(int(c), 1) for c in ctx] + [(15, 1), (16, 1), (17, 1), (31, 1)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=d, heads=heads, kv_heads=kv_heads, dtype=DT[dtype],
                                         seed=7)
    qd = q.to(DEV)
    odd = torch.empty(q.shape[0], q.shape[1], d + 1, dtype=qd.dtype, device=DEV)[:, :, :d]
    odd.copy_(qd)
    assert odd.stride(1) % 2 == 1 and odd.stride(2) == 1
    args = (kp.to(DEV), vp.to(DEV), bt.to(DEV), cl.to(DEV), ql.to(DEV), d ** -0.5)
    mma = pkg.paged_attention_cuda(qd, *args).float().cpu().numpy()
    assert "decode_mma" in pkg._lib.last_launches() and "decode_simt" not in pkg._lib.last_launches()
    simt = pkg.paged_attention_cuda(odd, *args).float().cpu().numpy()
    assert "decode_simt" in pkg._lib.last_launches() and "decode_mma" not in pkg._lib.last_launches()
    ref = oracle.paged_attention_gather(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), bt.numpy(),
                                        cl.numpy(), ql.numpy(), d ** -0.5, dtype)
    _close(mma, ref, dtype, "tensor-pipe decode")
    _close(simt, ref, dtype, "SIMT decode")
    np.testing.assert_allclose(mma, simt, atol=1e-2, rtol=1e-2)


PREFILL_LENGTHS = [(300, 300), (129, 129), (16, 16), (17, 17), (200, 57), (700, 700), (513, 100), (40, 3),
                   (5, 5), (130, 2), (256, 256), (1, 1), (90, 1)]


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("heads,kv_heads,d", [(32, 8, 128), (64, 8, 128), (12, 12, 64), (16, 8, 64), (8, 4, 128)])
def test_tensor_core_prefill_matches_oracle(pkg, oracle, dtype, heads, kv_heads, d):
    """Varlen paged prefill on tcgen05 for GQA groups 1/2/4/8 and head_dims 64/128:
    prompts shorter and longer than a tile, prefix-cache hits (query shorter than the
    context), contexts that end mid-block and mid-KV-tile, plus decode rows in the same
    call.  A query with an odd head stride sends the same rows through the generic
    kernel, which must agree."""
    q, kp, vp, bt, cl, ql = ragged_batch(PREFILL_LENGTHS, bs=16, d=d, heads=heads, kv_heads=kv_heads,
                                         dtype=DT[dtype], seed=11)
    qd = q.to(DEV)
    args = (kp.to(DEV), vp.to(DEV), bt.to(DEV), cl.to(DEV), ql.to(DEV), d ** -0.5)
    tc = pkg.paged_attention_cuda(qd, *args).float().cpu().numpy()
    assert {_pf(d), "decode_mma"} <= pkg._lib.last_launches() <= {_pf(d), "decode_mma", "combine"}
    odd = torch.empty(q.shape[0], q.shape[1], d + 1, dtype=qd.dtype, device=DEV)[:, :, :d]
    odd.copy_(qd)
    generic = pkg.paged_attention_cuda(odd, *args).float().cpu().numpy()
    assert {"generic", "decode_simt"} <= pkg._lib.last_launches() <= {"generic", "decode_simt", "combine"}
    ref = oracle.paged_attention_gather(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), bt.numpy(),
                                        cl.numpy(), ql.numpy(), d ** -0.5, dtype)
    _close(tc, ref, dtype, "tcgen05 prefill")
    _close(generic, ref, dtype, "generic prefill")
    assert pkg.read_device_error() == 0


def test_tensor_core_prefill_churn_shape(pkg, oracle):
    """BASELINE config 3's churn prompts (256..2048 tokens) at the Llama-8B shape: 3
    prompts through the tcgen05 kernel, one re-computed by the oracle."""
    rng = np.random.default_rng(5)
    lengths = [(int(n), int(n)) for n in rng.integers(256, 2049, size=3)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=128, heads=32, kv_heads=8, dtype=torch.bfloat16, seed=3)
    out = _run(pkg, q, kp, vp, bt, cl, ql, 128 ** -0.5).float().cpu().numpy()
    assert pkg._lib.last_launches() == {_pf()}
    pick = [int(np.argmin([c for c, _ in lengths]))]
    sub = compact_subbatch(q, kp, vp, bt, cl, ql, lengths, pick, 16)
    ref = oracle.paged_attention_gather(*sub, 128 ** -0.5, "bf16")
    _close(out[subset_rows(lengths, pick)], ref, "bf16")


def test_shared_prefix_blocks_match_oracle(pkg, oracle):
    """BASELINE config 4's structure: every block table starts with the same 8 physical
    blocks (a refcounted 128-token system prefix); prefix-hit prefills (query = the
    unique suffix, shorter than the context) and decodes read those blocks concurrently
    in one call, on the tcgen05 prefill and tensor-pipe decode kernels."""
    g = torch.Generator().manual_seed(31)
    bs, heads, kv_heads, d = 16, 32, 8, 128
    suffixes = [37, 200, 512, 16, 1, 1, 1, 1]      # four prefix-hit prefills, four decodes
    ctx = [128 + s + (40 if q == 1 else 0) for s, q in zip([37, 200, 512, 16, 90, 300, 5, 0], suffixes)]
    need = [-(-c // bs) for c in ctx]
    nb = 8 + sum(n - 8 for n in need) + 4
    perm = torch.randperm(nb, generator=g)
    tables = torch.zeros(len(ctx), max(need), dtype=torch.long)
    off = 8
    for i, n in enumerate(need):
        tables[i, :8] = perm[:8]                       # the shared prefix blocks
        tables[i, 8:n] = perm[off:off + n - 8]
        off += n - 8
    kp = torch.randn(nb, bs, kv_heads, d, generator=g).to(torch.bfloat16)
    vp = torch.randn(nb, bs, kv_heads, d, generator=g).to(torch.bfloat16)
    q = torch.randn(sum(suffixes), heads, d, generator=g).to(torch.bfloat16)
    cl = torch.tensor(ctx, dtype=torch.long)
    ql = torch.tensor(suffixes, dtype=torch.long)
    out = _run(pkg, q, kp, vp, tables, cl, ql, d ** -0.5).float().cpu().numpy()
    assert {_pf(), "decode_mma"} <= pkg._lib.last_launches()
    ref = oracle.paged_attention_gather(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), tables.numpy(),
                                        cl.numpy(), ql.numpy(), d ** -0.5, "bf16")
    _close(out, ref, "bf16", "shared prefix blocks")
    assert pkg.read_device_error() == 0


def _with_tiles(pkg, bt, cl, ql, num_tokens, nb, kv_heads, tile_tokens):
    """Device block tables carrying a plan tiled at `tile_tokens` query tokens per prefill
    tile (256 / G: the CTA-pair kernel; 128 / G: the single-CTA kernel)."""
    meta = pkg.StepMetadata.build(cl, ql, bt, num_tokens=num_tokens, pool_num_blocks=nb, block_size=16,
                                  num_kv_heads=kv_heads, device=DEV, prefill_tile_tokens=tile_tokens)
    return pkg.attach(bt.to(DEV), meta)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("heads,kv_heads", [(16, 16), (16, 8), (32, 8), (64, 8)])
def test_prefill_kernels_agree_with_each_other_and_oracle(pkg, oracle, monkeypatch, dtype, heads, kv_heads):
    """Every tcgen05 prefill kernel (persistent, single-CTA, CTA pair)
    on the same batch against the oracle and each other, for GQA groups 1/2/4/8 at
    head_dim 128: tiles whose second half has few or no tokens, prompts shorter than one
    tile, prefix hits, contexts ending mid-block and mid-KV-tile."""
    g = heads // kv_heads
    lengths = PREFILL_LENGTHS + [(256 // g + 1, 256 // g + 1), (128 // g, 128 // g), (128 // g + 3, 128 // g + 3),
                                 (1000, 256 // g), (333, 128 // g - 1)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=128, heads=heads, kv_heads=kv_heads, dtype=DT[dtype],
                                         seed=21)
    qd, kd, vd = q.to(DEV), kp.to(DEV), vp.to(DEV)
    cld, qld = cl.to(DEV), ql.to(DEV)
    ref = oracle.paged_attention_gather(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), bt.numpy(),
                                        cl.numpy(), ql.numpy(), 128 ** -0.5, dtype)
    outs = {}
    for kernel, rows in PREFILL_KERNELS:
        monkeypatch.setenv("PA_PREFILL_KERNEL", kernel)
        btd = _with_tiles(pkg, bt, cl, ql, q.shape[0], kp.shape[0], kv_heads, rows // g)
        out = pkg.paged_attention_cuda(qd, kd, vd, btd, cld, qld, 128 ** -0.5).float().cpu().numpy()
        assert _pf(rows) in pkg._lib.last_launches(), (kernel, rows, pkg._lib.last_launches())
        _close(out, ref, dtype, f"{kernel} prefill, {rows}-row tiles")
        outs[(kernel, rows)] = out
    for key, out in outs.items():
        np.testing.assert_allclose(out, outs[("per_tile", 128)], atol=1e-2, rtol=1e-2, err_msg=str(key))
    assert pkg.read_device_error() == 0


@pytest.mark.parametrize("kernel,rows", PREFILL_KERNELS)
def test_prefill_ignores_stale_rows_past_the_context(pkg, oracle, monkeypatch, kernel, rows):
    """The reference slices every sequence's keys to its context (attention.py:171-172),
    so whatever a freed-and-reused block holds past the context never reaches it.  Fill
    those rows of K and V with NaN: the tcgen05 kernels must give the oracle's result."""
    monkeypatch.setenv("PA_PREFILL_KERNEL", kernel)
    lengths = [(70, 70), (100, 37), (17, 17), (1000, 999), (130, 130)]
    heads, kv_heads = 32, 8
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=128, heads=heads, kv_heads=kv_heads,
                                         dtype=torch.bfloat16, seed=8)
    kp_bad, vp_bad = kp.clone(), vp.clone()
    for i, (c, _) in enumerate(lengths):
        last = int(bt[i, (c - 1) // 16])
        kp_bad[last, c % 16 or 16:] = float("nan")
        vp_bad[last, c % 16 or 16:] = float("nan")
    btd = _with_tiles(pkg, bt, cl, ql, q.shape[0], kp.shape[0], kv_heads, rows // (heads // kv_heads))
    out = pkg.paged_attention_cuda(q.to(DEV), kp_bad.to(DEV), vp_bad.to(DEV), btd, cl.to(DEV), ql.to(DEV),
                                   128 ** -0.5).float().cpu().numpy()
    assert _pf(rows) in pkg._lib.last_launches()
    assert np.isfinite(out).all()
    ref = oracle.paged_attention_gather(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), bt.numpy(),
                                        cl.numpy(), ql.numpy(), 128 ** -0.5, "bf16")
    _close(out, ref, "bf16", f"{kernel} prefill ({rows} rows) with NaN past the context")


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("kernel,rows", [("persistent", 128), ("per_tile", 128)])
def test_prefill_head_dim_64_kernels(pkg, oracle, monkeypatch, dtype, kernel, rows):
    """head_dim 64 (one 64-column half per row) on the tcgen05 prefill kernels that serve
    it, GQA group 4, with ragged prompts, prefix hits and a decode row in the batch."""
    monkeypatch.setenv("PA_PREFILL_KERNEL", kernel)
    heads, kv_heads = 16, 4
    lengths = [(300, 300), (77, 77), (513, 129), (64, 64), (1000, 1), (200, 33)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=64, heads=heads, kv_heads=kv_heads, dtype=DT[dtype],
                                         seed=31)
    btd = _with_tiles(pkg, bt, cl, ql, q.shape[0], kp.shape[0], kv_heads, rows // (heads // kv_heads))
    out = pkg.paged_attention_cuda(q.to(DEV), kp.to(DEV), vp.to(DEV), btd, cl.to(DEV), ql.to(DEV),
                                   64 ** -0.5).float().cpu().numpy()
    assert _pf(rows) in pkg._lib.last_launches()
    ref = oracle.paged_attention_gather(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), bt.numpy(),
                                        cl.numpy(), ql.numpy(), 64 ** -0.5, dtype)
    _close(out, ref, dtype, f"{kernel} prefill, head_dim 64, {rows}-row tiles")
    assert pkg.read_device_error() == 0


def _torch_gather_reference(q, kp, vp, bt, cl, ql, scale, rows=512):
    """The reference gather path's arithmetic on the GPU, for sizes the numpy oracle is too
    slow for, with the oracle's rounding points (attention.py:156-187): products computed
    in float32 and rounded to the pool dtype (the reference's half-precision matmuls
    return that dtype), the scaled scores rounded, softmax in float32, probabilities
    rounded before P.V, the output rounded.  Pinned against the oracle on a small case in
    the test that uses it."""
    def rnd(x):
        return x.to(vp.dtype).float()

    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    heads, bs, kvh = q.shape[1], kp.shape[1], kp.shape[2]
    start = 0
    for i in range(bt.shape[0]):
        c, n = int(cl[i]), int(ql[i])
        blocks = bt[i, :(c + bs - 1) // bs].to(q.device)
        k = kp[blocks].flatten(0, 1)[:c].float().repeat_interleave(heads // kvh, dim=1).transpose(0, 1)
        v = vp[blocks].flatten(0, 1)[:c].float().repeat_interleave(heads // kvh, dim=1).transpose(0, 1)
        for r0 in range(0, n, rows):
            r1 = min(n, r0 + rows)
            qq = q[start + r0:start + r1].float().transpose(0, 1)
            s = rnd(rnd(torch.matmul(qq, k.transpose(-1, -2))) * scale)
            qpos = torch.arange(c - n + r0, c - n + r1, device=q.device)
            s = s.masked_fill(torch.arange(c, device=q.device)[None, :] > qpos[:, None], float("-inf"))
            p = rnd(torch.softmax(s, dim=-1, dtype=torch.float32))
            out[start + r0:start + r1] = rnd(torch.matmul(p, v)).transpose(0, 1)
        start += n
    return out


@pytest.mark.parametrize("workload", ["config2-f32", "config2-bf16", "config3-decode", "config3-churn"])
def test_full_size_batches_every_sequence(pkg, oracle, workload):
    """BASELINE configs 2 and 3 at full size with EVERY sequence checked (the sampled
    tests above re-compute a few with the numpy oracle): config 2's 256 decode rows
    (GPT-2 heads, fp32 and bf16), config 3's 256 decode rows (32/8/128 bf16, contexts
    mean 4096 up to 16384) and a full step of 13 churn prompts (256..2048 tokens) through
    the tcgen05 prefill, against the gather path's arithmetic run in torch on the GPU
    (pinned to the oracle on two of the sequences here)."""
    torch.backends.cuda.matmul.allow_tf32 = False
    if workload.startswith("config2"):
        dt = workload.split("-")[1]
        ctx = lognormal_contexts(256, 1024, 0.9, 16, 8192, seed=0)
        lengths = [(int(c), 1) for c in ctx]
        heads, kv_heads, d, td = 12, 12, 64, DT[dt]
    elif workload == "config3-decode":
        dt = "bf16"
        ctx = lognormal_contexts(256, 4096 * np.exp(-0.405), 0.9, 128, 16384, seed=0)
        lengths = [(int(c), 1) for c in ctx]
        heads, kv_heads, d, td = 32, 8, 128, torch.bfloat16
    else:
        dt = "bf16"
        rng = np.random.default_rng(0)
        lengths = [(int(n), int(n)) for n in rng.integers(256, 2049, size=13)]
        heads, kv_heads, d, td = 32, 8, 128, torch.bfloat16
    batch = ragged_batch_device(lengths, bs=16, d=d, heads=heads, kv_heads=kv_heads, dtype=td, device=DEV)
    q, kp, vp, bt, cl, ql = batch
    out = pkg.paged_attention_cuda(q, kp, vp, bt.to(DEV), cl.to(DEV), ql.to(DEV), d ** -0.5)
    if workload == "config3-churn":
        assert pkg._lib.last_launches() == {_pf()}
    ref = _torch_gather_reference(q, kp, vp, bt, cl, ql, d ** -0.5).cpu().numpy()
    _close(out.float().cpu().numpy(), ref, dt, workload)
    # the torch restatement itself, pinned to the oracle on the shortest and longest rows
    picks = [int(np.argmin([c for c, _ in lengths])), int(np.argmax([c for c, _ in lengths]))]
    sub = compact_subbatch(*batch, lengths, picks, 16)
    want = oracle.paged_attention_gather(*sub, d ** -0.5, dt)
    _close(ref[subset_rows(lengths, picks)], want, dt, "torch restatement vs oracle")
    assert pkg.read_device_error() == 0


def test_long_context_prefill_matches_reference(pkg, oracle, monkeypatch):
    """Long rows of the tcgen05 prefill at the Llama-8B shape: a 4,600-token prompt and a
    prefix-cache hit of 700 new tokens over a 9,300-token context (plus a decode row),
    every row compared with the gather arithmetic in torch float32.  That torch reference
    is itself pinned to the oracle on a small batch first."""
    heads, kv_heads, d = 32, 8, 128
    small = [(300, 300), (200, 57), (90, 1)]
    q, kp, vp, bt, cl, ql = ragged_batch(small, bs=16, d=d, heads=heads, kv_heads=kv_heads, dtype=torch.bfloat16,
                                         seed=2)
    mine = _torch_gather_reference(q.to(DEV), kp.to(DEV), vp.to(DEV), bt, cl, ql, d ** -0.5, rows=64).cpu().numpy()
    ref = oracle.paged_attention_gather(q.float().numpy(), kp.float().numpy(), vp.float().numpy(), bt.numpy(),
                                        cl.numpy(), ql.numpy(), d ** -0.5, "bf16")
    np.testing.assert_allclose(mine, ref, atol=1e-2, rtol=1e-2)

    lengths = [(4600, 4600), (9300, 700), (12000, 1)]
    q, kp, vp, bt, cl, ql = ragged_batch_device(lengths, bs=16, d=d, heads=heads, kv_heads=kv_heads,
                                                dtype=torch.bfloat16, device=DEV, seed=6)
    ref = _torch_gather_reference(q, kp, vp, bt, cl, ql, d ** -0.5).cpu().numpy()
    for kernel, rows in PREFILL_KERNELS:
        monkeypatch.setenv("PA_PREFILL_KERNEL", kernel)
        btd = _with_tiles(pkg, bt, cl, ql, q.shape[0], kp.shape[0], kv_heads, rows // (heads // kv_heads))
        out = pkg.paged_attention_cuda(q, kp, vp, btd, cl.to(DEV), ql.to(DEV), d ** -0.5)
        assert {_pf(rows), "decode_mma"} <= pkg._lib.last_launches()
        _close(out.float().cpu().numpy(), ref, "bf16", f"long-context prefill ({kernel}, {rows} rows)")
    assert pkg.read_device_error() == 0
