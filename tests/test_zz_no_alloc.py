"""pa_paged_attention_fwd_noalloc, the entry point for callers that cannot allocate
device memory (a plug-in whose host framework owns all device memory, a serving loop
that cannot pay cudaMalloc's device-wide synchronisation).  It keeps its split-K scratch
in a static device array instead of a caller-provided workspace, and
pa_noalloc_read_device_error reads the kernels' error word inside that array.

Checked through the C ABI against the ordinary entry point on the same inputs: two calls
in a row (the second call finds the first call's scratch contents), a large batch
followed by a smaller one with fewer splits (stale partials would show), the error word
read back as 0 after good calls and with bit 1 after a block id that skipped the host
planner, and the rejection of a step whose scratch need exceeds the static array.  Each
test clears the sticky error word before it checks it, so the file passes alone in a
fresh process and after the rest of the suite.  This file is named to be collected last
so that a failure here never hides the rest of the suite.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from _batches import ragged_batch
from _golden import TOL

pytestmark = pytest.mark.gpu
DEV = "cuda"
CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def _noalloc(pkg, q, kp, vp, meta, scale):
    lib = pkg._lib.lib()
    out = torch.empty_like(q)
    rc = lib.pa_paged_attention_fwd_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), q.stride(2), q.shape[0], q.shape[1], q.shape[2],
        kp.data_ptr(), vp.data_ptr(), kp.shape[0], kp.shape[1], kp.shape[2], CODE[q.dtype], scale,
        ctypes.byref(meta.plan), meta.device_buffer.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
        torch.cuda.current_stream().cuda_stream)
    pkg._lib.check(rc)
    return out


def _error_word(pkg, clear: bool = True) -> int:
    word = ctypes.c_int32(-1)
    pkg._lib.check(pkg._lib.lib().pa_noalloc_read_device_error(int(clear), ctypes.byref(word),
                                                              torch.cuda.current_stream().cuda_stream))
    return int(word.value)


def _case(pkg, lengths, dtype, heads, kv_heads, d, seed):
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=d, heads=heads, kv_heads=kv_heads, dtype=dtype, seed=seed)
    q, kp, vp = q.to(DEV), kp.to(DEV), vp.to(DEV)
    scale = d ** -0.5
    ref = pkg.paged_attention_cuda(q, kp, vp, bt.to(DEV), cl.to(DEV), ql.to(DEV), scale)
    meta = pkg.StepMetadata.build(cl, ql, bt, num_tokens=q.shape[0], pool_num_blocks=kp.shape[0], block_size=16,
                                  num_kv_heads=kv_heads, device=DEV,
                                  prefill_tile_tokens=pkg.prefill_tile_tokens(heads, kv_heads, d))
    return q, kp, vp, meta, scale, ref


@pytest.mark.parametrize("dtype,heads,kv_heads,d", [(torch.bfloat16, 32, 8, 128), (torch.float32, 12, 12, 64)])
def test_noalloc_matches_workspace_entry_point_twice(pkg, dtype, heads, kv_heads, d):
    # decode rows with several splits each (combine pass), plus prefill rows
    lengths = [(1500, 1), (700, 1), (33, 1), (1, 1), (2900, 1), (64, 40), (90, 90)]
    q, kp, vp, meta, scale, ref = _case(pkg, lengths, dtype, heads, kv_heads, d, seed=4)
    assert meta.plan.num_combine_seqs > 0
    _error_word(pkg)  # start from a clear word whatever ran before in this process
    tol = TOL["f32" if dtype == torch.float32 else "bf16"]
    for _ in range(2):
        got = _noalloc(pkg, q, kp, vp, meta, scale)
        launched = pkg._lib.last_launches()
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(), **tol)
        if dtype == torch.bfloat16:  # the tensor-core decode and prefill both ran through it
            assert {"decode_mma", "combine"} <= launched and launched & {"prefill_tc", "prefill_persist"}
    assert _error_word(pkg) == 0


def test_noalloc_smaller_step_after_a_larger_one(pkg):
    """A step with fewer split-K partials after one with many: the smaller step must not
    read any of the larger step's partials left in the shared array."""
    big = [(4000, 1)] * 24 + [(900, 1)] * 40
    small = [(2100, 1), (17, 1), (300, 1), (640, 33)]
    _error_word(pkg)
    for lengths, seed in ((big, 11), (small, 12), (big, 13), (small, 14)):
        q, kp, vp, meta, scale, ref = _case(pkg, lengths, torch.bfloat16, 32, 8, 128, seed)
        got = _noalloc(pkg, q, kp, vp, meta, scale)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(), **TOL["bf16"])
    assert _error_word(pkg) == 0


def test_noalloc_error_word_reports_a_bad_block_id(pkg):
    """A block id past the pool that skipped the host planner (written straight into the
    device metadata) reaches the decode kernel's bounds check: the block is replaced by
    block 0 instead of being read, and bit 1 of the static scratch's error word is set
    and stays set until it is cleared."""
    q, kp, vp, meta, scale, _ = _case(pkg, [(300, 1), (70, 1)], torch.bfloat16, 32, 8, 128, seed=5)
    _error_word(pkg)  # clear whatever an earlier test left
    assert _error_word(pkg) == 0
    meta.device_buffer[int(meta.plan.off_block_tables) + 1] = kp.shape[0] + 1000
    _noalloc(pkg, q, kp, vp, meta, scale)
    _noalloc(pkg, q, kp, vp, meta, scale)
    assert _error_word(pkg, clear=False) & 1
    assert _error_word(pkg, clear=True) & 1
    assert _error_word(pkg) == 0


def test_noalloc_checks_arguments_before_sizing_its_scratch(pkg):
    """A bad head shape is a ValueError from the argument checks, not a scratch-size
    error (negative sizes would otherwise wrap to a huge scratch need)."""
    meta = pkg.StepMetadata.build(np.array([5]), np.array([1]), np.zeros((1, 1), dtype=np.int64), num_tokens=1,
                                  pool_num_blocks=1, block_size=16, num_kv_heads=1, device=DEV)
    lib = pkg._lib.lib()
    q = torch.zeros(1, 4, 64, dtype=torch.bfloat16, device=DEV)
    pool = torch.zeros(1, 16, 1, 64, dtype=torch.bfloat16, device=DEV)
    rc = lib.pa_paged_attention_fwd_noalloc(q.data_ptr(), 256, 64, 1, 1, -4, 64, pool.data_ptr(), pool.data_ptr(), 1,
                                            16, 1, 2, 0.125, ctypes.byref(meta.plan), meta.device_buffer.data_ptr(),
                                            q.data_ptr(), 256, 64, torch.cuda.current_stream().cuda_stream)
    assert rc == pkg._lib.PA_ERR_INVALID_ARGUMENT
    assert "positive" in lib.pa_last_error().decode()
    assert lib.pa_last_launches() == 0


def test_noalloc_rejects_steps_beyond_its_scratch(pkg):
    """A decode batch whose split-K partials need more than the static array is refused
    before any launch, with the size in the message."""
    b, ctx = 2048, 8192
    need = ctx // 16
    tables = np.zeros((b, need), dtype=np.int64)
    meta = pkg.StepMetadata.build(np.full(b, ctx), np.ones(b, dtype=np.int64), tables, num_tokens=b,
                                  pool_num_blocks=1, block_size=16, num_kv_heads=8, device=DEV)
    lib = pkg._lib.lib()
    assert lib.pa_workspace_bytes(ctypes.byref(meta.plan), 64, 128) > pkg._lib.PA_NOALLOC_SCRATCH_BYTES
    q = torch.zeros(b, 64, 128, dtype=torch.bfloat16, device=DEV)
    pool = torch.zeros(1, 16, 8, 128, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="static scratch holds"):
        _noalloc(pkg, q, pool, pool, meta, 128 ** -0.5)
