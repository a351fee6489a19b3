"""pa_paged_attention_fwd_noalloc, the entry point for callers that cannot allocate
device memory (a plug-in whose host framework owns all device memory, a serving loop
that cannot pay cudaMalloc's device-wide synchronisation).  It keeps its split-K scratch
in a static device array instead of a caller-provided workspace.

Checked through the C ABI against the ordinary entry point on the same inputs, for two
calls in a row (the second call finds the first call's scratch contents), plus the
rejection of a step whose scratch need exceeds the static array.  This file is named to
be collected last so that a failure here never hides the rest of the suite.
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


@pytest.mark.parametrize("dtype,heads,kv_heads,d", [(torch.bfloat16, 32, 8, 128), (torch.float32, 12, 12, 64)])
def test_noalloc_matches_workspace_entry_point_twice(pkg, dtype, heads, kv_heads, d):
    # decode rows with several splits each (combine pass), plus prefill rows
    lengths = [(1500, 1), (700, 1), (33, 1), (1, 1), (2900, 1), (64, 40), (90, 90)]
    q, kp, vp, bt, cl, ql = ragged_batch(lengths, bs=16, d=d, heads=heads, kv_heads=kv_heads, dtype=dtype, seed=4)
    q, kp, vp = q.to(DEV), kp.to(DEV), vp.to(DEV)
    scale = d ** -0.5
    ref = pkg.paged_attention_cuda(q, kp, vp, bt.to(DEV), cl.to(DEV), ql.to(DEV), scale)
    meta = pkg.StepMetadata.build(cl, ql, bt, num_tokens=q.shape[0], pool_num_blocks=kp.shape[0], block_size=16,
                                  num_kv_heads=kv_heads, device=DEV)
    assert meta.plan.num_combine_seqs > 0
    tol = TOL["f32" if dtype == torch.float32 else "bf16"]
    for _ in range(2):
        got = _noalloc(pkg, q, kp, vp, meta, scale)
        torch.cuda.synchronize()
        np.testing.assert_allclose(got.float().cpu().numpy(), ref.float().cpu().numpy(), **tol)


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
