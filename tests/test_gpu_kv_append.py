"""The fused K+V append is bit-exact against the reference's `_PagedCache.update`
(golden pool contents) and against the oracle's scatter at serving sizes."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from _golden import load

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _t(arr: np.ndarray, dt: str) -> torch.Tensor:
    if dt == "f32":
        return torch.from_numpy(np.ascontiguousarray(arr))
    return torch.from_numpy(np.ascontiguousarray(arr).view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_append_matches_reference_golden(pkg, dt):
    z = load(f"kv_append_{dt}")
    kp = _t(z["k_before"], dt).to(DEV)
    vp = _t(z["v_before"], dt).to(DEV)
    # The executor's view: [1, H, T, D] -> [T, H, D] (strided, paged_executor.py:119-121).
    key = _t(z["key"], dt).to(DEV)[0].transpose(0, 1)
    val = _t(z["value"], dt).to(DEV)[0].transpose(0, 1)
    assert not key.is_contiguous()
    slots = torch.from_numpy(z["write_slots"]).to(DEV)
    pkg.reshape_and_cache(key, val, kp, vp, slots)
    torch.cuda.synchronize()
    assert torch.equal(kp.cpu(), _t(z["k_after"], dt))
    assert torch.equal(vp.cpu(), _t(z["v_after"], dt))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("kv_heads,d", [(12, 64), (8, 128), (3, 8), (2, 12)])
def test_append_bit_exact_at_scale(pkg, oracle, dtype, kv_heads, d):
    """A decode step's worth of slots (256 tokens, random distinct slots) and a prefill's
    (2000 tokens) into a 4096-block pool; every other byte of the pool unchanged."""
    g = torch.Generator().manual_seed(kv_heads * d)
    nb, bs = 4096, 16
    for t in (256, 2000):
        kp = torch.randn(nb, bs, kv_heads, d, generator=g).to(dtype)
        vp = torch.randn(nb, bs, kv_heads, d, generator=g).to(dtype)
        slots = torch.randperm(nb * bs, generator=g)[:t]
        key = torch.randn(t, kv_heads, d, generator=g).to(dtype)
        val = torch.randn(t, kv_heads, d, generator=g).to(dtype)
        kd, vd = kp.to(DEV), vp.to(DEV)
        pkg.reshape_and_cache(key.to(DEV), val.to(DEV), kd, vd, slots.to(DEV))
        torch.cuda.synchronize()
        raw = torch.int16 if dtype != torch.float32 else torch.int32
        ref_k = oracle.kv_append(kp.view(raw).numpy(), slots.numpy(), key.view(raw).numpy())
        ref_v = oracle.kv_append(vp.view(raw).numpy(), slots.numpy(), val.view(raw).numpy())
        assert np.array_equal(kd.cpu().view(raw).numpy(), ref_k)
        assert np.array_equal(vd.cpu().view(raw).numpy(), ref_v)


def test_append_uses_planned_slot_mapping(pkg, oracle):
    """Slots from the step planner (new tokens only, paged_executor.py:245) land where the
    reference's block-table arithmetic says."""
    z = load("pack")
    meta = pkg.StepMetadata.build(z["context_lens"], z["query_lens"], z["block_tables"],
                                  num_tokens=int(z["query_lens"].sum()), pool_num_blocks=64, block_size=16,
                                  num_kv_heads=2, device=DEV)
    np.testing.assert_array_equal(meta.slot_mapping().cpu().numpy(), z["write_slots"])
    kp = torch.zeros(64, 16, 2, 8, device=DEV)
    vp = torch.zeros(64, 16, 2, 8, device=DEV)
    t = int(z["query_lens"].sum())
    key = torch.arange(t * 16, dtype=torch.float32, device=DEV).reshape(t, 2, 8)
    pkg.reshape_and_cache(key, -key, kp, vp, meta.slot_mapping())
    ref = oracle.kv_append(np.zeros((64, 16, 2, 8), np.float32), z["write_slots"], key.cpu().numpy())
    assert np.array_equal(kp.cpu().numpy(), ref)
    assert np.array_equal(vp.cpu().numpy(), -ref)
