"""Whole-block KV moves on the GPU: copy-on-write copies and swap-out / swap-in, against
the reference's own pool (golden vectors from kv_pool.py:142-182 and
paged_executor.py:265-270) and the oracle, bit for bit."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from _golden import load

pytestmark = pytest.mark.gpu
DEV = "cuda"
TORCH = {"f32": torch.float32, "bf16": torch.bfloat16}


def _to_torch(arr: np.ndarray, dt: str) -> torch.Tensor:
    """Golden array (float32, or raw 16-bit patterns for bf16) -> tensor of the dtype."""
    if dt == "f32":
        return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.float32))
    return torch.from_numpy(np.ascontiguousarray(arr, dtype=np.uint16).view(np.int16)).view(torch.bfloat16)


def _bits(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    return (t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)).numpy()


def _pool_from(pkg, k: torch.Tensor, v: torch.Tensor):
    L, NB, BS, H, D = k.shape
    pool = pkg.KVPool(L, NB, BS, H, D, k.dtype, DEV)
    for l in range(L):
        pool.k[l].copy_(k[l])
        pool.v[l].copy_(v[l])
    return pool


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_block_moves_match_reference_pool(pkg, dt):
    z = load(f"blocks_{dt}")
    pool = _pool_from(pkg, _to_torch(z["k_before"], dt), _to_torch(z["v_before"], dt))
    host = pkg.HostBlocks  # the class the reference's scheduler would receive
    h = pool.swap_out(z["swap_out_blocks"].tolist())
    assert isinstance(h, host) and len(h) == 4
    assert h.k[0].is_pinned()
    np.testing.assert_array_equal(_bits(torch.stack(h.k)), _bits(_to_torch(z["host_k"], dt)))
    np.testing.assert_array_equal(_bits(torch.stack(h.v)), _bits(_to_torch(z["host_v"], dt)))
    pool.swap_in(h, z["swap_in_blocks"].tolist())
    np.testing.assert_array_equal(_bits(torch.stack(pool.k)), _bits(_to_torch(z["k_after_swap_in"], dt)))
    np.testing.assert_array_equal(_bits(torch.stack(pool.v)), _bits(_to_torch(z["v_after_swap_in"], dt)))
    pool.copy_blocks(z["copy_pairs"].tolist())
    np.testing.assert_array_equal(_bits(torch.stack(pool.k)), _bits(_to_torch(z["k_after_copy"], dt)))
    np.testing.assert_array_equal(_bits(torch.stack(pool.v)), _bits(_to_torch(z["v_after_copy"], dt)))
    assert pool.read_error() == 0


def test_swap_in_accepts_per_layer_host_tensors(pkg, oracle):
    """A HostBlocks built the reference's way (separate per-layer CPU tensors) goes back
    through the per-layer staging copies."""
    g = torch.Generator().manual_seed(3)
    k = torch.randn(2, 12, 4, 2, 8, generator=g)
    v = torch.randn(2, 12, 4, 2, 8, generator=g)
    pool = _pool_from(pkg, k, v)
    hk = [torch.randn(3, 4, 2, 8, generator=g) for _ in range(2)]
    hv = [torch.randn(3, 4, 2, 8, generator=g) for _ in range(2)]
    pool.swap_in(pkg.HostBlocks(k=hk, v=hv), [7, 1, 10])
    ek, ev = oracle.swap_in(k.numpy(), v.numpy(), torch.stack(hk).numpy(), torch.stack(hv).numpy(), [7, 1, 10])
    np.testing.assert_array_equal(torch.stack(pool.k).cpu().numpy(), ek)
    np.testing.assert_array_equal(torch.stack(pool.v).cpu().numpy(), ev)


def test_more_layers_than_one_launch_holds(pkg, oracle):
    """130 layers: the C entry points split the pool pointers over two launches."""
    g = torch.Generator().manual_seed(5)
    k = torch.randn(130, 9, 4, 1, 8, generator=g)
    v = torch.randn(130, 9, 4, 1, 8, generator=g)
    pool = _pool_from(pkg, k, v)
    h = pool.swap_out([8, 0, 4])
    hk, hv = oracle.swap_out(k.numpy(), v.numpy(), [8, 0, 4])
    np.testing.assert_array_equal(torch.stack(h.k).numpy(), hk)
    np.testing.assert_array_equal(torch.stack(h.v).numpy(), hv)
    pool.swap_in(h, [1, 2, 3])
    pool.copy_blocks([(5, 6), (7, 0)])
    ek, ev = oracle.swap_in(k.numpy(), v.numpy(), hk, hv, [1, 2, 3])
    ek, ev = oracle.copy_block(ek, ev, [(5, 6), (7, 0)])
    np.testing.assert_array_equal(torch.stack(pool.k).cpu().numpy(), ek)
    np.testing.assert_array_equal(torch.stack(pool.v).cpu().numpy(), ev)


def test_serving_size_round_trip(pkg):
    """Llama-3-8B-shape pool (32 layers, 16 x 8 x 128 bf16 blocks): 200 blocks out, back
    into other blocks, byte-identical; copy-on-write of 64 blocks likewise."""
    L, NB = 32, 1024
    pool = pkg.KVPool(L, NB, 16, 8, 128, torch.bfloat16, DEV)
    g = torch.Generator(device=DEV).manual_seed(1)
    for t in pool.k + pool.v:
        t.normal_(generator=g)
    perm = torch.randperm(NB, generator=torch.Generator().manual_seed(2)).tolist()
    src, dst = perm[:200], perm[200:400]
    ref_k = [t[src].clone() for t in pool.k]
    h = pool.swap_out(src)
    pool.swap_in(h, dst)
    torch.cuda.synchronize()
    for l in range(L):
        assert torch.equal(pool.k[l][dst], ref_k[l])
    pairs = list(zip(perm[400:464], perm[464:528]))
    before = [t[[s for s, _ in pairs]].clone() for t in pool.v]
    pool.copy_blocks(pairs)
    for l in range(L):
        assert torch.equal(pool.v[l][[d for _, d in pairs]], before[l])
    assert pool.read_error() == 0


def test_block_move_contract_errors(pkg):
    pool = pkg.KVPool(2, 8, 4, 1, 8, torch.float32, DEV)
    with pytest.raises(ValueError, match="swap_in: 2 host blocks into 3 device blocks"):
        pool.swap_in(pool.swap_out([1, 2]), [3, 4, 5])
    with pytest.raises(ValueError, match="outside the pool"):
        pool.swap_out([8])
    with pytest.raises(ValueError, match="outside the pool"):
        pool.copy_blocks([(0, -1)])
    with pytest.raises(ValueError, match="distinct"):
        pool.copy_blocks([(0, 3), (1, 3)])
    with pytest.raises(ValueError, match="distinct"):
        pool.copy_blocks([(0, 3), (3, 4)])
    with pytest.raises(ValueError, match="distinct"):
        pool.swap_in(pool.swap_out([1, 2]), [5, 5])
    empty = pool.swap_out([])
    assert len(empty) == 0
    pool.swap_in(empty, [])
    pool.copy_blocks([])


def test_kernel_bounds_check_reports_bad_ids(pkg):
    """Ids that skip the host checks (straight through the C ABI) are caught by the
    kernel: the unit is skipped and bit 1 of the error word is set."""
    pool = pkg.KVPool(1, 4, 4, 1, 8, torch.float32, DEV)
    pool.k[0].fill_(1.0)
    pool.v[0].fill_(2.0)
    ids = torch.tensor([1, 7], dtype=torch.int32, device=DEV)
    stage = torch.full((1 * 2 * 2 * 4 * 8,), -5.0, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    arr = ctypes.c_void_p * 1
    rc = pkg._lib.lib().pa_gather_blocks(arr(pool.k[0].data_ptr()), arr(pool.v[0].data_ptr()), 1, 4, 4 * 8 * 4,
                                         ids.data_ptr(), 2, stage.data_ptr(), err.data_ptr(),
                                         torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) & 1
    st = stage.view(1, 2, 2, 32).cpu()
    assert torch.all(st[0, 0, 0] == 1.0) and torch.all(st[0, 1, 0] == 2.0)  # block 1 moved
    assert torch.all(st[0, :, 1] == -5.0)                                       # block 7 skipped
