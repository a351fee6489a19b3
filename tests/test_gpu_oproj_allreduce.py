"""The fused o_proj GEMM + all-reduce (tensor_parallel.FusedOProjAllReduce, the C ABI's
pa_oproj_allreduce) on one GPU, where it is the tcgen05 GEMM alone through the same two
kernels: its output is the float64 product rounded once to the storage dtype (within one
unit in the last place), for partial row tiles, strided activations, bf16 and fp16, and
across calls that reuse the output slots; the tensor-parallel layer gives the same result
through it as through torch.matmul.  The two-rank exchange is tested in
test_gpu_peer_allreduce.py."""

from __future__ import annotations

import importlib

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tp(pkg):
    return importlib.import_module(f"{pkg.__name__}.tensor_parallel")


def _case(rows, k, n, dtype, seed, a_stride=None):
    g = torch.Generator().manual_seed(seed)
    width = a_stride or k
    a_full = torch.randn(rows, width, generator=g).to(dtype)
    a = a_full[:, :k]
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(dtype)
    ref = a.double() @ w.double().t()
    return a_full.to(DEV)[:, :k], w.to(DEV), ref


def _assert_one_ulp(got: torch.Tensor, ref: torch.Tensor, dtype) -> None:
    """|got - ref| within one unit in the last place of the storage dtype (plus float32
    accumulation noise far below it)."""
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    err = (got.double().cpu() - ref).abs()
    bound = ulp * ref.abs() + 1e-4 * float(ref.abs().max())
    assert bool((err <= bound).all()), float((err - bound).max())


@pytest.mark.parametrize("rows,k,n,dtype,a_stride", [
    (512, 1024, 1024, torch.bfloat16, None),     # the config-5 tp8 shape, narrowed to n = 1024
    (200, 256, 512, torch.bfloat16, 320),        # partial last row tile, strided activations
    (1, 64, 256, torch.float16, None),           # one row, one k step, fp16
])
def test_single_rank_is_the_rounded_product(pkg, rows, k, n, dtype, a_stride):
    fused = _tp(pkg).FusedOProjAllReduce(512, n, dtype, device=DEV)
    a, w, ref = _case(rows, k, n, dtype, seed=rows + k, a_stride=a_stride)
    out = fused(a, w)
    torch.cuda.synchronize()
    fused.check()
    assert out.shape == (rows, n) and out.dtype == dtype
    _assert_one_ulp(out, ref, dtype)


def test_output_slots_survive_the_next_call(pkg):
    fused = _tp(pkg).FusedOProjAllReduce(256, 256, torch.bfloat16, device=DEV)
    outs, refs = [], []
    for i in range(5):
        a, w, ref = _case(256, 512, 256, torch.bfloat16, seed=10 + i)
        outs.append(fused(a, w))
        refs.append(ref)
        if i >= 1:                          # SLOTS = 2: the previous call's output is intact
            torch.cuda.synchronize()
            _assert_one_ulp(outs[i - 1], refs[i - 1], torch.bfloat16)
    torch.cuda.synchronize()
    fused.check()
    _assert_one_ulp(outs[-1], refs[-1], torch.bfloat16)


def test_tensor_parallel_layer_uses_the_fused_gemm(pkg):
    tp = _tp(pkg)
    from test_gpu_tensor_parallel import D, HEADS, KV_HEADS, _inputs, _layer_args

    batch = _inputs()
    qs, ks = tp.kv_head_shard(HEADS, KV_HEADS, 0, 1)
    w_o = tp.o_proj_shard(batch[8], HEADS, D, 0, 1, KV_HEADS).to(DEV)
    args = _layer_args(DEV, qs, ks, batch)
    rows = args[0].shape[0]
    n = w_o.shape[1]
    if n % 256:
        pytest.skip(f"d_model {n} is not a multiple of the fused GEMM's 256-column tile")
    fused = tp.FusedOProjAllReduce(rows, n, torch.bfloat16, device=DEV)
    got = tp.KVHeadParallelAttention(w_o=w_o, fused=fused)(*args).clone()
    args = _layer_args(DEV, qs, ks, batch)
    plain = tp.KVHeadParallelAttention(w_o=w_o)(*args)
    torch.cuda.synchronize()
    fused.check()
    torch.testing.assert_close(got.float(), plain.float(), rtol=2e-2, atol=2e-2)
