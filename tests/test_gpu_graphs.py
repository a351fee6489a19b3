"""CUDA-graph decode steps (graphs.DecodeStepGraph): a step captured once and replayed
with each step's metadata gives the same pool contents as the eager append (bitwise) and
the same attention as the eager kernels and the oracle, while the contexts grow from
step to step inside the bucket; a step that outgrows the bucket is refused."""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from _golden import TOL

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _setup(L=3, B=40, Hq=16, Hkv=4, D=128, seed=0):
    rng = np.random.default_rng(seed)
    ctx = np.clip(np.exp(rng.normal(np.log(300), 0.8, size=B)), 20, 900).astype(np.int64)
    width = 64                                      # 1,024 tokens per sequence fit the bucket
    nb = B * width + 8
    perm = rng.permutation(nb)
    tables = perm[:B * width].reshape(B, width).astype(np.int64)
    g = torch.Generator(device=DEV).manual_seed(seed)
    kp = [torch.randn(nb, 16, Hkv, D, generator=g, device=DEV).to(torch.bfloat16) for _ in range(L)]
    vp = [torch.randn(nb, 16, Hkv, D, generator=g, device=DEV).to(torch.bfloat16) for _ in range(L)]
    return ctx, tables, kp, vp, width


def test_replayed_decode_steps_match_eager_and_oracle(pkg, oracle):
    graphs = importlib.import_module(f"{pkg.__name__}.graphs")
    L, B, Hq, Hkv, D = 3, 40, 16, 4, 128
    ctx, tables, kp, vp, width = _setup(L, B, Hq, Hkv, D)
    kp_e = [t.clone() for t in kp]
    vp_e = [t.clone() for t in vp]
    gr = graphs.DecodeStepGraph(kp, vp, Hq, D ** -0.5, B, width)
    gen = torch.Generator(device=DEV).manual_seed(7)
    for step in range(5):
        c = ctx + 1 + step                              # this step's token is in the context
        gr.set_step(c, tables)
        for t in (gr.q, gr.k_new, gr.v_new):
            t.copy_(torch.randn(t.shape, generator=gen, device=DEV).to(t.dtype))
        if step == 0:
            gr.capture()                                # runs this step's launches once, then captures them
        else:
            gr.replay()
        # eager reference: the ordinary API on the cloned pools
        meta = pkg.StepMetadata.build(c, np.ones(B, np.int64), tables, num_tokens=B, pool_num_blocks=kp[0].shape[0],
                                      block_size=16, num_kv_heads=Hkv, device=DEV)
        bt = pkg.attach(torch.from_numpy(tables).to(DEV), meta)
        dummy = torch.zeros(1, dtype=torch.int64, device=DEV)
        for l in range(L):
            pkg.reshape_and_cache(gr.k_new[l], gr.v_new[l], kp_e[l], vp_e[l], meta.slot_mapping())
            out_e = pkg.paged_attention_cuda(gr.q[l], kp_e[l], vp_e[l], bt, dummy, dummy, D ** -0.5)
            torch.cuda.synchronize()
            assert torch.equal(kp[l], kp_e[l]) and torch.equal(vp[l], vp_e[l]), (step, l)
            np.testing.assert_allclose(gr.out[l].float().cpu().numpy(), out_e.float().cpu().numpy(), **TOL["bf16"])
        if step == 4:                                   # one layer against the oracle as well
            ref = oracle.paged_attention_gather(gr.q[0].float().cpu().numpy(), kp[0].float().cpu().numpy(),
                                                vp[0].float().cpu().numpy(), tables, c, np.ones(B, np.int64),
                                                D ** -0.5, "bf16")
            np.testing.assert_allclose(gr.out[0].float().cpu().numpy(), ref, **TOL["bf16"])
    assert gr.read_error() == 0


def test_step_outside_the_bucket_is_refused(pkg):
    graphs = importlib.import_module(f"{pkg.__name__}.graphs")
    ctx, tables, kp, vp, width = _setup(L=1, B=8)
    gr = graphs.DecodeStepGraph(kp, vp, 16, 128 ** -0.5, 8, 16)     # 256-token bucket
    with pytest.raises(graphs.BucketOverflow):
        gr.set_step(np.full(8, 300, np.int64), tables)
    gr.set_step(np.full(8, 200, np.int64), tables)
