"""End-to-end greedy-token parity through the HF model (BASELINE config 1 shape):
random-init GPT-2 124M in fp32 (seed 0), prompts of random token ids with lengths in
16..256, greedy decoding.  The CUDA executor (fused append + sm_100a attention + one-copy
metadata) and the oracle executor (the reference executor's algorithm with the numpy
gather path) run the same model on the same GPU; only the attention path differs, and
the north star requires identical greedy tokens.
"""

from __future__ import annotations

import importlib

import numpy as np
import pytest
import torch

from _engine import OracleExecutor, generate

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def gpt2():
    from transformers import GPT2Config, GPT2LMHeadModel

    torch.manual_seed(0)
    model = GPT2LMHeadModel(GPT2Config()).to(DEV).eval()
    return model


@pytest.fixture(scope="module")
def executor_mod(pkg):
    return importlib.import_module(f"{pkg.__name__}.executor")


def _prompts(n: int, seed: int):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 50257, size=int(rng.integers(16, 257))).tolist() for _ in range(n)]


def test_gpt2_fp32_greedy_tokens_match_gather_path(pkg, executor_mod, gpt2):
    prompts = _prompts(4, seed=0)
    nb, steps = 160, 24
    pool = pkg.KVPool.from_model(gpt2, num_blocks=nb, block_size=16)
    cuda_tokens = generate(executor_mod.CudaPagedExecutor(gpt2, None, pool), prompts, steps, nb)
    ref = OracleExecutor(gpt2, 12, nb, 16, 12, 64, "f32")
    ref_tokens = generate(ref, prompts, steps, nb)
    assert cuda_tokens == ref_tokens
    # Layer 0's K/V depend only on the embeddings, so both pools hold identical bytes.
    np.testing.assert_array_equal(pool.k[0].cpu().numpy(), ref.k[0])
    np.testing.assert_array_equal(pool.v[0].cpu().numpy(), ref.v[0])
    assert pkg.read_device_error() == 0


def test_gpt2_staggered_arrival_mixes_prefill_and_decode(pkg, executor_mod, gpt2):
    """Two prompts join mid-run, so their prefill runs in the same pass as the others'
    decodes (the reference's scheduler would split them; the kernels take both)."""
    prompts = _prompts(5, seed=1)
    nb, steps = 200, 16
    join = {4: [3], 9: [4]}
    pool = pkg.KVPool.from_model(gpt2, num_blocks=nb, block_size=16)
    cuda_tokens = generate(executor_mod.CudaPagedExecutor(gpt2, None, pool), prompts, steps, nb, join_at=join)
    ref_tokens = generate(OracleExecutor(gpt2, 12, nb, 16, 12, 64, "f32"), prompts, steps, nb, join_at=join)
    assert cuda_tokens == ref_tokens


def test_llama_shape_bf16_executor_first_tokens(pkg, executor_mod):
    """A reduced Llama-3 shape (GQA 32/8 heads of 128, bf16, 2 layers): the prefill pass's
    greedy token of every prompt agrees with the oracle executor's (later bf16 steps may
    legitimately flip a near-tied argmax, so they are not compared)."""
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    cfg = LlamaConfig(hidden_size=4096, intermediate_size=1024, num_attention_heads=32, num_key_value_heads=8,
                      head_dim=128, num_hidden_layers=2, vocab_size=4096, max_position_embeddings=4096)
    model = LlamaForCausalLM(cfg).to(DEV, torch.bfloat16).eval()
    prompts = [[t % 4096 for t in p] for p in _prompts(3, seed=2)]
    nb = 96
    pool = pkg.KVPool.from_model(model, num_blocks=nb, block_size=16)
    assert pool.num_kv_heads == 8 and pool.head_dim == 128 and pool.dtype == torch.bfloat16
    cuda_tokens = generate(executor_mod.CudaPagedExecutor(model, None, pool), prompts, 3, nb)
    ref_tokens = generate(OracleExecutor(model, 2, nb, 16, 8, 128, "bf16"), prompts, 3, nb)
    assert [t[0] for t in cuda_tokens] == [t[0] for t in ref_tokens]
