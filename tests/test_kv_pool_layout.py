"""The pool the kernels read, on CPU: the reference's block-major per-layer layout
(inference_server/core/kv_pool.py:106-139, tested by the reference's tests/test_kv_pool.py),
its flat slot addressing (block * block_size + offset, core/block_table.py:143-159, as the
reference's executor indexes pool.view(-1, Hkv, D)), sizes read off model configs the way
ModelDims.from_model does (kv_pool.py:47-61), and HostBlocks' length and byte count
(kv_pool.py:80-102)."""

from __future__ import annotations

import torch


def test_pool_is_block_major_per_layer_and_zeroed(pkg):
    pool = pkg.KVPool(3, 64, 4, 3, 8, torch.float32, "cpu")
    assert len(pool.k) == len(pool.v) == 3
    ptrs = set()
    for t in pool.k + pool.v:
        assert t.shape == (64, 4, 3, 8) and t.dtype == torch.float32 and t.is_contiguous()
        assert not bool(t.any())
        ptrs.add(t.data_ptr())
    assert len(ptrs) == 6                                # every layer's K and V is its own tensor
    assert pool.num_blocks == 64 and pool.block_size == 4 and pool.num_slots == 256


def test_flat_slot_is_block_times_block_size_plus_offset(pkg):
    pool = pkg.KVPool(1, 16, 4, 2, 8, torch.float32, "cpu")
    flat = pool.k[0].view(-1, 2, 8)                      # the reference executor's index_copy_ target
    for slot in (0, 3, 4, 37, 63):
        flat[slot] = float(slot + 1)
        assert bool((pool.k[0][slot // 4, slot % 4] == slot + 1).all())


def test_sizes_come_from_the_model_config(pkg):
    from transformers import GPT2Config, GPT2LMHeadModel, LlamaConfig, LlamaForCausalLM

    torch.manual_seed(0)
    gpt2 = GPT2LMHeadModel(GPT2Config(n_layer=2, n_embd=64, n_head=4, vocab_size=128, n_positions=64))
    pool = pkg.KVPool.from_model(gpt2, num_blocks=8, block_size=16)
    assert len(pool.k) == 2 and pool.k[0].shape == (8, 16, 4, 16) and pool.k[0].dtype == torch.float32

    llama = LlamaForCausalLM(LlamaConfig(hidden_size=64, num_attention_heads=8, num_key_value_heads=2,
                                         num_hidden_layers=3, intermediate_size=128, vocab_size=128))
    pool = pkg.KVPool.from_model(llama, num_blocks=8, block_size=16, dtype=torch.bfloat16)
    assert len(pool.v) == 3 and pool.v[0].shape == (8, 16, 2, 8) and pool.v[0].dtype == torch.bfloat16


def test_host_blocks_report_length_and_bytes(pkg):
    k = [torch.zeros(5, 16, 2, 8, dtype=torch.bfloat16) for _ in range(3)]
    v = [torch.zeros(5, 16, 2, 8, dtype=torch.bfloat16) for _ in range(3)]
    h = pkg.HostBlocks(k=k, v=v)
    assert len(h) == 5
    assert h.nbytes == 2 * 3 * 5 * 16 * 2 * 8 * 2
    assert len(pkg.HostBlocks(k=[], v=[])) == 0
