"""The CPU oracle against the reference's own outputs (committed golden vectors).

These pin the oracle before anything is compared with it: every attention case the
generator recorded from the reference's ``paged_attention_gather``, the reference
test-suite's known-answer ``_token_map`` case, ``_pack`` over real reference sequences
and the pool after ``_PagedCache.update``.
"""

from __future__ import annotations

import numpy as np
import pytest

from _golden import attention_cases, decode_stored, load, load_attention

CASES = attention_cases()


def test_golden_set_is_complete():
    # 9 reference test shapes + 2 more padding seeds + GQA + non-pow2 + 2 half dtypes
    # + 7 block-size-16 serving shapes.
    assert len(CASES) == 22


@pytest.mark.parametrize("case", CASES)
def test_oracle_matches_reference_gather(case, oracle):
    g = load_attention(case)
    out = oracle.paged_attention_gather(g["query"], g["k_pool"], g["v_pool"], g["block_tables"],
                                        g["context_lens"], g["query_lens"], g["scale"], g["dtype"])
    assert out.shape == g["out"].shape
    if g["dtype"] == "f32":
        np.testing.assert_allclose(out, g["out"], atol=2e-6, rtol=2e-6)
    else:
        # Same rounding points as torch; residual differences come from the float32
        # accumulation order inside the two matmuls, then one half-precision rounding.
        ulp = 2.0 ** -7 if g["dtype"] == "bf16" else 2.0 ** -10
        np.testing.assert_allclose(out, g["out"], atol=2 * ulp, rtol=2 * ulp)


MIRROR_CASES = sorted(load("mirror").keys())


@pytest.mark.parametrize("case", MIRROR_CASES)
def test_mirror_matches_reference_mirror(case, oracle):
    """The secondary oracle: the reference's PyTorch mirror of its Triton kernel
    (attention_triton.py:309-384: per-block online softmax, float32 throughout) against
    this oracle's restatement, on the same inputs."""
    g = load_attention(case)
    want = decode_stored(load("mirror")[case], g["dtype"])
    out = oracle.paged_attention_mirror(g["query"], g["k_pool"], g["v_pool"], g["block_tables"],
                                        g["context_lens"], g["query_lens"], g["scale"], g["dtype"])
    if g["dtype"] == "f32":
        np.testing.assert_allclose(out, want, atol=2e-6, rtol=2e-6)
    else:  # float32 summation order, then one rounding to the storage dtype
        ulp = 2.0 ** -7 if g["dtype"] == "bf16" else 2.0 ** -10
        np.testing.assert_allclose(out, want, atol=ulp, rtol=ulp)


@pytest.mark.parametrize("case", MIRROR_CASES)
def test_mirror_agrees_with_gather(case, oracle):
    """The two reference algorithms (gather path and the kernel mirror) agree within the
    reference's own tolerance for its mirror tier (tests/test_paged_attention_triton.py:97-128:
    1e-5 in fp32; the half cases within the 2e-2 kernel-tier bound)."""
    g = load_attention(case)
    out = oracle.paged_attention_mirror(g["query"], g["k_pool"], g["v_pool"], g["block_tables"],
                                        g["context_lens"], g["query_lens"], g["scale"], g["dtype"])
    tol = 1e-5 if g["dtype"] == "f32" else 2e-2
    np.testing.assert_allclose(out, g["out"], atol=tol, rtol=tol)


def test_token_map_known_answer(oracle):
    """tests/test_paged_attention_triton.py:140-147 of the reference."""
    s, p, cu = oracle.token_map([6, 10, 4], [1, 3, 4])
    assert s.tolist() == [0, 1, 1, 1, 2, 2, 2, 2]
    assert p.tolist() == [5, 7, 8, 9, 0, 1, 2, 3]
    assert cu.tolist() == [0, 1, 4, 8]


@pytest.mark.parametrize("tag", ["known", "random"])
def test_token_map_matches_reference(tag, oracle):
    z = load("token_map")
    s, p, cu = oracle.token_map(z[f"{tag}_context_lens"], z[f"{tag}_query_lens"])
    np.testing.assert_array_equal(s, z[f"{tag}_seq_idx"])
    np.testing.assert_array_equal(p, z[f"{tag}_q_pos"])
    np.testing.assert_array_equal(cu, z[f"{tag}_cu"])


def test_pack_matches_reference(oracle):
    z = load("pack")
    seqs = [(z["blocks"][i][: z["num_blocks_per_seq"][i]].tolist(), int(z["num_cached"][i]),
             int(z["num_new"][i])) for i in range(len(z["num_cached"]))]
    got = oracle.pack_step(seqs, int(z["block_size"]))
    for key in ("write_slots", "block_tables", "context_lens", "query_lens", "ends", "position_ids"):
        np.testing.assert_array_equal(got[key], z[key], err_msg=key)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_kv_append_matches_reference(dt, oracle):
    z = load(f"kv_append_{dt}")
    # [1, H, T, D] -> [T, H, D], the layout _PagedCache.update scatters.
    key = z["key"][0].transpose(1, 0, 2)
    val = z["value"][0].transpose(1, 0, 2)
    np.testing.assert_array_equal(oracle.kv_append(z["k_before"], z["write_slots"], key), z["k_after"])
    np.testing.assert_array_equal(oracle.kv_append(z["v_before"], z["write_slots"], val), z["v_after"])


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_block_moves_match_reference(dt, oracle):
    """swap_out / swap_in (kv_pool.py:142-182) and _copy_block (paged_executor.py:265-270)
    of the reference pool, bit for bit (half dtypes compared as raw patterns)."""
    z = load(f"blocks_{dt}")
    hk, hv = oracle.swap_out(z["k_before"], z["v_before"], z["swap_out_blocks"])
    np.testing.assert_array_equal(hk, z["host_k"])
    np.testing.assert_array_equal(hv, z["host_v"])
    k1, v1 = oracle.swap_in(z["k_before"], z["v_before"], hk, hv, z["swap_in_blocks"])
    np.testing.assert_array_equal(k1, z["k_after_swap_in"])
    np.testing.assert_array_equal(v1, z["v_after_swap_in"])
    k2, v2 = oracle.copy_block(k1, v1, z["copy_pairs"].tolist())
    np.testing.assert_array_equal(k2, z["k_after_copy"])
    np.testing.assert_array_equal(v2, z["v_after_copy"])
    with pytest.raises(ValueError, match="host blocks into"):
        oracle.swap_in(z["k_before"], z["v_before"], hk, hv, z["swap_in_blocks"][:-1])


def test_slots_raise_past_capacity(oracle):
    with pytest.raises(IndexError):
        oracle.slots([3, 1], 16, 33)
    assert oracle.slots([3, 1], 16, 18).tolist() == list(range(48, 64)) + [16, 17]


def test_oracle_contract_errors(oracle):
    """Same ValueError texts as the reference's _check (tests/test_paged_attention.py:165-179)."""
    g = load_attention("prefill_on_boundary")
    args = (g["query"], g["k_pool"], g["v_pool"], g["block_tables"])
    with pytest.raises(ValueError, match="query_len exceeds context_len"):
        oracle.paged_attention_gather(*args, g["context_lens"] - 1, g["query_lens"], g["scale"])
    with pytest.raises(ValueError, match="query_lens sum"):
        oracle.paged_attention_gather(g["query"][:-1], *args[1:], g["context_lens"], g["query_lens"], g["scale"])


def test_bf16_rounding_is_nearest_even(oracle):
    x = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8, -2.5, np.inf, 1e-40], dtype=np.float32)
    r = oracle.round_to(x, "bf16")
    assert r[0] == 1.0                      # tie -> even
    assert r[1] == 1.0 + 2.0 ** -6          # tie -> even (up)
    assert r[2] == -2.5 and np.isinf(r[3])


def test_oracle_executor_reproduces_reference_greedy_tokens():
    """The oracle executor (tests/_engine.py) that the GPU token-parity tests compare the
    CUDA executor against reproduces the reference's own PagedExecutor token for token
    (random-init GPT-2 124M, fp32, CPU; golden made by the reference)."""
    import torch
    from transformers import GPT2Config, GPT2LMHeadModel

    from _engine import OracleExecutor, generate

    z = load("gpt2_greedy_cpu")
    prompts = [p.tolist() for p in np.split(z["prompts"], np.cumsum(z["prompt_lens"])[:-1])]
    torch.manual_seed(0)
    model = GPT2LMHeadModel(GPT2Config()).eval()
    nb = int(z["num_blocks"])
    tokens = generate(OracleExecutor(model, 12, nb, 16, 12, 64, "f32"), prompts, int(z["steps"]), nb)
    assert tokens == z["tokens"].tolist()
