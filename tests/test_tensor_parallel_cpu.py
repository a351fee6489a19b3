"""KV-head tensor parallelism, host logic on CPU: two gloo ranks each run their shard of
one attention layer (heads, KV pool slice, o_proj row slice, all-reduce) and must equal
the single-device layer; a rank that leaves before the collective makes the other fail
within the process-group timeout instead of hanging.

The attention and append inside the ranks are the CPU oracle wrapped in the kernels'
signatures (the CUDA kernels themselves are covered by the -m gpu tests); what is
tested here is the sharding arithmetic and the collective.
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
HEADS, KV_HEADS, D, D_MODEL, BS = 16, 4, 32, 64, 16
LENGTHS = [(40, 1), (70, 1), (33, 33), (20, 7)]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs():
    sys.path.insert(0, str(ROOT / "tests"))
    from _batches import ragged_batch

    q, kp, vp, bt, cl, ql = ragged_batch(LENGTHS, bs=BS, d=D, heads=HEADS, kv_heads=KV_HEADS, seed=3)
    g = torch.Generator().manual_seed(9)
    t = q.shape[0]
    k_new = torch.randn(t, KV_HEADS, D, generator=g)
    v_new = torch.randn(t, KV_HEADS, D, generator=g)
    w = torch.randn(D_MODEL, HEADS * D, generator=g) / (HEADS * D) ** 0.5     # nn.Linear weight [out, in]
    from oracle import paged_attention_oracle as oracle

    seqs = [(bt[i, :-(-c // BS)].tolist(), c - n, n) for i, (c, n) in enumerate(LENGTHS)]
    slots = torch.from_numpy(oracle.pack_step(seqs, BS)["write_slots"])
    return q, kp, vp, bt, cl, ql, k_new, v_new, w, slots


def _oracle_fns():
    from oracle import paged_attention_oracle as oracle

    def attention(q, k_pool, v_pool, bt, cl, ql, scale):
        return torch.from_numpy(oracle.paged_attention_gather(q.numpy(), k_pool.numpy(), v_pool.numpy(), bt.numpy(),
                                                              cl.numpy(), ql.numpy(), scale, "f32"))

    def append(k, v, k_pool, v_pool, slots):
        k_pool.copy_(torch.from_numpy(oracle.kv_append(k_pool.numpy(), slots.numpy(), k.numpy())))
        v_pool.copy_(torch.from_numpy(oracle.kv_append(v_pool.numpy(), slots.numpy(), v.numpy())))

    return attention, append


def _worker(rank: int, world: int, port: int, out_dir: str, leave_early: bool) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, str(ROOT))
    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    from __graft_entry__ import import_package

    import_package()
    import importlib

    tp = importlib.import_module("llm_inference_server_b200.tensor_parallel")
    q, kp, vp, bt, cl, ql, k_new, v_new, w, slots = _inputs()
    qs, ks = tp.kv_head_shard(HEADS, KV_HEADS, rank, world)
    attention, append = _oracle_fns()
    layer = tp.KVHeadParallelAttention(w_o=tp.o_proj_shard(w, HEADS, D, rank, world, KV_HEADS),
                                       attention=attention, append=append)
    if leave_early and rank == 1:
        os._exit(0)                       # leaves between steps, nothing in flight
    try:
        out = layer(q[:, qs].contiguous(), k_new[:, ks].contiguous(), v_new[:, ks].contiguous(),
                    kp[:, :, ks].contiguous(), vp[:, :, ks].contiguous(), bt, cl, ql, D ** -0.5, slots)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), out.numpy())
    except Exception as exc:  # the collective failed: record it for the parent
        Path(out_dir, f"rank{rank}.err").write_text(type(exc).__name__ + ": " + str(exc)[:200])
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _spawn(world: int, tmp_path, leave_early: bool = False):
    ctx = torch.multiprocessing.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), leave_early)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
    return procs


def test_shards_cover_every_head_once():
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import import_package

    import_package()
    import importlib

    tp = importlib.import_module("llm_inference_server_b200.tensor_parallel")
    for world in (1, 2, 4, 8):
        qh, kh = [], []
        for r in range(world):
            qs, ks = tp.kv_head_shard(64, 8, r, world)
            qh += list(range(64))[qs]
            kh += list(range(8))[ks]
            assert all(h // 8 in range(8)[ks] for h in range(64)[qs])   # a GQA group stays together
        assert qh == list(range(64)) and kh == list(range(8))
    with pytest.raises(ValueError):
        tp.kv_head_shard(64, 8, 0, 3)


def test_two_rank_kv_head_parallel_layer_matches_single_device(tmp_path):
    _spawn(2, tmp_path)
    q, kp, vp, bt, cl, ql, k_new, v_new, w, slots = _inputs()
    attention, append = _oracle_fns()
    append(k_new, v_new, kp, vp, slots)
    ref = attention(q, kp, vp, bt, cl, ql, D ** -0.5).reshape(q.shape[0], -1) @ w.t()
    for r in range(2):
        assert not (tmp_path / f"rank{r}.err").exists(), (tmp_path / f"rank{r}.err").read_text()
        np.testing.assert_allclose(np.load(tmp_path / f"rank{r}.npy"), ref.numpy(), atol=1e-5, rtol=1e-5)


def test_a_rank_that_leaves_fails_the_other_within_the_timeout(tmp_path):
    """Rank 1 exits before the all-reduce; rank 0's collective must raise (process-group
    timeout 5 s) rather than wait forever."""
    _spawn(2, tmp_path, leave_early=True)
    err = tmp_path / "rank0.err"
    assert err.exists(), "rank 0 completed a collective its peer never joined"
    assert not (tmp_path / "rank0.npy").exists()
