"""KV-head tensor parallelism on GPUs (BASELINE config 5 shape, reduced d_model): two
ranks over NCCL, each with the sm_100a append + attention kernels on its 4 of 8 KV heads
and its row slice of o_proj, one all-reduce; the result must match the single-GPU layer.
Skipped where fewer than two GPUs are visible (run it with a 2-GPU allocation)."""

from __future__ import annotations

import datetime
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
HEADS, KV_HEADS, D, D_MODEL = 64, 8, 128, 1024
LENGTHS = [(900, 1), (3000, 1), (17, 1), (300, 300), (1200, 40)]


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _inputs():
    sys.path.insert(0, str(ROOT / "tests"))
    from _batches import ragged_batch
    from oracle import paged_attention_oracle as oracle

    q, kp, vp, bt, cl, ql = ragged_batch(LENGTHS, bs=16, d=D, heads=HEADS, kv_heads=KV_HEADS,
                                         dtype=torch.bfloat16, seed=21)
    g = torch.Generator().manual_seed(22)
    t = q.shape[0]
    k_new = torch.randn(t, KV_HEADS, D, generator=g).to(torch.bfloat16)
    v_new = torch.randn(t, KV_HEADS, D, generator=g).to(torch.bfloat16)
    w = (torch.randn(D_MODEL, HEADS * D, generator=g) / (HEADS * D) ** 0.5).to(torch.bfloat16)
    seqs = [(bt[i, :-(-c // 16)].tolist(), c - n, n) for i, (c, n) in enumerate(LENGTHS)]
    slots = torch.from_numpy(oracle.pack_step(seqs, 16)["write_slots"])
    return q, kp, vp, bt, cl, ql, k_new, v_new, w, slots


def _layer_args(dev, qs, ks, batch):
    q, kp, vp, bt, cl, ql, k_new, v_new, w, slots = batch
    return (q[:, qs].contiguous().to(dev), k_new[:, ks].contiguous().to(dev), v_new[:, ks].contiguous().to(dev),
            kp[:, :, ks].contiguous().to(dev), vp[:, :, ks].contiguous().to(dev), bt.to(dev), cl.to(dev),
            ql.to(dev), D ** -0.5, slots.to(dev))


def _worker(rank: int, world: int, port: int, out_dir: str) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    sys.path.insert(0, str(ROOT))
    import importlib

    import torch.distributed as dist

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from __graft_entry__ import import_package

        import_package()
        tp = importlib.import_module("llm_inference_server_b200.tensor_parallel")
        batch = _inputs()
        qs, ks = tp.kv_head_shard(HEADS, KV_HEADS, rank, world)
        layer = tp.KVHeadParallelAttention(w_o=tp.o_proj_shard(batch[8], HEADS, D, rank, world, KV_HEADS).to(dev))
        out = layer(*_layer_args(dev, qs, ks, batch))
        torch.cuda.synchronize(dev)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), out.float().cpu().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_gpu_kv_head_parallel_layer_matches_single_gpu(pkg, tmp_path):
    ctx = torch.multiprocessing.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert not p.is_alive() and p.exitcode == 0, f"rank exit code {p.exitcode}"
    import importlib

    tp = importlib.import_module(f"{pkg.__name__}.tensor_parallel")
    batch = _inputs()
    dev = torch.device("cuda", 0)
    full = tp.KVHeadParallelAttention(w_o=batch[8].t().contiguous().to(dev))
    ref = full(*_layer_args(dev, slice(0, HEADS), slice(0, KV_HEADS), batch)).float().cpu().numpy()
    for r in range(2):
        np.testing.assert_allclose(np.load(tmp_path / f"rank{r}.npy"), ref, atol=2e-2, rtol=2e-2)
