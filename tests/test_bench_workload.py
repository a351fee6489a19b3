"""The benchmark's workload arithmetic, on CPU: the seeded batches it times and the
algorithmic bytes / FLOPs its rooflines divide by.  The context-length calibration meets
the stated clipped mean, block tables never alias (the fused append writes every new
token to a distinct slot), and attention_bytes / prefill_flops equal brute-force counts of
what the decode and causal prefill passes must touch."""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


@pytest.mark.parametrize("mean,sigma,lo,hi", [(4096.0, 0.9, 128, 16384), (8192.0, 0.9, 128, 32768)])
def test_clipped_lognormal_meets_the_stated_mean(mean, sigma, lo, hi):
    mu = bench.clipped_lognormal_mu(mean, sigma, lo, hi)
    x = np.clip(np.exp(np.random.default_rng(0).normal(mu, sigma, size=2_000_000)), lo, hi)
    assert abs(x.mean() / mean - 1.0) < 5e-3


def _small(**kw):
    args = dict(batch=24, layers=2, heads=8, kv_heads=2, head_dim=64, block_size=16, mean_ctx=300.0, lo=20,
                hi=900, sigma=0.9, seed=3, max_steps=5, churn=0.25, prompt_lo=17, prompt_hi=90)
    args.update(kw)
    return bench.Workload(**args)


def test_block_tables_never_alias():
    wl = _small()
    used = []
    for i, c in enumerate(wl.ctx0):
        n = -(-(int(c) + 5) // 16)                     # the last step's context still fits
        row = wl.tables[i, :n]
        assert (row >= 0).all() and (row < wl.num_blocks).all()
        used.extend(row.tolist())
    for row in wl.churn_tables[:wl.n_churn]:
        used.extend(row.tolist())
    assert len(used) == len(set(used))


def test_attention_bytes_is_the_brute_force_count():
    wl = _small()
    for step in (0, 3):
        for elem in (2, 4):
            ctx = wl.context_lens(step)
            kv = sum(int(c) * wl.kv_heads * wl.head_dim * elem for c in ctx) * 2            # K and V, once
            qo = wl.batch * wl.heads * wl.head_dim * elem * 2                                # q in, out
            ids = sum(-(-int(c) // wl.block_size) for c in ctx) * 4                          # int32 block ids
            assert wl.attention_bytes(step, elem) == kv + qo + ids + 8 * wl.batch


def test_prefill_flops_count_causal_keys_only():
    wl = _small()
    for step in range(5):
        visible = sum(t + 1 for n in wl.prompt_lens(step) for t in range(int(n)))          # keys 0..t
        assert wl.prefill_flops(step) == pytest.approx(4.0 * wl.heads * wl.head_dim * visible, rel=1e-12)


def test_config3_workload_is_the_recorded_one():
    """Seed 0 of BASELINE config 3 (the default bench line): 256 contexts of mean ~4096
    summing to 1,058,916 tokens at step 0, 13 churn prompts per step."""
    w = bench.WORKLOADS["config3"]
    wl = bench.Workload(batch=256, layers=32, heads=w["heads"], kv_heads=w["kv_heads"], head_dim=w["head_dim"],
                        block_size=16, mean_ctx=w["mean_ctx"], lo=w["lo"], hi=w["hi"], sigma=0.9, seed=0,
                        max_steps=36, churn=w["churn"])
    assert int(wl.ctx0.sum()) == 1_058_916
    assert wl.n_churn == 13
    assert 128 <= wl.ctx0.min() and wl.ctx0.max() <= 16384
    assert 256 <= wl.prompts.min() and wl.prompts.max() <= 2048


# ------------------------------------------------------------------ ServeSim vs the reference
def _sim_log(requests, num_blocks, max_running, steps):
    sim = bench.ServeSim(num_blocks, 16, max_running)
    seqs = [bench.SimSeq(i, p, m) for i, (p, m) in enumerate(requests)]
    for s in seqs:
        sim.add(s)
    log = []
    for _ in range(steps):
        if not sim.has_work:
            break
        batch = sim.schedule()
        if batch:
            log.append([(f"r{s.sid}", s.feed) for s in batch])
            sim.finish_pass(batch)
    return log, sim.preemptions, sim.completed


def _reference_log(requests, num_blocks, max_running, steps, monkeypatch):
    import _reference

    _reference.require()
    sys.path.insert(0, str(_reference.REF))
    import importlib

    config = importlib.import_module("inference_server.config")
    scheduler = importlib.import_module("inference_server.core.scheduler")
    allocator = importlib.import_module("inference_server.core.block_allocator")
    sequence = importlib.import_module("inference_server.core.sequence")
    monkeypatch.setattr(config.CONFIG, "block_size", 16)
    monkeypatch.setattr(config.CONFIG, "max_running", max_running)
    monkeypatch.setattr(config.CONFIG, "preemption", "recompute")
    monkeypatch.setattr(config.CONFIG, "max_queue_depth", 10_000)

    class Counting:
        def __init__(self):
            self.log = []

        def execute(self, seqs):
            self.log.append([(s.seq_id, len(s.next_input_ids)) for s in seqs])
            for s in seqs:
                s.num_cached += len(s.next_input_ids)
            return [1] * len(seqs)

    ex = Counting()
    sched = scheduler.Scheduler(ex, -1, allocator=allocator.BlockAllocator(num_blocks), pool=None)
    for i, (p, m) in enumerate(requests):
        sched.add(sequence.Sequence(seq_id=f"r{i}", prompt_token_ids=[7] * p, max_tokens=m))
    for _ in range(steps):
        if not sched.has_work:
            break
        sched.step()
    st = sched.stats()
    return ex.log, st["preemptions"], st["completed"]


@pytest.mark.parametrize("num_blocks,max_running,seed", [(40, 8, 0), (64, 16, 1), (2000, 32, 2)])
def test_serve_sim_takes_the_reference_schedulers_decisions(num_blocks, max_running, seed, monkeypatch):
    """config 5's serving run uses ServeSim in place of the reference Scheduler; on the
    same requests both run the same passes in the same order (sequences, tokens fed),
    preempt as often and complete as many requests — including pools small enough that
    recompute preemption fires repeatedly."""
    rng = np.random.default_rng(seed)
    reqs = [(int(rng.integers(20, 300)), int(rng.integers(5, 90))) for _ in range(24)]
    reqs = [(p, m) for p, m in reqs if -(-(p + m - 1) // 16) <= num_blocks]
    sim = _sim_log(reqs, num_blocks, max_running, 5000)
    ref = _reference_log(reqs, num_blocks, max_running, 5000, monkeypatch)
    assert sim[0] == ref[0]
    assert sim[1:] == ref[1:]
    if num_blocks <= 64:
        assert sim[1] > 0
