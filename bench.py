"""Benchmark of the paged-attention hot path on B200 (one JSON line on rank 0).

Workload (the shape the north star's >=70 %-of-HBM target is quoted
on): Llama-3-8B-shape GQA attention, 32 query heads / 8 KV heads / head_dim 128, bf16,
32 layers, KV block size 16; a continuous batch of 256 sequences whose contexts are
lognormal with mean 4096 clipped to 128..16384 (seed 0 per rank), with ~5 % per-step
admit/evict churn whose new prompts (256..2048 tokens) run through varlen paged
prefill.  Synthetic data: pools, queries and new K/V rows are N(0,1); block tables are a
seeded permutation of the pool (non-contiguous, unsorted).  The pools are real
per-layer allocations (about 140 GB of KV for 32 layers), so every layer streams its
own ~4.3 GB from HBM; each layer's KV is far larger than the 126 MB L2, which is this
benchmark's answer to L2 flushing.

One step = what the reference's scheduler runs for that batch (it never mixes prefill
and decode in one pass, inference_server/core/scheduler.py:425-437):
  1. a prefill pass for the 13 newly admitted prompts — their metadata, then per layer
     the fused K+V append of their tokens and tcgen05 varlen prefill attention;
  2. a decode pass for all 256 sequences — metadata, then per layer the append of the
     256 new tokens and split-K decode attention (tensor-pipe MMA) + combine.
Decode contexts grow by one token per step.  Tokens generated per step: 256 + 13.

* ``value``  generated tokens/s with inputs resident in HBM (per-step metadata uploaded
  before the timed region), CUDA events on the launching stream, max over ranks.
* ``e2e``    the same through the public API with HOST buffers: every step plans and
  uploads its metadata, copies each layer's q / new K / new V from pinned host memory
  and reads each layer's attention output back.  The uploads and read-backs run on two
  copy streams into double-buffered device slots, overlapped with the neighbouring
  layers' compute (PCIe carries both directions at once), as a serving loop would.
* ``roofline``  the decode attention launches (the dominant kernel): algorithmic bytes
  (K+V of every context once, q and out, block ids, lengths) over their CUDA-event time,
  against the measured HBM copy peak.  ``prefill_roofline``: the prefill attention
  launches' causal FLOPs over their time, against the measured sustained bf16 peak.
* ``cpu_baseline``  the CPU oracle (a numpy port of the reference's gather path) on a
  bounded sample of the same workload, on this host's cores.

Multi-GPU: request-level replicas, one process per GPU, each with its own batch and
pools; no collective on the data path (``scaling: weak``).  ``--impl reference`` times
the reference algorithm's CPU port instead (rank 0 only).
"""

from __future__ import annotations

import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged decode tok/s at 1/2/4/8 B200; paged-attn HBM GB/s vs 8 TB/s peak"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS_SUSTAINED = 1400.0
NOMINAL_HBM_GBS = 8000.0


def clipped_lognormal_mu(mean: float, sigma: float, lo: float, hi: float) -> float:
    """mu such that E[clip(exp(N(mu, sigma)), lo, hi)] == mean (bisection on the closed
    form), so "mean 4096 clipped to 128..16384" holds after the clip."""
    from math import erf, exp, log, sqrt

    def cdf(x):
        return 0.5 * (1.0 + erf(x / sqrt(2.0)))

    def clipped_mean(mu):
        a, b = (log(lo) - mu) / sigma, (log(hi) - mu) / sigma
        mid = exp(mu + sigma * sigma / 2) * (cdf(b - sigma) - cdf(a - sigma))
        return lo * cdf(a) + mid + hi * (1.0 - cdf(b))

    a, b = log(lo), log(hi)
    for _ in range(100):
        m = 0.5 * (a + b)
        a, b = (m, b) if clipped_mean(m) < mean else (a, m)
    return 0.5 * (a + b)


class Workload:
    """The seeded batch of one rank: decode sequences plus per-step churn prompts."""

    def __init__(self, batch: int, layers: int, heads: int, kv_heads: int, head_dim: int, block_size: int,
                 mean_ctx: float, lo: int, hi: int, sigma: float, seed: int, max_steps: int, churn: float,
                 prompt_lo: int = 256, prompt_hi: int = 2048, median_ctx: float | None = None):
        self.batch, self.layers, self.heads, self.kv_heads = batch, layers, heads, kv_heads
        self.head_dim, self.block_size = head_dim, block_size
        rng = np.random.default_rng(seed)
        mu = np.log(median_ctx) if median_ctx else clipped_lognormal_mu(mean_ctx, sigma, lo, hi)
        self.ctx0 = np.clip(np.exp(rng.normal(mu, sigma, size=batch)), lo, hi).astype(np.int64)
        need = -(-(self.ctx0 + max_steps) // block_size)
        self.n_churn = int(round(churn * batch))
        churn_width = -(-prompt_hi // block_size)
        self.num_blocks = int(need.sum()) + self.n_churn * churn_width + 16
        perm = rng.permutation(self.num_blocks)
        self.tables = np.zeros((batch, int(need.max())), dtype=np.int64)
        off = 0
        for i, n in enumerate(need):
            self.tables[i, :n] = perm[off:off + n]
            off += n
        self.churn_tables = np.zeros((max(self.n_churn, 1), churn_width), dtype=np.int64)
        for i in range(self.n_churn):
            self.churn_tables[i] = perm[off:off + churn_width]
            off += churn_width
        self.query_lens = np.ones(batch, dtype=np.int64)
        # prompt lengths of every step's churn (uniform 256..2048, seeded)
        self.prompts = rng.integers(prompt_lo, prompt_hi + 1, size=(max_steps, max(self.n_churn, 1)))

    def context_lens(self, step: int) -> np.ndarray:
        return self.ctx0 + step

    def prompt_lens(self, step: int) -> np.ndarray:
        return self.prompts[step, :self.n_churn].astype(np.int64)

    def attention_bytes(self, step: int, elem: int) -> int:
        """Algorithmic HBM bytes of one layer's decode attention at `step`."""
        ctx = self.context_lens(step)
        kv = int(ctx.sum()) * self.kv_heads * self.head_dim * 2 * elem
        qo = 2 * self.batch * self.heads * self.head_dim * elem
        ids = int((-(-ctx // self.block_size)).sum()) * 4
        return kv + qo + ids + 8 * self.batch

    def prefill_flops(self, step: int) -> float:
        """Causal attention FLOPs of one layer's prefill pass at `step`:
        4 * Hq * D * sum over prompts of sum_{t<L} (t + 1)."""
        lens = self.prompt_lens(step).astype(np.float64)
        return float(4.0 * self.heads * self.head_dim * np.sum(lens * (lens + 1) / 2))


def _measured_peaks() -> tuple[float, float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), float(d["bf16_tflops_sustained"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS_SUSTAINED, "fallback"


class QuietHost:
    """Keeps Python's cyclic garbage collector out of a timed region: everything alive is
    collected once and frozen (no later collection walks it) and automatic collection is
    off until the region ends.  The enqueue loops here run only ~100 ms ahead of the GPU,
    and a full collection in a process with torch loaded takes about that long, so one
    would idle the GPU inside a single launch's event pair."""

    def __enter__(self):
        gc.collect()
        gc.freeze()
        self._enabled = gc.isenabled()
        gc.disable()
        return self

    def __exit__(self, *exc):
        if self._enabled:
            gc.enable()
        gc.unfreeze()
        return False


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms during timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.rows: list[list[str]] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu_index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is None:
            return False
        time.sleep(0.2)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)
        return False

    def summary(self) -> dict:
        rows = self.rows
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows]
        mx = [num(r[2]) for r in rows]
        power = [num(r[3]) for r in rows]
        reasons = set()
        for r in rows:
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                 r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        pw = [p for p in power if p is not None]
        loaded = [s for s, p in zip(sm, power) if s is not None and p is not None and pw and p > 0.5 * max(pw)]
        sm_ok = [s for s in sm if s is not None]
        capped = sum(1 for r in rows if r[8].lower().startswith("active"))
        return {"sm_mhz": statistics.median(loaded or sm_ok) if sm_ok else None,
                "sm_max_mhz": max([m for m in mx if m is not None], default=None),
                "reasons": sorted(reasons), "samples": len(rows), "power_w_max": max(pw) if pw else None,
                "sm_mhz_min": min(loaded or sm_ok) if sm_ok else None,
                "sw_power_cap_frac": capped / len(rows)}


# ------------------------------------------------------------------ CPU legs (oracle)
def _sample_for_cpu(wl: Workload, nseq: int, step: int, dtype: str, seed: int):
    """A bounded sample of the workload for the CPU oracle: the first `nseq` decode
    sequences at `step`, with their own blocks only (float32 arrays holding bf16 values)."""
    g = torch.Generator().manual_seed(seed)
    ctx = wl.context_lens(step)[:nseq]
    need = -(-ctx // wl.block_size)
    nb = int(need.sum())
    shape = (nb, wl.block_size, wl.kv_heads, wl.head_dim)
    tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
    kp = torch.randn(shape, generator=g).to(tdt).float().numpy()
    vp = torch.randn(shape, generator=g).to(tdt).float().numpy()
    tables = np.zeros((nseq, int(need.max())), dtype=np.int64)
    off = 0
    for i, n in enumerate(need):
        tables[i, :n] = np.arange(off, off + n)
        off += n
    q = torch.randn(nseq, wl.heads, wl.head_dim, generator=g).to(tdt).float().numpy()
    knew = torch.randn(nseq, wl.kv_heads, wl.head_dim, generator=g).to(tdt).float().numpy()
    vnew = torch.randn(nseq, wl.kv_heads, wl.head_dim, generator=g).to(tdt).float().numpy()
    slots = np.array([tables[i, (c - 1) // wl.block_size] * wl.block_size + (c - 1) % wl.block_size
                      for i, c in enumerate(ctx)], dtype=np.int64)
    return q, kp, vp, tables, ctx, np.ones(nseq, dtype=np.int64), knew, vnew, slots


def _blas_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 0) for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(max(n)) if n else 1
    except Exception:
        return 1


def _oracle_layer_timer(wl: Workload, nseq: int, dtype: str = "bf16"):
    """One layer of the oracle's decode step (KV append + gather-path attention) on a
    sample of `nseq` sequences; returns a function that runs it and returns seconds."""
    from oracle import paged_attention_oracle as oracle

    q, kp, vp, tables, ctx, ql, knew, vnew, slots = _sample_for_cpu(wl, nseq, 0, dtype, seed=1234)
    scale = wl.head_dim ** -0.5

    def one():
        t0 = time.perf_counter()
        kp2 = oracle.kv_append(kp, slots, knew)
        vp2 = oracle.kv_append(vp, slots, vnew)
        oracle.paged_attention_gather(q, kp2, vp2, tables, ctx, ql, scale, dtype)
        return time.perf_counter() - t0

    return one, ctx


def _cpu_sample_text(wl: Workload, nseq: int, ctx, reps: int, dtype: str = "bf16") -> str:
    how = "bf16 emulated in float32 numpy" if dtype == "bf16" else "float32 numpy"
    return (f"{nseq} decode sequences of the workload (contexts {ctx.tolist()}), {reps} repetitions of one layer "
            f"of the oracle's KV append + gather-path attention ({how}), scaled to "
            f"{wl.layers} layers and to decode tokens/s; churn prefill not included; host has "
            f"{os.cpu_count()} CPUs")


REF_DIR = ROOT / "baseline" / "_ref"


def _reference_modules():
    """The unmodified reference server installed in ``baseline/_ref`` (by
    ``baseline/install_reference.py``), or None when it is not installed.  Its modules
    are imported as they are; ``DEVICE`` defaults to ``cpu`` for its config."""
    if not (REF_DIR / "inference_server" / "core" / "attention.py").exists():
        return None
    import importlib
    import types

    os.environ.setdefault("DEVICE", "cpu")
    if str(REF_DIR) not in sys.path:
        sys.path.append(str(REF_DIR))
    names = dict(config="config", attention="core.attention", paged_executor="core.paged_executor",
                 kv_pool="core.kv_pool", block_allocator="core.block_allocator", scheduler="core.scheduler",
                 sequence="core.sequence")
    return types.SimpleNamespace(**{k: importlib.import_module(f"inference_server.{v}") for k, v in names.items()})


class ReferenceStepSample:
    """One layer of the reference's own step on the host CPU, on a bounded sample of the
    workload, scaled to the whole step.

    The sample runs, unchanged, the reference's KV append (``_PagedCache.update``,
    inference_server/core/paged_executor.py:116-125) and gather attention
    (``paged_attention_gather``, core/attention.py:92-187) on a ``PagedKVPool`` holding
    one layer, in the workload's dtype, with ``torch.set_num_threads(os.cpu_count())``:

    * decode: ``nseq`` sequences that include the batch's longest one.  The reference's
      batched decode pads every row to the longest context of the batch
      (core/attention.py:130-153), so the full batch costs ``batch / nseq`` times the
      sample;
    * prefill (workloads with churn): the first ``npf`` churn prompts of step 0 through
      the per-sequence ragged loop (core/attention.py:156-187), whose dense scores cost
      grows with prompt length squared; scaled by the step's sum of squared prompt
      lengths over the sample's.

    ``step_seconds = layers * (t_decode * batch / nseq + t_prefill * prefill_scale)`` and
    the value is the step's generated tokens (batch + churn prompts) over that.
    """

    def __init__(self, ref, wl: "Workload", nseq: int, npf: int, dtype: str, seed: int = 1234):
        self.ref, self.wl = ref, wl
        torch.set_num_threads(os.cpu_count() or 1)
        self.cores = torch.get_num_threads()
        tdt = torch.bfloat16 if dtype == "bf16" else torch.float32
        g = torch.Generator().manual_seed(seed)
        bs, Hq, Hkv, D = wl.block_size, wl.heads, wl.kv_heads, wl.head_dim
        ctx_all = wl.context_lens(0)
        longest = int(np.argmax(ctx_all))
        sel = [longest] + [i for i in range(wl.batch) if i != longest][:max(nseq, 1) - 1]
        self.ctx = ctx_all[sel].astype(np.int64)
        self.plen = wl.prompt_lens(0)[:npf].astype(np.int64) if wl.n_churn and npf else np.zeros(0, np.int64)
        need_d, need_p = -(-self.ctx // bs), -(-self.plen // bs)
        nb = int(need_d.sum() + need_p.sum()) + 1
        dims = ref.kv_pool.ModelDims(num_layers=1, num_kv_heads=Hkv, head_dim=D, dtype=tdt)
        self.pool = ref.kv_pool.PagedKVPool(dims, num_blocks=nb, block_size=bs, device="cpu")
        self.pool.k[0].copy_(torch.randn(self.pool.k[0].shape, generator=g))
        self.pool.v[0].copy_(torch.randn(self.pool.v[0].shape, generator=g))
        perm = torch.randperm(nb, generator=g).tolist()

        def layout(lens, q_lens):
            nonlocal perm
            rows, slots = [], []
            for c, q in zip(lens.tolist(), q_lens.tolist()):
                n = -(-c // bs)
                blocks, perm = perm[:n], perm[n:]
                rows.append(blocks)
                slots += [blocks[p // bs] * bs + p % bs for p in range(c - q, c)]
            width = max(len(r) for r in rows)
            tables = torch.tensor([r + [0] * (width - len(r)) for r in rows], dtype=torch.long)
            return tables, torch.tensor(slots, dtype=torch.long)

        def case(lens, q_lens):
            tables, slots = layout(lens, q_lens)
            t = int(q_lens.sum())
            return dict(q=torch.randn(t, Hq, D, generator=g).to(tdt),
                        k=torch.randn(1, Hkv, t, D, generator=g).to(tdt), v=torch.randn(1, Hkv, t, D, generator=g).to(tdt),
                        tables=tables, slots=slots, ctx=torch.from_numpy(lens), ql=torch.from_numpy(q_lens))

        self.decode = case(self.ctx, np.ones_like(self.ctx))
        self.prefill = case(self.plen, self.plen) if len(self.plen) else None
        self.scale = D ** -0.5
        full_sq = float(np.sum(wl.prompt_lens(0).astype(np.float64) ** 2)) if wl.n_churn else 0.0
        self.pf_scale = full_sq / float(np.sum(self.plen.astype(np.float64) ** 2)) if len(self.plen) else 0.0
        self.dec_scale = wl.batch / len(self.ctx)
        self.last = (0.0, 0.0)

    def _layer(self, c) -> float:
        pe, attention = self.ref.paged_executor, self.ref.attention
        t0 = time.perf_counter()
        sc = pe._StepContext(write_slots=c["slots"], block_tables=c["tables"], context_lens=c["ctx"],
                             query_lens=c["ql"], pool=self.pool)
        pe._PagedCache(sc).update(c["k"], c["v"], 0)
        attention.paged_attention_gather(c["q"], self.pool.k[0], self.pool.v[0], c["tables"], c["ctx"], c["ql"],
                                         self.scale)
        return time.perf_counter() - t0

    def step_seconds(self) -> float:
        """Runs the sample once; returns the scaled seconds of one whole step."""
        t_dec = self._layer(self.decode)
        t_pf = self._layer(self.prefill) if self.prefill is not None else 0.0
        self.last = (t_dec, t_pf)
        return self.wl.layers * (t_dec * self.dec_scale + t_pf * self.pf_scale)

    @property
    def tokens_per_step(self) -> int:
        return self.wl.batch + self.wl.n_churn

    def describe(self, reps: int) -> str:
        pf = (f"; prefill: churn prompts {self.plen.tolist()} through the ragged loop, scaled x{self.pf_scale:.2f} "
              f"(sum of squared prompt lengths) to the step's {self.wl.n_churn} prompts") if len(self.plen) else ""
        return (f"the reference's own _PagedCache.update + paged_attention_gather (baseline/_ref, unchanged) on "
                f"one layer, {str(self.pool.k[0].dtype).replace('torch.', '')}, torch CPU with "
                f"{self.cores} threads; decode: {len(self.ctx)} sequences incl. the batch's longest (contexts "
                f"{self.ctx.tolist()}), padded rows scaled x{self.dec_scale:.0f} to the batch of {self.wl.batch}"
                f"{pf}; x{self.wl.layers} layers; {reps} repetitions; last decode/prefill layer "
                f"{self.last[0] * 1e3:.0f}/{self.last[1] * 1e3:.0f} ms; host has {os.cpu_count()} CPUs")


def _cpu_leg(args, wl: "Workload", dtype: str) -> dict | None:
    """The CPU baseline beside the GPU line: the reference's own code when it is
    installed (``kind: reference``), else the numpy port (``kind: port``)."""
    ref = _reference_modules()
    if ref is not None:
        s = ReferenceStepSample(ref, wl, args.cpu_sample_seqs, args.cpu_sample_prompts, dtype)
        s.step_seconds()                                           # warm-up
        t_end = time.perf_counter() + args.cpu_budget_s
        reps = []
        while len(reps) < 2 or time.perf_counter() < t_end:
            reps.append(s.step_seconds())
        return {"value": s.tokens_per_step / float(np.mean(reps)), "unit": "tok/s", "cores": s.cores,
                "kind": "reference", "sample": s.describe(len(reps))}
    one, ctx = _oracle_layer_timer(wl, args.cpu_sample_seqs, dtype)
    one()
    t_end = time.perf_counter() + args.cpu_budget_s
    reps = []
    while len(reps) < 2 or time.perf_counter() < t_end:
        reps.append(one())
    return {"value": args.cpu_sample_seqs / (float(np.mean(reps)) * wl.layers), "unit": "tok/s",
            "cores": _blas_threads(), "kind": "port",
            "sample": "reference not installed in baseline/_ref; " + _cpu_sample_text(wl, args.cpu_sample_seqs, ctx,
                                                                                      len(reps), dtype)}


def run_reference(args, rank: int, world: int) -> None:
    """``--impl reference``: the reference's own CPU path on this host's cores, rank 0
    only.  Attention workloads time ``ReferenceStepSample`` (each step = one run of the
    sample, scaled to a whole step); ``config1`` serves a bounded sample of its requests
    through the reference's Scheduler + PagedExecutor.  Falls back to the numpy port,
    saying so in ``kind``, when the reference is not installed."""
    if rank != 0:
        return
    dt = WORKLOADS[args.workload]["dtype"]
    if args.workload == "config1":
        cpu = _c1_cpu_sample(args)
        value, ms, wl_cfg = cpu["value"], None, {"workload": "BASELINE config 1 (see the GPU line)",
                                                "model": "gpt2-124m (random-init)"}
        steps, sample = 1, cpu
    else:
        wl = _make_workload(args, rank, max_steps=1)
        ref = _reference_modules()
        if ref is not None:
            s = ReferenceStepSample(ref, wl, args.cpu_sample_seqs, args.cpu_sample_prompts, dt)
            for _ in range(args.warmup):
                s.step_seconds()
            times, wall = [], []
            for _ in range(args.steps):
                t0 = time.perf_counter()
                times.append(s.step_seconds())
                wall.append(time.perf_counter() - t0)
            value = s.tokens_per_step / float(np.mean(times))
            sample = {"value": value, "unit": "tok/s", "cores": s.cores, "kind": "reference",
                      "sample": s.describe(len(times)),
                      "extrapolated_ms_per_full_step": float(np.mean(times)) * 1e3}
            times = wall
        else:
            one, ctx = _oracle_layer_timer(wl, args.cpu_sample_seqs, dt)
            for _ in range(args.warmup):
                one()
            times = [one() for _ in range(args.steps)]
            value = args.cpu_sample_seqs / (float(np.mean(times)) * wl.layers)
            sample = {"value": value, "unit": "tok/s", "cores": _blas_threads(), "kind": "port",
                      "sample": "reference not installed in baseline/_ref; " +
                                _cpu_sample_text(wl, args.cpu_sample_seqs, ctx, len(times), dt)}
        ms, wl_cfg, steps = float(np.mean(times)) * 1e3, _config(args, wl, world), args.steps
    # ms_per_step: wall time of one timed sample step on this host (the value extrapolates
    # the sample to the whole step; see cpu_baseline.sample)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": dt, "data": "synthetic",
        "config": wl_cfg,
        "cpu_baseline": sample,
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "host_cpus": os.cpu_count(),
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
WORKLOADS = {
    # BASELINE config 3 (the default line): Llama-3-8B shape with churn prefill.
    "config3": dict(heads=32, kv_heads=8, head_dim=128, dtype="bf16", mean_ctx=4096.0, median_ctx=None,
                    lo=128, hi=16384, layers=32, churn=0.05),
    # the isolated paged-decode microbenchmark, GPT-2 heads.
    "config2-f32": dict(heads=12, kv_heads=12, head_dim=64, dtype="f32", mean_ctx=0.0, median_ctx=1024.0,
                        lo=16, hi=8192, layers=1, churn=0.0),
    "config2-bf16": dict(heads=12, kv_heads=12, head_dim=64, dtype="bf16", mean_ctx=0.0, median_ctx=1024.0,
                         lo=16, hi=8192, layers=1, churn=0.0),
    # Llama-3-70B-shape decode with KV heads sharded over the GPUs
    # (--gpus N = tensor-parallel size), o_proj row-split, one all-reduce per layer.
    "config5": dict(heads=64, kv_heads=8, head_dim=128, dtype="bf16", mean_ctx=8192.0, median_ctx=None,
                    lo=128, hi=32768, layers=80, churn=0.0, batch=512, d_model=8192),
    "config5-decode": dict(heads=64, kv_heads=8, head_dim=128, dtype="bf16", mean_ctx=8192.0, median_ctx=None,
                    lo=128, hi=32768, layers=80, churn=0.0, batch=512, d_model=8192),
    # the serving engine end to end, GPT-2 124M random-init, fp32.
    "config1": dict(heads=12, kv_heads=12, head_dim=64, dtype="f32", mean_ctx=0.0, median_ctx=None,
                    lo=0, hi=0, layers=12, churn=0.0, batch=32),
    # prefix sharing on the Llama-3-8B shape (8 shared 16-token blocks).
    "config4": dict(heads=32, kv_heads=8, head_dim=128, dtype="bf16", mean_ctx=0.0, median_ctx=None,
                    lo=0, hi=0, layers=32, churn=0.0, batch=64),
    # Whole-block moves on the config-3 pool shape: copy-on-write and swap-out / swap-in.
    # config 5's per-rank o_proj alone (rows = batch, k = heads * head_dim / --tp, n = d_model).
    "oproj": dict(heads=64, kv_heads=8, head_dim=128, dtype="bf16", mean_ctx=0.0, median_ctx=None,
                  lo=0, hi=0, layers=1, churn=0.0, batch=512, d_model=8192),
    "blocks": dict(heads=32, kv_heads=8, head_dim=128, dtype="bf16", mean_ctx=0.0, median_ctx=None,
                   lo=0, hi=0, layers=32, churn=0.0),
}

def run_tp(args, rank: int, world: int, local_rank: int) -> None:
    """``--workload config5``: BASELINE config 5 decode (Llama-3-70B attention shape: 64 q
    / 8 kv heads, head_dim 128, bf16, 80 layers, d_model 8192, batch 512, contexts
    lognormal mean 8192 clipped 128..32768) with the KV heads sharded over the
    ``--gpus N`` ranks (tensor_parallel.KVHeadParallelAttention: fused append, paged
    attention over the rank's heads, the rank's row slice of o_proj, one NCCL all-reduce
    of [batch, d_model] per layer).  Every rank serves the same batch, so the total work
    is fixed (``scaling: strong``).  The 80 layer calls cycle over as many physical
    per-layer pools as fit in 55 % of HBM (layer l uses pool l mod P); each call still
    streams its whole KV (GBs, far above L2) and appends its own new tokens."""
    import importlib

    from __graft_entry__ import import_package

    pkg = import_package()
    tpm = importlib.import_module(f"{pkg.__name__}.tensor_parallel")
    w = WORKLOADS["config5"]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if w["kv_heads"] % world:
        raise SystemExit(f"config5 shards {w['kv_heads']} KV heads; {world} ranks do not divide them")
    L, B, D, DM = args.layers, args.batch, w["head_dim"], w["d_model"]
    steps_total = args.warmup + args.steps
    wl = Workload(batch=B, layers=L, heads=w["heads"], kv_heads=w["kv_heads"], head_dim=D, block_size=16,
                  mean_ctx=w["mean_ctx"], lo=w["lo"], hi=w["hi"], sigma=0.9, seed=args.seed, max_steps=steps_total + 1,
                  churn=0.0)
    qs, ks = tpm.kv_head_shard(w["heads"], w["kv_heads"], rank, world)
    Hq, Hkv = qs.stop - qs.start, ks.stop - ks.start
    per_layer = wl.num_blocks * 16 * Hkv * D * 2 * 2
    P = max(1, min(L, int(0.55 * torch.cuda.get_device_properties(dev).total_memory // per_layer)))
    g = torch.Generator(device=dev).manual_seed(args.seed + 100 * rank)
    shape = (wl.num_blocks, 16, Hkv, D)
    k_pools = [torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=g) for _ in range(P)]
    v_pools = [torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=g) for _ in range(P)]
    q = [torch.randn(B, Hq, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(L)]
    kn = [torch.randn(B, Hkv, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(L)]
    vn = [torch.randn(B, Hkv, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(L)]
    w_o = [(torch.randn(Hq * D, DM, generator=g, device=dev) / (w["heads"] * D) ** 0.5).to(torch.bfloat16)
           for _ in range(L)]
    bt = torch.from_numpy(wl.tables).to(dev)
    sm = pkg.metadata.sm_count(dev)
    tile = _prefill_tile(pkg, args, Hq, Hkv, D)
    dummy = torch.zeros(1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def plan(s):
        return pkg.StepMetadata.plan_host(wl.context_lens(s), wl.query_lens, wl.tables, num_tokens=B,
                                          pool_num_blocks=wl.num_blocks, block_size=16, num_kv_heads=Hkv, sm=sm,
                                          prefill_tile_tokens=tile, pinned=True)

    metas = [plan(s).upload(dev) for s in range(steps_total)]
    layers = [tpm.KVHeadParallelAttention(w_o=w_o[l]) for l in range(L)]
    reducer = (tpm.PeerAllReduce(B * DM, torch.bfloat16, device=dev, timeout_s=10.0)
               if world > 1 and args.allreduce == "peer" else None)
    # --allreduce fused: the o_proj GEMM and its all-reduce in one collective (at tp1 the
    # same kernels run the GEMM alone); weights kept K-major for it
    fused = (tpm.FusedOProjAllReduce(B, DM, torch.bfloat16, device=dev, timeout_s=10.0)
             if args.allreduce == "fused" else None)
    w_nk = [w.t().contiguous() for w in w_o] if fused is not None else None

    def step(meta, marks=None, host=None):
        slots = meta.slot_mapping()
        bta = pkg.attach(bt, meta)
        out = None
        for l in range(L):
            if host is not None:   # e2e: this layer's q / new K / new V come from pinned host memory
                q[0].copy_(host[0], non_blocking=True)
                kn[0].copy_(host[1], non_blocking=True)
                vn[0].copy_(host[2], non_blocking=True)
                ql, kl, vl = q[0], kn[0], vn[0]
            else:
                ql, kl, vl = q[l], kn[l], vn[l]
            kp, vp = k_pools[l % P], v_pools[l % P]
            if marks is not None:
                marks[l][0].record(stream)
            pkg.reshape_and_cache(kl, vl, kp, vp, slots)
            attn = pkg.paged_attention_cuda(ql, kp, vp, bta, dummy, dummy, D ** -0.5)
            if marks is not None:
                marks[l][1].record(stream)
            a2 = attn.reshape(B, -1)
            if fused is not None:      # GEMM + all-reduce together (timed as the o_proj span)
                partial = fused(a2, w_nk[l])
            elif reducer is not None:  # the GEMM writes into the peer-mapped slot
                partial = torch.matmul(a2, layers[l].w_o, out=reducer.slot((B, DM)))
            else:
                partial = a2 @ layers[l].w_o
            if marks is not None:
                marks[l][2].record(stream)
            if fused is not None:
                pass
            elif reducer is not None:
                reducer.all_reduce_(partial)
            elif world > 1:
                torch.distributed.all_reduce(partial)
            if marks is not None:
                marks[l][3].record(stream)
            out = partial
        return out

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    clocks = ClockSampler(dev.index)
    with clocks, QuietHost():
        for s in range(args.warmup):
            step(metas[s])
        barrier()
        torch.cuda.synchronize(dev)
        marks = [[[ev() for _ in range(4)] for _ in range(L)] for _ in range(args.steps)]
        t0, t1 = ev(), ev()
        t0.record(stream)
        host_step_ms = []
        for k in range(args.steps):
            th = time.perf_counter()
            step(metas[args.warmup + k], marks[k])
            host_step_ms.append((time.perf_counter() - th) * 1e3)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        elapsed = t0.elapsed_time(t1)
        attn_kernels = pkg._lib.last_launches()      # this library's kernels per attention call
        attn_ms = float(np.mean([m[0].elapsed_time(m[1]) for mk in marks for m in mk]))
        # rank 0's spread: per-layer attention spans and the host's enqueue time per step
        # (a span far above the kernels' own time means the GPU waited for the host)
        spans = [m[0].elapsed_time(m[1]) for mk in marks for m in mk]
        spread = {"attn_span_ms_min_p50_max": [round(min(spans), 3), round(float(np.median(spans)), 3),
                                               round(max(spans), 3)],
                  "attn_span_ms_first_step": [round(x, 3) for x in spans[:L]],
                  "host_enqueue_ms_per_step": [round(x, 2) for x in host_step_ms]}
        gemm_ms = float(np.mean([m[1].elapsed_time(m[2]) for mk in marks for m in mk]))
        ar_ms = float(np.mean([m[2].elapsed_time(m[3]) for mk in marks for m in mk]))

        # e2e: metadata planned and uploaded every step, each layer's inputs from pinned
        # host memory, the step's output (last layer, [batch, d_model]) read back.
        host = [q[0].cpu().pin_memory(), kn[0].cpu().pin_memory(), vn[0].cpu().pin_memory()]
        out_host = torch.empty(B, DM, dtype=torch.bfloat16).pin_memory()
        for s in range(args.warmup):
            out_host.copy_(step(plan(s).upload(dev), host=host), non_blocking=True)
        barrier()
        torch.cuda.synchronize(dev)
        e0, e1 = ev(), ev()
        e0.record(stream)
        words = 0
        for k in range(args.steps):
            m = plan(args.warmup + k)
            words += int(m.plan.words)
            out_host.copy_(step(m.upload(dev), host=host), non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = e0.elapsed_time(e1)
    assert pkg.read_device_error(dev) == 0, "a kernel set the device error word"
    if reducer is not None:
        reducer.check()
        reducer.close()
        barrier()
    times = torch.tensor([elapsed, e2e_ms, attn_ms, gemm_ms, ar_ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(times, op=torch.distributed.ReduceOp.MAX)
    elapsed, e2e_ms, attn_ms, gemm_ms, ar_ms = times.tolist()
    if rank != 0:
        return
    timed = [args.warmup + k for k in range(args.steps)]
    ctx_sum = float(np.mean([wl.context_lens(s).sum() for s in timed]))
    attn_bytes = (ctx_sum * Hkv * D * 2 * 2 + 2 * B * Hq * D * 2 + ctx_sum / 16 * 4 + 2 * B * Hkv * D * 2 * 2)
    hbm_peak, bf16_peak, peak_kind = _measured_peaks()
    achieved = attn_bytes / (attn_ms / 1e3) / 1e9
    ar_bytes = B * DM * 2
    backend = ("fused with the o_proj GEMM (pa_oproj_allreduce: pushes from the GEMM epilogue over NVLink)"
               if fused is not None else "NCCL" if reducer is None else
               "peer memory (pa_peer_allreduce: two-shot over NVLink, GEMM output written into the peer-mapped slot)")
    line = {
        "metric": METRIC, "value": B * args.steps / (elapsed / 1e3), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "BASELINE config 5: Llama-3-70B-shape GQA decode (64 q / 8 kv heads, head_dim 128, "
                               f"bf16, {L} layers, d_model {DM}), batch {B}, contexts lognormal mean 8192 clipped "
                               f"128..32768, KV heads sharded over {world} GPU(s) with a row-split o_proj and one "
                               "all-reduce per layer",
                   "model": "llama3-70b-shape attention + o_proj (random-init)", "global_batch": B, "layers": L,
                   "kv_heads_per_gpu": Hkv, "q_heads_per_gpu": Hq, "sum_context_step0": int(wl.ctx0.sum()),
                   "seq_len": "ragged (mean 8192)", "physical_layer_pools": P,
                   "l2": f"each layer call streams {per_layer / 1e9:.2f} GB of KV (>> 126 MB L2); {L} layer calls "
                         f"cycle over {P} physical pools",
                   "parallelism": (f"tp{world} (KV-head sharding; {backend} all-reduce after o_proj)")
                                  if world > 1 else "tp1"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_source": f"{peak_kind} HBM copy", "traffic": None,
                     "kernel": "per-rank KV append + decode paged attention per layer (tensor-pipe MMA + combine)",
                     "algorithmic_bytes_per_launch": attn_bytes, "avg_launch_ms": attn_ms},
        "o_proj": {"avg_ms": gemm_ms, "tflops": 2 * B * Hq * D * DM / (gemm_ms / 1e3) / 1e12,
                   "peak_tflops": bf16_peak,
                   "kernel": ("pa_oproj_allreduce: tcgen05 GEMM whose epilogue stores tiles into their owners' "
                              "staging over NVLink, then the owners' sums stored into every rank (GEMM and "
                              "all-reduce timed together here)") if fused is not None
                             else "torch bf16 matmul (cuBLAS)"},
        "all_reduce": None if world == 1 or fused is not None else {
            "avg_ms": ar_ms, "bytes": ar_bytes, "bus_gbs": 2 * (world - 1) / world * ar_bytes / (ar_ms / 1e3) / 1e9,
            "backend": backend},
        "cpu_baseline": None,
        "e2e": {"value": B * args.steps / (e2e_ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": words * 4 // args.steps + L * B * (Hq + 2 * Hkv) * D * 2,
                "d2h_bytes_per_step": B * DM * 2, "ms_per_step": e2e_ms / args.steps},
        "launch_spread": spread,
        "gpu_launches": args.steps * L * (1 + len(attn_kernels) + (1 if reducer is not None else 0)
                                          + (2 if fused is not None else 0)),
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


SERVE_POOL_FRACTION = 0.90     # config 5: the pool takes ~90 % of the HBM left after weights and buffers
SERVE_MAX_PASS_TOKENS = 131072 # tokens one pass may feed (four 32k-token recomputes)
SERVE_OPROJ_CHUNK = 16384      # prefill passes run o_proj + all-reduce in chunks of this many tokens


def run_serve_tp(args, rank: int, world: int, local_rank: int) -> None:
    """``--workload config5``: BASELINE config 5 served as stated — Llama-3-70B attention
    shape (64 q / 8 kv heads, head_dim 128, bf16, 80 layers, d_model 8192), 512 requests
    with contexts lognormal mean 8192 clipped 128..32768, KV heads sharded over the
    ``--gpus N`` ranks with a row-split o_proj and one all-reduce per layer, and each
    rank's 80-layer pool sized to ~90 % of the HBM left after the o_proj weights and the
    pass buffers, so the batch is bounded by the pool and recompute preemption fires.

    Scheduling is ``ServeSim`` (the reference scheduler's policy, checked step for step
    against it on CPU): a pass is either the admitted sequences' prefill (whole history;
    a preempted victim's recompute included) through the tcgen05 varlen prefill kernel,
    or one decode token for every running sequence.  The run starts from a steady state:
    requests are admitted in order while they fit, as if their prompts had been prefilled
    (their KV resident, random); the rest wait.  Output lengths are lognormal with median
    64 (sigma 0.9, clipped 1..512), borrowed from config 4 because config 5 states none.
    Per pass and layer: fused K+V append, paged attention over the rank's heads, the
    rank's o_proj row slice, all-reduce (decode: the peer-memory kernel; prefill: NCCL in
    chunks of 16k tokens).  value = tokens sampled / time (both pass kinds sample one
    token per sequence); the line splits the time by pass kind and by operation."""
    import importlib

    from __graft_entry__ import import_package

    pkg = import_package()
    tpm = importlib.import_module(f"{pkg.__name__}.tensor_parallel")
    w = WORKLOADS["config5"]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if w["kv_heads"] % world:
        raise SystemExit(f"config5 shards {w['kv_heads']} KV heads; {world} ranks do not divide them")
    L, NREQ, D, DM, BS = args.layers, args.batch, w["head_dim"], w["d_model"], 16
    qs, ks = tpm.kv_head_shard(w["heads"], w["kv_heads"], rank, world)
    Hq, Hkv = qs.stop - qs.start, ks.stop - ks.start
    rng = np.random.default_rng(args.seed)
    mu = clipped_lognormal_mu(w["mean_ctx"], 0.9, w["lo"], w["hi"])
    prompts = np.clip(np.exp(rng.normal(mu, 0.9, size=NREQ)), w["lo"], w["hi"]).astype(np.int64)
    outs = np.clip(np.exp(rng.normal(np.log(64.0), 0.9, size=NREQ)), 1, 512).astype(np.int64)

    # ---- weights and pass buffers first, then the pool from what is left
    g = torch.Generator(device=dev).manual_seed(args.seed + 100 * rank)
    w_o = [(torch.randn(Hq * D, DM, generator=g, device=dev) / (w["heads"] * D) ** 0.5).to(torch.bfloat16)
           for _ in range(L)]
    T = SERVE_MAX_PASS_TOKENS
    q_buf = torch.randn(T, Hq, D, generator=g, device=dev).to(torch.bfloat16)
    k_new = torch.randn(T, Hkv, D, generator=g, device=dev).to(torch.bfloat16)
    v_new = torch.randn(T, Hkv, D, generator=g, device=dev).to(torch.bfloat16)
    proj = torch.empty(SERVE_OPROJ_CHUNK, DM, dtype=torch.bfloat16, device=dev)
    reducer = (tpm.PeerAllReduce(NREQ * DM, torch.bfloat16, device=dev, timeout_s=10.0)
               if world > 1 and args.allreduce == "peer" else None)
    torch.cuda.synchronize(dev)
    free_b, total_b = torch.cuda.mem_get_info(dev)
    # the attention output of the largest pass is allocated per pass: keep room for it
    budget = free_b - T * Hq * D * 2 - (2 << 30)
    block_bytes = L * 2 * BS * Hkv * D * 2
    nb = int(SERVE_POOL_FRACTION * budget // block_bytes)
    shape = (nb, BS, Hkv, D)
    k_pools = [torch.empty(shape, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    v_pools = [torch.empty(shape, dtype=torch.bfloat16, device=dev) for _ in range(L)]
    for t in k_pools + v_pools:
        t.normal_(generator=g)
    pool_bytes = 2 * L * nb * BS * Hkv * D * 2

    sim = ServeSim(nb, BS, max_running=NREQ)
    seqs = [SimSeq(i, int(p), int(o)) for i, (p, o) in enumerate(zip(prompts, outs))]
    resident = 0
    for s in seqs:
        if resident == len(sim.running) and sim.admit_resident(s):
            resident += 1
        else:
            sim.add(s)
    # the largest pass's attention output and a generous split-K workspace are cached
    # before timing, so the timed passes allocate nothing new from the nearly full HBM
    pkg.attention._workspace(dev, 64 << 20)
    tmp = torch.empty(T * Hq * D, dtype=torch.bfloat16, device=dev)
    del tmp
    sm = pkg.metadata.sm_count(dev)
    tile = _prefill_tile(pkg, args, Hq, Hkv, D)
    dummy = torch.zeros(1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)
    launches = [0]

    def plan(batch):
        width = max(len(s.blocks) for s in batch)
        tables = np.zeros((len(batch), width), dtype=np.int64)
        for i, s in enumerate(batch):
            tables[i, :len(s.blocks)] = s.blocks
        ctx = np.array([s.after_next for s in batch], dtype=np.int64)
        ql = np.array([s.feed for s in batch], dtype=np.int64)
        meta = pkg.StepMetadata.plan_host(ctx, ql, tables, num_tokens=int(ql.sum()), pool_num_blocks=nb,
                                          block_size=BS, num_kv_heads=Hkv, sm=sm, prefill_tile_tokens=tile,
                                          pinned=True)
        return meta, torch.from_numpy(tables).to(dev, non_blocking=True)

    def run_pass(batch, marks):
        meta, bt = plan(batch)
        tokens = meta.num_tokens
        if tokens > T:
            raise SystemExit(f"config5: a pass feeds {tokens} tokens (> {T}); raise SERVE_MAX_PASS_TOKENS")
        meta = meta.upload(dev)
        slots = meta.slot_mapping()
        bta = pkg.attach(bt, meta)
        decode = not any(s.prefilling for s in batch)
        for l in range(L):
            marks[l][0].record(stream)
            pkg.reshape_and_cache(k_new[:tokens], v_new[:tokens], k_pools[l], v_pools[l], slots)
            attn = pkg.paged_attention_cuda(q_buf[:tokens], k_pools[l], v_pools[l], bta, dummy, dummy, D ** -0.5)
            launches[0] += 1 + bin(pkg._lib.lib().pa_last_launches()).count("1")
            marks[l][1].record(stream)
            a2 = attn.reshape(tokens, -1)
            if decode:
                out = (torch.matmul(a2, w_o[l], out=reducer.slot((tokens, DM))) if reducer is not None
                       else a2 @ w_o[l])
                marks[l][2].record(stream)
                if reducer is not None:
                    reducer.all_reduce_(out)
                    launches[0] += 1
                elif world > 1:
                    torch.distributed.all_reduce(out)
                marks[l][3].record(stream)
            else:
                for c0 in range(0, tokens, SERVE_OPROJ_CHUNK):
                    c1 = min(tokens, c0 + SERVE_OPROJ_CHUNK)
                    torch.matmul(a2[c0:c1], w_o[l], out=proj[:c1 - c0])
                    if world > 1:
                        torch.distributed.all_reduce(proj[:c1 - c0])
                marks[l][2].record(stream)        # o_proj and its all-reduce timed together
                marks[l][3].record(stream)
        return decode, tokens

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def one_step(record):
        batch = sim.schedule()
        if not batch:
            return None
        marks = [[ev() for _ in range(4)] for _ in range(L)]
        decode, tokens = run_pass(batch, marks)
        sim.finish_pass(batch)
        if record is not None:
            record.append((decode, len(batch), tokens, marks))
        return decode

    clocks = ClockSampler(dev.index)
    with clocks, QuietHost():
        for _ in range(args.warmup):
            one_step(None)
        barrier()
        torch.cuda.synchronize(dev)
        pre0, rec0, done0, launches[0] = sim.preemptions, sim.recompute_tokens, sim.completed, 0
        passes: list = []
        t0, t1 = ev(), ev()
        t0.record(stream)
        while len(passes) < args.steps and sim.has_work:
            one_step(passes)
        t1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        elapsed = t0.elapsed_time(t1)
    assert pkg.read_device_error(dev) == 0, "a kernel set the device error word"
    if reducer is not None:
        reducer.check()
        reducer.close()
        barrier()

    def span(kind, a, b):
        return float(sum(m[a].elapsed_time(m[b]) for d, _, _, mk in passes if d == kind for m in mk))

    sampled = sum(n for _, n, _, _ in passes)
    stats = torch.tensor([elapsed, span(True, 0, 1), span(True, 1, 2), span(True, 2, 3), span(False, 0, 1),
                          span(False, 1, 3)], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(stats, op=torch.distributed.ReduceOp.MAX)
    elapsed, dec_attn, dec_gemm, dec_ar, pre_attn, pre_proj = stats.tolist()
    if rank != 0:
        return
    n_dec = sum(1 for d, _, _, _ in passes if d)
    n_pre = len(passes) - n_dec
    dec_tokens = sum(n for d, n, _, _ in passes if d)
    pre_tokens = sum(t for d, _, t, _ in passes if not d)
    line = {
        "metric": METRIC, "value": sampled / (elapsed / 1e3), "unit": "tok/s", "n_gpus": world,
        "steps": len(passes), "warmup": args.warmup, "ms_per_step": elapsed / max(1, len(passes)),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "BASELINE config 5 served: Llama-3-70B-shape GQA (64 q / 8 kv heads, head_dim 128, "
                               f"bf16, {L} layers, d_model {DM}), {NREQ} requests with contexts lognormal mean 8192 "
                               "clipped 128..32768 (outputs lognormal median 64, clipped 1..512), KV heads sharded "
                               f"over {world} GPU(s), row-split o_proj + one all-reduce per layer; the reference "
                               "scheduler's policy (prefill-priority passes, recompute preemption) over a pool of "
                               f"~90 % of free HBM",
                   "model": "llama3-70b-shape attention + o_proj (random-init)", "requests": NREQ, "layers": L,
                   "kv_heads_per_gpu": Hkv, "q_heads_per_gpu": Hq,
                   "pool_blocks": nb, "pool_gb": round(pool_bytes / 1e9, 1),
                   "pool_frac_of_hbm": round(pool_bytes / total_b, 3),
                   "resident_at_start": resident, "running_at_end": len(sim.running),
                   "waiting_at_end": len(sim.waiting) + len(sim.preempted),
                   "l2": "every layer's pool is its own allocation (GBs, >> 126 MB L2)",
                   "parallelism": f"tp{world} (KV-head sharding)" if world > 1 else "tp1"},
        "passes": {"decode": n_dec, "prefill": n_pre, "decode_tokens_sampled": dec_tokens,
                   "prefill_tokens_fed": pre_tokens, "preemptions": sim.preemptions - pre0,
                   "recompute_tokens": sim.recompute_tokens - rec0, "completed": sim.completed - done0},
        "time_split_ms": {"decode_attention": dec_attn, "decode_o_proj": dec_gemm, "decode_all_reduce": dec_ar,
                          "prefill_attention": pre_attn, "prefill_o_proj_and_all_reduce": pre_proj,
                          "total": elapsed},
        "all_reduce_share_of_decode_passes": (dec_ar / (dec_attn + dec_gemm + dec_ar)) if n_dec else None,
        "cpu_baseline": None,
        "e2e": None,
        "gpu_launches": launches[0],
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


class SimSeq:
    """One request in ``ServeSim``: token counts only (no token ids are needed to drive
    the attention path)."""

    __slots__ = ("sid", "prompt_len", "max_tokens", "generated", "num_cached", "blocks", "state", "preempted_step",
                 "preemptions")

    def __init__(self, sid: int, prompt_len: int, max_tokens: int):
        self.sid, self.prompt_len, self.max_tokens = sid, prompt_len, max_tokens
        self.generated, self.num_cached, self.blocks = 0, 0, []
        self.state, self.preempted_step, self.preemptions = "waiting", -1, 0

    @property
    def total_len(self) -> int:
        return self.prompt_len + self.generated

    @property
    def feed(self) -> int:
        """Tokens of the next pass: the whole history when nothing is cached (prefill or
        a recompute), else the one token sampled last."""
        return self.total_len - self.num_cached

    @property
    def prefilling(self) -> bool:
        return self.num_cached == 0 or self.feed > 1

    @property
    def after_next(self) -> int:
        return self.num_cached + self.feed


class ServeSim:
    """The reference scheduler's policy (inference_server/core/scheduler.py:184-437) over
    token counts, for config 5's pool-bound serving run.  Restated, not imported, so the
    bench runs where the reference is not installed; ``tests/test_bench_workload.py``
    checks it step for step against the reference ``Scheduler`` with a fake executor.

    Per step: evict finished sequences (their blocks freed); admit preempted sequences
    first, then waiting ones, FIFO with head-of-line blocking, while a slot is free and
    the sequence's next-pass blocks fit in the free list less the running set's own
    next-pass growth, never on the step it was preempted; select the prefilling
    sequences if any, else every running one; grow each selected sequence's blocks in
    batch order, preempting the most recently admitted running sequence on exhaustion
    (recompute: its blocks freed, nothing cached, back to the front of the preempted
    queue).  The caller runs the pass and then calls ``finish_pass``.  Blocks come from
    a LIFO free list like the reference allocator's."""

    def __init__(self, num_blocks: int, block_size: int, max_running: int):
        self.num_blocks, self.bs, self.max_running = num_blocks, block_size, max_running
        self.free = list(reversed(range(num_blocks)))
        self.waiting: list[SimSeq] = []
        self.preempted: list[SimSeq] = []
        self.running: list[SimSeq] = []
        self.step_count = 0
        self.preemptions = 0
        self.recompute_tokens = 0       # tokens re-prefilled after a preemption
        self.completed = 0

    def blocks_for(self, n: int) -> int:
        return -(-n // self.bs)

    def add(self, seq: SimSeq) -> None:
        if self.blocks_for(seq.prompt_len + seq.max_tokens - 1) > self.num_blocks:
            raise ValueError(f"request {seq.sid} cannot fit the pool even alone")
        self.waiting.append(seq)

    def admit_resident(self, seq: SimSeq) -> bool:
        """Steady-state start: admit `seq` as if its prompt had been prefilled and its
        first token sampled (its KV is resident), if it fits by the admission rule."""
        seq.num_cached, seq.generated = seq.prompt_len, 1
        if len(self.running) >= self.max_running or not self._fits(seq):
            seq.num_cached, seq.generated = 0, 0
            return False
        self._grow_to(seq, seq.num_cached)
        seq.state = "running"
        self.running.append(seq)
        return True

    @property
    def has_work(self) -> bool:
        return bool(self.waiting or self.preempted or self.running)

    # ---------------------------------------------------------------- the policy
    def _needed(self, s: SimSeq) -> int:
        return self.blocks_for(s.after_next) - len(s.blocks)

    def _fits(self, s: SimSeq) -> bool:
        reserved = sum(self._needed(r) for r in self.running)
        return self._needed(s) <= len(self.free) - reserved

    def _grow_to(self, s: SimSeq, tokens: int) -> bool:
        need = self.blocks_for(tokens) - len(s.blocks)
        if need <= 0:
            return True
        if need > len(self.free):
            return False
        s.blocks += [self.free.pop() for _ in range(need)]
        return True

    def _release(self, s: SimSeq) -> None:
        self.free += s.blocks
        s.blocks = []

    def _preempt(self, v: SimSeq) -> None:
        self._release(v)
        self.running.remove(v)
        v.num_cached, v.state, v.preempted_step = 0, "preempted", self.step_count
        v.preemptions += 1
        self.preempted.insert(0, v)
        self.preemptions += 1

    def schedule(self) -> list[SimSeq]:
        """Steps 1-3 of a scheduler step; returns the batch to execute (maybe empty)."""
        self.step_count += 1
        done = [s for s in self.running if s.state == "finished"]
        for s in done:
            self._release(s)
        self.running = [s for s in self.running if s.state != "finished"]
        while len(self.running) < self.max_running:
            queue = self.preempted if self.preempted else self.waiting
            if not queue:
                break
            s = queue[0]
            if s.preempted_step == self.step_count or not self._fits(s):
                break
            queue.pop(0)
            s.state = "running"
            self.running.append(s)
        pre = [s for s in self.running if s.prefilling]
        batch = pre if pre else list(self.running)
        pending = list(batch)
        while pending:
            s = pending[0]
            if self._grow_to(s, s.after_next):
                pending.pop(0)
                continue
            victim = self.running[-1]
            self._preempt(victim)
            if victim in pending:
                pending.remove(victim)
            if victim in batch:
                batch.remove(victim)
        return batch

    def finish_pass(self, batch: list[SimSeq]) -> None:
        """Step 5: the pass cached every fed token and sampled one per sequence."""
        for s in batch:
            if s.num_cached == 0 and s.preemptions:
                self.recompute_tokens += s.feed
            s.num_cached = s.after_next
            s.generated += 1
            if s.generated >= s.max_tokens:
                s.state = "finished"
                self.completed += 1


class PrefixWorkload:
    """BASELINE config 4 as a seeded continuous batch: `batch` running requests, each a
    shared 128-token system prefix (the same 8 physical blocks in every block table, as
    the reference's prefix cache refcounts them) plus a unique suffix of 32..512 tokens;
    outputs lognormal with median 64 (sigma 0.9, capped at 512).  A finished request's
    slot is refilled by a new request, whose suffix is prefilled over the cached prefix
    (query_len < context_len).  Each slot owns a private block range after the prefix."""

    PREFIX, BS = 128, 16

    def __init__(self, batch: int, seed: int, max_steps: int):
        rng = np.random.default_rng(seed)
        self.batch = batch
        per_slot = -(-(512 + 512) // self.BS) + 1
        self.num_blocks = self.PREFIX // self.BS + batch * per_slot + 16
        perm = rng.permutation(self.num_blocks)
        prefix = perm[:self.PREFIX // self.BS]
        self.tables = np.zeros((batch, self.PREFIX // self.BS + per_slot), dtype=np.int64)
        for i in range(batch):
            self.tables[i, :len(prefix)] = prefix
            self.tables[i, len(prefix):] = perm[len(prefix) + i * per_slot:len(prefix) + (i + 1) * per_slot]
        new_req = lambda: (int(rng.integers(32, 513)), int(np.clip(np.exp(rng.normal(np.log(64), 0.9)), 1, 512)))
        suffix, out_len, gen = [], [], []
        for _ in range(batch):
            sfx, o = new_req()
            suffix.append(sfx)
            out_len.append(o)
            gen.append(int(rng.integers(0, o)))
        # per step: decode contexts of the running batch, and the admitted requests' suffixes
        self.decode_ctx, self.admit = [], []
        for _ in range(max_steps):
            admit = []
            for i in range(batch):
                if gen[i] >= out_len[i]:                      # finished: refill the slot
                    suffix[i], out_len[i] = new_req()
                    gen[i] = 1                                 # the prefill pass produces token 1
                    admit.append((i, suffix[i]))
            self.admit.append(admit)
            self.decode_ctx.append(np.array([self.PREFIX + suffix[i] + gen[i] for i in range(batch)], dtype=np.int64))
            for i in range(batch):
                gen[i] += 1

    def prefill_flops(self, step: int, heads: int, head_dim: int) -> float:
        total = 0.0
        for _, q in self.admit[step]:
            ctx = self.PREFIX + q
            total += q * (ctx - q) + q * (q + 1) / 2            # visible keys of the q new tokens
        return 4.0 * heads * head_dim * total


def run_prefix(args, rank: int, world: int, local_rank: int) -> None:
    """``--workload config4``: per step, a prefill pass for the requests admitted this step
    (their suffixes over the shared, cached prefix blocks: query_len < context_len) and a
    decode pass for the running batch, 32 Llama-3-8B-shape layers each (fused append, then
    paged attention).  Request-level replicas across GPUs (scaling: weak)."""
    from __graft_entry__ import import_package

    pkg = import_package()
    w = WORKLOADS["config4"]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    L, B, Hq, Hkv, D = args.layers, args.batch, w["heads"], w["kv_heads"], w["head_dim"]
    steps_total = args.warmup + args.steps
    wl = PrefixWorkload(B, args.seed + rank, steps_total + 1)
    g = torch.Generator(device=dev).manual_seed(args.seed + 100 * rank)
    shape = (wl.num_blocks, 16, Hkv, D)
    k_pools = [torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=g) for _ in range(L)]
    v_pools = [torch.empty(shape, dtype=torch.bfloat16, device=dev).normal_(generator=g) for _ in range(L)]
    t_pre = max(max((sum(q for _, q in a) for a in wl.admit), default=1), 1)
    dec = _Pass(L, B, Hq, Hkv, D, torch.bfloat16, dev, g)
    pre = _Pass(L, t_pre, Hq, Hkv, D, torch.bfloat16, dev, g)
    bt = torch.from_numpy(wl.tables).to(dev)
    sm = pkg.metadata.sm_count(dev)
    tile = _prefill_tile(pkg, args, Hq, Hkv, D)
    dummy = torch.zeros(1, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def plan_decode(s):
        return pkg.StepMetadata.plan_host(wl.decode_ctx[s], np.ones(B, dtype=np.int64), wl.tables, num_tokens=B,
                                          pool_num_blocks=wl.num_blocks, block_size=16, num_kv_heads=Hkv, sm=sm,
                                          prefill_tile_tokens=tile, pinned=True)

    def plan_prefill(s):
        a = wl.admit[s]
        if not a:
            return None
        rows = np.array([i for i, _ in a])
        q = np.array([x for _, x in a], dtype=np.int64)
        return pkg.StepMetadata.plan_host(wl.PREFIX + q, q, wl.tables[rows], num_tokens=int(q.sum()),
                                          pool_num_blocks=wl.num_blocks, block_size=16, num_kv_heads=Hkv, sm=sm,
                                          prefill_tile_tokens=tile, pinned=True)

    metas = [(plan_decode(s).upload(dev), (lambda m: m.upload(dev) if m is not None else None)(plan_prefill(s)))
             for s in range(steps_total)]
    bts_pre = {s: torch.from_numpy(wl.tables[[i for i, _ in wl.admit[s]]]).to(dev)
               for s in range(steps_total) if wl.admit[s]}
    launches = [0]
    host = {"dec": [dec.q[0].cpu().pin_memory(), dec.k[0].cpu().pin_memory(), dec.v[0].cpu().pin_memory()],
            "pre": [pre.q[0].cpu().pin_memory(), pre.k[0].cpu().pin_memory(), pre.v[0].cpu().pin_memory()],
            "out": torch.empty(max(B, t_pre), Hq, D, dtype=torch.bfloat16).pin_memory()}
    moved = [0, 0]

    def run_pass(meta, rows_bt, inp, tokens, marks=None, src=None):
        slots = meta.slot_mapping()
        bta = pkg.attach(rows_bt, meta)
        for l in range(L):
            if src is not None:     # e2e: this layer's inputs from pinned host memory, output read back
                for dst, h in zip((inp.q[0], inp.k[0], inp.v[0]), src):
                    dst[:tokens].copy_(h[:tokens], non_blocking=True)
                    moved[0] += h[:tokens].numel() * 2
                ql, kl, vl = inp.q[0][:tokens], inp.k[0][:tokens], inp.v[0][:tokens]
            else:
                ql, kl, vl = inp.q[l][:tokens], inp.k[l][:tokens], inp.v[l][:tokens]
            pkg.reshape_and_cache(kl, vl, k_pools[l], v_pools[l], slots)
            if marks is not None:
                marks[l][0].record(stream)
            out = pkg.paged_attention_cuda(ql, k_pools[l], v_pools[l], bta, dummy, dummy, D ** -0.5)
            if marks is not None:
                marks[l][1].record(stream)
            launches[0] += 1 + len(pkg._lib.last_launches())
            if src is not None:
                host["out"][:tokens].copy_(out, non_blocking=True)
                moved[1] += out.numel() * 2

    graph = None
    if args.graphs:                 # the decode pass as one captured CUDA graph per step
        import importlib

        graphs = importlib.import_module(f"{pkg.__name__}.graphs")
        graph = graphs.DecodeStepGraph(k_pools, v_pools, Hq, D ** -0.5, B, wl.tables.shape[1], device=dev)
        for l in range(L):
            graph.q[l].copy_(dec.q[l])
            graph.k_new[l].copy_(dec.k[l])
            graph.v_new[l].copy_(dec.v[l])

    def decode_graph(s, marks=None, src=None):
        graph.set_step(wl.decode_ctx[s], wl.tables)
        if src is not None:
            for dst, h in zip((graph.q, graph.k_new, graph.v_new), src):
                for l in range(L):
                    dst[l].copy_(h[:B], non_blocking=True)
                moved[0] += L * h[:B].numel() * 2
            moved[0] += 4 * graph.words
        if marks is not None:
            marks[0][0].record(stream)
        if graph.graph is None:
            graph.capture()
        else:
            graph.replay()
        if marks is not None:
            marks[0][1].record(stream)
        launches[0] += L * 3
        if src is not None:
            for l in range(L):
                host["out"][:B].copy_(graph.out[l], non_blocking=True)
            moved[1] += L * B * Hq * D * 2

    def step(s, md=None, mp=None, e2e=False):
        if e2e:                     # plan and upload this step's metadata inside the timed region
            dm = plan_decode(s) if graph is None else None
            pm = plan_prefill(s)
            moved[0] += 4 * ((int(dm.plan.words) if dm is not None else 0) + (int(pm.plan.words) if pm is not None else 0))
            dm, pm = (dm.upload(dev) if dm is not None else None), (pm.upload(dev) if pm is not None else None)
        else:
            dm, pm = metas[s]
        if pm is not None:
            run_pass(pm, bts_pre[s], pre, pm.num_tokens, mp, host["pre"] if e2e else None)
        if graph is not None:
            decode_graph(s, md, host["dec"] if e2e else None)
        else:
            run_pass(dm, bt, dec, B, md, host["dec"] if e2e else None)

    clocks = ClockSampler(dev.index)
    with clocks, QuietHost():
        for s in range(args.warmup):
            step(s)
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize(dev)
        md = [[[ev(), ev()] for _ in range(L)] for _ in range(args.steps)]
        mp = [[[ev(), ev()] for _ in range(L)] for _ in range(args.steps)]
        launches[0] = 0
        t0, t1 = ev(), ev()
        t0.record(stream)
        for k in range(args.steps):
            step(args.warmup + k, md[k], mp[k])
        t1.record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
        gpu_launches = launches[0]
        for s in range(args.warmup):
            step(s, e2e=True)
        torch.cuda.synchronize(dev)
        moved[0] = moved[1] = 0
        e0, e1 = ev(), ev()
        e0.record(stream)
        for k in range(args.steps):
            step(args.warmup + k, e2e=True)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        if world > 1:
            torch.distributed.barrier()
    assert pkg.read_device_error(dev) == 0, "a kernel set the device error word"
    timed = [args.warmup + k for k in range(args.steps)]
    elapsed = t0.elapsed_time(t1)
    e2e_ms = e0.elapsed_time(e1)
    dec_ms = (float(np.mean([m[0].elapsed_time(m[1]) for mk in md for m in mk])) if graph is None else
              float(np.mean([mk[0][0].elapsed_time(mk[0][1]) for mk in md])) / L)   # a replay covers all layers
    pre_list = [m[0].elapsed_time(m[1]) for k, mk in enumerate(mp) if metas[timed[k]][1] is not None for m in mk]
    pre_ms = float(np.sum(pre_list)) / L / args.steps if pre_list else 0.0   # per layer, averaged over steps
    times = torch.tensor([elapsed, dec_ms, pre_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(times, op=torch.distributed.ReduceOp.MAX)
    elapsed, dec_ms, pre_ms, e2e_ms = times.tolist()
    if rank != 0:
        return
    tokens = sum(B + len(wl.admit[s]) for s in timed) * world
    ctx_sum = float(np.mean([wl.decode_ctx[s].sum() for s in timed]))
    dec_bytes = ctx_sum * Hkv * D * 2 * 2 + 2 * B * Hq * D * 2 + ctx_sum / 16 * 4 + 8 * B
    hbm_peak, bf16_peak, peak_kind = _measured_peaks()
    pre_flops = float(np.mean([wl.prefill_flops(s, Hq, D) for s in timed]))
    admitted = float(np.mean([len(wl.admit[s]) for s in timed]))
    line = {
        "metric": METRIC, "value": tokens / (elapsed / 1e3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"BASELINE config 4: prefix sharing on the Llama-3-8B shape (32 q / 8 kv heads, "
                               f"head_dim 128, bf16, {L} layers); concurrency {B}; every request = the shared "
                               "128-token prefix (8 physical blocks in every block table) + a unique 32..512-token "
                               "suffix prefilled over the cached prefix; outputs lognormal median 64",
                   "model": "llama3-8b-shape attention hot path (random-init)", "global_batch": B * world,
                   "layers": L, "admitted_per_step": admitted, "seq_len": "ragged (prefix 128 + suffix + output)",
                   "l2": "decode K/V of the whole batch per layer exceeds L2 except the shared prefix blocks, "
                         "which every sequence re-reads (L2 hits); no flush",
                   "parallelism": f"replicas x{world} (request-level data parallel, no collectives)",
                   "decode_pass": "one CUDA graph per step (captured append + attention for all layers)"
                   if graph is not None else "eager launches"},
        "roofline": {"bound": "hbm", "achieved": dec_bytes / (dec_ms / 1e3) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                     "frac": dec_bytes / (dec_ms / 1e3) / 1e9 / hbm_peak, "peak_source": f"{peak_kind} HBM copy",
                     "traffic": None, "kernel": "decode paged attention per layer (tensor-pipe MMA + combine); "
                     "algorithmic bytes count each sequence's prefix blocks, which L2 serves after the first read",
                     "algorithmic_bytes_per_launch": dec_bytes, "avg_launch_ms": dec_ms},
        "prefill_roofline": {"bound": "tensor", "achieved": pre_flops / (pre_ms / 1e3) / 1e12 if pre_ms else None,
                             "peak": bf16_peak, "unit": "TFLOP/s",
                             "kernel": "prefix-hit prefill paged attention per layer (tcgen05, query_len < context_len)",
                             "causal_flops_per_step_layer": pre_flops, "avg_ms_per_step_layer": pre_ms},
        "cpu_baseline": None,
        "e2e": {"value": tokens / (e2e_ms / 1e3), "unit": "tok/s", "h2d_bytes_per_step": moved[0] // args.steps,
                "d2h_bytes_per_step": moved[1] // args.steps, "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": gpu_launches,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


class _Alloc:
    def __init__(self, n: int):
        self.free = list(range(n))[::-1]

    def allocate(self) -> int:
        if not self.free:
            raise MemoryError("pool exhausted")
        return self.free.pop()


class _Table:
    """The attributes the executor reads from the reference's BlockTable."""

    def __init__(self, alloc: _Alloc, block_size: int):
        self.alloc, self.block_size, self.blocks = alloc, block_size, []

    @property
    def capacity(self) -> int:
        return len(self.blocks) * self.block_size

    def ensure_capacity(self, n: int) -> None:
        while self.capacity < n:
            self.blocks.append(self.alloc.allocate())

    def ensure_private(self, logical, copy=None):
        return None

    def release(self) -> None:
        self.alloc.free.extend(reversed(self.blocks))
        self.blocks = []


class _Req:
    """The attributes the executor reads from the reference's Sequence."""

    def __init__(self, prompt, out_len: int):
        self.prompt_token_ids, self.max_tokens = list(prompt), int(out_len)
        self.output_token_ids: list[int] = []
        self.num_cached = 0
        self.block_table = None

    @property
    def next_input_ids(self):
        return (self.prompt_token_ids + self.output_token_ids)[self.num_cached:]


def _c1_requests(n: int, seed: int):
    """BASELINE config 1's workload: prompts of random token ids, length uniform 16..256;
    output lengths lognormal (median 30, sigma 0.9) capped at 512."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(16, 257, size=n)
    outs = np.clip(np.exp(rng.normal(np.log(30), 0.9, size=n)), 1, 512).astype(int)
    return [(rng.integers(0, 50257, size=int(l)).tolist(), int(o)) for l, o in zip(lens, outs)]


def _serve(executor, requests, concurrency: int, num_blocks: int, block_size: int = 16) -> tuple[int, int]:
    """Closed-loop continuous batching in the reference scheduler's shape (admit while a
    slot and blocks are free; a pass is either the admitted prompts' prefill or one decode
    token for every running request, never both).  Returns (generated tokens, passes)."""
    alloc = _Alloc(num_blocks)
    waiting = [_Req(p, o) for p, o in requests]
    running: list[_Req] = []
    generated = passes = 0
    while waiting or running:
        new = []
        while waiting and len(running) + len(new) < concurrency:
            r = waiting[0]
            r.block_table = _Table(alloc, block_size)
            r.block_table.ensure_capacity(len(r.prompt_token_ids) + 1)
            new.append(waiting.pop(0))
        batch = new if new else running
        for r in batch:
            r.block_table.ensure_capacity(r.num_cached + len(r.next_input_ids))
        toks = executor.execute(batch)
        passes += 1
        for r, t in zip(batch, toks):
            r.output_token_ids.append(int(t))
        generated += len(batch)
        running += new
        for r in [r for r in running if len(r.output_token_ids) >= r.max_tokens]:
            r.block_table.release()
            running.remove(r)
    return generated, passes


def run_engine(args, rank: int, world: int, local_rank: int) -> None:
    """``--workload config1``: BASELINE config 1 end to end — a random-init GPT-2 124M
    (fp32, ``torch.manual_seed(0)``) served by the paged executor with the sm_100a
    attention (CudaPagedExecutor), 2,048-block pool of 16-token blocks, 200 requests
    (prompts 16..256 random ids, outputs lognormal median 30 capped at 512), greedy, at
    concurrency 4 and ``--batch`` (32).  Time = the whole closed-loop run (host
    scheduling, HF model, our append + attention kernels, token read-back every pass)."""
    from transformers import GPT2Config, GPT2LMHeadModel

    from __graft_entry__ import import_package

    pkg = import_package()
    executor_mod = __import__(f"{pkg.__name__}.executor", fromlist=["CudaPagedExecutor"])
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    torch.manual_seed(0)
    model = GPT2LMHeadModel(GPT2Config()).to(dev).eval()
    pool = pkg.KVPool.from_model(model, num_blocks=2048)
    ex = executor_mod.CudaPagedExecutor(model, None, pool, decode_graphs=args.graphs)
    reqs = _c1_requests(200, args.seed + rank)
    results = {}
    clocks = ClockSampler(dev.index)
    with clocks, QuietHost():
        _serve(ex, _c1_requests(8, 99), 4, 2048)          # warm-up: kernels, cuBLAS, allocator
        if args.graphs:   # capture every (batch, width) bucket the timed runs will meet
            for conc in sorted({4, args.batch}):
                _serve(ex, _c1_requests(200, 99), conc, 2048)
        torch.cuda.synchronize(dev)
        for conc in sorted({4, args.batch}):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            gen, passes = _serve(ex, reqs, conc, 2048)
            b.record()
            torch.cuda.synchronize(dev)
            results[conc] = (gen, passes, a.elapsed_time(b))
    if rank != 0:
        return
    gen, passes, ms = results[args.batch]
    hbm_peak, _, peak_kind = _measured_peaks()
    weights = sum(p.numel() * p.element_size() for p in model.parameters())
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = _c1_cpu_sample(args)
    line = {
        "metric": METRIC, "value": gen / (ms / 1e3), "unit": "tok/s", "n_gpus": world, "steps": passes,
        "warmup": 1, "ms_per_step": ms / passes, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": "BASELINE config 1: GPT-2 124M random-init (seed 0, fp32) served end to end by the "
                               "paged executor with ATTENTION=cuda; 2,048-block pool, block 16; 200 requests of random "
                               "token ids (prompts 16..256, outputs lognormal median 30 capped at 512); greedy",
                   "model": "gpt2-124m (random-init)", "concurrency": args.batch, "requests": 200,
                   "decode_graphs": bool(args.graphs),
                   "passes": passes, "generated_tokens": gen,
                   "at_concurrency_4": {"tok_s": results[4][0] / (results[4][2] / 1e3), "passes": results[4][1],
                                        "ms": results[4][2]},
                   "l2": "the model's 498 MB of fp32 weights are re-read every pass (> 126 MB L2)",
                   "parallelism": f"replicas x{world}"},
        "roofline": {"bound": "hbm", "achieved": weights * passes / (ms / 1e3) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                     "frac": weights * passes / (ms / 1e3) / 1e9 / hbm_peak, "peak_source": f"{peak_kind} HBM copy",
                     "traffic": None, "kernel": "whole forward pass: model weights read once per pass (the pass is "
                     "weight-bandwidth and host-overhead bound at this batch size)",
                     "algorithmic_bytes_per_launch": weights, "avg_launch_ms": ms / passes},
        "cpu_baseline": cpu,
        "e2e": {"value": gen / (ms / 1e3), "unit": "tok/s",
                "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
                "note": "the value is already end to end: token ids in from the host, greedy ids read back every pass"},
        "gpu_launches": None,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def _c1_cpu_sample(args) -> dict:
    """BASELINE config 1 on the host CPU through the reference's own engine parts: its
    ``Scheduler`` (admission, prefill-priority selection, growth), ``BlockAllocator``,
    ``PagedKVPool`` and ``PagedExecutor`` with ``ATTENTION=gather`` on ``DEVICE=cpu``,
    all imported unchanged from ``baseline/_ref``, serving a bounded sample of the 200
    requests (the first 8, at concurrency 4) with a random-init GPT-2 (seed 0, fp32).
    Falls back to the oracle port under the bench's own loop when the reference is not
    installed."""
    from transformers import GPT2Config, GPT2LMHeadModel

    torch.set_num_threads(os.cpu_count() or 1)
    torch.manual_seed(0)
    model = GPT2LMHeadModel(GPT2Config()).eval()
    sample = _c1_requests(200, args.seed)[:8]
    ref = _reference_modules()
    if ref is None:
        sys.path.insert(0, str(ROOT / "tests"))
        from _engine import OracleExecutor

        ex = OracleExecutor(model, 12, 2048, 16, 12, 64)
        t = time.perf_counter()
        gen, passes = _serve(ex, sample[:4], 4, 2048)
        dt = time.perf_counter() - t
        return {"value": gen / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "port",
                "sample": f"reference not installed in baseline/_ref; the first 4 of the 200 requests at concurrency "
                          f"4 ({gen} tokens, {passes} passes): GPT-2 on the host CPU with the oracle's KV append and "
                          "gather-path attention"}
    C = ref.config.CONFIG
    saved = {k: getattr(C, k) for k in ("device", "attention", "max_running", "block_size", "prefix_caching")}
    try:
        C.device, C.attention, C.max_running, C.block_size, C.prefix_caching = "cpu", "gather", 4, 16, False
        pool = ref.kv_pool.PagedKVPool.from_model(model, num_blocks=2048, block_size=16, device="cpu")
        ex = ref.paged_executor.PagedExecutor(model, None, pool)
        alloc = ref.block_allocator.BlockAllocator(2048)
        sched = ref.scheduler.Scheduler(ex, -1, allocator=alloc, pool=pool)
        seqs = [ref.sequence.Sequence(seq_id=f"r{i}", prompt_token_ids=p, max_tokens=o)
                for i, (p, o) in enumerate(sample)]
        for q in seqs:
            sched.add(q)
        t = time.perf_counter()
        passes = 0
        while sched.has_work:
            sched.step()
            passes += 1
        dt = time.perf_counter() - t
    finally:
        for k, v in saved.items():
            setattr(C, k, v)
    gen = sum(len(q.output_token_ids) for q in seqs)
    return {"value": gen / dt, "unit": "tok/s", "cores": torch.get_num_threads(), "kind": "reference",
            "sample": f"the reference's Scheduler + PagedExecutor (ATTENTION=gather, DEVICE=cpu; baseline/_ref, "
                      f"unchanged) serving the first 8 of the 200 requests at concurrency 4 ({gen} tokens, {passes} "
                      f"passes, {dt:.1f} s) with GPT-2 random-init fp32 on {torch.get_num_threads()} threads"}


BLOCK_POOL_BLOCKS = 16384   # per layer: 16384 x [16, 8, 128] bf16 = 512 MB for K and V
BLOCK_COW_PAIRS = 256       # copy-on-write pairs per step
BLOCK_SWAP = 64             # blocks swapped out and back in per step (a 1,024-token sequence)


def _blocks_cpu_sample(args) -> dict:
    """The oracle's copy_block (the reference's per-layer block copies, in numpy) on a
    host-sized sample of the blocks workload: GB/s read + written."""
    from oracle import paged_attention_oracle as oracle

    block_bytes = 16 * WORKLOADS["blocks"]["kv_heads"] * WORKLOADS["blocks"]["head_dim"] * 2
    ks = np.zeros((4, 2048, block_bytes // 2), dtype=np.uint16)
    vs = np.zeros_like(ks)
    pairs = list(zip(range(0, 128), range(1024, 1152)))
    reps, t_end = [], time.perf_counter() + min(args.cpu_budget_s, 5.0)
    while len(reps) < 3 or time.perf_counter() < t_end:
        a = time.perf_counter()
        oracle.copy_block(ks, vs, pairs)
        reps.append(time.perf_counter() - a)
    moved = 2 * len(pairs) * 4 * 2 * block_bytes
    return {"value": moved / float(np.median(reps)) / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"oracle copy_block: {len(pairs)} pairs x 4 layers x K,V of {block_bytes} B blocks (the "
                      f"reference's per-layer copies, numpy), {len(reps)} repetitions; includes the oracle's "
                      "copy of the input pools"}


def run_oproj(args, rank: int, world: int, local_rank: int) -> None:
    """``--workload oproj``: config 5's per-rank output projection on one GPU -- rows =
    ``--batch`` (512), k = 64 heads x 128 / ``--tp``, n = d_model 8192, bf16 -- through the
    fused collective's kernels with one rank (the tcgen05 GEMM whose epilogue stages the
    tiles, then the owner pass that writes the output) and through cuBLAS (torch.matmul).
    Each step runs one call per weight copy, cycling over enough copies (>= 256 MB) that a
    call's weights are not left in the 126 MB L2 by the previous one.  CUDA events on the
    launching stream; one JSON line."""
    import importlib

    from __graft_entry__ import import_package

    pkg = import_package()
    tpm = importlib.import_module(f"{pkg.__name__}.tensor_parallel")
    w = WORKLOADS["oproj"]
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    rows, n = args.batch, w["d_model"]
    k = w["heads"] * w["head_dim"] // args.tp
    copies = max(2, -(-256 * 2 ** 20 // (n * k * 2)))
    g = torch.Generator(device=dev).manual_seed(args.seed)
    a = torch.randn(rows, k, generator=g, device=dev).to(torch.bfloat16)
    w_nk = [(torch.randn(n, k, generator=g, device=dev) / k ** 0.5).to(torch.bfloat16) for _ in range(copies)]
    w_kn = [t.t().contiguous() for t in w_nk]
    fused = tpm.FusedOProjAllReduce(rows, n, torch.bfloat16, device=dev)
    out = torch.empty(rows, n, dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev)

    def timed(fn):
        for _ in range(args.warmup):
            for c in range(copies):
                fn(c)
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            for c in range(copies):
                fn(c)
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / (args.steps * copies)

    clocks = ClockSampler(dev.index)
    with clocks, QuietHost():
        fused_ms = timed(lambda c: fused(a, w_nk[c]))
        cublas_ms = timed(lambda c: torch.matmul(a, w_kn[c], out=out))
    fused.check()
    flops = 2.0 * rows * k * n
    _, bf16_peak, peak_kind = _measured_peaks()
    line = {
        "metric": "config-5 o_proj per call: fused tcgen05 GEMM (+ owner pass) vs cuBLAS", "unit": "TFLOP/s",
        "value": flops / (fused_ms / 1e3) / 1e12, "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": fused_ms * copies, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"o_proj of one rank at tp{args.tp}: [{rows}, {k}] x [{k}, {n}] bf16",
                   "weight_copies": copies, "l2": f"{copies} weight copies of {n * k * 2 / 2 ** 20:.0f} MB cycled"},
        "fused_us": fused_ms * 1e3, "cublas_us": cublas_ms * 1e3,
        "cublas_tflops": flops / (cublas_ms / 1e3) / 1e12,
        "roofline": {"bound": "tensor", "achieved": flops / (fused_ms / 1e3) / 1e12, "peak": bf16_peak,
                     "unit": "TFLOP/s", "frac": flops / (fused_ms / 1e3) / 1e12 / bf16_peak,
                     "peak_source": f"{peak_kind} sustained bf16", "traffic": None,
                     "kernel": "oproj_push_kernel + oproj_gather_kernel (one rank)"},
        "cpu_baseline": None, "e2e": None,
        "gpu_launches": 2 * (args.warmup + args.steps) * copies,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_blocks(args, rank: int, world: int, local_rank: int) -> None:
    """``--workload blocks``: one step = copy-on-write of BLOCK_COW_PAIRS blocks in every
    layer (one launch), then swap-out of BLOCK_SWAP blocks to pinned host memory and
    swap-in into other blocks (kv_pool.py:142-182's operations, one gather / scatter
    launch and one PCIe copy each).  ``value`` = copy-on-write GB/s (bytes read + written
    by the device-resident copy kernel); ``e2e`` = swap round-trip GB/s over PCIe."""
    from __graft_entry__ import import_package

    pkg = import_package()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = WORKLOADS["blocks"]
    L, NB, P, S = args.layers, BLOCK_POOL_BLOCKS, BLOCK_COW_PAIRS, BLOCK_SWAP
    pool = pkg.KVPool(L, NB, 16, w["kv_heads"], w["head_dim"], torch.bfloat16, dev)
    g = torch.Generator(device=dev).manual_seed(args.seed + rank)
    for t in pool.k + pool.v:
        t.normal_(generator=g)
    block_bytes = 16 * w["kv_heads"] * w["head_dim"] * 2
    rng = np.random.default_rng(args.seed + rank)
    plans = []
    for _ in range(args.warmup + args.steps):
        perm = rng.permutation(NB).tolist()
        plans.append((list(zip(perm[:P], perm[P:2 * P])), perm[2 * P:2 * P + S], perm[2 * P + S:2 * P + 2 * S]))
    copy_bytes = 2 * P * L * 2 * block_bytes      # read + write
    swap_bytes = S * L * 2 * block_bytes          # each direction
    stream = torch.cuda.current_stream(dev)
    ev = lambda: torch.cuda.Event(enable_timing=True)

    def step(s, marks=None):
        pairs, out_b, in_b = plans[s]
        if marks:
            marks[0].record(stream)
        pool.copy_blocks(pairs)
        if marks:
            marks[1].record(stream)
        host = pool.swap_out(out_b)
        if marks:
            marks[2].record(stream)
        pool.swap_in(host, in_b)
        if marks:
            marks[3].record(stream)

    clocks = ClockSampler(dev.index)
    with clocks, QuietHost():
        for s in range(args.warmup):
            step(s)
        torch.cuda.synchronize(dev)
        marks = [[ev() for _ in range(4)] for _ in range(args.steps)]
        t0, t1 = ev(), ev()
        t0.record(stream)
        for k in range(args.steps):
            step(args.warmup + k, marks[k])
        t1.record(stream)
        torch.cuda.synchronize(dev)
    assert pool.read_error() == 0
    total_ms = t0.elapsed_time(t1)
    cow_ms = float(np.mean([m[0].elapsed_time(m[1]) for m in marks]))
    out_ms = float(np.mean([m[1].elapsed_time(m[2]) for m in marks]))
    in_ms = float(np.mean([m[2].elapsed_time(m[3]) for m in marks]))
    if rank != 0:
        return
    hbm_peak, _, peak_kind = _measured_peaks()
    achieved = copy_bytes / (cow_ms / 1e3) / 1e9

    cpu = _blocks_cpu_sample(args) if world == 1 and not args.no_cpu_baseline else None
    line = {
        "metric": "KV block moves: copy-on-write GB/s (device) and swap round trip GB/s (PCIe)",
        "value": achieved, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"block moves on the Llama-3-8B pool shape: {L} layers x {NB} blocks of "
                               f"[16, 8, 128] bf16; per step {P} copy-on-write pairs, {S} blocks swapped out "
                               "and back into other blocks", "layers": L, "pool_blocks": NB,
                   "cow_pairs": P, "swap_blocks": S, "l2": "each step moves >= 0.5 GB, far above the 126 MB L2"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_source": f"{peak_kind} HBM copy", "traffic": None,
                     "kernel": "block_copy_kernel (copy-on-write, all layers in one launch)",
                     "algorithmic_bytes_per_launch": copy_bytes, "avg_launch_ms": cow_ms},
        "cpu_baseline": cpu,
        "e2e": {"value": 2 * swap_bytes / ((out_ms + in_ms) / 1e3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": swap_bytes, "d2h_bytes_per_step": swap_bytes,
                "swap_out_ms": out_ms, "swap_in_ms": in_ms,
                "swap_out_gbs": swap_bytes / (out_ms / 1e3) / 1e9, "swap_in_gbs": swap_bytes / (in_ms / 1e3) / 1e9},
        "gpu_launches": 3 * args.steps,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def _make_workload(args, rank: int, max_steps: int) -> Workload:
    w = WORKLOADS[args.workload]
    return Workload(batch=args.batch, layers=args.layers, heads=w["heads"], kv_heads=w["kv_heads"],
                    head_dim=w["head_dim"], block_size=16, mean_ctx=w["mean_ctx"], lo=w["lo"], hi=w["hi"],
                    sigma=0.9, seed=args.seed + rank, max_steps=max_steps, churn=args.churn,
                    median_ctx=w["median_ctx"])


def _config(args, wl: Workload, world: int) -> dict:
    if args.workload == "config3":
        desc = ("BASELINE config 3: Llama-3-8B-shape GQA paged attention (32 q / 8 kv heads, head_dim 128, "
                "bf16, 32 layers, block 16), batch 256, contexts lognormal mean 4096 clipped 128..16384, "
                f"{wl.n_churn} churn prompts of 256..2048 tokens per step through varlen paged prefill")
        model = "llama3-8b-shape attention hot path (random-init)"
    else:
        desc = (f"BASELINE config 2: isolated paged-decode attention microbenchmark, GPT-2 shape (12 heads, "
                f"head_dim 64, {WORKLOADS[args.workload]['dtype']}, block 16), batch 256, contexts lognormal "
                f"median 1024 clipped 16..8192, {wl.layers} layer(s) per step")
        model = "gpt2-shape attention (random-init)"
    return {
        "workload": desc,
        "model": model,
        "global_batch": wl.batch * world,
        "batch_per_gpu": wl.batch,
        "churn_prompts_per_step": wl.n_churn,
        "layers": wl.layers,
        "heads": wl.heads, "kv_heads": wl.kv_heads, "head_dim": wl.head_dim, "block_size": wl.block_size,
        "sum_context_step0": int(wl.ctx0.sum()),
        "seq_len": "ragged (mean 4096)",
        "l2": f"inputs larger than L2 (each layer's KV is {wl.attention_bytes(0, 2 if args.workload != 'config2-f32' else 4) / 1e9:.2f} GB vs 126 MB L2); no flush",
        "parallelism": f"replicas x{world} (request-level data parallel, no collectives)",
        "step": "prefill pass for the churn prompts + decode pass for the batch; per layer: fused K+V append, "
                "then paged attention",
    }


class _Pass:
    """Device-resident per-layer inputs of one pass (decode or prefill)."""

    def __init__(self, L, tokens, Hq, Hkv, D, dtype, dev, g):
        self.q = [torch.randn(tokens, Hq, D, generator=g, device=dev).to(dtype) for _ in range(L)]
        self.k = [torch.randn(tokens, Hkv, D, generator=g, device=dev).to(dtype) for _ in range(L)]
        self.v = [torch.randn(tokens, Hkv, D, generator=g, device=dev).to(dtype) for _ in range(L)]
        self.free = [None, None]   # e2e: event after the last read of each device input slot


def run_cuda(args, rank: int, world: int, local_rank: int) -> None:
    from __graft_entry__ import import_package

    pkg = import_package()
    lib = pkg._lib.lib()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    steps_total = args.warmup + args.steps
    wl = _make_workload(args, rank, max_steps=steps_total + 1)
    L, B, Hq, Hkv, D, BS = wl.layers, wl.batch, wl.heads, wl.kv_heads, wl.head_dim, wl.block_size
    f32 = WORKLOADS[args.workload]["dtype"] == "f32"
    dtype, elem = (torch.float32, 4) if f32 else (torch.bfloat16, 2)
    tile = _prefill_tile(pkg, args, Hq, Hkv, D)
    sm = pkg.metadata.sm_count(dev)

    # ---- device-resident inputs
    g = torch.Generator(device=dev).manual_seed(args.seed + 100 * rank)
    pool_shape = (wl.num_blocks, BS, Hkv, D)
    k_pools = [torch.empty(pool_shape, dtype=dtype, device=dev).normal_(generator=g) for _ in range(L)]
    v_pools = [torch.empty(pool_shape, dtype=dtype, device=dev).normal_(generator=g) for _ in range(L)]
    dec = _Pass(L, B, Hq, Hkv, D, dtype, dev, g)
    t_pre_max = max(int(wl.prompts[:, :wl.n_churn].sum(axis=1).max()), 1) if wl.n_churn else 1
    pre = _Pass(L, t_pre_max, Hq, Hkv, D, dtype, dev, g)
    bt_dec = torch.from_numpy(wl.tables).to(dev)
    bt_pre = torch.from_numpy(wl.churn_tables).to(dev)
    scale = D ** -0.5

    def plan_decode(step: int):
        m = pkg.StepMetadata.plan_host(wl.context_lens(step), wl.query_lens, wl.tables, num_tokens=B,
                                       pool_num_blocks=wl.num_blocks, block_size=BS, num_kv_heads=Hkv, sm=sm,
                                       prefill_tile_tokens=tile, pinned=True)
        return m.upload(dev)

    def plan_prefill(step: int):
        lens = wl.prompt_lens(step)
        m = pkg.StepMetadata.plan_host(lens, lens, wl.churn_tables[:wl.n_churn], num_tokens=int(lens.sum()),
                                       pool_num_blocks=wl.num_blocks, block_size=BS, num_kv_heads=Hkv, sm=sm,
                                       prefill_tile_tokens=tile, pinned=True)
        return m.upload(dev)

    metas_d = [plan_decode(s) for s in range(steps_total)]
    metas_p = [plan_prefill(s) for s in range(steps_total)] if wl.n_churn else [None] * steps_total
    dummy_lens = torch.zeros(1, dtype=torch.int64, device=dev)
    _reserve_for_timing(pkg, dev, [m for m in metas_d + metas_p if m is not None], Hq, D, dtype,
                        max(B, t_pre_max))
    torch.cuda.synchronize(dev)
    stream = torch.cuda.current_stream(dev)
    launches = [0]

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def run_pass(meta, bt, inp, tokens, ev=None):
        """Per layer: fused append of the pass's new tokens, then attention."""
        slots = meta.slot_mapping()
        bt = pkg.attach(bt, meta)
        for layer in range(L):
            q, k, v = inp.q[layer][:tokens], inp.k[layer][:tokens], inp.v[layer][:tokens]
            pkg.reshape_and_cache(k, v, k_pools[layer], v_pools[layer], slots)
            if ev is not None:
                ev[layer][0].record(stream)
            out = pkg.paged_attention_cuda(q, k_pools[layer], v_pools[layer], bt, dummy_lens, dummy_lens, scale)
            if ev is not None:
                ev[layer][1].record(stream)
            launches[0] += 1 + bin(lib.pa_last_launches()).count("1")   # append + attention kernels

    # e2e copy streams: PCIe is full duplex, so layer l+1's inputs travel up (h2d) and
    # layer l-1's output travels down (d2h) while layer l computes; a step then costs
    # about the larger of its upload, its read-back and its compute, not their sum.
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    nslot = min(2, L)                   # device input slots per pass (double buffering)

    def run_pass_host(meta, bt, inp, tokens, q_src, kv_src, out_host):
        """run_pass with each layer's q / new K / new V copied from pinned host memory
        into a device slot and each layer's attention output read back to the host."""
        slots = meta.slot_mapping()
        bt = pkg.attach(bt, meta)
        loaded = [torch.cuda.Event() for _ in range(L)]

        def load(layer: int):
            s = layer % nslot
            if inp.free[s] is None:     # first use of the slot: after everything before it
                h2d.wait_stream(stream)
            else:                       # after the last attention that read this slot
                h2d.wait_event(inp.free[s])
            with torch.cuda.stream(h2d):
                inp.q[s][:tokens].copy_(q_src[0][:tokens], non_blocking=True)
                inp.k[s][:tokens].copy_(kv_src[0][:tokens], non_blocking=True)
                inp.v[s][:tokens].copy_(kv_src[1][:tokens], non_blocking=True)
            loaded[layer].record(h2d)

        for layer in range(nslot):
            load(layer)
        for layer in range(L):
            s = layer % nslot
            stream.wait_event(loaded[layer])
            q, k, v = inp.q[s][:tokens], inp.k[s][:tokens], inp.v[s][:tokens]
            pkg.reshape_and_cache(k, v, k_pools[layer], v_pools[layer], slots)
            out = pkg.paged_attention_cuda(q, k_pools[layer], v_pools[layer], bt, dummy_lens, dummy_lens, scale)
            done = torch.cuda.Event()
            done.record(stream)
            inp.free[s] = done
            if layer + nslot < L:
                load(layer + nslot)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                out_host[:tokens].copy_(out, non_blocking=True)
            out.record_stream(d2h)      # the allocator keeps `out` until its read-back ends

    def events():
        return [[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(L)]

    def device_step(s: int, ev_d=None, ev_p=None):
        if wl.n_churn:
            mp = metas_p[s]
            run_pass(mp, bt_pre, pre, mp.num_tokens, ev_p)
        run_pass(metas_d[s], bt_dec, dec, B, ev_d)

    clocks = ClockSampler(dev.index)
    with clocks, QuietHost():
        # ---- value: device-resident inputs
        for s in range(args.warmup):
            device_step(s)
        barrier()
        torch.cuda.synchronize(dev)
        launches[0] = 0
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev_d = [events() for _ in range(args.steps)]
        ev_p = [events() for _ in range(args.steps)]
        alloc0 = _allocator_counts(dev)
        start.record(stream)
        t_host = time.perf_counter()
        host_step_ms = []
        for k in range(args.steps):
            t0 = time.perf_counter()
            device_step(args.warmup + k, ev_d[k], ev_p[k])
            host_step_ms.append((time.perf_counter() - t0) * 1e3)
        end.record(stream)
        host_enqueue_ms = (time.perf_counter() - t_host) * 1e3
        alloc1 = _allocator_counts(dev)
        torch.cuda.synchronize(dev)
        barrier()
        gpu_launches = launches[0]
        elapsed_ms = start.elapsed_time(end)
        dec_ms = [ev_d[k][l][0].elapsed_time(ev_d[k][l][1]) for k in range(args.steps) for l in range(L)]
        pre_ms = ([ev_p[k][l][0].elapsed_time(ev_p[k][l][1]) for k in range(args.steps) for l in range(L)]
                  if wl.n_churn else [0.0])

        # ---- e2e: host buffers through the public API
        q_host_d = [dec.q[0].cpu().pin_memory()]
        kv_host_d = [dec.k[0].cpu().pin_memory(), dec.v[0].cpu().pin_memory()]
        out_host_d = torch.empty(B, Hq, D, dtype=dtype).pin_memory()
        q_host_p = [pre.q[0].cpu().pin_memory()]
        kv_host_p = [pre.k[0].cpu().pin_memory(), pre.v[0].cpu().pin_memory()]
        out_host_p = torch.empty(t_pre_max, Hq, D, dtype=dtype).pin_memory()
        h2d_bytes, d2h_bytes = [], []

        def e2e_step(s: int):
            h2d = d2h = 0
            if wl.n_churn:
                mp = plan_prefill(s)
                tp = mp.num_tokens
                run_pass_host(mp, bt_pre, pre, tp, q_host_p, kv_host_p, out_host_p)
                h2d += int(mp.plan.words) * 4 + L * tp * (Hq + 2 * Hkv) * D * elem
                d2h += L * tp * Hq * D * elem
            md = plan_decode(s)
            run_pass_host(md, bt_dec, dec, B, q_host_d, kv_host_d, out_host_d)
            h2d += int(md.plan.words) * 4 + L * B * (Hq + 2 * Hkv) * D * elem
            d2h += L * B * Hq * D * elem
            h2d_bytes.append(h2d)
            d2h_bytes.append(d2h)

        for s in range(args.warmup):
            e2e_step(s)
        barrier()
        torch.cuda.synchronize(dev)
        h2d_bytes.clear()
        d2h_bytes.clear()
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e_start.record(stream)
        for k in range(args.steps):
            e2e_step(args.warmup + k)
        stream.wait_stream(d2h)            # the last read-back is inside the timed region
        e_end.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = e_start.elapsed_time(e_end)
    assert pkg.read_device_error(dev) == 0, "a kernel set the device error word"

    # ---- max over ranks, plus every rank's own figures (a slow rank vs a power-capped node)
    timed = [args.warmup + k for k in range(args.steps)]
    csum = clocks.summary()
    my_dec_gbs = float(np.mean([wl.attention_bytes(s, elem) for s in timed])) / (float(np.mean(dec_ms)) / 1e3) / 1e9
    my_pre_tflops = (float(np.mean([wl.prefill_flops(s) for s in timed])) / (float(np.mean(pre_ms)) / 1e3) / 1e12
                     if wl.n_churn else 0.0)
    mine = torch.tensor([elapsed_ms, e2e_ms, float(np.mean(dec_ms)), float(np.mean(pre_ms)), my_dec_gbs, my_pre_tflops,
                         float(csum.get("sm_mhz") or 0.0), float(csum.get("sw_power_cap_frac") or 0.0),
                         float(csum.get("power_w_max") or 0.0)], dtype=torch.float64, device=dev)
    if world > 1:
        every = torch.empty(world, mine.numel(), dtype=torch.float64, device=dev)
        torch.distributed.all_gather_into_tensor(every, mine)
    else:
        every = mine[None]
    every = every.cpu().numpy()
    elapsed_ms, e2e_ms, dec_avg_ms, pre_avg_ms = (float(x) for x in every[:, :4].max(axis=0))
    if rank != 0:
        return
    per_rank = {"step_ms": [round(float(x) / args.steps, 3) for x in every[:, 0]],
                "decode_gbs": [round(float(x), 1) for x in every[:, 4]],
                "prefill_tflops": [round(float(x), 1) for x in every[:, 5]] if wl.n_churn else None,
                "sm_mhz_median": [float(x) for x in every[:, 6]],
                "sw_power_cap_frac": [round(float(x), 3) for x in every[:, 7]],
                "power_w_max": [round(float(x), 1) for x in every[:, 8]]}

    tokens = (B + wl.n_churn) * args.steps * world
    value = tokens / (elapsed_ms / 1e3)
    e2e_value = tokens / (e2e_ms / 1e3)
    bytes_per_call = float(np.mean([wl.attention_bytes(s, elem) for s in timed]))
    achieved = bytes_per_call / (dec_avg_ms / 1e3) / 1e9
    hbm_peak, bf16_peak, peak_kind = _measured_peaks()
    traffic = (_traffic_per_call(float(np.mean([wl.context_lens(s).sum() for s in timed])))
               if args.workload == "config3" else None)
    pre_flops = float(np.mean([wl.prefill_flops(s) for s in timed])) if wl.n_churn else 0.0
    pre_tflops = pre_flops / (pre_avg_ms / 1e3) / 1e12 if wl.n_churn else None

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_leg(args, wl, "f32" if f32 else "bf16")

    # rank 0's per-launch spread (CUDA events per layer): shows a bimodal launch population
    def pct(xs, digits):
        return [round(float(x), digits) for x in (min(xs), *np.percentile(xs, [10, 50, 90]), max(xs))]

    spread = {"decode_ms_min_p10_p50_p90_max": pct(dec_ms, 4), "prefill_tflops_min_p10_p50_p90_max": None}
    if wl.n_churn:
        rates = [wl.prefill_flops(timed[i // L]) / (t / 1e3) / 1e12 for i, t in enumerate(pre_ms)]
        spread["prefill_tflops_min_p10_p50_p90_max"] = pct(rates, 1)
        slow = [(i // L, i % L, round(pre_ms[i], 3)) for i, r in enumerate(rates) if r < 0.5 * float(np.median(rates))]
        spread["prefill_slow_launches_step_layer_ms"] = slow[:8]
    # host time to enqueue the whole timed loop, and one step's enqueue right after the
    # pre-timing synchronize (empty launch queue, so no blocking: the host's own cost)
    spread["host_enqueue_ms"] = round(host_enqueue_ms, 2)
    spread["host_first_step_ms"] = round(host_step_ms[0], 2)
    spread["host_slowest_step_ms"] = [int(np.argmax(host_step_ms)), round(max(host_step_ms), 2)]
    # device allocations and allocator retries (free-and-retry after a failed cudaMalloc,
    # which synchronises the device) inside the timed loop: both should be 0
    spread["allocator_in_timed_loop"] = {k: alloc1[k] - alloc0[k] for k in alloc0}

    source = "MEASURED_PEAKS.json" if peak_kind == "measured" else "fallback"
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32" if f32 else "bf16", "data": "synthetic",
        "config": _config(args, wl, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                     "frac": achieved / hbm_peak, "peak_source": f"{peak_kind} HBM copy ({source} hbm_gbs)",
                     "frac_of_nominal_8tbs": achieved / NOMINAL_HBM_GBS, "traffic": traffic,
                     "kernel": "decode paged attention per layer (split-K decode + combine; "
                               + ("SIMT fp32" if f32 else "tensor-pipe MMA") + ")",
                     "algorithmic_bytes_per_launch": bytes_per_call, "avg_launch_ms": dec_avg_ms},
        "prefill_roofline": None if not wl.n_churn else {
            "bound": "tensor", "achieved": pre_tflops, "peak": bf16_peak, "unit": "TFLOP/s",
            "frac": pre_tflops / bf16_peak, "peak_source": f"{peak_kind} sustained bf16 ({source})",
            "kernel": "prefill paged attention per layer (tcgen05 varlen prefill)",
            "causal_flops_per_launch": pre_flops, "avg_launch_ms": pre_avg_ms,
            "prompt_tokens_per_step": float(np.mean([wl.prompt_lens(s).sum() for s in timed]))},
        "launch_spread": spread,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": int(np.mean(h2d_bytes)),
                "d2h_bytes_per_step": int(np.mean(d2h_bytes)), "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": gpu_launches,
        "clocks": csum,
        "per_rank": per_rank,
        "decode_splits": {"split_blocks": metas_d[0].plan.split_blocks, "items": metas_d[0].plan.num_decode_items,
                          "combine_seqs": metas_d[0].plan.num_combine_seqs},
    }
    print(json.dumps(line), flush=True)


def _prefill_tile(pkg, args, Hq: int, Hkv: int, D: int) -> int:
    """Query tokens per prefill tile: the library's choice, or ``--prefill-tile-rows``
    (256 selects the CTA-pair kernel, 128 the single-CTA kernel) divided by the group."""
    if args.prefill_tile_rows:
        return args.prefill_tile_rows // (Hq // Hkv)
    return pkg.metadata.prefill_tile_tokens(Hq, Hkv, D)


def _allocator_counts(dev) -> dict:
    """Cumulative counters of torch's caching allocator on `dev`: segments obtained from
    cudaMalloc and free-and-retry passes."""
    st = torch.cuda.memory_stats(dev)
    return {"device_allocs": int(st.get("num_device_alloc", 0)), "alloc_retries": int(st.get("num_alloc_retries", 0))}


def _reserve_for_timing(pkg, dev, metas, heads: int, head_dim: int, dtype, max_tokens: int) -> None:
    """Size the library's workspace for the largest plan and leave cached blocks for the
    largest attention outputs before any timed region, so no allocation (a cudaMalloc,
    or the caching allocator freeing and retrying when HBM is nearly full) happens while
    launches are being timed.  A layer's output is allocated while the previous layer's
    is still referenced, so up to three of the largest size can be live at once (the
    timed loop's allocator counters confirm none is made there)."""
    lib = pkg._lib.lib()
    ws = max(int(lib.pa_workspace_bytes(pkg._lib.ctypes.byref(m.plan), heads, head_dim)) for m in metas)
    pkg.attention._workspace(dev, ws)
    tmp = [torch.empty(max_tokens * heads * head_dim, dtype=dtype, device=dev) for _ in range(3)]
    del tmp


def _traffic_per_call(ctx_tokens: float):
    """DRAM bytes per decode launch from the committed ncu summary, scaled from the
    captured case to this workload by context tokens (traffic grows with the K/V bytes
    streamed, which are proportional to them)."""
    p = ROOT / "profiles" / "paged_decode_splitk_traffic.txt"
    if not p.exists():
        return None
    try:
        kv = dict(line.split("=", 1) for line in p.read_text().splitlines()
                  if "=" in line and not line.startswith("#"))
        return float(kv["dram_bytes_per_launch"]) / float(kv["context_tokens"]) * ctx_tokens
    except Exception:
        return None


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["cuda", "reference"], default="cuda")
    ap.add_argument("--batch", type=int, default=None, help="default: the workload's (256; 512 for config5)")
    ap.add_argument("--layers", type=int, default=None, help="default: the workload's (32 for config3)")
    ap.add_argument("--churn", type=float, default=None,
                    help="fraction of the batch re-admitted per step (default: the workload's, 0.05 for config3)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="config3",
                    help="config3 (default headline), BASELINE config 2's isolated decode microbenchmark, "
                         "config5 (70B shape, KV heads sharded over --gpus), or blocks (copy-on-write and swap "
                         "moves)")
    ap.add_argument("--cpu-sample-seqs", type=int, default=4,
                    help="decode sequences in the CPU baseline's sample (the batch's longest among them)")
    ap.add_argument("--cpu-sample-prompts", type=int, default=2, help="churn prompts in the CPU baseline's sample")
    ap.add_argument("--cpu-budget-s", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--prefill-tile-rows", type=int, default=0,
                    help="(token, head) rows per prefill tile: 256 = CTA-pair kernel, 128 = single-CTA kernel "
                         "(default: the library's choice)")
    ap.add_argument("--graphs", action="store_true",
                    help="config4: run the decode pass as a captured CUDA graph per step; config1: the executor's "
                         "all-decode passes as captured graphs of the whole model forward")
    ap.add_argument("--tp", type=int, default=2, help="oproj: the tensor-parallel size whose per-rank k is run")
    ap.add_argument("--allreduce", choices=["peer", "nccl", "fused"], default="peer",
                    help="config5: the o_proj all-reduce over NVLink peer memory (default), NCCL, or fused "
                         "with the o_proj GEMM into one peer-memory collective")
    args = ap.parse_args()
    if args.layers is None:
        args.layers = WORKLOADS[args.workload]["layers"]
    if args.batch is None:
        args.batch = WORKLOADS[args.workload].get("batch", 256)
    if args.churn is None:
        args.churn = WORKLOADS[args.workload]["churn"]
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        if args.impl == "cuda":
            torch.cuda.set_device(local_rank)
            torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                                 device_id=torch.device("cuda", local_rank))
        else:
            torch.distributed.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    try:
        if args.impl == "reference":
            if args.workload == "oproj":
                if rank == 0:
                    print(json.dumps({"impl": "reference", "unavailable": "the reference has no tensor-parallel "
                                      "o_proj (no multi-GPU path); --workload oproj is a GEMM microbenchmark"}))
            elif args.workload == "blocks":
                if rank == 0:
                    cpu = _blocks_cpu_sample(args)
                    print(json.dumps({"impl": "reference", "metric": "KV block moves: copy-on-write GB/s (device) "
                                      "and swap round trip GB/s (PCIe)", "value": cpu["value"], "unit": "GB/s",
                                      "n_gpus": world, "higher_is_better": True, "cpu_baseline": cpu,
                                      "e2e": {"value": cpu["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                                              "d2h_bytes_per_step": 0}}), flush=True)
            else:
                run_reference(args, rank, world)
        elif args.workload == "blocks":
            run_blocks(args, rank, world, local_rank)
        elif args.workload == "config5":
            run_serve_tp(args, rank, world, local_rank)
        elif args.workload == "config5-decode":
            run_tp(args, rank, world, local_rank)
        elif args.workload == "oproj":
            run_oproj(args, rank, world, local_rank)
        elif args.workload == "config4":
            run_prefix(args, rank, world, local_rank)
        elif args.workload == "config1":
            run_engine(args, rank, world, local_rank)
        else:
            run_cuda(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
