"""Benchmark of the paged-attention hot path on B200 (one JSON line on rank 0).

Workload (the shape the north star's >=70 %-of-HBM target is quoted
on): Llama-3-8B-shape GQA decode, 32 query heads / 8 KV heads / head_dim 128, bf16,
32 layers, KV block size 16, a continuous batch of 256 sequences whose contexts are
lognormal with mean 4096 clipped to 128..16384 (seed 0 per rank).  Synthetic data:
pools, queries and new K/V rows are N(0,1); block tables are a seeded permutation of
the pool (non-contiguous, unsorted).  The pools are real per-layer allocations
(about 138 GB of KV for 32 layers), so every layer streams its own 4.3 GB from HBM;
each layer's KV is far larger than the 126 MB L2, which is this benchmark's answer to
L2 flushing.

One step = one decode step of the hot path for the whole batch: the step's ragged
metadata (planned on the host), then for each of the 32 layers the fused K+V append
of the 256 new tokens and paged attention over every sequence's context (split-K
decode + combine).  Contexts grow by one token per step, as in real decode.

* ``value``  decode tokens/s with inputs resident in HBM (per-step metadata uploaded
  before the timed region), timed with CUDA events, max over ranks.
* ``e2e``    the same through the public API with HOST buffers: every step plans its
  metadata on the host and uploads it, copies each layer's q / new K / new V from pinned
  host memory, and reads each layer's attention output back.
* ``roofline``  the paged-attention launch (decode + combine) per layer: algorithmic
  bytes (K+V of every context once, q and out, block ids, lengths) over its CUDA-event
  duration, against the measured HBM copy peak.
* ``cpu_baseline``  the CPU oracle (a numpy port of the reference's gather path) on a
  bounded sample of the same workload, on this host's cores.

Multi-GPU: request-level replicas, one process per GPU, each with its own batch and
pools; no collective on the data path (``scaling: weak``).  ``--impl reference`` times
the reference algorithm's CPU port instead (rank 0 only).
"""

from __future__ import annotations

import argparse
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
    """The seeded decode batch of one rank."""

    def __init__(self, batch: int, layers: int, heads: int, kv_heads: int, head_dim: int, block_size: int,
                 mean_ctx: float, lo: int, hi: int, sigma: float, seed: int, max_steps: int):
        self.batch, self.layers, self.heads, self.kv_heads = batch, layers, heads, kv_heads
        self.head_dim, self.block_size = head_dim, block_size
        rng = np.random.default_rng(seed)
        mu = clipped_lognormal_mu(mean_ctx, sigma, lo, hi)
        self.ctx0 = np.clip(np.exp(rng.normal(mu, sigma, size=batch)), lo, hi).astype(np.int64)
        need = -(-(self.ctx0 + max_steps) // block_size)
        self.num_blocks = int(need.sum()) + 16
        perm = rng.permutation(self.num_blocks)
        self.tables = np.zeros((batch, int(need.max())), dtype=np.int64)
        off = 0
        for i, n in enumerate(need):
            self.tables[i, :n] = perm[off:off + n]
            off += n
        self.query_lens = np.ones(batch, dtype=np.int64)

    def context_lens(self, step: int) -> np.ndarray:
        return self.ctx0 + step

    def attention_bytes(self, step: int, elem: int) -> int:
        """Algorithmic HBM bytes of one layer's paged attention at `step`."""
        ctx = self.context_lens(step)
        kv = int(ctx.sum()) * self.kv_heads * self.head_dim * 2 * elem
        qo = 2 * self.batch * self.heads * self.head_dim * elem
        ids = int((-(-ctx // self.block_size)).sum()) * 4
        return kv + qo + ids + 8 * self.batch


def _measured_hbm() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 100 ms during timing."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None

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
        self.rows = []
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
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        power = [float(r[3]) for r in rows if r[3].replace(".", "").isdigit()]
        reasons = set()
        for r in rows:
            for name, val in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"),
                                 r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        loaded = [s for s, p in zip(sm, power) if p > 0.5 * max(power)] if power else sm
        return {"sm_mhz": statistics.median(loaded or sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows), "power_w_max": max(power) if power else None}


# ------------------------------------------------------------------ CPU legs (oracle)
def _sample_for_cpu(wl: Workload, nseq: int, step: int, dtype: str, seed: int):
    """A bounded sample of the workload for the CPU oracle: the first `nseq` sequences at
    `step`, with their own blocks only (float32 arrays holding bf16 values)."""
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


def cpu_layer_seconds(wl: Workload, nseq: int, dtype: str, budget_s: float, min_reps: int = 2):
    """Mean wall time of one layer of the oracle's decode step (KV append + gather-path
    attention) on the sample, repeated until `budget_s` is spent."""
    from oracle import paged_attention_oracle as oracle

    q, kp, vp, tables, ctx, ql, knew, vnew, slots = _sample_for_cpu(wl, nseq, 0, dtype, seed=1234)
    scale = wl.head_dim ** -0.5
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < min_reps or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        kp2 = oracle.kv_append(kp, slots, knew)
        vp2 = oracle.kv_append(vp, slots, vnew)
        oracle.paged_attention_gather(q, kp2, vp2, tables, ctx, ql, scale, dtype)
        times.append(time.perf_counter() - t0)
    return float(np.mean(times)), len(times)


def run_reference(args, rank: int, world: int) -> None:
    """`--impl reference`: the reference algorithm's CPU port, rank 0 only."""
    if rank != 0:
        return
    wl = _make_workload(args, rank, max_steps=1)
    nseq = args.cpu_sample_seqs
    from oracle import paged_attention_oracle as oracle

    q, kp, vp, tables, ctx, ql, knew, vnew, slots = _sample_for_cpu(wl, nseq, 0, "bf16", seed=1234)
    scale = wl.head_dim ** -0.5

    def one_step():
        t0 = time.perf_counter()
        kp2 = oracle.kv_append(kp, slots, knew)
        vp2 = oracle.kv_append(vp, slots, vnew)
        oracle.paged_attention_gather(q, kp2, vp2, tables, ctx, ql, scale, "bf16")
        return time.perf_counter() - t0

    for _ in range(args.warmup):
        one_step()
    times = [one_step() for _ in range(args.steps)]
    sec_layer = float(np.mean(times))
    value = nseq / (sec_layer * wl.layers)
    threads = _blas_threads()
    sample = (f"{nseq} sequences (contexts {ctx.tolist()}) of the workload, one layer per step of the oracle's "
              f"KV append + gather-path attention (bf16 emulated in float32 numpy), scaled to {wl.layers} layers")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec_layer * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _config(args, wl, world),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "host_cpus": os.cpu_count(),
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ GPU arm
def _make_workload(args, rank: int, max_steps: int) -> Workload:
    return Workload(batch=args.batch, layers=args.layers, heads=32, kv_heads=8, head_dim=128, block_size=16,
                    mean_ctx=4096.0, lo=128, hi=16384, sigma=0.9, seed=args.seed + rank, max_steps=max_steps)


def _config(args, wl: Workload, world: int) -> dict:
    return {
        "workload": "BASELINE config 3: Llama-3-8B-shape GQA paged decode (32 q / 8 kv heads, head_dim 128, "
                    "bf16, 32 layers, block 16), batch 256, contexts lognormal mean 4096 clipped 128..16384",
        "model": "llama3-8b-shape attention hot path (random-init)",
        "global_batch": wl.batch * world,
        "batch_per_gpu": wl.batch,
        "layers": wl.layers,
        "heads": wl.heads, "kv_heads": wl.kv_heads, "head_dim": wl.head_dim, "block_size": wl.block_size,
        "sum_context_step0": int(wl.ctx0.sum()),
        "seq_len": "ragged (mean 4096)",
        "l2": "inputs larger than L2 (each layer's KV is ~4.3 GB vs 126 MB L2); no flush",
        "parallelism": f"replicas x{world} (request-level data parallel, no collectives)",
        "step": "plan metadata, then per layer: fused K+V append of 256 new tokens + paged decode attention",
    }


def run_cuda(args, rank: int, world: int, local_rank: int) -> None:
    from __graft_entry__ import import_package

    pkg = import_package()
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    steps_total = args.warmup + args.steps
    wl = _make_workload(args, rank, max_steps=steps_total + 1)
    L, B, Hq, Hkv, D, BS = wl.layers, wl.batch, wl.heads, wl.kv_heads, wl.head_dim, wl.block_size
    dtype = torch.bfloat16
    elem = 2

    # ---- device-resident inputs
    g = torch.Generator(device=dev).manual_seed(args.seed + 100 * rank)
    pool_shape = (wl.num_blocks, BS, Hkv, D)
    k_pools, v_pools = [], []
    for _ in range(L):
        k_pools.append(torch.empty(pool_shape, dtype=dtype, device=dev).normal_(generator=g))
        v_pools.append(torch.empty(pool_shape, dtype=dtype, device=dev).normal_(generator=g))
    q_dev = [torch.randn(B, Hq, D, generator=g, device=dev).to(dtype) for _ in range(L)]
    k_new = [torch.randn(B, Hkv, D, generator=g, device=dev).to(dtype) for _ in range(L)]
    v_new = [torch.randn(B, Hkv, D, generator=g, device=dev).to(dtype) for _ in range(L)]
    bt_dev = torch.from_numpy(wl.tables).to(dev)
    ql_dev = torch.from_numpy(wl.query_lens).to(dev)
    scale = D ** -0.5

    def plan(step: int, upload: bool = True):
        ctx = wl.context_lens(step)
        m = pkg.StepMetadata.plan_host(ctx, wl.query_lens, wl.tables, num_tokens=B,
                                       pool_num_blocks=wl.num_blocks, block_size=BS, num_kv_heads=Hkv,
                                       sm=pkg.metadata.sm_count(dev), pinned=True)
        if upload:
            m.upload(dev)
        return m

    metas = [plan(s) for s in range(steps_total)]
    ctx_dev = [torch.from_numpy(wl.context_lens(s)).to(dev) for s in range(steps_total)]
    torch.cuda.synchronize(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    stream = torch.cuda.current_stream(dev)
    launches_per_step = L * (2 + (1 if metas[0].plan.num_combine_seqs > 0 else 0))

    def device_step(s: int, ev=None):
        meta = metas[s]
        bt = pkg.attach(bt_dev, meta)
        slots = meta.slot_mapping()
        for layer in range(L):
            pkg.reshape_and_cache(k_new[layer], v_new[layer], k_pools[layer], v_pools[layer], slots)
            if ev is not None:
                ev[layer][0].record(stream)
            pkg.paged_attention_cuda(q_dev[layer], k_pools[layer], v_pools[layer], bt, ctx_dev[s], ql_dev, scale)
            if ev is not None:
                ev[layer][1].record(stream)

    clocks = ClockSampler(dev.index)
    with clocks:
        # ---- value: device-resident inputs
        for s in range(args.warmup):
            device_step(s)
        barrier()
        torch.cuda.synchronize(dev)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        layer_events = [[[torch.cuda.Event(enable_timing=True) for _ in range(2)] for _ in range(L)]
                        for _ in range(args.steps)]
        start.record(stream)
        for k in range(args.steps):
            device_step(args.warmup + k, layer_events[k])
        end.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        elapsed_ms = start.elapsed_time(end)
        attn_ms = [layer_events[k][l][0].elapsed_time(layer_events[k][l][1])
                   for k in range(args.steps) for l in range(L)]

        # ---- e2e: host buffers through the public API
        q_host = [t.cpu().pin_memory() for t in q_dev]
        k_host = [t.cpu().pin_memory() for t in k_new]
        v_host = [t.cpu().pin_memory() for t in v_new]
        out_host = [torch.empty(B, Hq, D, dtype=dtype).pin_memory() for _ in range(L)]
        q_buf = [torch.empty_like(t) for t in q_dev]
        k_buf = [torch.empty_like(t) for t in k_new]
        v_buf = [torch.empty_like(t) for t in v_new]
        ctx_host = [torch.from_numpy(wl.context_lens(s)) for s in range(steps_total)]
        meta_bytes = []

        def e2e_step(s: int):
            meta = plan(s)            # host planning + one metadata upload
            meta_bytes.append(int(meta.plan.words) * 4)
            bt = pkg.attach(bt_dev, meta)
            slots = meta.slot_mapping()
            for layer in range(L):
                q_buf[layer].copy_(q_host[layer], non_blocking=True)
                k_buf[layer].copy_(k_host[layer], non_blocking=True)
                v_buf[layer].copy_(v_host[layer], non_blocking=True)
                pkg.reshape_and_cache(k_buf[layer], v_buf[layer], k_pools[layer], v_pools[layer], slots)
                out = pkg.paged_attention_cuda(q_buf[layer], k_pools[layer], v_pools[layer], bt, ctx_host[s],
                                               ctx_host[s], scale)
                out_host[layer].copy_(out, non_blocking=True)

        for s in range(args.warmup):
            e2e_step(s)
        barrier()
        torch.cuda.synchronize(dev)
        e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        meta_bytes.clear()
        e_start.record(stream)
        for k in range(args.steps):
            e2e_step(args.warmup + k)
        e_end.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e2e_ms = e_start.elapsed_time(e_end)
    assert pkg.read_device_error(dev) == 0, "a kernel set the device error word"

    # ---- max over ranks
    times = torch.tensor([elapsed_ms, e2e_ms, float(np.mean(attn_ms))], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(times, op=torch.distributed.ReduceOp.MAX)
    elapsed_ms, e2e_ms, attn_avg_ms = times.tolist()
    if rank != 0:
        return

    tokens = B * args.steps * world
    value = tokens / (elapsed_ms / 1e3)
    e2e_value = tokens / (e2e_ms / 1e3)
    bytes_per_call = float(np.mean([wl.attention_bytes(args.warmup + k, elem) for k in range(args.steps)]))
    achieved = bytes_per_call / (attn_avg_ms / 1e3) / 1e9
    peak, peak_kind = _measured_hbm()
    traffic = _traffic_per_call(float(np.mean([wl.context_lens(args.warmup + k).sum()
                                               for k in range(args.steps)])))

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        sec_layer, reps = cpu_layer_seconds(wl, args.cpu_sample_seqs, "bf16", args.cpu_budget_s)
        cpu = {"value": args.cpu_sample_seqs / (sec_layer * L), "unit": "tok/s", "cores": _blas_threads(),
               "kind": "port",
               "sample": f"{args.cpu_sample_seqs} sequences of the workload (contexts "
                         f"{wl.context_lens(0)[:args.cpu_sample_seqs].tolist()}), {reps} repetitions of one layer "
                         f"of the oracle's KV append + gather-path attention (bf16 emulated in float32 numpy), "
                         f"scaled to {L} layers; host has {os.cpu_count()} CPUs"}

    h2d = float(np.mean(meta_bytes)) + L * (q_host[0].numel() + 2 * k_host[0].numel()) * elem
    d2h = L * out_host[0].numel() * elem
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _config(args, wl, world),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6.65 TB/s",
                     "frac_of_nominal_8tbs": achieved / NOMINAL_HBM_GBS, "traffic": traffic,
                     "kernel": "paged attention per layer (split-K decode + combine)",
                     "algorithmic_bytes_per_launch": bytes_per_call, "avg_launch_ms": attn_avg_ms},
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": "tok/s", "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                "ms_per_step": e2e_ms / args.steps},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
        "decode_splits": {"split_blocks": metas[0].plan.split_blocks, "items": metas[0].plan.num_decode_items,
                          "combine_seqs": metas[0].plan.num_combine_seqs},
    }
    print(json.dumps(line), flush=True)


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
    ap.add_argument("--batch", type=int, default=256)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--cpu-sample-seqs", type=int, default=4)
    ap.add_argument("--cpu-budget-s", type=float, default=15.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
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
            run_reference(args, rank, world)
        else:
            run_cuda(args, rank, world, local_rank)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
