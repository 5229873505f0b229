#!/usr/bin/env python
"""Paged decode attention throughput on B200 (one decode step per iteration).

Default workload: config 3 -- batch 256, GQA 32/8, head_dim 128, FP16 pages
of 16 tokens, context lengths LogNormal(ln 8192, sigma=0.5) clipped to
[512, 32768], sharded by sequence across the N GPUs (greedy length
balancing), every GPU with its own TensorPagedKVCache and device pool, no
collective.  A step is the SDK's decode transaction for the whole shard:
pkv_step_begin (decode locks, reserve one token per sequence, page-table
patch upload), pkv_paged_decode_append (the new K/V rows stored by the
decode kernel itself, then paged SDPA; --unfused: pkv_kv_append and
pkv_paged_decode as two calls), and pkv_step_end (commit lengths, release
locks).

  value  tokens/s of the whole job with Q and new K/V rows already in HBM
         (total tokens of all ranks / max over ranks of the device step time)
  e2e    the same step with Q and new K/V copied from pinned host memory and
         the attention output copied back every step
  roofline  the decode kernel: algorithmic bytes per launch (K+V of every
         visible token, Q, O, block table) / mean launch time (CUDA events)
  cpu_baseline  the SDK's own CPU attention (tensor_sdpa_f32 built from its
         sources, oracle/_ref) on a sample of the same sequences, all host
         threads; rank 0 at N=1 only

--impl reference times only that SDK CPU path (rank 0; other ranks exit).
Run under torchrun for N > 1 (RANK/LOCAL_RANK/WORLD_SIZE from the env).
"""
from __future__ import annotations

import argparse
import dataclasses
import datetime
import json
import math
import os
import pathlib
import statistics
import sys
import threading
import time
import time

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from inference_c_b200 import workloads as W  # noqa: E402

FALLBACK_HBM_GBS = 6650.0


def parse_args():
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawTextHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=100)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--config", type=int, choices=[2, 3, 4, 5, 6, 7], default=3)
    p.add_argument("--chunk", type=int, default=0, help="decode split size in tokens (0: auto)")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--cpu-seconds", type=float, default=12.0,
                   help="wall-time budget of the cpu_baseline sample")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--head-dim", type=int, choices=[64, 128], default=0,
                   help="configs 2, 3 and 7: run the configuration with this head size "
                        "instead of its 128 (decode: 64 takes the paired tensor-core path); a "
                        "variant, not a BASELINE.json configuration, named so in "
                        "config.workload")
    p.add_argument("--comm", choices=["pkv", "torch", "peer"], default="pkv",
                   help="config 4 all-gather: the library's NCCL communicator with a host "
                        "deadline (pkv_comm_*), torch.distributed's all_gather_into_tensor "
                        "(NCCL), or the library's peer-store all-gather over NVLink "
                        "(pkv_peer_*, an A/B variant)")
    p.add_argument("--unfused", action="store_true",
                   help="decode configs: append with pkv_kv_append and decode with "
                        "pkv_paged_decode (two launches) instead of the one-launch "
                        "pkv_paged_decode_append (an A/B variant)")
    p.add_argument("--prefill-batch", type=int, default=0,
                   help="config 5 only: sequences per step (default: the config's 8; smaller "
                        "values make small cases for profiling)")
    return p.parse_args()


def peak_hbm() -> tuple[float, str]:
    f = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(f.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per algorithmic
# byte of one paged_decode_tc_kernel launch, from single-launch ncu captures
# of this bench's own command (summaries: profiles/decode_tc_cfg2.md,
# decode_tc_cfg3.md, decode_tc_cfg4.md).  A declared measurement, not read
# at run time; roofline.traffic scales it to this run's algorithmic bytes.
DECODE_DRAM_PER_ALG_BYTE = {2: 1.015, 3: 1.001, 4: 1.007}


def traffic_ratio(cfg: int):
    return DECODE_DRAM_PER_ALG_BYTE.get(cfg)


def metric_name(cfg: int) -> str:
    return ("paged decode attention tokens/s (config %d: append 1 token per sequence + paged "
            "SDPA per step)" % cfg)


def decode_config(cfg: int, head_dim: int = 0):
    """The workload of a decode configuration, optionally at another head
    size (a variant: the name says so)."""
    c = W.CONFIGS[cfg]
    if head_dim and head_dim != c.head_dim:
        c = dataclasses.replace(c, head_dim=head_dim,
                                name=f"{c.name} -- variant at head_dim {head_dim}")
    return c


def config_block(cfg: int, n: int, chunk: int, head_dim: int = 0) -> dict:
    c = decode_config(cfg, head_dim)
    d = {"workload": c.name, "batch": c.batch, "q_heads": c.q_heads, "kv_heads": c.kv_heads,
         "head_dim": c.head_dim, "block_size": c.block_size, "storage": "f16",
         "accumulate": "f32", "decode_chunk_tokens": chunk,
         "parallelism": f"sequence-sharded over {n} GPU(s), one page pool per GPU, no collective",
         "l2": "no flush needed: every step reads all visible pages (> 126 MB L2)"}
    if cfg == 3:
        d["lognormal_sigma"] = W.CFG3_SIGMA
        d["lengths"] = "LogNormal(ln 8192, 0.5) clipped [512, 32768]"
    else:
        d["lengths"] = "U[1024, 4096]"
    return d


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while running."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, uuid: str):
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            u = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
            self._h = pynvml.nvmlDeviceGetHandleByUUID(u)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h) & ~0x1
            except Exception:
                pass
            time.sleep(0.01)

    def __enter__(self):
        if self._nv is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join()

    def summary(self) -> dict:
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": [n for b, n in self.REASONS.items() if self.reasons & b]}


def auto_chunk(lengths: np.ndarray, kv_heads: int, sms: int = 148) -> int:
    """Split size giving ~24 units per persistent CTA (2 CTAs per SM)."""
    units = float(lengths.sum()) * kv_heads / (sms * 2 * 24)
    c = int(math.ceil(max(units, 128) / 64.0) * 64)
    return min(c, 4096)


# ---------------------------------------------------------------------------
# SDK CPU path (oracle/_ref): the reference arm and cpu_baseline
# ---------------------------------------------------------------------------

def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def host_sample_job(cfg: int, lengths: np.ndarray, picks: np.ndarray, seed: int):
    """RefJob over host-generated FP16 pages for the chosen sequences."""
    from oracle import oracle as O
    c = W.CONFIGS[cfg]
    rng = np.random.default_rng(seed + 99)
    L = lengths[picks]
    pages = (L + 15) // 16
    rows = int(pages.sum()) * 16
    k = rng.standard_normal((rows, c.kv_width), dtype=np.float32).astype(np.float16).view(np.uint16)
    v = rng.standard_normal((rows, c.kv_width), dtype=np.float32).astype(np.float16).view(np.uint16)
    q = rng.standard_normal((len(picks), c.q_heads, c.head_dim), dtype=np.float32).astype(
        np.float16).view(np.uint16)
    tables = np.zeros((len(picks), int(pages.max())), np.uint32)
    at = 0
    for i, n in enumerate(pages):
        tables[i, :n] = np.arange(at, at + n)
        at += n
    return O.RefJob("f16", q, None, k, v, c.kv_heads, c.head_dim, 16, tables, L, c.q_heads,
                    c.scale, False)


def stratified(lengths: np.ndarray, n: int) -> np.ndarray:
    order = np.argsort(lengths, kind="stable")
    idx = np.linspace(0, len(order) - 1, num=max(1, min(n, len(order)))).round().astype(int)
    return np.unique(order[idx])


def calibrate_sample(cfg: int, lengths: np.ndarray, threads: int, budget_s: float, seed: int):
    """Sequences per sample so that one run of the SDK path takes ~budget_s."""
    probe = stratified(lengths, threads)
    job = host_sample_job(cfg, lengths, probe, seed)
    t = job.run(threads)
    job.close()
    per_round = max(t, 1e-3)  # one sequence per thread, in parallel
    rounds = max(1, int(budget_s / per_round))
    picks = stratified(lengths, min(len(lengths), rounds * threads))
    # bound host memory: at most ~300k context tokens (~2.5 GB widened to FP32)
    while len(picks) > 1 and int(lengths[picks].sum()) > 300_000:
        picks = stratified(lengths, len(picks) // 2)
    return picks


def sdk_cpu_rate(cfg: int, lengths: np.ndarray, budget_s: float, seed: int,
                 repeats: int = 1) -> tuple[list[float], dict]:
    threads = cpu_threads()
    picks = calibrate_sample(cfg, lengths, threads, budget_s, seed)
    job = host_sample_job(cfg, lengths, picks, seed)
    times = [job.run(threads) for _ in range(repeats)]
    job.close()
    rates = [len(picks) / t for t in times]
    info = {"cores": min(threads, len(picks)), "kind": "reference",
            "sample": (f"{len(picks)} of {len(lengths)} sequences (stratified by length, "
                       f"{int(lengths[picks].sum())} tokens of context) through the SDK's "
                       f"tensor_sdpa_f32 built from its sources; gather+widen untimed")}
    return rates, info


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    lengths = W.context_lengths(args.config, args.seed)
    threads = cpu_threads()
    steps, warmup = args.steps, args.warmup
    budget = max(0.05, 150.0 / max(1, steps + warmup))  # whole run within a few minutes
    picks = calibrate_sample(args.config, lengths, threads, budget, args.seed)
    job = host_sample_job(args.config, lengths, picks, args.seed)
    for _ in range(warmup):
        job.run(threads)
    times = [job.run(threads) for _ in range(steps)]
    job.close()
    t = statistics.mean(times)
    value = len(picks) / t
    line = {
        "metric": metric_name(args.config), "value": value, "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": steps, "warmup": warmup, "ms_per_step": t * 1e3,
        "higher_is_better": True, "scaling": "strong" if args.config == 3 else "weak",
        "vs_baseline": None, "dtype": "f16", "data": "synthetic (seeded N(0,1) FP16)",
        "impl": "reference",
        "config": config_block(args.config, args.gpus, 0),
        "cpu_baseline": {"value": value, "unit": "tokens/s",
                         "cores": min(threads, len(picks)),  # one sequence per thread
                         "kind": "reference",
                         "sample": (f"each step: {len(picks)} of {len(lengths)} sequences "
                                    "(stratified by length) through the SDK's tensor_sdpa_f32 "
                                    "on all host threads; gather+widen untimed")},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------

def run_ours(args) -> None:
    import torch

    import inference_c_b200 as P

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    P.load()
    cfg = args.config
    c = decode_config(cfg, args.head_dim)
    if cfg == 3:
        all_len = W.context_lengths(3, args.seed)
        shard = W.shard_by_length(all_len, world)[rank]
        lengths = all_len[shard]
        total_seqs = len(all_len)
    else:  # config 2 is a per-GPU batch of 32: weak scaling, one seed per rank
        lengths = W.context_lengths(2, args.seed + rank)
        total_seqs = len(lengths) * world
    n = len(lengths)
    steps, warmup = args.steps, args.warmup
    e2e_steps = 0 if args.no_e2e else steps
    grow = 2 * warmup + steps + e2e_steps + 2
    chunk = args.chunk or auto_chunk(lengths + grow // 2, c.kv_heads)

    # ---- cache, pool, fragmented tables, context import ----
    pages_final = (lengths + grow + 15) // 16
    pool_pages = int(math.ceil(pages_final.sum() * 1.1)) + 16
    max_pages = int(pages_final.max()) + 1
    cache = P.PagedKVCache(16, pool_pages, n)
    pool = P.PagedPool(cache, local, P.PKV_DTYPE_F16, 1, c.kv_heads, c.head_dim, n, max_pages)
    seqs = [cache.sequence_create() for _ in range(n)]
    pages_now = (lengths + 15) // 16
    picks = np.repeat(np.arange(n), pages_now)
    picks = picks[W.permutation(args.seed + 7, len(picks), stream=rank)]
    have = np.zeros(n, np.int64)
    for b in picks:  # one page at a time, sequences in seeded random order
        have[b] += 1
        assert cache.reserve(seqs[b], int(min(lengths[b], 16 * have[b])))
    pool.step_begin(seqs, lengths.tolist())  # the whole context is this step's new rows
    batch = pool.step_batch()
    layer = pool.layer(0)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank)
    off_all = np.concatenate([[0], np.cumsum(lengths)])
    start = 0
    while start < n:  # import ~128 MB of rows at a time
        stop = start
        while stop < n and (off_all[stop + 1] - off_all[start]) * c.kv_width <= (64 << 20):
            stop += 1
        stop = max(stop, start + 1)
        counts = np.zeros(n, np.int64)
        counts[start:stop] = lengths[start:stop]
        offs = torch.from_numpy(np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)).to(dev)
        rows = int(counts.sum())
        kr = torch.randn(rows, c.kv_width, generator=gen, device=dev).half()
        vr = torch.randn(rows, c.kv_width, generator=gen, device=dev).half()
        P.kv_import(layer, batch, kr, vr, offs)
        del kr, vr
        start = stop
    pool.step_end(True)
    torch.cuda.synchronize()

    q = torch.randn(n, c.q_heads, c.head_dim, generator=gen, device=dev).half()
    newk = torch.randn(n, c.kv_width, generator=gen, device=dev).half()
    newv = torch.randn(n, c.kv_width, generator=gen, device=dev).half()
    out = torch.empty(n, c.q_heads, c.head_dim, dtype=torch.float16, device=dev)
    max_len = int(lengths.max()) + grow
    ws = P.decode_workspace(n, c.q_heads, c.head_dim, max_len, chunk, device=dev)
    stream = torch.cuda.current_stream()
    cur = lengths.copy()
    launches = {"n": 0}
    bytes_log: list[float] = []
    kv_bytes_per_token = c.kv_width * 2 * 2

    stepper = P.DecodeStepper(pool, layer, seqs, q, newk, newv, out, c.scale, max_len, ws, chunk,
                              stream, fused=not args.unfused)

    def step(i: int | None, bufs=None):
        """One SDK transaction for the shard: step_begin (one staging kernel),
        append + paged decode (one kernel; two with --unfused), step_end,
        through the C ABI with the arguments bound once (DecodeStepper).
        Nothing else is put on the stream between the kernels, so each one's
        launch and prologue overlap the one before it (programmatic dependent
        launch)."""
        nonlocal cur
        if bufs is not None:
            stepper.bind(*bufs)
        stepper.step()
        cur = cur + 1
        if i is not None:
            launches["n"] += 3 if args.unfused else 2  # staging, (append,) decode
            bytes_log.append(float(cur.sum()) * kv_bytes_per_token + 2 * q.numel() * 2 +
                             float(((cur + 15) // 16).sum()) * 4)

    def barrier():
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid))
    with sampler:
        for _ in range(warmup):
            step(None)
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(steps):
            step(i)
        t1.record(stream)
        barrier()
        ms_step = t0.elapsed_time(t1) / steps
        # ---- the decode kernel alone, for the roofline: an open step with no
        # new tokens, K launches each bracketed by events ----
        pool.step_begin(seqs, [0] * n)
        b0 = pool.step_batch()
        ev_a = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ev_b = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        for i in range(steps):
            ev_a[i].record(stream)
            P.paged_decode(layer, b0, q, out, c.scale, max_len, ws, chunk)
            ev_b[i].record(stream)
        pool.step_end(True)
        torch.cuda.synchronize()
        dec_ms = [a.elapsed_time(b) for a, b in zip(ev_a, ev_b)]
        dec_bytes = float(cur.sum()) * kv_bytes_per_token + 2 * q.numel() * 2 + \
            float(((cur + 15) // 16).sum()) * 4
        # ---- e2e: host buffers in, output back, every step.  Two buffer sets:
        # step i+1's uploads (copy stream) overlap step i's kernels, step i's
        # download overlaps step i+1 ----
        e2e = None
        if e2e_steps:
            copy = torch.cuda.Stream(device=dev)
            h_q = [torch.empty(q.shape, dtype=q.dtype, pin_memory=True).copy_(q.cpu())
                   for _ in range(2)]
            h_k = [torch.empty(newk.shape, dtype=newk.dtype, pin_memory=True).copy_(newk.cpu())
                   for _ in range(2)]
            h_v = [torch.empty(newv.shape, dtype=newv.dtype, pin_memory=True).copy_(newv.cpu())
                   for _ in range(2)]
            h_o = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
            d_q = [torch.empty_like(q) for _ in range(2)]
            d_k = [torch.empty_like(newk) for _ in range(2)]
            d_v = [torch.empty_like(newv) for _ in range(2)]
            d_o = [torch.empty_like(out) for _ in range(2)]
            up_done = [torch.cuda.Event() for _ in range(2)]
            step_done = [torch.cuda.Event() for _ in range(2)]
            used = [False, False]

            def upload(s_: int):
                with torch.cuda.stream(copy):
                    if used[s_]:
                        copy.wait_event(step_done[s_])  # step s_-2 no longer reads them
                    d_q[s_].copy_(h_q[s_], non_blocking=True)
                    d_k[s_].copy_(h_k[s_], non_blocking=True)
                    d_v[s_].copy_(h_v[s_], non_blocking=True)
                    up_done[s_].record(copy)

            def e2e_run(k: int):
                upload(0)
                for i in range(k):
                    s_ = i & 1
                    if i + 1 < k:
                        upload(s_ ^ 1)
                    stream.wait_event(up_done[s_])
                    step(None, (d_q[s_], d_k[s_], d_v[s_], d_o[s_]))
                    step_done[s_].record(stream)
                    used[s_] = True
                    with torch.cuda.stream(copy):
                        copy.wait_event(step_done[s_])
                        h_o[s_].copy_(d_o[s_], non_blocking=True)

            e2e_run(warmup)
            barrier()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            e2e_run(e2e_steps)
            stream.wait_stream(copy)  # the last download is inside the timed region
            e1.record(stream)
            barrier()
            e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
            h2d = (h_q[0].numel() + h_k[0].numel() + h_v[0].numel()) * 2
            d2h = h_o[0].numel() * 2
            e2e = {"value": total_seqs / (e2e_ms / 1e3), "unit": "tokens/s",
                   "ms_per_step": e2e_ms, "h2d_bytes_per_step": h2d * world,
                   "d2h_bytes_per_step": d2h * world,
                   "api": ("pkv_step_begin/pkv_kv_append/pkv_paged_decode/pkv_step_end"
                           if args.unfused else
                           "pkv_step_begin/pkv_paged_decode_append/pkv_step_end") +
                          " (DecodeStepper) + pinned host<->device copies on a second stream, "
                          "double-buffered"}
    fault = P.device_fault(local)
    if fault:
        raise SystemExit(f"device fault code {fault} recorded during the bench")
    ms_max = max_over_ranks(ms_step)
    mean_dec = statistics.mean(dec_ms)
    alg_bytes = dec_bytes
    peak, peak_kind = peak_hbm()
    achieved = alg_bytes / (mean_dec / 1e3) / 1e9
    ratio = traffic_ratio(cfg) if c.head_dim == 128 else None  # captured at head_dim 128
    per_rank = {"rank": rank, "decode_ms": mean_dec, "gbs": achieved, "seqs": n,
                "tokens": int(cur.sum())}
    gathered = [per_rank]
    if dist is not None:
        gathered = [None] * world
        dist.all_gather_object(gathered, per_rank)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            rates, info = sdk_cpu_rate(cfg, lengths, args.cpu_seconds, args.seed)
            cpu = {"value": rates[0], "unit": "tokens/s", **info}
        except FileNotFoundError as e:
            cpu = {"value": None, "unit": "tokens/s", "cores": cpu_threads(), "kind": "reference",
                   "sample": f"unavailable: {e}"}
    if rank == 0:
        line = {
            "metric": metric_name(cfg),
            "value": total_seqs / (ms_max / 1e3),
            "unit": "tokens/s",
            "n_gpus": world, "steps": steps, "warmup": warmup, "ms_per_step": ms_max,
            "higher_is_better": True,
            "scaling": "strong" if cfg == 3 else "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic: seeded N(0,1) FP16 Q/K/V on the device, seeded lengths",
            "config": config_block(cfg, world, chunk, args.head_dim),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": None if ratio is None else ratio * alg_bytes,
                         "traffic_source": (f"declared ncu ratio {ratio} DRAM bytes per "
                                            f"algorithmic byte (capture summarised in "
                                            f"profiles/decode_tc_cfg{cfg}.md) x this run's "
                                            f"algorithmic bytes"),
                         "peak_kind": peak_kind, "kernel": "paged_decode_kernel",
                         "algorithmic_bytes_per_launch": alg_bytes,
                         "mean_launch_ms": mean_dec,
                         "launch_timing": "CUDA events around each of K decode launches on the "
                                          "launch stream, in a decode-only loop right after "
                                          "the timed steps (same pages, lengths after them)",
                         "per_rank": gathered},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches["n"],
            "clocks": sampler.summary(),
        }
        print(json.dumps(line), flush=True)
    cache.free()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# Config 5: chunked prefill over the paged cache
# ---------------------------------------------------------------------------

def prefill_flops(past: int, chunk: int, batch: int, q_heads: int, d: int) -> float:
    """QK^T and PV FLOPs of causal chunked prefill (the chunk sees the past
    and itself causally)."""
    return float(batch) * q_heads * 4 * d * (chunk * past + chunk * (chunk + 1) / 2)


def measured_peak_tflops() -> tuple[float, str]:
    f = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(f.read_text())["bf16_tflops"]), "measured (burst)"
    except Exception:
        return 1590.0, "fallback"


def cfg5_block() -> dict:
    c = W.CONFIGS[5]
    return {"workload": c.name, "batch": c.batch, "q_heads": c.q_heads, "kv_heads": c.kv_heads,
            "head_dim": c.head_dim, "block_size": c.block_size, "storage": "bf16",
            "accumulate": "f32 (TMEM)", "past": W.CFG5_PAST, "chunk": W.CFG5_CHUNK,
            "causal": "within the chunk (SDK offset kv_len - q_len)",
            "parallelism": "one GPU",
            "l2": "no flush needed: 335 MB of pages + 134 MB of new rows per step (> 126 MB L2)"}


def sdk_prefill_rate(budget_s: float, seed: int) -> tuple[float, dict]:
    """SDK tensor_sdpa_f32 on a slice of config 5: one sequence, one KV head
    (its 4 query heads), the chunk's last n rows, sized to ~budget_s."""
    from oracle import oracle as O
    c = W.CONFIGS[5]
    threads = cpu_threads()
    rng = np.random.default_rng(seed + 5)
    L = W.CFG5_PAST + W.CFG5_CHUNK
    pages = (L + 15) // 16
    k = rng.standard_normal((pages * 16, c.kv_width), dtype=np.float32)
    v = rng.standard_normal((pages * 16, c.kv_width), dtype=np.float32)
    kb, vb = W.f32_to_bf16_bits(k), W.f32_to_bf16_bits(v)
    qrows = W.f32_to_bf16_bits(rng.standard_normal((W.CFG5_CHUNK, c.q_heads, c.head_dim),
                                                   dtype=np.float32))
    tables = np.arange(pages, dtype=np.uint32)[None, :]
    group = c.q_heads // c.kv_heads

    def job(rows, kv_n):
        return O.RefJob("bf16", qrows, np.array([0, W.CFG5_CHUNK], np.int32), kb, vb, c.kv_heads,
                        c.head_dim, 16, tables, np.array([L]), c.q_heads, c.scale, True,
                        kv_head0=0, kv_head_n=kv_n, tail_rows=rows)

    probe = job(16, 1)
    t = probe.run(1)
    probe.close()
    rows = int(max(16, min(W.CFG5_CHUNK, 16 * budget_s / max(t, 1e-4))))
    kv_n = max(1, min(c.kv_heads, threads))
    j = job(rows, kv_n)
    sec = j.run(1)  # one tensor_sdpa_f32 call: the SDK CPU path is single-threaded per call
    j.close()
    flops = kv_n * group * 4 * c.head_dim * sum(W.CFG5_PAST + W.CFG5_CHUNK - rows + i + 1
                                               for i in range(rows))
    info = {"cores": 1, "kind": "reference",
            "sample": (f"one tensor_sdpa_f32 call (causal) on the last {rows} chunk rows of one "
                       f"sequence, {kv_n} KV head(s) x {group} query heads; gather+widen untimed")}
    return flops / sec / 1e12, info


def run_prefill(args) -> None:
    import torch

    import inference_c_b200 as P

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1 and rank != 0:
        return  # config 5 is a one-GPU configuration
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    P.load()
    c = W.CONFIGS[5]
    B, past, chunk = args.prefill_batch or c.batch, W.CFG5_PAST, W.CFG5_CHUNK
    L = past + chunk
    pool_pages = B * ((L + 15) // 16) + 16
    cache = P.PagedKVCache(16, pool_pages, B)
    pool = P.PagedPool(cache, local, P.PKV_DTYPE_BF16, 1, c.kv_heads, c.head_dim, B,
                       (L + 15) // 16 + 1)
    seqs = [cache.sequence_create() for _ in range(B)]
    for r in range(1, (past + 15) // 16 + 1):  # interleaved: fragmented tables
        for s_ in seqs:
            cache.reserve(s_, min(past, 16 * r))
    gen = torch.Generator(device=dev).manual_seed(args.seed)
    pool.step_begin(seqs, [past] * B)
    layer = pool.layer(0)
    kr = torch.randn(B * past, c.kv_width, generator=gen, device=dev).bfloat16()
    vr = torch.randn(B * past, c.kv_width, generator=gen, device=dev).bfloat16()
    P.kv_import(layer, pool.step_batch(), kr, vr, pool.step_row_offsets())
    pool.step_end(True)
    del kr, vr
    newk = torch.randn(B * chunk, c.kv_width, generator=gen, device=dev).bfloat16()
    newv = torch.randn(B * chunk, c.kv_width, generator=gen, device=dev).bfloat16()
    q = torch.randn(B * chunk, c.q_heads, c.head_dim, generator=gen, device=dev).bfloat16()
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream()
    steps, warmup = args.steps, args.warmup
    ea = [torch.cuda.Event(enable_timing=True) for _ in range(4 * steps)]

    def step(i=None):
        # the SDK transaction for a 2048-token chunk per sequence, rolled back
        # at the end so every step appends the same chunk at the same positions
        pool.step_begin(seqs, [chunk] * B)
        b = pool.step_batch()
        offs = pool.step_row_offsets()
        if i is not None:
            ea[4 * i].record(stream)
        P.kv_append(layer, b, newk, newv, offs)
        if i is not None:
            ea[4 * i + 1].record(stream)
            ea[4 * i + 2].record(stream)
        P.paged_prefill(layer, b, q, offs, out, c.scale, chunk, True)
        if i is not None:
            ea[4 * i + 3].record(stream)
        pool.step_end(False)

    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid))
    with sampler:
        for _ in range(warmup):
            step()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(steps):
            step(i)
        t1.record(stream)
        torch.cuda.synchronize()
    fault = P.device_fault(local)
    if fault:
        raise SystemExit(f"device fault code {fault} recorded during the bench")
    ms_step = t0.elapsed_time(t1) / steps
    app_ms = statistics.mean(ea[4 * i].elapsed_time(ea[4 * i + 1]) for i in range(steps))
    pf_ms = statistics.mean(ea[4 * i + 2].elapsed_time(ea[4 * i + 3]) for i in range(steps))
    flops = prefill_flops(past, chunk, B, c.q_heads, c.head_dim)
    peak, kind = measured_peak_tflops()
    hbm, hbm_kind = peak_hbm()
    app_bytes = 2 * 2 * B * chunk * c.kv_width * 2  # K and V rows: read + written
    cpu = None
    if not args.no_cpu_baseline:
        try:
            rate, info = sdk_prefill_rate(args.cpu_seconds, args.seed)
            cpu = {"value": rate, "unit": "TFLOP/s", **info}
        except FileNotFoundError as e:
            cpu = {"value": None, "unit": "TFLOP/s", "kind": "reference", "cores": 1,
                   "sample": f"unavailable: {e}"}
    line = {
        "metric": "chunked prefill attention TFLOP/s over the paged cache (config 5: append "
                  "2048-token chunks + causal prefill per step)",
        "value": flops / (ms_step / 1e3) / 1e12, "unit": "TFLOP/s", "n_gpus": 1,
        "steps": steps, "warmup": warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) BF16 Q/K/V on the device",
        "config": {**cfg5_block(), "batch": B},
        "tokens_per_s": B * chunk / (ms_step / 1e3),
        "roofline": {"bound": "tensor", "achieved": flops / (pf_ms / 1e3) / 1e12, "peak": peak,
                     "unit": "TFLOP/s", "frac": flops / (pf_ms / 1e3) / 1e12 / peak,
                     "traffic": None, "peak_kind": kind, "kernel": "paged_prefill_tc_kernel",
                     "algorithmic_flops_per_launch": flops, "mean_launch_ms": pf_ms,
                     "mma_flops_issued_per_launch": flops * 1.5,
                     "note": "PV runs twice (16-bit P high and low halves), so the tensor "
                             "pipe issues 1.5x the algorithmic FLOPs"},
        "append_roofline": {"bound": "hbm", "achieved": app_bytes / (app_ms / 1e3) / 1e9,
                            "peak": hbm, "unit": "GB/s",
                            "frac": app_bytes / (app_ms / 1e3) / 1e9 / hbm,
                            "kernel": "kv_rows_kernel (append)", "bytes_per_launch": app_bytes,
                            "mean_launch_ms": app_ms, "peak_kind": hbm_kind},
        "cpu_baseline": cpu,
        "e2e": None,
        "gpu_launches": 3 * steps,
        "clocks": sampler.summary(),
    }
    print(json.dumps(line), flush=True)
    cache.free()


# ---------------------------------------------------------------------------
# Config 4: one 131072-token sequence, KV heads split across the GPUs
# ---------------------------------------------------------------------------

def run_cfg4(args) -> None:
    import torch

    import inference_c_b200 as P

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    c = W.CONFIGS[4]
    if c.kv_heads % world:
        raise SystemExit(f"config 4 splits {c.kv_heads} KV heads; --gpus must divide it")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    P.load()
    comm = peer = None
    if dist is not None and args.comm == "peer":
        nbytes = (c.kv_heads // world) * (c.q_heads // c.kv_heads) * c.head_dim * 2
        peer = P.PeerGather(local, world, rank, nbytes)
        handles = [None] * world
        dist.all_gather_object(handles, peer.ipc_handle)
        peer.connect(handles)
    if dist is not None and args.comm == "pkv":
        # the library's non-blocking NCCL communicator: a peer that never joins
        # or stalls ends the wait at the deadline (and the step rolls back)
        box = [P.comm_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        comm = P.Comm(box[0], world, rank, local, timeout_s=60.0)
    kvl = c.kv_heads // world                 # KV heads owned by this rank
    qhl = kvl * (c.q_heads // c.kv_heads)     # their query heads
    steps, warmup = args.steps, args.warmup
    grow = 2 * warmup + 2 * steps + 2
    L0 = W.CFG4_TOKENS
    need = (L0 + grow + 15) // 16
    rng = np.random.default_rng(args.seed + 4)
    gaps = rng.integers(0, 4, need)           # filler pages before each real page
    pool_pages = need + int(gaps.sum()) + 16
    cache = P.PagedKVCache(16, pool_pages, 2)
    pool = P.PagedPool(cache, local, P.PKV_DTYPE_F16, 1, kvl, c.head_dim, 1, need + 1)
    seq, filler = cache.sequence_create(), cache.sequence_create()
    have_f = 0
    for i in range(need):  # same seeded interleaving on every rank: identical tables
        have_f += int(gaps[i])
        if gaps[i]:
            assert cache.reserve(filler, 16 * have_f)
        assert cache.reserve(seq, 16 * (i + 1))
    assert cache.release(filler)
    cache.set_length(seq, 0)
    cache.reserve(seq, L0)
    gen = torch.Generator(device=dev).manual_seed(args.seed * 1000 + rank)
    pool.step_begin([seq], [L0])
    layer = pool.layer(0)
    kv = kvl * c.head_dim
    for start in range(0, L0, 32768):  # this rank's heads only
        n = min(32768, L0 - start)
        kr = torch.randn(n, kv, generator=gen, device=dev).half()
        vr = torch.randn(n, kv, generator=gen, device=dev).half()
        offs = torch.tensor([0, n], dtype=torch.int32, device=dev)
        b = pool.step_batch()
        lens = torch.tensor([start + n], dtype=torch.int32, device=dev)
        P.kv_append(layer, P.PkvBatch(b.block_tables, b.table_stride, lens.data_ptr(), 1), kr,
                    vr, offs)
        torch.cuda.synchronize()
    pool.step_end(True)
    q = torch.randn(1, qhl, c.head_dim, generator=gen, device=dev).half()
    newk = torch.randn(1, kv, generator=gen, device=dev).half()
    newv = torch.randn(1, kv, generator=gen, device=dev).half()
    out = torch.empty(1, qhl, c.head_dim, dtype=torch.float16, device=dev)
    full = torch.empty(world, qhl, c.head_dim, dtype=torch.float16, device=dev)
    max_len = L0 + grow
    ws = P.decode_workspace(1, qhl, c.head_dim, max_len, device=dev)
    stream = torch.cuda.current_stream()
    cur = [L0]

    stepper = P.DecodeStepper(pool, layer, [seq], q, newk, newv, out, c.scale, max_len, ws, 0,
                              stream, fused=not args.unfused)

    def step(q_in=None, k_in=None, v_in=None, full_out=None):
        """Transaction, append, decode of this rank's heads (DecodeStepper:
        the C calls with their arguments bound once), then the all-gather of
        every rank's head outputs.  No events between the kernels, so their
        launches overlap (programmatic dependent launch)."""
        if q_in is not None:
            stepper.bind(q_in, k_in, v_in, out)
        stepper.step()
        cur[0] += 1
        dst = full if full_out is None else full_out
        if comm is not None:
            comm.all_gather(out, dst, stream, timeout_s=10.0)  # per-head outputs, NVLink
        elif peer is not None:
            peer.all_gather(out, dst, stream, timeout_s=5.0)
        elif dist is not None:
            dist.all_gather_into_tensor(dst, out)
        else:
            dst.copy_(out)

    def barrier():
        if comm is not None:
            comm.wait(stream, timeout_s=60.0)  # the collectives of this rank finished
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def gather_only():
        if comm is not None:
            comm.all_gather(out, full, stream, timeout_s=10.0)
        elif peer is not None:
            peer.all_gather(out, full, stream, timeout_s=5.0)
        else:
            dist.all_gather_into_tensor(full, out)

    def timed(fn, k, align=False):
        """Mean device ms of fn() over k calls, CUDA events on the stream;
        align: barrier + synchronize before each call (no rank skew)."""
        ms = []
        for _ in range(k):
            if align:
                barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            if align:
                torch.cuda.synchronize()
            ms.append((a, b))
        torch.cuda.synchronize()
        return statistics.mean(x.elapsed_time(y) for x, y in ms)

    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid))
    with sampler:
        for _ in range(warmup):
            step()
        barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for i in range(steps):
            step()
        t1.record(stream)
        barrier()
        ms = max_over_ranks(t0.elapsed_time(t1) / steps)
        # the decode kernel(s) alone (open step, no new token), and the
        # all-gather alone after a barrier (its latency without rank skew)
        pool.step_begin([seq], [0])
        b0 = pool.step_batch()
        dec = timed(lambda: P.paged_decode(layer, b0, q, out, c.scale, max_len, ws), steps)
        pool.step_end(True)
        ag = timed(gather_only, steps, align=True) if dist is not None else 0.0
        # e2e: host buffers, double-buffered on a copy stream (as config 3)
        copy = torch.cuda.Stream(device=dev)
        h_q = [torch.empty(q.shape, dtype=q.dtype, pin_memory=True).copy_(q.cpu())
               for _ in range(2)]
        h_k = [torch.empty(newk.shape, dtype=newk.dtype, pin_memory=True).copy_(newk.cpu())
               for _ in range(2)]
        h_v = [torch.empty(newv.shape, dtype=newv.dtype, pin_memory=True).copy_(newv.cpu())
               for _ in range(2)]
        h_o = [torch.empty(full.shape, dtype=full.dtype, pin_memory=True) for _ in range(2)]
        d_q = [torch.empty_like(q) for _ in range(2)]
        d_k = [torch.empty_like(newk) for _ in range(2)]
        d_v = [torch.empty_like(newv) for _ in range(2)]
        d_f = [torch.empty_like(full) for _ in range(2)]
        up_done = [torch.cuda.Event() for _ in range(2)]
        step_done = [torch.cuda.Event() for _ in range(2)]
        used = [False, False]

        def upload(s_):
            with torch.cuda.stream(copy):
                if used[s_]:
                    copy.wait_event(step_done[s_])
                d_q[s_].copy_(h_q[s_], non_blocking=True)
                d_k[s_].copy_(h_k[s_], non_blocking=True)
                d_v[s_].copy_(h_v[s_], non_blocking=True)
                up_done[s_].record(copy)

        def e2e_run(k):
            upload(0)
            for i in range(k):
                s_ = i & 1
                if i + 1 < k:
                    upload(s_ ^ 1)
                stream.wait_event(up_done[s_])
                step(d_q[s_], d_k[s_], d_v[s_], d_f[s_])
                step_done[s_].record(stream)
                used[s_] = True
                with torch.cuda.stream(copy):
                    copy.wait_event(step_done[s_])
                    h_o[s_].copy_(d_f[s_], non_blocking=True)

        e2e_run(warmup)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        e2e_run(steps)
        stream.wait_stream(copy)
        e1.record(stream)
        barrier()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / steps)
        h_q, h_k, h_v, h_o = h_q[0], h_k[0], h_v[0], h_o[0]
    fault = P.device_fault(local)
    if fault:
        raise SystemExit(f"device fault code {fault} recorded during the bench")
    peak, peak_kind = peak_hbm()
    alg = cur[0] * kv * 2 * 2 + 2 * q.numel() * 2  # the decode-only launches' length
    gbs = alg / (dec / 1e3) / 1e9
    if rank == 0:
        line = {
            "metric": "paged decode attention tokens/s (config 4: one 131072-token sequence, "
                      "KV heads split across GPUs, NCCL all-gather of per-head outputs)",
            "value": 1.0 / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16",
            "data": "synthetic: seeded N(0,1) FP16 on the device; seeded fragmented block table",
            "config": {"workload": c.name, "tokens": L0, "q_heads": c.q_heads,
                       "kv_heads": c.kv_heads, "head_dim": c.head_dim, "block_size": 16,
                       "kv_heads_per_gpu": kvl,
                       "parallelism": (f"KV-head split over {world} GPU(s) + "
                                       + ("peer-store all-gather" if peer is not None
                                          else "NCCL all-gather")),
                       "l2": "no flush needed: 512 MiB of pages per step at one GPU"},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peak, "unit": "GB/s",
                         "frac": gbs / peak, "traffic": None, "peak_kind": peak_kind,
                         "kernel": "paged_decode_tc_kernel (+ merge kernel when split wide)",
                         "algorithmic_bytes_per_launch": alg, "mean_launch_ms": dec},
            "allgather_ms": ag,
            "allgather_timing": "the all-gather alone, each call after a barrier and "
                                "synchronize (latency without rank skew)",
            "allgather_api": ("pkv_comm_all_gather (NCCL, joined under a host deadline)"
                              if comm is not None else
                              "pkv_peer_all_gather (peer stores over NVLink, bounded waits)"
                              if peer is not None else
                              "torch.distributed all_gather_into_tensor (NCCL)"),
            "cpu_baseline": None,
            "e2e": {"value": 1.0 / (e2e_ms / 1e3), "unit": "tokens/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": (h_q.numel() + h_k.numel() + h_v.numel()) * 2 * world,
                    "d2h_bytes_per_step": h_o.numel() * 2},
            # staging, (append,) decode, merge (+ the peer gather; NCCL's own not counted)
            "gpu_launches": steps * (3 + bool(args.unfused) + (peer is not None)),
            "clocks": sampler.summary(),
        }
        print(json.dumps(line), flush=True)
    cache.free()
    if comm is not None:
        comm.wait(stream, timeout_s=60.0)
        comm.destroy()
    if peer is not None:
        torch.cuda.synchronize()
        dist.barrier()  # no rank still stores into another's area
        peer.destroy()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# Config 6: the SDK's paged decoder entry point end to end
# ---------------------------------------------------------------------------

CFG6 = dict(layers=4, hidden=4096, inter=14336, qh=32, kvh=8, hd=128, vocab=32000,
            context=4096, tokens=16, block=16)


def cfg6_block() -> dict:
    c = CFG6
    return {"workload": ("cfg6: Llama-3-8B-shaped decoder, 4 of its 32 layers, F16 weights, "
                         "GQA 32/8, d=128, vocab 32000, 4096-token context; a step = one "
                         "tensor_attention_decode_sequence_paged call generating 16 tokens"),
            **c, "storage": "TENSOR_PAGED_KV_F16", "weights": "host arrays, device copies "
            "cached after the first call (as the SDK's CUDA backend)",
            "l2": "no flush needed: each token streams 2.0 GB of weights (> 126 MB L2)"}


def cfg6_model(seed: int):
    """Seeded F16 weights (host, uint16 bits) and a 4096-token prefix."""
    import torch
    c = CFG6
    g = torch.Generator().manual_seed(seed)
    kvw = c["kvh"] * c["hd"]

    def mat(o, i, gain=1.0):
        return (torch.randn(o, i, generator=g) * (gain / i ** 0.5)).half().numpy().view(np.uint16)

    def vec(n):
        return (1 + 0.1 * torch.randn(n, generator=g)).half().numpy().view(np.uint16)

    h, it = c["hidden"], c["inter"]
    layers = [[vec(h), mat(h, h), mat(kvw, h), mat(kvw, h), mat(h, h, 0.5), vec(h), mat(it, h),
               mat(it, h), mat(h, it, 0.5)] for _ in range(c["layers"])]
    emb = torch.randn(c["vocab"], h, generator=g).half().numpy().view(np.uint16)
    head = mat(c["vocab"], h, 4.0)
    cap = c["context"] + c["tokens"] * 64
    kc = [torch.randn(cap, kvw, generator=g).half().numpy().view(np.uint16)
          for _ in range(c["layers"])]
    vc = [torch.randn(cap, kvw, generator=g).half().numpy().view(np.uint16)
          for _ in range(c["layers"])]
    return layers, emb, vec(h), head, kc, vc, cap


def cfg6_bytes_per_token(context: int) -> float:
    """Weight bytes every token streams (all layer matrices and norms, lm_head,
    one embedding row) plus the visible K/V rows of every layer."""
    c = CFG6
    h, it, kvw = c["hidden"], c["inter"], c["kvh"] * c["hd"]
    layer = 2 * (h * h + 2 * kvw * h + h * h + 3 * it * h + 2 * h)
    return c["layers"] * (layer + context * kvw * 2 * 2) + 2 * c["vocab"] * h + 2 * h


def run_decoder(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # one sequence: a single-GPU configuration
    import torch
    c = CFG6
    torch.cuda.set_device(0)
    layers, emb, fnorm, head, kc, vc, cap = cfg6_model(args.seed)
    steps, warmup = args.steps, args.warmup
    pages = (cap + c["block"] - 1) // c["block"]
    ref = args.impl == "reference"
    if ref:
        from oracle import oracle as O
        if not O.ref_cuda_available():
            print(json.dumps({"impl": "reference", "unavailable":
                              "oracle/_ref/libref_cuda.so (the SDK's CUDA backend) not built"}))
            return
        dec = O.RefCudaDecoder(c["block"], pages)

        def call(initial, count, past):
            return dec.decode(1, 0, layers, emb, initial, count, kc, vc, past, c["hidden"],
                              c["inter"], c["qh"], c["kvh"], c["hd"], 1e-5, 500000.0, fnorm,
                              head, c["vocab"])
    else:
        import inference_c_b200 as P
        P.load()
        cache = P.PagedKVCache(c["block"], pages, 1)
        seq = cache.sequence_create()

        def call(initial, count, past):
            return P.decode_sequence_paged(cache, seq, P.TENSOR_PAGED_KV_F16, layers, emb,
                                           initial, count, kc, vc, past, c["hidden"], c["inter"],
                                           c["qh"], c["kvh"], c["hd"], 1e-5, 500000.0, fnorm,
                                           head, c["vocab"])
    # first call: prefix import of the 4096-token context and weight upload (untimed)
    past = c["context"]
    toks = call(1, 1, past)
    assert toks is not None, "decoder call failed"
    past += 1
    token = toks[-1]
    sampler = ClockSampler(str(torch.cuda.get_device_properties(0).uuid))
    times = []
    with sampler:
        for i in range(warmup + steps):
            t0 = time.perf_counter()
            toks = call(token, c["tokens"], past)
            dt = time.perf_counter() - t0
            assert toks is not None, "decoder call failed"
            token, past = toks[-1], past + c["tokens"]
            if i >= warmup:
                times.append(dt)
    ms = statistics.mean(times) * 1e3
    tps = c["tokens"] / (ms / 1e3)
    mid_context = c["context"] + 1 + c["tokens"] * (warmup + steps / 2)
    bpt = cfg6_bytes_per_token(int(mid_context))
    hbm, hbm_kind = peak_hbm()
    gbs = bpt * tps / 1e9
    line = {
        "metric": "paged decoder tokens/s (config 6: tensor_attention_decode_sequence_paged, "
                  "16 greedy tokens per call)",
        "value": tps, "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic: seeded N(0,1)-scaled F16 weights and context",
        "config": cfg6_block(),
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                     "frac": gbs / hbm, "traffic": None, "peak_kind": hbm_kind,
                     "bytes_per_token": bpt,
                     "note": "whole call timed on the host clock (the API is synchronous): "
                             "weights + visible K/V per token over the call time"},
        "e2e": {"value": tps, "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4 * c["tokens"],
                "api": "tensor_attention_decode_sequence_paged (host token in, host tokens out)"},
        "gpu_launches": None,
        "clocks": sampler.summary(),
    }
    if ref:
        line["impl"] = "reference"
        line["cpu_baseline"] = {"value": None, "unit": "tokens/s", "cores": 0,
                                "kind": "reference",
                                "sample": "the SDK's own CUDA backend (attention_cuda.cu) built "
                                          "from its sources, on the same GPU; the SDK has no CPU "
                                          "decoder"}
        dec.close()
    else:
        line["gpu_launches"] = c["tokens"] * (9 * c["layers"] + 3) * steps
        cache.free()
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# Config 7: dense FP16 SDPA (tensor_sdpa_f16's backend) on the prefill kernel
# ---------------------------------------------------------------------------

CFG7 = dict(batch=1, q_heads=32, kv_heads=8, q_len=4096, kv_len=4096, head_dim=128, causal=True)


def cfg7_flops(c=CFG7) -> float:
    off = c["kv_len"] - c["q_len"]
    keys = sum(min(c["kv_len"], off + i + 1) for i in range(c["q_len"]))
    return 4.0 * c["head_dim"] * c["batch"] * c["q_heads"] * keys


def run_dense(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch
    c = dict(CFG7)
    if args.head_dim:
        c["head_dim"] = args.head_dim
    d = c["head_dim"]
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(args.seed)
    B, Hq, Hkv, Lq, Lk = c["batch"], c["q_heads"], c["kv_heads"], c["q_len"], c["kv_len"]
    q = torch.randn(B, Hq, Lq, d, generator=g, device=dev).half()
    k = torch.randn(B, Hkv, Lk, d, generator=g, device=dev).half()
    v = torch.randn(B, Hkv, Lk, d, generator=g, device=dev).half()
    out = torch.empty_like(q)
    scale = 1 / math.sqrt(d)
    flops = cfg7_flops(c)
    peak, kind = measured_peak_tflops()
    steps, warmup = args.steps, args.warmup
    block = {"workload": f"cfg7: dense causal FP16 SDPA, B=1, GQA 32/8, 4096 x 4096, d={d} "
                         "(tensor_sdpa_f16's backend)"
                         + ("" if d == 128 else " -- variant at head_dim 64"), **c}
    sampler = ClockSampler(str(torch.cuda.get_device_properties(dev).uuid))
    h_q, h_k, h_v = (t.cpu().numpy().view(np.uint16) for t in (q, k, v))
    if args.impl == "reference":
        from oracle import oracle as O
        if not O.ref_cuda_available():
            print(json.dumps({"impl": "reference", "unavailable":
                              "oracle/_ref/libref_cuda.so (the SDK's CUDA backend) not built"}))
            return
        run = O.ref_cuda_sdpa_f16
        call = lambda: run(h_q, h_k, h_v, scale, True)
    else:
        import inference_c_b200 as P
        P.load()
        call = lambda: P.sdpa_f16_host(h_q, h_k, h_v, scale, True)
    # e2e: the backend hook with host tensors (upload, attention, download)
    with sampler:
        for _ in range(warmup):
            assert call() is not None
        t0 = time.perf_counter()
        for _ in range(steps):
            call()
        e2e_ms = (time.perf_counter() - t0) / steps * 1e3
        dev_ms = None
        if args.impl != "reference":
            s = torch.cuda.current_stream()
            for _ in range(warmup):
                P.sdpa_f16(q, k, v, out, scale, True)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(steps):
                P.sdpa_f16(q, k, v, out, scale, True)
            e1.record(s)
            torch.cuda.synchronize()
            dev_ms = e0.elapsed_time(e1) / steps
    ms = dev_ms if dev_ms is not None else e2e_ms
    value = flops / (ms / 1e3) / 1e12
    bytes_h = (q.numel() + k.numel() + v.numel()) * 2
    line = {
        "metric": "dense causal SDPA TFLOP/s (config 7: tensor_sdpa_f16's backend)",
        "value": value, "unit": "TFLOP/s", "n_gpus": 1, "steps": steps, "warmup": warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f16", "data": "synthetic: seeded N(0,1) FP16", "config": block,
        "roofline": {"bound": "tensor", "achieved": value, "peak": peak, "unit": "TFLOP/s",
                     "frac": value / peak, "traffic": None, "peak_kind": kind,
                     "algorithmic_flops_per_call": flops,
                     "note": "device entry with resident tensors (query and output read "
                             "and written in place by the prefill kernel)"},
        "e2e": {"value": flops / (e2e_ms / 1e3) / 1e12, "unit": "TFLOP/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": bytes_h, "d2h_bytes_per_step": q.numel() * 2,
                "api": "run_f16 backend hook with host tensors (pkv_sdpa_f16_host)"},
        "gpu_launches": 4 * steps,
        "clocks": sampler.summary(),
    }
    if args.impl == "reference":
        line["impl"] = "reference"
        line["gpu_launches"] = None
        line["cpu_baseline"] = {"value": None, "unit": "TFLOP/s", "cores": 0, "kind": "reference",
                                "sample": "the SDK's own CUDA backend dense sdpa (run_f16, "
                                          "attention_cuda.cu:71-99) on the same GPU"}
        line["roofline"] = None
    print(json.dumps(line), flush=True)


def run_prefill_reference(args) -> None:
    """--impl reference for config 5: the SDK's tensor_sdpa_f32 on a bounded
    slice of the workload each step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    steps, warmup = args.steps, args.warmup
    budget = max(0.05, 150.0 / max(1, steps + warmup))
    rates, info = [], None
    for i in range(warmup + steps):
        r, info = sdk_prefill_rate(budget, args.seed)
        if i >= warmup:
            rates.append(r)
    value = statistics.mean(rates)
    print(json.dumps({
        "metric": "chunked prefill attention TFLOP/s over the paged cache (config 5: append "
                  "2048-token chunks + causal prefill per step)",
        "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": steps,
        "warmup": warmup, "ms_per_step": None, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) BF16)",
        "impl": "reference", "config": cfg5_block(),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", **info},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0}}), flush=True)


def main():
    args = parse_args()
    if args.config == 7:
        run_dense(args)
    elif args.config == 6:
        run_decoder(args)
    elif args.config == 5:
        run_prefill_reference(args) if args.impl == "reference" else run_prefill(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.config == 4:
        run_cfg4(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
