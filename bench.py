#!/usr/bin/env python3
"""Benchmark of the GQA decode hot path (Llama-3-8B shape).

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``

One step = one decode over the HBM-resident cache of one batch: B=64
sequences x 32 query heads over 8 KV heads, head_dim 128, 4096 cached tokens,
bf16 ~ N(0,1)*0.5 (seed 1).  Under torchrun each rank runs its own batch of
64 sequences (weak scaling: global batch = 64 x N; batch sharding has no
data-path collective).  The metric is the KV-stream bandwidth, GB/s =
sum(len) x Hkv x D x 2 (K and V) x 2 bytes / step time, summed over ranks,
with queries/s = sequences / step time beside it.

* ``value``: device time of K timed steps (CUDA events on the launching
  stream, barrier + synchronize on both sides, max over ranks); inputs are
  resident (1 GiB per step, larger than L2, so no flush is needed).
* ``e2e``: the same metric through the public API with host buffers:
  ``AttentionAccelerator.run_query`` with pinned host q/o (H2D of q, decode,
  D2H of o, synchronous), wall-clock over K steps.
* ``roofline``: the decode kernel's algorithmic bytes per launch / its mean
  launch time, against the measured HBM copy bandwidth.
* ``cpu_baseline``: the CPU oracle (restatement of the reference's
  ``cpu_attention_numpy``) on the same workload, on this host's cores.
* ``--impl reference``: times that CPU path (the reference's own implementation
  of the path is SystemVerilog RTL plus this NumPy CPU model, so the CPU model
  is what runs here) on rank 0 and prints its own line.
"""

from __future__ import annotations

import os

# The CPU baseline parallelises over (sequence, kv-head) pairs with one
# thread per core, so the BLAS inside each NumPy call runs single-threaded;
# like the reference harness (sw/board_performance.py:13-17) this is set
# before NumPy is imported.
for _name in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS", "NUMEXPR_NUM_THREADS"):
    os.environ.setdefault(_name, "1")

import argparse
import json
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "GQA decode KV-stream GB/s (% of HBM peak) & queries/s at 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
# ncu summaries per workload (dram traffic per launch of the full workload)
PROFILE_SUMMARIES = {"llama3_8b_decode": ROOT / "profiles" / "decode_llama3_8b_cfg2.txt",
                     "ragged_decode_stress": ROOT / "profiles" / "decode_tc_ragged_cfg3.txt"}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[2, 3, 4, 5, 6], default=2,
                    help="BASELINE config (2 = the headline Llama-3-8B decode; 5 = chunked prefill); "
                         "6 = the layer prologue (RMSNorm + QKV projection + RoPE) of config 5's new tokens")
    ap.add_argument("--batch", type=int, default=None,
                    help="config 2/4: sequences per rank (default 64 / 8); config 3: the first N of its 256 "
                         "ragged sequences (a smaller case for profiling)")
    ap.add_argument("--seq-len", type=int, default=None)
    ap.add_argument("--splits", type=int, default=0, help="force the split count (0 = planner)")
    ap.add_argument("--chunk", type=int, default=0)
    ap.add_argument("--paged", type=int, default=0, metavar="PAGE_SIZE",
                    help="configs 2/3: decode from a paged cache (page pool in shuffled page order, block "
                         "table) instead of the contiguous cache; 0 = contiguous")
    ap.add_argument("--paged-order", choices=["random", "sequential"], default="random",
                    help="page assignment of the paged cache (random permutation or consecutive pages)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU-baseline sample time")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def measured_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except (ValueError, KeyError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def profiled_traffic(workload: str):
    """dram bytes per launch from the workload's committed ncu summary, if present."""
    path = PROFILE_SUMMARIES.get(workload)
    if path is None or not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            try:
                return int(float(line.split(":", 1)[1].strip()))
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling every 200 ms during the timed region."""

    FIELDS = ("timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_uuid: str | None):
        self.path = Path(tempfile.mkstemp(prefix="lara_clocks_", suffix=".csv")[1])
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if gpu_uuid:
            cmd += ["-i", gpu_uuid]
        self.proc = None
        try:
            self.fh = self.path.open("w")
            self.proc = subprocess.Popen(cmd, stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        t0 = time.time()
        while self.proc is not None and time.time() - t0 < 5.0 and self.path.stat().st_size == 0:
            time.sleep(0.05)
        self.t_start = self.t_end = None

    def start(self):
        self.t_start = time.time()

    def stop(self):
        self.t_end = time.time()
        time.sleep(0.25)
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        rows = []
        if self.proc is not None and self.path.exists():
            for line in self.path.read_text().splitlines():
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 10:
                    continue
                try:
                    ts = time.mktime(time.strptime(parts[0].split(".")[0], "%Y/%m/%d %H:%M:%S"))
                    rows.append((ts, float(parts[2]), float(parts[3]), parts[6:10], parts[5]))
                except ValueError:
                    continue
        try:
            self.path.unlink()
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        lo, hi = (self.t_start or 0) - 1.0, (self.t_end or 1e18) + 1.0
        inside = [r for r in rows if lo <= r[0] <= hi] or rows
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in inside for i, v in enumerate(r[3]) if v.lower().startswith("active")})
        return {"sm_mhz": statistics.median(r[1] for r in inside), "sm_max_mhz": max(r[2] for r in inside),
                "reasons": reasons, "samples": len(inside)}


class CpuOracle:
    """The CPU oracle's decode over (sequence, kv-head) pairs on a thread pool."""

    def __init__(self, q, k, v, lens, threads: int):
        import concurrent.futures as cf

        import oracle

        self.q, self.k, self.v, self.lens = q, k, v, lens
        self.threads = max(1, threads)
        self.pool = cf.ThreadPoolExecutor(max_workers=self.threads)
        self._decode = oracle.decode_attention

    def step(self, pairs) -> None:
        chunks = [pairs[i::self.threads] for i in range(min(self.threads, len(pairs)))]
        list(self.pool.map(lambda ps: self._decode(self.q, self.k, self.v, self.lens, pairs=ps), chunks))

    def close(self) -> None:
        self.pool.shutdown()


def cpu_pass_times(q, k, v, lens, pairs, threads: int, repeats: int = 5, seconds: float = 0.0):
    """One warm-up pass, then timed passes of the CPU oracle over ``pairs``.

    Passes are timed one by one with ``perf_counter_ns`` (the reference's
    harness: 1 warm-up + 5 repeats, sw/board_performance.py:195-204); at least
    ``repeats`` are taken, and more until ``seconds`` have passed.  Returns
    (KV bytes per pass, list of pass seconds)."""
    nbytes = sum(int(lens[b]) for b, _ in pairs) * k.shape[3] * 4
    runner = CpuOracle(q, k, v, lens, threads)
    times = []
    try:
        runner.step(pairs)
        t_start = time.perf_counter()
        while len(times) < repeats or time.perf_counter() - t_start < seconds:
            t0 = time.perf_counter_ns()
            runner.step(pairs)
            times.append((time.perf_counter_ns() - t0) * 1e-9)
    finally:
        runner.close()
    return nbytes, times


def pass_stats(times) -> dict:
    """min / median / p95 / max of pass times in seconds (sw/board_performance.py:321-331)."""
    a = np.asarray(times, np.float64)
    return {"repeats": int(a.size), "min_s": round(float(a.min()), 5), "median_s": round(float(np.median(a)), 5),
            "p95_s": round(float(np.percentile(a, 95)), 5), "max_s": round(float(a.max()), 5)}


def cpu_baseline_runs(q, k, v, lens, pairs, cores: int, seconds: float, one_thread_pass_s: float = 1.5):
    """The oracle on all ``cores`` threads over ``pairs``, then on one thread over
    a prefix of ``pairs`` sized for about ``one_thread_pass_s`` per pass.

    Returns (all-core GB/s, its stats, one-thread GB/s, its stats, pairs in the one-thread sample)."""
    nb, t_all = cpu_pass_times(q, k, v, lens, pairs, cores, 5, seconds)
    st_all = pass_stats(t_all)
    n1 = max(1, min(len(pairs), int(len(pairs) * one_thread_pass_s / max(st_all["median_s"] * cores, 1e-9))))
    nb1, t_one = cpu_pass_times(q, k, v, lens, pairs[:n1], 1, 5)
    st_one = pass_stats(t_one)
    return nb / st_all["median_s"] / 1e9, st_all, nb1 / st_one["median_s"] / 1e9, st_one, n1


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------

def run_reference(args, rank: int, world: int) -> int:
    """CPU reference path (oracle port of cpu_attention_numpy), rank 0 only.

    Each of the K timed steps decodes a bounded sample of the workload's
    (sequence, kv-head) pairs, sized by a calibration so the K steps take
    about a minute; the value is the sample's KV bytes over its time."""
    if rank != 0:
        return 0
    import concurrent.futures as cf

    import oracle
    from lara_b200.workloads import CONFIGS

    cfg = CONFIGS[2]
    B = args.batch or cfg.batch
    L = args.seq_len or cfg.seq_len
    Hkv, D = cfg.n_kv_heads, cfg.head_dim
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    pack = oracle.fp32_to_bf16_u16
    rng = np.random.default_rng(cfg.seed)
    nb = min(B, max(1, -(-cores // Hkv)) * 2)  # sequences held on the host for the samples
    q = pack(rng.standard_normal((nb, cfg.n_q_heads, D), dtype=np.float32) * np.float32(cfg.std))
    k = pack(rng.standard_normal((nb, Hkv, L, D), dtype=np.float32) * np.float32(cfg.std))
    v = pack(rng.standard_normal((nb, Hkv, L, D), dtype=np.float32) * np.float32(cfg.std))
    lens = np.full(nb, L, np.int32)
    all_pairs = [(b, h) for b in range(nb) for h in range(Hkv)]
    runner = CpuOracle(q, k, v, lens, cores)
    calib = all_pairs[:min(len(all_pairs), cores)]
    runner.step(calib)
    t0 = time.perf_counter()
    runner.step(calib)
    t_batch = time.perf_counter() - t0  # wall time of `cores` pairs in parallel
    budget = min(2.0, 60.0 / max(args.steps, 1))
    n_pairs = int(max(1, min(len(all_pairs), budget / max(t_batch, 1e-6) * len(calib))))
    sample = all_pairs[:n_pairs]
    for _ in range(min(args.warmup, 3)):
        runner.step(sample)
    step_s = []
    for _ in range(args.steps):
        t0 = time.perf_counter_ns()
        runner.step(sample)
        step_s.append((time.perf_counter_ns() - t0) * 1e-9)
    t = sum(step_s) / max(args.steps, 1)
    runner.close()
    nbytes = n_pairs * L * D * 2 * 2
    # the same harness on one thread (1 warm-up + 5 repeats over a smaller prefix)
    n1 = max(1, min(n_pairs, int(n_pairs * 1.5 / max(t * cores, 1e-9))))
    nb1, t_one = cpu_pass_times(q, k, v, lens, sample[:n1], 1, 5)
    st_one = pass_stats(t_one)
    value = nbytes / t / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg.name, "global_batch": B * world, "seq_len": L, "n_q_heads": cfg.n_q_heads,
                   "n_kv_heads": Hkv, "head_dim": D},
        "queries_per_s": round(n_pairs / Hkv / t, 2),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"{n_pairs} (sequence, kv-head) pairs x {L} tokens per step (of {B * Hkv}); the "
                                   f"reference's implementation of this path is CPU NumPy "
                                   f"(sw/board_performance.py:158-192), run as the oracle port on {cores} threads",
                         "pass_seconds": pass_stats(step_s),
                         "single_thread": {"value": round(nb1 / st_one["median_s"] / 1e9, 3), "unit": "GB/s",
                                           "cores": 1, "sample": f"first {n1} pairs of the same sample",
                                           "pass_seconds": st_one}},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _setup_decode(args, cfg, rank, world, dev):
    """Inputs, step function and per-rank bytes for configs 2/3/4.

    Config 2: each rank runs its own batch (weak scaling).  Config 3: the 256
    ragged sequences are partitioned across ranks by token count (strong).
    Config 4: every sequence's tokens are split across ranks (split-KV,
    strong); the step is partial decode + NCCL all-gather + LSE combine."""
    import torch

    from lara_b200 import ops, parallel
    from lara_b200.workloads import make_decode_inputs

    info = {}
    if cfg.name == "llama3_8b_decode":
        B = args.batch or cfg.batch
        L = args.seq_len or cfg.seq_len
        q, k, v, lens = make_decode_inputs(cfg, dev, batch=B, seq_len=L, seed=cfg.seed + 1000 * rank)
        scaling, global_batch = "weak", B * world
    elif cfg.name == "ragged_decode_stress":
        all_lens = cfg.lens(args.batch)  # --batch N: the first N sequences (small profiling case)
        mine = parallel.balanced_partition(all_lens, world)[rank] if world > 1 else list(range(len(all_lens)))
        L = int(all_lens[mine].max())
        q, k, v, lens = make_decode_inputs(cfg, dev, lens=all_lens[mine], capacity=L, seed=cfg.seed + 1000 * rank)
        B = len(mine)
        scaling, global_batch = "strong", len(all_lens)
        info["sequences_on_rank0"] = len(mine)
    else:  # long-context split-KV
        B = args.batch or cfg.batch
        L_total = args.seq_len or cfg.seq_len
        start, L = parallel.token_range(L_total, world, rank)
        # every rank draws its own token slice (seeded by rank); q is shared
        q, k, v, lens = make_decode_inputs(cfg, dev, batch=B, seq_len=L, seed=cfg.seed + 1000 * rank)
        g = torch.Generator(device=dev)
        g.manual_seed(cfg.seed)
        q = (torch.randn(q.shape, generator=g, device=dev) * cfg.std).to(torch.bfloat16)
        scaling, global_batch = "strong", B
        info["tokens_per_rank"] = L
    lens_np = lens.cpu().numpy()
    nbytes = cfg.kv_bytes(lens_np)
    o = torch.empty_like(q)
    if cfg.name == "long_context_splitkv" and world > 1:
        dec = parallel.SplitKVDecoder(B, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, L, dev, lens_local=lens_np)
        plan = dec.decoder.plan

        def step():
            dec(q, k, v, lens, out=o)
        launches = 3  # partial decode, NCCL all-gather, combine
    elif args.paged:
        import math

        from lara_b200 import _native

        dec = ops.Decoder(B, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, L, dev, lens=lens_np,
                          num_splits=args.splits, chunk_tokens=args.chunk)
        plan = dec.plan
        ps = int(args.paged)
        pps = math.ceil(L / ps)
        npg = [math.ceil(int(n) / ps) for n in lens_np]
        total = sum(npg)
        perm = (torch.randperm(total, generator=torch.Generator().manual_seed(7)) if args.paged_order == "random"
                else torch.arange(total)).to(dev)
        table = torch.full((B, pps), -1, dtype=torch.int32, device=dev)
        kp = torch.empty((total, cfg.n_kv_heads, ps, cfg.head_dim), dtype=k.dtype, device=dev)
        vp = torch.empty_like(kp)
        base = 0
        for b in range(B):
            n = npg[b]
            if n == 0:
                continue
            pages = perm[base:base + n]
            table[b, :n] = pages.to(torch.int32)
            for src, dst in ((k, kp), (v, vp)):
                rows = src[b, :, : n * ps] if n * ps <= L else torch.nn.functional.pad(src[b], (0, 0, 0, n * ps - L))
                dst.index_copy_(0, pages, rows.reshape(cfg.n_kv_heads, n, ps, cfg.head_dim).permute(1, 0, 2, 3))
            base += n
        del k, v
        torch.cuda.empty_cache()
        k, v = kp, vp
        stream = torch.cuda.current_stream(dev)
        scale = 1.0 / math.sqrt(cfg.head_dim)

        def step():
            _native.check(_native.lib.lara_gqa_decode_paged(
                q.data_ptr(), kp.data_ptr(), vp.data_ptr(), table.data_ptr(), lens.data_ptr(), o.data_ptr(), B,
                cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, ps, pps, total, scale, plan.num_splits,
                plan.chunk_tokens, dec.workspace.data_ptr(), dec.workspace.numel(), stream.cuda_stream),
                "decode_paged")
        launches = 1
        info["paged"] = {"page_size": ps, "pages": total, "page_order": ("random permutation (seed 7)" if args.paged_order == "random" else "sequential"),
                         "layout": "[pages][Hkv][page_size][D]"}
    else:
        dec = ops.Decoder(B, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, L, dev, lens=lens_np,
                          num_splits=args.splits, chunk_tokens=args.chunk)
        plan = dec.plan

        def step():
            dec(q, k, v, lens, out=o)
        launches = 1
    info.update({"splits": plan.num_splits, "chunk_tokens": plan.chunk_tokens})
    ws = dec.decoder.workspace if hasattr(dec, "decoder") else dec.workspace
    return dict(q=q, k=k, v=v, lens=lens, lens_np=lens_np, o=o, B=B, L=L, nbytes=nbytes, step=step, ws=ws,
                scaling=scaling, global_batch=global_batch, info=info, launches=launches)


def run_ours(args, rank: int, world: int, local_rank: int) -> int:
    import torch
    import torch.distributed as dist

    from lara_b200 import ops
    from lara_b200.workloads import CONFIGS

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = CONFIGS[args.config]
    S = _setup_decode(args, cfg, rank, world, dev)
    q, k, v, lens, lens_np, o, B, L, nbytes = (S[x] for x in ("q", "k", "v", "lens", "lens_np", "o", "B", "L",
                                                              "nbytes"))
    step = S["step"]
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if ops.workspace_status(S["ws"]) != 0:
        raise RuntimeError("decode kernel reported a device error status during warm-up")

    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        uuid = None
    sampler = ClockSampler(uuid)
    barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.start()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    sampler.stop()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    clocks = sampler.summary()
    if ops.workspace_status(S["ws"]) != 0:
        raise RuntimeError("decode kernel reported a device error status")

    # e2e through the public API with pinned host buffers
    e2e_ms = None
    h2d = d2h = 0
    e2e_api = None
    if not args.no_e2e:
        q_host = q.view(torch.int16).cpu().pin_memory()
        o_host = torch.empty_like(q_host).pin_memory()
        qn = q_host.numpy().view(np.uint16)
        on = o_host.numpy().view(np.uint16)
        e2e_steps = max(10, args.steps // 4)
        if (world == 1 or cfg.name != "long_context_splitkv") and not args.paged:
            import ctypes

            from lara_b200 import _native
            from lara_b200.attn_driver import AttentionAccelerator

            with AttentionAccelerator(device=local_rank) as acc:
                acc.configure_heads(cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, max_seq_len=L, batch=B)
                # device-resident cache load through the C ABI (on_device = 1)
                _native.check(_native.lib.lara_kv_load(acc._ctx, k.data_ptr(), v.data_ptr(),
                                                       lens_np.ctypes.data_as(ctypes.c_void_p), L, 1), "kv_load")
                for _ in range(max(3, min(args.warmup, 20))):
                    acc.run_query(qn, out=on)
                barrier()
                t0 = time.perf_counter()
                for _ in range(e2e_steps):
                    acc.run_query(qn, out=on)
                e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
                barrier()
            e2e_api = "AttentionAccelerator.run_query (pinned host q/o)"
        else:
            qd, od = q.view(torch.int16), o.view(torch.int16)

            def e2e_step():
                qd.copy_(q_host, non_blocking=True)
                step()
                o_host.copy_(od, non_blocking=True)
                torch.cuda.synchronize(dev)
            for _ in range(3):
                e2e_step()
            barrier()
            t0 = time.perf_counter()
            for _ in range(e2e_steps):
                e2e_step()
            e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
            barrier()
            e2e_api = ("lara_gqa_decode_paged with pinned host q/o copies" if args.paged else
                       "lara_b200.parallel.SplitKVDecoder with pinned host q/o copies")
        h2d, d2h = qn.nbytes, on.nbytes
        if not np.array_equal(on, o.view(torch.int16).cpu().numpy().view(np.uint16)):
            raise RuntimeError("API output differs from the timed kernel output")

    # max over ranks; bytes summed over ranks
    total_bytes = nbytes
    if world > 1:
        t = torch.tensor([ms, e2e_ms or 0.0], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = float(t[0]), (float(t[1]) if e2e_ms is not None else None)
        nb = torch.tensor([nbytes], dtype=torch.float64, device=dev)
        dist.all_reduce(nb, op=dist.ReduceOp.SUM)
        total_bytes = int(nb.item())

    if rank != 0:
        return 0
    peak, peak_kind = measured_peak()
    value = total_bytes / (ms * 1e-3) / 1e9
    achieved = nbytes / (ms * 1e-3) / 1e9  # this GPU's bytes over the step
    full_size = args.batch is None and args.seq_len is None
    traffic = profiled_traffic(cfg.name) if full_size and not args.paged else None
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
        # bounded sample: as many whole sequences as fit ~4 GB of bf16 on the host
        per_seq = [int(x) * cfg.n_kv_heads * cfg.head_dim * 4 for x in lens_np]
        nseq, acc_b = 0, 0
        while nseq < B and (nseq == 0 or acc_b + per_seq[nseq] <= 4 << 30):
            acc_b += per_seq[nseq]
            nseq += 1
        Ls = int(lens_np[:nseq].max())
        qn_, kn_, vn_ = (t[:nseq, :, :Ls].contiguous() if t.dim() == 4 else t[:nseq].contiguous()
                         for t in (q, k, v))
        qn_, kn_, vn_ = (t.view(torch.int16).cpu().numpy().view(np.uint16) for t in (qn_, kn_, vn_))
        pairs = [(b, h) for b in range(nseq) for h in range(cfg.n_kv_heads)]
        gbs, st_all, gbs1, st_one, n1 = cpu_baseline_runs(qn_, kn_, vn_, lens_np[:nseq], pairs, cores,
                                                          args.cpu_seconds)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"passes over {nseq} of {B} sequences ({int(lens_np[:nseq].sum())} tokens, "
                         f"{len(pairs)} (sequence, kv-head) pairs) on {cores} threads, value from the median "
                         f"pass; oracle restatement of sw/board_performance.py:158-192",
               "pass_seconds": st_all,
               "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
                                 "sample": f"first {n1} (sequence, kv-head) pairs of the same sample",
                                 "pass_seconds": st_one}}
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": S["scaling"],
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg.name, "global_batch": S["global_batch"], "batch_per_gpu": B, "seq_len": L,
                   "n_q_heads": cfg.n_q_heads, "n_kv_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim,
                   "parallelism": {"llama3_8b_decode": f"batch-sharded x{world}",
                                   "ragged_decode_stress": f"token-balanced batch partition x{world}",
                                   "long_context_splitkv": f"split-KV x{world} (NCCL all-gather + LSE combine)"
                                   }[cfg.name],
                   "l2": "inputs larger than L2, no flush", **S["info"]},
        "queries_per_s": round(S["global_batch"] / (ms * 1e-3), 1),
        "pct_hbm_peak": round(100.0 * achieved / peak, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6650 GB/s", "algorithmic_bytes_per_launch": nbytes},
        "cpu_baseline": cpu,
        "e2e": None if e2e_ms is None else {
            "value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 5),
            "api": e2e_api},
        "gpu_launches": args.steps * S["launches"],
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_prefill(args, rank: int, world: int, local_rank: int) -> int:
    """Config 5: chunked prefill on the tensor cores (TFLOP/s).

    One step = append the 2048 new K/V tokens of every sequence at position
    8192 (lengths reset first) + causal attention of the 2048 new queries over
    cache + self.  Sequences are split across ranks (weak scaling: each rank
    runs config 5's 4 sequences)."""
    import ctypes

    import torch
    import torch.distributed as dist

    from lara_b200 import _native, ops
    from lara_b200.workloads import PREFILL, make_prefill_inputs

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = PREFILL
    q, k, v, kn, vn, lens0 = make_prefill_inputs(cfg, dev)
    B, n, C = cfg.batch, cfg.new, cfg.cached
    Lmax = C + n
    lens = lens0.clone()
    nb = int(_native.lib.lara_prefill_workspace_bytes(B, n, cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, Lmax))
    ws = ops.new_workspace(nb, dev)
    o = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)
    scale = 1.0 / (cfg.head_dim ** 0.5)

    def step():
        lens.copy_(lens0)
        ops.kv_append(k, v, lens, kn, vn, workspace=ws)
        _native.check(_native.lib.lara_gqa_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens0.data_ptr(),
                                                   o.data_ptr(), B, n, cfg.n_q_heads, cfg.n_kv_heads,
                                                   cfg.head_dim, Lmax, 1, scale, ws.data_ptr(), ws.numel(),
                                                   stream.cuda_stream), "prefill")

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if ops.workspace_status(ws) != 0:
        raise RuntimeError("prefill reported a device error status")
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.start()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    sampler.stop()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    # kernel-only time of the attention launch (for the roofline)
    ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    lens.copy_(lens0)
    ka.record(stream)
    for _ in range(max(3, args.steps // 4)):
        _native.check(_native.lib.lara_gqa_prefill(q.data_ptr(), k.data_ptr(), v.data_ptr(), lens0.data_ptr(),
                                                   o.data_ptr(), B, n, cfg.n_q_heads, cfg.n_kv_heads,
                                                   cfg.head_dim, Lmax, 1, scale, ws.data_ptr(), ws.numel(),
                                                   stream.cuda_stream), "prefill")
    kb.record(stream)
    torch.cuda.synchronize(dev)
    k_ms = ka.elapsed_time(kb) / max(3, args.steps // 4)
    clocks = sampler.summary()
    o_kernel = o.clone()

    # e2e: the driver API with page-locked host buffers -- every step the
    # chunk's q and new K/V go host->device and the output comes back
    # (AttentionAccelerator.run_prefill_chunk, pipelined by sequence), after
    # truncate_kv rewinds the previous step's append
    e2e_ms, h2d, d2h = None, 0, 0
    if not args.no_e2e:
        import numpy as np

        from lara_b200.attn_driver import AttentionAccelerator

        def pinned_words(t):
            h = t.cpu().view(torch.int16).pin_memory()
            return h, h.numpy().view(np.uint16)

        (qh, q_np), (knh, kn_np), (vnh, vn_np) = (pinned_words(t) for t in (q, kn, vn))
        oh, o_np = pinned_words(torch.empty_like(q))
        lens0_np = lens0.cpu().numpy().astype(np.int32)
        acc = AttentionAccelerator(device=local_rank)
        acc.configure_heads(cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, max_seq_len=Lmax, batch=B)
        acc.load_kv(k[:, :, :C].contiguous().cpu().view(torch.int16).numpy().view(np.uint16),
                    v[:, :, :C].contiguous().cpu().view(torch.int16).numpy().view(np.uint16), lens0_np)

        def e2e_step():
            acc.truncate_kv(lens0_np)
            acc.run_prefill_chunk(q_np, kn_np, vn_np, causal=True, out=o_np)

        for _ in range(2):
            e2e_step()
        n_e2e = max(3, min(args.steps, 20))
        barrier()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            e2e_step()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / n_e2e
        acc.close()
        if not torch.equal(oh, o_kernel.cpu().view(torch.int16)):
            raise RuntimeError("API output differs from the timed kernel output")
        h2d = qh.numel() * 2 + knh.numel() * 2 + vnh.numel() * 2
        d2h = oh.numel() * 2
    if world > 1:
        t = torch.tensor([ms, k_ms, e2e_ms or 0.0], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, k_ms = float(t[0]), float(t[1])
        e2e_ms = float(t[2]) if e2e_ms is not None else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = prefill_cpu_baseline(cfg, q, k, v, args.cpu_seconds)
    if rank != 0:
        return 0
    flops = cfg.flops()
    peak = 1415.2
    peak_src = "fallback 1400 TFLOP/s sustained"
    pp = ROOT / "MEASURED_PEAKS.json"
    if pp.exists():
        try:
            peak = float(json.loads(pp.read_text())["bf16_tflops_sustained"])
            peak_src = "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
        except (ValueError, KeyError):
            pass
    achieved = flops / (k_ms * 1e-3) / 1e12
    line = {
        "metric": "chunked-prefill attention TFLOP/s (tensor-core path)", "value": round(flops * world / (ms * 1e-3) / 1e12, 2),
        "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": cfg.name, "batch_per_gpu": B, "new_tokens": n, "cached_tokens": C,
                   "n_q_heads": cfg.n_q_heads, "n_kv_heads": cfg.n_kv_heads, "head_dim": cfg.head_dim,
                   "causal": True, "step": "length reset + K/V append + attention",
                   "p_precision": "bf16 RNE (LARA_TC_SPLIT_P=0)" if os.environ.get("LARA_TC_SPLIT_P") == "0"
                   else "P_hi + P_lo"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_src,
                     "algorithmic_flop_per_launch": flops, "attention_kernel_ms": round(k_ms, 4)},
        "cpu_baseline": cpu,
        "e2e": None if e2e_ms is None else {
            "value": round(flops * world / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
            "api": "AttentionAccelerator.run_prefill_chunk (page-locked host q, k_new, v_new, o; truncate_kv "
                   "rewinds the chunk each step)"},
        "gpu_launches": args.steps * 3, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    return 0


def prefill_cpu_baseline(cfg, q, k, v, seconds: float) -> dict:
    """The CPU oracle's chunked prefill (oracle.prefill_attention, the causal rule of
    sw/board_performance.py:174-177 over cache + self) for the kv-head groups of
    sequence 0, timed per pass on all host cores and on one thread."""
    import concurrent.futures as cf

    import torch

    import oracle

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    B, n, Hq, D = q.shape
    Hkv, C = cfg.n_kv_heads, cfg.cached
    G = Hq // Hkv
    words = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    qw = words(q[0]).transpose(1, 0, 2)[None]          # [1, Hq, n, D]
    kw, vw = words(k[0])[None], words(v[0])[None]      # [1, Hkv, Lmax, D], chunk already appended
    kv_len = np.array([C + n])
    flop_group = G * (n * C + n * (n + 1) // 2) * 4 * D

    def unit(g):
        oracle.prefill_attention(qw[:, g * G:(g + 1) * G], kw[:, g:g + 1], vw[:, g:g + 1], kv_len, C, causal=True)

    def passes(threads, groups, repeats, min_s):
        times = []
        with cf.ThreadPoolExecutor(max_workers=threads) as pool:
            list(pool.map(unit, groups))  # warm-up
            t_start = time.perf_counter()
            while len(times) < repeats or time.perf_counter() - t_start < min_s:
                t0 = time.perf_counter_ns()
                list(pool.map(unit, groups))
                times.append((time.perf_counter_ns() - t0) * 1e-9)
        return times

    groups = list(range(Hkv))
    t_all = passes(min(cores, Hkv), groups, 3, seconds)
    st_all = pass_stats(t_all)
    t_one = passes(1, groups[:1], 3, 0.0)
    st_one = pass_stats(t_one)
    return {"value": round(flop_group * len(groups) / st_all["median_s"] / 1e12, 5), "unit": "TFLOP/s",
            "cores": min(cores, Hkv), "kind": "port",
            "sample": f"the {Hkv} kv-head groups of sequence 0 ({G} query heads each, {n} queries over {C} cached "
                      f"+ self), one group per thread; value from the median pass",
            "pass_seconds": st_all,
            "single_thread": {"value": round(flop_group / st_one["median_s"] / 1e12, 5), "unit": "TFLOP/s",
                              "cores": 1, "sample": "kv-head group 0 of sequence 0", "pass_seconds": st_one}}


def run_prologue(args, rank: int, world: int, local_rank: int) -> int:
    """Config 6: the run_layer prologue of config 5's chunk on the tensor cores.

    One step = RMSNorm + fused QKV projection / RoPE / head scatter for the
    2048 new tokens of each of config 5's 4 sequences (Llama-3-8B: hidden
    4096 -> 32 q + 8 k + 8 v heads of 128; positions 8192 + t) in one batched
    call (3 launches: RoPE table, RMSNorm, persistent projection).  Weights
    bf16 [4096][6144], N(0,1)/64."""
    import torch
    import torch.distributed as dist

    from lara_b200 import _native, ops

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    B, L, hidden, hq, hkv, D, base_pos = 4, 2048, 4096, 32, 8, 128, 8192
    n_total = (hq + 2 * hkv) * D
    g = torch.Generator(device=dev)
    g.manual_seed(6)
    x = torch.randn((B, L, hidden), generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn((hidden, n_total), generator=g, device=dev) / 64.0).to(torch.bfloat16)
    rms = (1.0 + 0.1 * torch.randn((hidden,), generator=g, device=dev)).to(torch.bfloat16)
    q = torch.empty((B, hq, L, D), dtype=torch.bfloat16, device=dev)
    k = torch.empty((B, hkv, L, D), dtype=torch.bfloat16, device=dev)
    v = torch.empty_like(k)
    nb = int(_native.lib.lara_layer_prologue_workspace_bytes(B, L, hidden))
    wss = [ops.new_workspace(nb, dev)]
    stream = torch.cuda.current_stream(dev)

    def step():
        _native.check(_native.lib.lara_layer_prologue(
            x.data_ptr(), rms.data_ptr(), w.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
            B, L, hidden, hq, hkv, D, base_pos, base_pos, 1e-5, 10000.0, wss[0].data_ptr(), wss[0].numel(),
            stream.cuda_stream), "layer_prologue")

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if any(ops.workspace_status(ws) != 0 for ws in wss):
        raise RuntimeError("prologue reported a device error status")
    uuid = None
    try:
        uuid = "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        pass
    sampler = ClockSampler(uuid)
    barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler.start()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    sampler.stop()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    clocks = sampler.summary()
    outs_kernel = [t.clone() for t in (q, k, v)]

    # e2e: ops.layer_prologue with the hidden states from pinned host memory and
    # q/k/v read back every step (weights resident)
    e2e_ms, h2d, d2h = None, 0, 0
    if not args.no_e2e:
        xh = x.cpu().pin_memory()
        hosts = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in (q, k, v)]
        xd = torch.empty_like(x)

        def e2e_step():
            xd.copy_(xh, non_blocking=True)
            ops.layer_prologue(xd, w, rms, n_q_heads=hq, n_kv_heads=hkv, head_dim=D, q_pos_base=base_pos,
                               kv_pos_base=base_pos, workspace=wss[0], out=(q, k, v))
            for hb, t in zip(hosts, (q, k, v)):
                hb.copy_(t, non_blocking=True)
            stream.synchronize()

        for _ in range(2):
            e2e_step()
        n_e2e = max(3, min(args.steps, 20))
        barrier()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            e2e_step()
        e2e_ms = (time.perf_counter() - t0) * 1e3 / n_e2e
        for hb, t in zip(hosts, outs_kernel):
            if not torch.equal(hb.view(torch.int16), t.cpu().view(torch.int16)):
                raise RuntimeError("API output differs from the timed kernel output")
        h2d = xh.numel() * 2
        d2h = sum(hb.numel() * 2 for hb in hosts)
    if world > 1:
        t = torch.tensor([ms, e2e_ms or 0.0], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t[0])
        e2e_ms = float(t[1]) if e2e_ms is not None else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = prologue_cpu_baseline(x, w, rms, hq, hkv, D, base_pos, args.cpu_seconds)
    if rank != 0:
        return 0
    flops = 2.0 * B * L * hidden * n_total
    peak, peak_src = 1415.2, "fallback 1400 TFLOP/s sustained"
    pp = ROOT / "MEASURED_PEAKS.json"
    if pp.exists():
        try:
            peak = float(json.loads(pp.read_text())["bf16_tflops_sustained"])
            peak_src = "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
        except (ValueError, KeyError):
            pass
    achieved = flops / (ms * 1e-3) / 1e12
    line = {
        "metric": "layer prologue TFLOP/s (RMSNorm + QKV projection + RoPE, tensor-core path)",
        "value": round(achieved * world, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "llama3_8b_qkv_prologue_of_cfg5_chunk", "sequences_per_gpu": B, "tokens": L,
                   "hidden": hidden, "n_q_heads": hq, "n_kv_heads": hkv, "head_dim": D, "position_base": base_pos,
                   "weights": "bf16 [4096][6144] (50 MB, read once per launch from L2/HBM)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_src,
                     "algorithmic_flop_per_step": flops,
                     "note": "step time includes the RMSNorm and RoPE-table kernels (3 launches per step)"},
        "cpu_baseline": cpu,
        "e2e": None if e2e_ms is None else {
            "value": round(flops * world / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms, 4),
            "api": "ops.layer_prologue (pinned host x in, q/k/v out)"},
        "gpu_launches": args.steps * 3, "clocks": clocks,
    }
    print(json.dumps(line), flush=True)
    return 0


def prologue_cpu_baseline(x, w, rms, hq, hkv, D, base_pos, seconds: float) -> dict:
    """The CPU oracle's layer prologue (oracle.prologue.layer_prologue: RMSNorm, fp64
    projection, RoPE) on 8 blocks of 32 tokens of sequence 0, one block per thread."""
    import concurrent.futures as cf

    import torch

    from oracle import prologue as oracle_prologue

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    words = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)  # noqa: E731
    blocks, tok = 8, 32
    xw = words(x[0, :blocks * tok])
    ww, rw = words(w), words(rms)
    hidden, n_total = ww.shape
    flop_block = 2.0 * tok * hidden * n_total

    def unit(i):
        oracle_prologue.layer_prologue(xw[i * tok:(i + 1) * tok], ww, rw, n_q_heads=hq, n_kv_heads=hkv,
                                       head_dim=D, q_pos_base=base_pos + i * tok, kv_pos_base=base_pos + i * tok)

    def passes(threads, ids, repeats, min_s):
        times = []
        with cf.ThreadPoolExecutor(max_workers=threads) as pool:
            list(pool.map(unit, ids))
            t_start = time.perf_counter()
            while len(times) < repeats or time.perf_counter() - t_start < min_s:
                t0 = time.perf_counter_ns()
                list(pool.map(unit, ids))
                times.append((time.perf_counter_ns() - t0) * 1e-9)
        return times

    threads = min(cores, blocks)
    st_all = pass_stats(passes(threads, list(range(blocks)), 3, seconds))
    st_one = pass_stats(passes(1, [0], 3, 0.0))
    return {"value": round(flop_block * blocks / st_all["median_s"] / 1e12, 5), "unit": "TFLOP/s", "cores": threads,
            "kind": "port",
            "sample": f"{blocks} blocks of {tok} tokens of sequence 0, one block per thread; value from the median pass",
            "pass_seconds": st_all,
            "single_thread": {"value": round(flop_block / st_one["median_s"] / 1e12, 5), "unit": "TFLOP/s",
                              "cores": 1, "sample": f"one block of {tok} tokens", "pass_seconds": st_one}}


def main() -> int:
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.gpus != world and world != 1:
        print(f"warning: --gpus {args.gpus} but WORLD_SIZE={world}", file=sys.stderr)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    import datetime

    import torch
    import torch.distributed as dist

    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.config == 5:
            return run_prefill(args, rank, world, local_rank)
        if args.config == 6:
            return run_prologue(args, rank, world, local_rank)
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    raise SystemExit(main())
