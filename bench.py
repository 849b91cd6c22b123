#!/usr/bin/env python3
"""Benchmark of the GQA decode hot path (Llama-3-8B shape).

``python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]``

One step = one decode over the HBM-resident cache of config 2's batch: 64
sequences x 32 query heads over 8 KV heads, head_dim 128, 4096 cached tokens,
bf16 ~ N(0,1)*0.5 (seed 1).  Under torchrun the global batch of 64 is split
across the ranks as BASELINE config 2 states (``"scaling": "strong"``: 64/N
sequences per GPU, no data-path collective); ``--weak`` gives every rank its
own 64 sequences instead.  The metric is the KV-stream bandwidth, GB/s =
sum(len) x Hkv x D x 2 (K and V) x 2 bytes / step time, summed over ranks,
with queries/s = sequences / step time beside it.

* ``value``: device time of K timed steps (CUDA events on the launching
  stream, barrier + synchronize on both sides, max over ranks).  Inputs are
  HBM-resident and larger than L2: a rank whose cache is smaller than 4x L2
  rotates over copies of it, so consecutive steps never read the same bytes.
* launch: the K timed steps are captured into one CUDA graph and replayed
  (``--eager``: a host launch per step); the split-KV step, which holds an
  NCCL collective, is launched from the host.
* ``e2e``: the same metric through the public API with host buffers:
  ``AttentionAccelerator.run_query`` with pinned host q/o (H2D of q, decode,
  D2H of o, synchronous), wall-clock over the steps, max over ranks.
* ``roofline``: the decode kernel's algorithmic bytes per launch / its mean
  launch time, against the measured HBM copy bandwidth.
* ``cpu_baseline``: the CPU oracle (restatement of the reference's
  ``cpu_attention_numpy``) on the same workload, on this host's cores (N=1).
* ``split_kv`` / ``ragged`` / ``prefill``: BASELINE configs 4, 3 and 5 at the
  same N in the same run (config 4: each sequence's 1,048,576 tokens split
  across the ranks, partial decode + NCCL all-gather + LSE combine; config 3:
  256 ragged sequences, token-balanced across ranks; config 5: chunked prefill
  on the tensor cores, (sequence, kv head) units split across ranks), each
  with its own value, roofline and a parity check.
* ``parity``: after the timed regions rank 0 checks sampled (sequence, kv
  head) outputs of every record against the CPU oracle (the checker, outside
  the timed regions): worst floored and strict ulp, and the fp64-anchored
  bound ``|gpu - fp64| <= 2 ulp(fp64) + |golden - fp64|``.
* ``--impl reference``: times the reference's CPU implementation of the path
  (the reference is SystemVerilog RTL plus this NumPy CPU model, so the CPU
  model is what runs here) on rank 0 and prints its own line.
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
import math
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
PREFILL_METRIC = "chunked-prefill attention TFLOP/s (tensor-core path)"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_SUSTAINED = 1400.0
L2_BYTES = 126.5e6          # B200 L2
ROTATE_BYTES = 4 * L2_BYTES  # a rank's per-step inputs are rotated up to this working set
# ncu summaries per workload (dram traffic per launch of the full single-GPU workload)
PROFILE_SUMMARIES = {"llama3_8b_decode": ROOT / "profiles" / "decode_llama3_8b_cfg2.txt",
                     "ragged_decode_stress": ROOT / "profiles" / "decode_tc_ragged_cfg3.txt"}


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, choices=[2, 3, 4, 5, 6], default=2,
                    help="BASELINE config of the main line (2 = the headline Llama-3-8B decode; 5 = chunked "
                         "prefill); 6 = the layer prologue (RMSNorm + QKV projection + RoPE) of config 5's new tokens")
    ap.add_argument("--weak", action="store_true",
                    help="config 2: every rank decodes its own 64 sequences (weak scaling) instead of its share "
                         "of the global batch of 64")
    ap.add_argument("--batch", type=int, default=None,
                    help="config 2: global batch (default 64; per rank with --weak); config 4: sequences (default "
                         "8); config 3: the first N of its 256 ragged sequences (a smaller case for profiling)")
    ap.add_argument("--seq-len", type=int, default=None)
    ap.add_argument("--splits", type=int, default=0, help="force the split count (0 = planner)")
    ap.add_argument("--chunk", type=int, default=0)
    ap.add_argument("--paged", type=int, default=0, metavar="PAGE_SIZE",
                    help="configs 2/3: decode from a paged cache (page pool in shuffled page order, block "
                         "table) instead of the contiguous cache; 0 = contiguous")
    ap.add_argument("--paged-order", choices=["random", "sequential"], default="random",
                    help="page assignment of the paged cache (random permutation or consecutive pages)")
    ap.add_argument("--no-extra", action="store_true",
                    help="config 2: skip the config 3/4/5 records (split_kv, ragged, prefill)")
    ap.add_argument("--extra-steps", type=int, default=200,
                    help="timed steps of each config 3/4/5 record (at most --steps)")
    ap.add_argument("--no-parity", action="store_true", help="skip the post-timing oracle checks")
    ap.add_argument("--eager", action="store_true",
                    help="launch every timed step from the host instead of replaying a CUDA graph of them")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="target CPU-baseline sample time")
    return ap.parse_args(argv)


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


def profiled_traffic(workload: str, nbytes: int):
    """DRAM bytes per launch from the workload's committed ncu summary, scaled by
    the algorithmic bytes this launch processes (the K/V stream is read once, so
    traffic grows in proportion); None when no summary covers the workload."""
    path = PROFILE_SUMMARIES.get(workload)
    if path is None or not path.exists():
        return None, None
    traffic = algo = None
    for line in path.read_text().splitlines():
        try:
            if line.startswith("traffic_bytes_per_launch:"):
                traffic = int(float(line.split(":", 1)[1].split()[0]))
            elif line.startswith("algorithmic_bytes_per_launch:"):
                algo = int(float(line.split(":", 1)[1].split()[0]))
        except (ValueError, IndexError):
            return None, None
    if traffic is None or not algo:
        return None, None
    if nbytes == algo:
        return traffic, f"ncu capture of this workload ({path.name})"
    return int(round(traffic * nbytes / algo)), (f"ncu capture {path.name} scaled by algorithmic bytes "
                                                 f"({traffic / algo:.4f} x)")


def measured_tensor_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops_sustained"]), \
                "measured (MEASURED_PEAKS.json bf16_tflops_sustained)"
        except (ValueError, KeyError):
            pass
    return FALLBACK_BF16_SUSTAINED, f"fallback {FALLBACK_BF16_SUSTAINED:.0f} TFLOP/s sustained"


def rotation_count(rank_bytes: int) -> int:
    """Copies of a rank's per-step inputs to rotate over so that consecutive
    steps' working set is at least 4x L2 (no step re-reads the last one's bytes
    from L2)."""
    return max(1, math.ceil(ROTATE_BYTES / max(int(rank_bytes), 1)))


def workload_config(cfgnum: int, global_batch: int, seq_len) -> dict:
    """The workload a line is quoted on; identical between the two arms."""
    from lara_b200.workloads import CONFIGS, PREFILL

    if cfgnum == 5:
        c = PREFILL
        return {"workload": c.name, "global_batch": c.batch, "new_tokens": c.new, "cached_tokens": c.cached,
                "n_q_heads": c.n_q_heads, "n_kv_heads": c.n_kv_heads, "head_dim": c.head_dim, "causal": True}
    c = CONFIGS[cfgnum]
    return {"workload": c.name, "global_batch": int(global_batch), "seq_len": seq_len, "n_q_heads": c.n_q_heads,
            "n_kv_heads": c.n_kv_heads, "head_dim": c.head_dim}


class Collectives:
    """Barrier / max / sum over ranks (NCCL); no-ops on one process."""

    def __init__(self, world: int, local_rank: int, dev):
        self.world, self.local_rank, self.dev = world, local_rank, dev

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier(device_ids=[self.local_rank])

    def reduce(self, values, op: str):
        if self.world == 1:
            return [float(x) for x in values]
        import torch
        import torch.distributed as dist

        t = torch.tensor([float(x) for x in values], dtype=torch.float64, device=self.dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
        return [float(x) for x in t.tolist()]


def timed_steps(step, steps: int, stream, comm: Collectives, sampler=None, graph: bool = False) -> float:
    """Mean ms per step of `steps` back-to-back calls step(i), by CUDA events on
    `stream`, with a barrier and a synchronize on both sides.

    With `graph` the `steps` calls are first captured into one CUDA graph (and
    replayed once, untimed), and the timed region is one replay of it: the
    same kernels on the same buffers, without a host launch per kernel, as a
    serving loop replays its decode step.  Small steps (tens of microseconds at
    8 sequences per GPU) are otherwise paced by the host's launch rate."""
    import torch

    g = None
    if graph:
        g = torch.cuda.CUDAGraph()
        # thread-local capture: other threads of the process (the process
        # group's watchdog, the clock sampler) keep their CUDA calls
        with torch.cuda.graph(g, capture_error_mode="thread_local"):
            for i in range(steps):
                step(i)
        g.replay()
        torch.cuda.synchronize(stream.device)
    comm.barrier()
    torch.cuda.synchronize(stream.device)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if sampler is not None:
        sampler.start()
    ev0.record(stream)
    if g is not None:
        g.replay()
    else:
        for i in range(steps):
            step(i)
    ev1.record(stream)
    torch.cuda.synchronize(stream.device)
    if sampler is not None:
        sampler.stop()
    comm.barrier()
    del g
    return ev0.elapsed_time(ev1) / steps


def gpu_uuid(dev):
    import torch

    try:
        return "GPU-" + str(torch.cuda.get_device_properties(dev).uuid)
    except Exception:
        return None


# ---------------------------------------------------------------------------
# parity checks (the CPU oracle as the checker, after the timed regions)
# ---------------------------------------------------------------------------

def _words(t) -> np.ndarray:
    import torch

    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


class ParityTally:
    """Worst-case aggregate of oracle.bf16_parity_error over checked head groups."""

    def __init__(self):
        self.r = {"groups": 0, "elements": 0, "max_ulp": 0.0, "max_ulp_strict": 0.0, "n_over_strict": 0,
                  "anchored_ratio": 0.0, "n_over_anchored": 0, "n_over_plain": 0, "excess_kappa_u": 0.0,
                  "eps_golden_u": 0.0, "finite": True}

    def add(self, got_words, gold, g64, tensor_core: bool = False):
        import oracle

        e = oracle.bf16_parity_error(got_words, gold, g64, oracle.TC_SPLIT_P_KAPPA if tensor_core else 0.0)
        r = self.r
        r["groups"] += 1
        r["elements"] += e["n"]
        r["max_ulp"] = max(r["max_ulp"], e["max_ulp"])
        r["max_ulp_strict"] = max(r["max_ulp_strict"], e["max_ulp_strict"])
        r["n_over_strict"] += e["n_over_strict"]
        r["anchored_ratio"] = max(r["anchored_ratio"], e["anchored_ratio"])
        r["n_over_anchored"] += e["n_over_anchored"]
        r["n_over_plain"] += e["n_over_plain"]
        r["excess_kappa_u"] = max(r["excess_kappa_u"], e["excess_kappa_u"])
        r["eps_golden_u"] = max(r["eps_golden_u"], e["eps_golden_u"])
        r["finite"] = r["finite"] and e["finite"]

    def result(self, what: str) -> dict:
        import oracle

        r = dict(self.r)
        r["max_ulp"] = round(r["max_ulp"], 3)
        r["max_ulp_strict"] = round(r["max_ulp_strict"], 3)
        r["anchored_ratio"] = round(r["anchored_ratio"], 4)
        r["ok"] = bool(r["finite"] and r["groups"] > 0 and r["max_ulp"] <= oracle.PARITY_ULPS
                       and r["n_over_anchored"] == 0)
        r["checked"] = what
        return r


def check_decode_groups(cfg, pairs, q_local, seqs, o_local, kv_rows, tensor_core: bool) -> ParityTally:
    """Oracle check of decode outputs: for each (local index, kv head), the G
    query heads of that group.  kv_rows(i, h) returns the sequence's full K/V
    rows of head h as device tensors [n, D]."""
    import oracle

    G = cfg.group
    tally = ParityTally()
    qw, ow = _words(q_local), _words(o_local)
    for i, h in pairs:
        k_rows, v_rows = kv_rows(i, h)
        n = k_rows.shape[0]
        kw = _words(k_rows)[None, None]
        vw = _words(v_rows)[None, None]
        qs = qw[i:i + 1, h * G:(h + 1) * G]
        gold = oracle.decode_attention(qs, kw, vw, np.array([n]))
        g64 = oracle.decode_attention_fp64(qs, kw, vw, np.array([n]))
        tally.add(ow[i, h * G:(h + 1) * G], gold[0], g64[0], tensor_core)
    return tally


# ---------------------------------------------------------------------------
# decode records (configs 2, 3, 4)
# ---------------------------------------------------------------------------

def decode_record(args, cfgnum: int, rank: int, world: int, dev, comm: Collectives, *, steps: int, warmup: int,
                  main: bool) -> dict:
    """Build, time and check one decode workload on this rank.  Every rank
    calls this with the same arguments (it contains collectives)."""
    import torch

    from lara_b200 import ops, parallel
    from lara_b200.workloads import CONFIGS, decode_shard

    cfg = CONFIGS[cfgnum]
    Hq, Hkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    stream = torch.cuda.current_stream(dev)
    run = {}
    tok0, tokn = 0, None
    if cfgnum == 2:
        Bg = (args.batch if main and args.batch else cfg.batch)
        L = (args.seq_len if main and args.seq_len else cfg.seq_len)
        if main and args.weak:
            seqs = [rank * Bg + i for i in range(Bg)]
            lens_all = np.full(Bg * world, L, np.int32)
            global_batch, scaling = Bg * world, "weak"
        else:
            s0, cnt = parallel.batch_range(Bg, world, rank)
            seqs = list(range(s0, s0 + cnt))
            lens_all = np.full(Bg, L, np.int32)
            global_batch, scaling = Bg, "strong"
        seq_len = L
        run["parallelism"] = f"batch-sharded x{world}, {len(seqs)} sequences on rank {rank}"
    elif cfgnum == 3:
        lens_all = cfg.lens(args.batch if main else None)
        seqs = parallel.balanced_partition(lens_all, world)[rank] if world > 1 else list(range(len(lens_all)))
        global_batch, scaling = len(lens_all), "strong"
        seq_len = f"ragged {int(lens_all.min())}..{int(lens_all.max())} (sum {int(lens_all.sum())})"
        run["parallelism"] = f"token-balanced batch partition x{world}, {len(seqs)} sequences on rank {rank}"
    else:
        Bg = (args.batch if main and args.batch else cfg.batch)
        Ltot = (args.seq_len if main and args.seq_len else cfg.seq_len)
        tok0, tokn = parallel.token_range(Ltot, world, rank)
        seqs = list(range(Bg))
        lens_all = np.full(Bg, Ltot, np.int32)
        global_batch, scaling, seq_len = Bg, "strong", Ltot
        run["parallelism"] = (f"split-KV x{world}: tokens [{tok0}, {tok0 + tokn}) of every sequence on rank "
                              f"{rank}, partial decode + NCCL all-gather + LSE combine" if world > 1 else
                              "one GPU (split-KV merged inside the decode kernel)")
    q, k, v, lens = decode_shard(cfg, dev, seqs, lens_all, token_start=tok0, token_count=tokn)
    lens_np = lens.cpu().numpy()
    B, cap = len(seqs), k.shape[2]
    nbytes = cfg.kv_bytes(lens_np)
    paged = main and bool(args.paged)
    R = 1 if paged else rotation_count(nbytes + 2 * q.numel() * 2)
    copies = [(k, v)] + [(k.clone(), v.clone()) for _ in range(R - 1)]
    o = torch.empty_like(q)
    split = cfgnum == 4 and world > 1
    if split:
        dec = parallel.SplitKVDecoder(B, Hq, Hkv, D, cap, dev, lens_local=lens_np)
        plan, ws, launches = dec.decoder.plan, dec.decoder.workspace, 2  # partial decode + combine (+ NCCL)

        def step(i):
            kc, vc = copies[i % R]
            dec(q, kc, vc, lens, out=o)
    elif paged:
        step, plan, ws, launches, pinfo = _paged_step(args, cfg, q, k, v, lens, lens_np, o, dev)
        run["paged"] = pinfo
        copies = None
    else:
        dec = ops.Decoder(B, Hq, Hkv, D, cap, dev, lens=lens_np, num_splits=args.splits if main else 0,
                          chunk_tokens=args.chunk if main else 0)
        plan, ws, launches = dec.plan, dec.workspace, 1

        def step(i):
            kc, vc = copies[i % R]
            dec(q, kc, vc, lens, out=o)
    run.update({"splits": plan.num_splits, "chunk_tokens": plan.chunk_tokens,
                "kernel": ops.decode_kernel(Hq, Hkv, D), "input_copies": R,
                "l2": (f"inputs larger than L2: {R} copies of the rank's {nbytes / 1e6:.1f} MB cache rotated, "
                       f"{R * nbytes / 1e6:.0f} MB between re-reads" if R > 1 else
                       f"inputs larger than L2 ({nbytes / 1e6:.0f} MB per step per rank), no flush")})
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if ops.workspace_status(ws) != 0:
        raise RuntimeError(f"{cfg.name}: decode kernel reported a device error status during warm-up")
    sampler = ClockSampler(gpu_uuid(dev)) if main else None
    use_graph = not args.eager and not split  # the split-KV step holds an NCCL collective
    run["launch"] = "CUDA graph of the timed steps, replayed once" if use_graph else "host launch per step"
    ms = timed_steps(step, steps, stream, comm, sampler, graph=use_graph)
    clocks = sampler.summary() if sampler is not None else None
    if ops.workspace_status(ws) != 0:
        raise RuntimeError(f"{cfg.name}: decode kernel reported a device error status")

    e2e_ms, h2d, d2h, e2e_api = None, 0, 0, None
    if main and not args.no_e2e:
        e2e_ms, h2d, d2h, e2e_api = _decode_e2e(args, cfg, q, copies, lens_np, o, B, cap, step, steps, comm, dev,
                                                split or paged)
    ms_max, e2e_max = comm.reduce([ms, e2e_ms or 0.0], "max")
    total_bytes = int(comm.reduce([nbytes], "sum")[0])

    # parity: rank 0 checks sampled (sequence, kv head) groups
    parity = None
    if rank == 0 and not args.no_parity and B > 0:
        if split:
            def kv_rows(i, h):
                _, kf, vf, _ = decode_shard(cfg, dev, [seqs[i]], lens_all)
                return kf[0, h], vf[0, h]
            pairs = [(0, 1), (B - 1, Hkv - 2)]
        else:
            def kv_rows(i, h):
                n = int(lens_np[i])
                return k[i, h, :n], v[i, h, :n]
            if cfgnum == 3:
                order = np.argsort(lens_np)
                pick = sorted({int(order[-1]), int(order[0]), int(order[len(order) // 2])})
                pairs = [(i, seqs[i] % Hkv) for i in pick]
            else:
                pairs = sorted({(0, 0), (0, Hkv - 3), (B // 2, Hkv // 2), (B - 1, Hkv - 1)})
        on_tc = ops.decode_kernel(Hq, Hkv, D) == "tensor"
        parity = check_decode_groups(cfg, pairs, q, seqs, o, kv_rows, on_tc).result(
            f"{len(pairs)} (sequence, kv head) groups of rank 0: {[(seqs[i], h) for i, h in pairs]}")
    comm.barrier()
    rec = {
        "config": workload_config(cfgnum, global_batch, seq_len),
        "value": round(total_bytes / (ms_max * 1e-3) / 1e9, 2), "unit": "GB/s", "ms_per_step": round(ms_max, 5),
        "steps": steps, "warmup": warmup, "scaling": scaling,
        "queries_per_s": round(global_batch / (ms_max * 1e-3), 1),
        "gpu_launches": steps * launches, "run": run, "parity": parity,
        "_rank_bytes": nbytes, "_rank_ms": ms, "_total_bytes": total_bytes, "_clocks": clocks,
        "_e2e": None if not e2e_ms else {"ms": e2e_max, "h2d": h2d, "d2h": d2h, "api": e2e_api},
        "_cpu_inputs": (q, k, v, lens_np) if main else None, "_cfg": cfg,
    }
    peak, peak_kind = measured_peak()
    achieved = nbytes / (ms * 1e-3) / 1e9
    traffic, traffic_src = profiled_traffic(cfg.name, nbytes) if not paged else (None, None)
    rec["roofline"] = {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                       "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_source": traffic_src,
                       "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                       else "fallback 6650 GB/s", "algorithmic_bytes_per_launch": nbytes,
                       "note": "rank 0's bytes over its step time" + (
                           " (the step includes the NCCL all-gather and the combine launch)" if split else "")}
    if not main:
        del rec["_cpu_inputs"], rec["_clocks"], rec["_e2e"]
    del copies, k, v
    torch.cuda.empty_cache()
    return rec


def _decode_e2e(args, cfg, q, copies, lens_np, o, B, cap, step, steps, comm, dev, device_api_only):
    """The decode through the public API with pinned host q/o: H2D of q, decode,
    D2H of o, synchronous; one context per rotated cache copy."""
    import ctypes

    import torch

    from lara_b200 import _native
    from lara_b200.attn_driver import AttentionAccelerator

    q_host = q.view(torch.int16).cpu().pin_memory()
    o_host = torch.empty_like(q_host).pin_memory()
    qn, on = q_host.numpy().view(np.uint16), o_host.numpy().view(np.uint16)
    e2e_steps = max(10, steps // 4)
    Hq, Hkv, D = cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim
    if not device_api_only:
        accs = []
        try:
            for kc, vc in copies:
                acc = AttentionAccelerator(device=dev.index)
                accs.append(acc)
                acc.configure_heads(Hq, Hkv, D, max_seq_len=cap, batch=B)
                # device-resident cache load through the C ABI (on_device = 1)
                _native.check(_native.lib.lara_kv_load(acc._ctx, kc.data_ptr(), vc.data_ptr(),
                                                       lens_np.ctypes.data_as(ctypes.c_void_p), cap, 1), "kv_load")
            for i in range(max(3, min(args.warmup, 20))):
                accs[i % len(accs)].run_query(qn, out=on)
            comm.barrier()
            t0 = time.perf_counter()
            for i in range(e2e_steps):
                accs[i % len(accs)].run_query(qn, out=on)
            e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
            comm.barrier()
        finally:
            for acc in accs:
                acc.close()
        api = "AttentionAccelerator.run_query (pinned host q/o)"
    else:
        qd, od = q.view(torch.int16), o.view(torch.int16)

        def e2e_step(i):
            qd.copy_(q_host, non_blocking=True)
            step(i)
            o_host.copy_(od, non_blocking=True)
            torch.cuda.synchronize(dev)
        for i in range(3):
            e2e_step(i)
        comm.barrier()
        t0 = time.perf_counter()
        for i in range(e2e_steps):
            e2e_step(i)
        e2e_ms = (time.perf_counter() - t0) * 1e3 / e2e_steps
        comm.barrier()
        api = ("lara_gqa_decode_paged with pinned host q/o copies" if args.paged else
               "lara_b200.parallel.SplitKVDecoder with pinned host q/o copies")
    if not np.array_equal(on, o.view(torch.int16).cpu().numpy().view(np.uint16)):
        raise RuntimeError("API output differs from the timed kernel output")
    return e2e_ms, qn.nbytes, on.nbytes, api


def _paged_step(args, cfg, q, k, v, lens, lens_np, o, dev):
    """Paged cache built from the contiguous one: page pool in shuffled (or
    sequential) page order plus a block table; the step decodes from it."""
    import torch

    from lara_b200 import _native, ops

    B, L = q.shape[0], k.shape[2]
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
    scale = 1.0 / math.sqrt(cfg.head_dim)

    def step(i):
        _native.check(_native.lib.lara_gqa_decode_paged(
            q.data_ptr(), kp.data_ptr(), vp.data_ptr(), table.data_ptr(), lens.data_ptr(), o.data_ptr(), B,
            cfg.n_q_heads, cfg.n_kv_heads, cfg.head_dim, ps, pps, total, scale, plan.num_splits,
            plan.chunk_tokens, dec.workspace.data_ptr(), dec.workspace.numel(),
            torch.cuda.current_stream(dev).cuda_stream),  # the capture stream while a graph records
            "decode_paged")
    info = {"page_size": ps, "pages": total,
            "page_order": "random permutation (seed 7)" if args.paged_order == "random" else "sequential",
            "layout": "[pages][Hkv][page_size][D]"}
    return step, plan, dec.workspace, 1, info


# ---------------------------------------------------------------------------
# prefill record (config 5)
# ---------------------------------------------------------------------------

def prefill_record(args, rank: int, world: int, dev, comm: Collectives, *, steps: int, warmup: int,
                   main: bool) -> dict:
    """Config 5 on this rank's (sequence, kv head) units: one step = reset the
    cached lengths, append the 2048 new K/V tokens, causal attention of the new
    queries over cache + self (tensor cores).  Every rank calls this."""
    import torch

    from lara_b200 import _native, ops
    from lara_b200.workloads import PREFILL, prefill_launch_groups, prefill_shard, prefill_units

    cfg = PREFILL
    G, D, C, n = cfg.n_q_heads // cfg.n_kv_heads, cfg.head_dim, cfg.cached, cfg.new
    stream = torch.cuda.current_stream(dev)
    scale = 1.0 / math.sqrt(D)
    lib = _native.lib
    pieces = prefill_units(cfg, world, rank)
    parts = []
    for b, nseq, h0, nh in prefill_launch_groups(cfg, pieces):
        q, k, v, kn, vn, lens0 = prefill_shard(cfg, dev, b, h0, nh, nseq)
        wsb = int(lib.lara_prefill_workspace_bytes(nseq, n, nh * G, nh, D, C + n))
        rank_bytes = sum(t.numel() * 2 for t in (q, k, v, kn, vn)) + q.numel() * 2
        parts.append({"b": b, "nb": nseq, "h0": h0, "nh": nh, "lens0": lens0, "ws": ops.new_workspace(wsb, dev),
                      "bytes": rank_bytes,
                      "copies": [{"q": q, "k": k, "v": v, "kn": kn, "vn": vn, "o": torch.empty_like(q),
                                  "lens": lens0.clone()}]})
    R = rotation_count(sum(p["bytes"] for p in parts)) if parts else 1
    for p in parts:
        c0 = p["copies"][0]
        for _ in range(R - 1):
            p["copies"].append({key: t.clone() for key, t in c0.items()})
    pairs_per_head = n * C + n * (n + 1) // 2
    flops = sum(p["nb"] * p["nh"] * G * pairs_per_head * 4 * D for p in parts)

    def attend(p, c):
        _native.check(lib.lara_gqa_prefill(c["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(),
                                           p["lens0"].data_ptr(), c["o"].data_ptr(), p["nb"], n, p["nh"] * G, p["nh"], D,
                                           C + n, 1, scale, p["ws"].data_ptr(), p["ws"].numel(),
                                           torch.cuda.current_stream(dev).cuda_stream), "prefill")

    def step(i):
        for p in parts:
            c = p["copies"][i % R]
            c["lens"].copy_(p["lens0"])
            ops.kv_append(c["k"], c["v"], c["lens"], c["kn"], c["vn"], workspace=p["ws"])
            attend(p, c)

    for i in range(warmup):
        step(i)
    torch.cuda.synchronize(dev)
    if any(ops.workspace_status(p["ws"]) != 0 for p in parts):
        raise RuntimeError("prefill reported a device error status during warm-up")
    sampler = ClockSampler(gpu_uuid(dev)) if main else None
    use_graph = not args.eager
    ms = timed_steps(step, steps, stream, comm, sampler, graph=use_graph)
    clocks = sampler.summary() if sampler is not None else None
    # kernel-only rate of the attention launches (the roofline's denominator time)
    k_steps = max(3, steps // 4)
    k_ms = timed_steps(lambda i: [attend(p, p["copies"][i % R]) for p in parts], k_steps, stream, comm,
                       graph=use_graph)
    if any(ops.workspace_status(p["ws"]) != 0 for p in parts):
        raise RuntimeError("prefill reported a device error status")

    e2e = None
    if main and not args.no_e2e:
        e2e = _prefill_e2e(args, cfg, parts, comm, dev)
    ms_max, k_ms_max, e2e_ms = comm.reduce([ms, k_ms, e2e["ms"] if e2e else 0.0], "max")
    total_flops = comm.reduce([flops], "sum")[0]

    parity = None
    if rank == 0 and not args.no_parity and parts:
        import oracle

        p = parts[0]
        c = p["copies"][0]
        tally = ParityTally()
        kw_all, vw_all = _words(c["k"]), _words(c["v"])
        if not (np.array_equal(kw_all[:, :, C:], _words(c["kn"])) and np.array_equal(vw_all[:, :, C:],
                                                                                     _words(c["vn"]))):
            tally.r["finite"] = False  # the append did not land where it should
        qw, ow = _words(c["q"][:1]), _words(c["o"][:1])
        for i0 in (127, n - 2):
            qs = qw[:, i0:i0 + 2].transpose(0, 2, 1, 3)
            args_ = (qs, kw_all[:1], vw_all[:1], np.array([C + n]), C + i0)
            gold = oracle.prefill_attention(*args_, causal=True)[0]
            g64 = oracle.prefill_attention(*args_, causal=True, dtype=np.float64, kappa=True)[0]
            tally.add(ow[0, i0:i0 + 2].transpose(1, 0, 2), gold, g64, os.environ.get("LARA_ATTN_PATH") != "stream")
        parity = tally.result(f"query rows 127-128 and {n - 2}-{n - 1} of sequence {p['b']}, kv heads "
                              f"{p['h0']}..{p['h0'] + p['nh'] - 1} (all their query heads); appended K/V compared "
                              f"word for word")
    comm.barrier()
    peak, peak_src = measured_tensor_peak()
    achieved = flops / (k_ms * 1e-3) / 1e12
    rec = {
        "config": workload_config(5, cfg.batch, None),
        "value": round(total_flops / (ms_max * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "ms_per_step": round(ms_max, 4),
        "steps": steps, "warmup": warmup, "scaling": "strong",
        "gpu_launches": steps * 3 * len(parts),
        "run": {"parallelism": f"(sequence, kv head) units split x{world}: rank {rank} holds "
                               f"{[(b, f'kv {h0}..{h0 + nh - 1}') for b, h0, nh in pieces]}, "
                               f"{len(parts)} launch group(s)",
                "step": "length reset + K/V append + attention (3 kernels per launch group: append, length "
                        "update, prefill)",
                "launch": "CUDA graph of the timed steps, replayed once" if use_graph else "host launch per step",
                "p_precision": "bf16 RNE (LARA_TC_SPLIT_P=0)" if os.environ.get("LARA_TC_SPLIT_P") == "0"
                else "P_hi + P_lo", "input_copies": R,
                "l2": f"{R} copies of the rank's inputs rotated (>= 4x L2 between re-reads)" if R > 1
                else "inputs larger than 4x L2"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(achieved / peak, 4), "traffic": None, "peak_source": peak_src,
                     "algorithmic_flop_per_launch": flops, "attention_kernel_ms": round(k_ms, 4),
                     "attention_kernel_ms_max_over_ranks": round(k_ms_max, 4)},
        "parity": parity,
    }
    if main:
        rec["_clocks"] = clocks
        rec["_e2e"] = None if e2e is None else dict(e2e, ms=e2e_ms)
        rec["_total_flops"] = total_flops
        rec["_cpu"] = (parts[0]["copies"][0] if parts else None)
    for p in parts:
        p["copies"].clear()
    torch.cuda.empty_cache()
    return rec


def _prefill_e2e(args, cfg, parts, comm, dev) -> dict:
    """AttentionAccelerator.run_prefill_chunk with page-locked host buffers:
    every step the chunk's q and new K/V go host->device and the output comes
    back (pipelined by sequence), after truncate_kv rewinds the last append."""
    import torch

    from lara_b200.attn_driver import AttentionAccelerator

    G, D, C, n = cfg.n_q_heads // cfg.n_kv_heads, cfg.head_dim, cfg.cached, cfg.new
    accs, jobs = [], []
    h2d = d2h = 0
    try:
        for p in parts:
            c = p["copies"][0]

            def pinned(t):
                h = t.cpu().view(torch.int16).pin_memory()
                return h, h.numpy().view(np.uint16)
            (qh, qn), (knh, knn), (vnh, vnn) = (pinned(t) for t in (c["q"], c["kn"], c["vn"]))
            oh, on = pinned(torch.empty_like(c["q"]))
            acc = AttentionAccelerator(device=dev.index)
            accs.append(acc)
            acc.configure_heads(p["nh"] * G, p["nh"], D, max_seq_len=C + n, batch=p["nb"])
            acc.load_kv(_words(c["k"][:, :, :C]), _words(c["v"][:, :, :C]), np.full(p["nb"], C, np.int32))
            jobs.append((acc, qn, knn, vnn, on, c["o"], p["nb"]))
            h2d += sum(x.numel() * 2 for x in (qh, knh, vnh))
            d2h += oh.numel() * 2

        def e2e_step():
            for acc, qn, knn, vnn, on, _, nseq in jobs:
                acc.truncate_kv(np.full(nseq, C, np.int32))
                acc.run_prefill_chunk(qn, knn, vnn, causal=True, out=on)
        for _ in range(2):
            e2e_step()
        n_e2e = max(3, min(args.steps, 20))
        comm.barrier()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            e2e_step()
        ms = (time.perf_counter() - t0) * 1e3 / n_e2e
        comm.barrier()
        for acc, qn, knn, vnn, on, o_dev, _ in jobs:
            if not np.array_equal(on, _words(o_dev)):
                raise RuntimeError("API output differs from the timed kernel output")
    finally:
        for acc in accs:
            acc.close()
    return {"ms": ms, "h2d": h2d, "d2h": d2h,
            "api": "AttentionAccelerator.run_prefill_chunk (page-locked host q, k_new, v_new, o; truncate_kv "
                   "rewinds the chunk each step)"}


# ---------------------------------------------------------------------------
# arms
# ---------------------------------------------------------------------------

def _public(rec: dict) -> dict:
    return {k: v for k, v in rec.items() if not k.startswith("_")}


def run_ours(args, rank: int, world: int, local_rank: int) -> int:
    import torch

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    comm = Collectives(world, local_rank, dev)
    if args.config == 5:
        return _print_prefill_main(args, rank, world, dev, comm)
    main = decode_record(args, args.config, rank, world, dev, comm, steps=args.steps, warmup=args.warmup, main=True)
    extras = {}
    if (args.config == 2 and not args.no_extra and args.batch is None and args.seq_len is None
            and not args.paged):
        ks = max(1, min(args.steps, args.extra_steps))
        kw = max(3, min(args.warmup, 20))
        extras["split_kv"] = decode_record(args, 4, rank, world, dev, comm, steps=ks, warmup=kw, main=False)
        extras["ragged"] = decode_record(args, 3, rank, world, dev, comm, steps=ks, warmup=kw, main=False)
        extras["prefill"] = prefill_record(args, rank, world, dev, comm, steps=ks, warmup=kw, main=False)
    if rank != 0:
        return 0
    cfg = main["_cfg"]
    cpu = None
    if not args.no_cpu_baseline and world == 1:
        cpu = _decode_cpu_baseline(args, cfg, *main["_cpu_inputs"])
    e2e = main["_e2e"]
    line = {
        "metric": METRIC, "value": main["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": main["ms_per_step"], "higher_is_better": True,
        "scaling": main["scaling"], "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) x std per BASELINE config, drawn per sequence and token block)",
        "config": main["config"], "run": main["run"],
        "queries_per_s": main["queries_per_s"],
        "pct_hbm_peak": round(100.0 * main["roofline"]["frac"], 2),
        "roofline": main["roofline"],
        "cpu_baseline": cpu,
        "e2e": None if e2e is None else {
            "value": round(main["_total_bytes"] / (e2e["ms"] * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"], "ms_per_step": round(e2e["ms"], 5),
            "api": e2e["api"]},
        "gpu_launches": main["gpu_launches"],
        "clocks": main["_clocks"],
        "parity": main["parity"],
    }
    for name, rec in extras.items():
        line[name] = _public(rec)
    print(json.dumps(line), flush=True)
    # a timed region that ran less work than it counts would read far above the
    # copy-bandwidth / GEMM peak that the roofline divides by
    implausible = [n for n, r in [("main", main)] + list(extras.items()) if r["roofline"]["frac"] > 1.5]
    if implausible:
        print(f"roofline fraction above 1.5 for: {implausible}", file=sys.stderr)
        return 1
    bad = [n for n, r in [("main", main)] + list(extras.items()) if r.get("parity") and not r["parity"]["ok"]]
    if bad:
        print(f"parity check failed for: {bad}", file=sys.stderr)
        return 1
    return 0


def _print_prefill_main(args, rank, world, dev, comm) -> int:
    rec = prefill_record(args, rank, world, dev, comm, steps=args.steps, warmup=args.warmup, main=True)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and rec["_cpu"] is not None:
        from lara_b200.workloads import PREFILL

        c = rec["_cpu"]
        cpu = prefill_cpu_baseline(PREFILL, c["q"], c["k"], c["v"], args.cpu_seconds)
    if rank != 0:
        return 0
    e2e = rec["_e2e"]
    line = {
        "metric": PREFILL_METRIC, "value": rec["value"], "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) x 0.5 per sequence)",
        "config": rec["config"], "run": rec["run"], "roofline": rec["roofline"], "cpu_baseline": cpu,
        "e2e": None if e2e is None else {
            "value": round(rec["_total_flops"] / (e2e["ms"] * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
            "h2d_bytes_per_step": e2e["h2d"], "d2h_bytes_per_step": e2e["d2h"], "ms_per_step": round(e2e["ms"], 4),
            "api": e2e["api"]},
        "gpu_launches": rec["gpu_launches"], "clocks": rec["_clocks"], "parity": rec["parity"],
    }
    print(json.dumps(line), flush=True)
    return 0 if (rec["parity"] is None or rec["parity"]["ok"]) else 1


def _decode_cpu_baseline(args, cfg, q, k, v, lens_np) -> dict:
    """The CPU oracle over a bounded sample of the rank's sequences (as many
    whole sequences as fit ~4 GB of bf16 on the host), all cores and one."""
    import torch

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    B = q.shape[0]
    per_seq = [int(x) * cfg.n_kv_heads * cfg.head_dim * 4 for x in lens_np]
    nseq, acc_b = 0, 0
    while nseq < B and (nseq == 0 or acc_b + per_seq[nseq] <= 4 << 30):
        acc_b += per_seq[nseq]
        nseq += 1
    Ls = int(lens_np[:nseq].max())
    qn_, kn_, vn_ = (t[:nseq, :, :Ls].contiguous() if t.dim() == 4 else t[:nseq].contiguous() for t in (q, k, v))
    qn_, kn_, vn_ = (t.view(torch.int16).cpu().numpy().view(np.uint16) for t in (qn_, kn_, vn_))
    pairs = [(b, h) for b in range(nseq) for h in range(cfg.n_kv_heads)]
    gbs, st_all, gbs1, st_one, n1 = cpu_baseline_runs(qn_, kn_, vn_, lens_np[:nseq], pairs, cores, args.cpu_seconds)
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"passes over {nseq} of {B} sequences ({int(lens_np[:nseq].sum())} tokens, "
                      f"{len(pairs)} (sequence, kv-head) pairs) on {cores} threads, value from the median "
                      f"pass; oracle restatement of sw/board_performance.py:158-192",
            "pass_seconds": st_all,
            "single_thread": {"value": round(gbs1, 3), "unit": "GB/s", "cores": 1,
                              "sample": f"first {n1} (sequence, kv-head) pairs of the same sample",
                              "pass_seconds": st_one}}


def run_reference(args, rank: int, world: int) -> int:
    """CPU reference path (oracle port of cpu_attention_numpy), rank 0 only.

    Each of the K timed steps decodes a bounded sample of config 2's (sequence,
    kv-head) pairs, sized by a calibration so the K steps take about a minute;
    the value is the sample's KV bytes over its time.  The line's ``config`` is
    the workload our arm is quoted on at the same N."""
    if rank != 0:
        return 0
    import oracle
    from lara_b200.workloads import CONFIGS

    cfg = CONFIGS[2]
    Bg = args.batch or cfg.batch
    global_batch = Bg * world if args.weak else Bg
    L = args.seq_len or cfg.seq_len
    Hkv, D = cfg.n_kv_heads, cfg.head_dim
    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    pack = oracle.fp32_to_bf16_u16
    rng = np.random.default_rng(cfg.seed)
    nb = min(Bg, max(1, -(-cores // Hkv)) * 2)  # sequences held on the host for the samples
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
        "scaling": "weak" if args.weak else "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) x 0.5)",
        "config": workload_config(2, global_batch, L),
        "queries_per_s": round(n_pairs / Hkv / t, 2),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"per step, {n_pairs} of the workload's {global_batch * Hkv} (sequence, kv-head) "
                                   f"pairs x {L} tokens (a bounded sample; GB/s is a per-byte rate, so it compares "
                                   f"with the GPU's at the same config); the reference's implementation of this "
                                   f"path is CPU NumPy (sw/board_performance.py:158-192), run as the oracle port "
                                   f"on {cores} threads, rank 0 only",
                         "pass_seconds": pass_stats(step_s),
                         "single_thread": {"value": round(nb1 / st_one["median_s"] / 1e9, 3), "unit": "GB/s",
                                           "cores": 1, "sample": f"first {n1} pairs of the same sample",
                                           "pass_seconds": st_one}},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
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
        if args.config == 6:
            return run_prologue(args, rank, world, local_rank)
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1 and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    raise SystemExit(main())
