"""Benchmark of the fused top-k / top-p sampling path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints ONE JSON line (rank 0). The metric is BASELINE.json's: µs per sampling call at
B=1, V=151936, k=50, p=0.9, BF16 (the C1 anchor; lower is better), plus HBM GB/s at B=1024 against
the measured peak (the C3 config, reported in `roofline`).

* A step is one sampling call on one batch. `value` is the amortised device time per call over
  exactly K back-to-back steps, inputs resident in HBM, cold L2: the steps rotate over enough
  distinct input buffers to exceed 2x L2 (126 MB). A short device spin before the start event
  lets the host queue the calls ahead of the GPU, so a small K measures device latency rather
  than the host's first launches into an idle GPU; `no_queue_fill_us` is the same K calls
  without it.
* `e2e` is the same metric through the public API with host buffers, every step inside the timed
  region: `fused.sample_fused` on pinned host logits, which the kernel reads over PCIe in place,
  writing the id into a pinned host tensor (`staged_us`: the same with copy-engine transfers, an
  upload into a device buffer and a download of the id).
* `roofline` is the B=1024 call (311 MB of logits per call, two rotating buffers > 2x L2). At that
  batch the call is the streaming path's two launches (slice kernel, then row merge); the time
  is the CUDA-event time of the whole call, so `achieved` (algorithmic bytes B*V*2 + B*8 over it)
  charges the row merge to the slice kernel. Peak: MEASURED_PEAKS.json's burst HBM copy bandwidth.
* `cpu_baseline` / `--impl reference` time the reference's own CPU implementation of the path,
  benchmarks/reference.py:sample_eager(check_inputs=False) built into oracle/_ref by
  `make -C oracle` (the oracle port of it when that is missing), on all host threads, on a
  bounded sample of C1 calls.
* `adversarial` (one GPU): µs per call of the four adversarial configurations at B=8,
  V=151936, FP16 (16 distinct values at k=1024; top-p only at k=V, the wide path; greedy; rows
  with +-inf and the most negative finite value), cold L2. `lm_head` (one GPU): the LM-head
  producer against the GEMM alone and GEMM + one sampler call.
* N > 1 (torchrun, one process per GPU): weak scaling of the anchor (each rank samples its own
  B=1 row; value = max over ranks), plus the B=1024 batch-sharded config (rows split across
  ranks, no collective on the data path) and the vocab-sharded tensor-parallel config (B=32,
  V=256000 split into N shards, candidates all-gathered over NCCL, merged and sampled on every
  rank). All multi-GPU times are CUDA-event times, max over ranks.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
METRIC = "µs/sampling call (B=1,V=151936,k=50,p=.9 BF16); HBM GB/s at B=1024 vs peak"
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0

C1 = dict(B=1, V=151936, k=50, p=0.9)
C3 = dict(B=1024, V=151936, k=50, p=0.95)
C4 = dict(B=32, V=256000, k=64, p=0.9)


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# ---------------------------------------------------------------------------------------------
# environment
# ---------------------------------------------------------------------------------------------


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (burst copy, measured)"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback 6.65 TB/s (earlier measurement on this pool)"


def committed_traffic():
    """DRAM bytes of one B=1024 call (slice + row-merge launches) from the committed ncu summary."""
    p = ROOT / "profiles" / "fs_slice_kernel_b1024.md"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_call:"):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 50 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------------
# synthetic inputs (seeded, generated on the device)
# ---------------------------------------------------------------------------------------------


def anchor_buffers(n, B, V, device, seed=1234):
    """C1: N(0, 2^2) bf16 with 20 distinct random ids per row boosted by +8. All n buffers come
    from one generation pass (rows of one tensor, each buffer its own memory)."""
    g = torch.Generator(device=device).manual_seed(seed)
    rng = np.random.default_rng(seed)
    idx = np.stack([rng.choice(V, 20, replace=False) for _ in range(n * B)])
    x = torch.randn(n * B, V, generator=g, device=device) * 2.0
    x.scatter_add_(1, torch.from_numpy(idx).to(device), torch.full((n * B, 20), 8.0, device=device))
    x = x.to(torch.bfloat16)
    return [x[i * B:(i + 1) * B] for i in range(n)]


def zipf_buffers(n, B, V, device, seed=7, sigma=3.0, s=1.1):
    """C3: N(0, 3^2) plus a per-row Zipf(1.1) log-bias over a random permutation of ids."""
    g = torch.Generator(device=device).manual_seed(seed)
    ranks = torch.arange(1, V + 1, device=device, dtype=torch.float32)
    bias = -s * torch.log(ranks)
    bias = bias - bias.mean()
    out = []
    for _ in range(n):
        x = torch.randn(B, V, generator=g, device=device) * sigma
        for r0 in range(0, B, 128):
            rows = min(128, B - r0)
            perm = torch.rand(rows, V, generator=g, device=device).argsort(dim=-1)
            x[r0:r0 + rows].scatter_add_(1, perm, bias.expand(rows, V))
        out.append(x.to(torch.bfloat16))
        del x
    torch.cuda.synchronize()
    return out


def tp_logits(B, V, device, seed=11, sigma=2.5):
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(B, V, generator=g, device=device) * sigma).to(torch.bfloat16)


# ---------------------------------------------------------------------------------------------
# timing helpers
# ---------------------------------------------------------------------------------------------


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


QUEUE_FILL_US = 200  # device spin ahead of the start event (see timed_steps)


def timed_steps(fn, steps, warmup, world, queue_fill=True):
    """Warm-up, then exactly `steps` calls between CUDA events on the current stream with a
    barrier + synchronize on both sides. Returns the device ms of the timed region. Step indices
    continue past the warm-up (fn(warmup + i)), so a timed step never reuses the input buffer of a
    warm-up step.

    queue_fill: a device spin of QUEUE_FILL_US is enqueued before the start event, so the host
    has issued the first calls by the time the GPU reaches them and the events time the calls'
    amortised device latency, not the host's first launches into an idle GPU (the reference's
    harness gets the same by calibrating thousands of calls per sample). The spin is outside the
    events; the timed region holds exactly the `steps` calls."""
    for i in range(warmup):
        fn(i)
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    if queue_fill:
        torch.cuda._sleep(int(QUEUE_FILL_US * 2000))  # cycles at about 2 GHz
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for i in range(steps):
        fn(warmup + i)
    e.record()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    return s.elapsed_time(e)


# ---------------------------------------------------------------------------------------------
# the CPU side: the reference's own sample_eager (built into oracle/_ref by `make -C oracle`),
# else the oracle port of it
# ---------------------------------------------------------------------------------------------


def reference_cpu_impl():
    """(fn(x, k, p), kind, description) of the CPU implementation to time: the reference's own
    benchmarks/reference.py:sample_eager(check_inputs=False) when oracle/_ref holds it, else the
    oracle's port of it."""
    refpkg = ROOT / "oracle" / "_ref" / "refpkg"
    if (refpkg / "benchmarks" / "reference.py").exists():
        sys.path.insert(0, str(refpkg))
        try:
            from benchmarks.reference import sample_eager

            return (lambda x, k, p, i: sample_eager(x, k, p, check_inputs=False), "reference",
                    "benchmarks/reference.py:sample_eager(check_inputs=False), the reference's own code "
                    "(torch CPU FP32 stable sort + softmax + cumsum + multinomial)")
        except Exception as e:  # noqa: BLE001
            log(f"reference sample_eager unavailable ({e}); timing the oracle port")
        finally:
            sys.path.remove(str(refpkg))
    sys.path.insert(0, str(ROOT))
    from oracle import sampler_oracle as orc

    return (lambda x, k, p, i: orc.sample(x, k, p, seed=1, offset=i), "port",
            "the oracle port of benchmarks/reference.py:sample_eager (oracle/_ref not built)")


def cpu_reference_time(B, V, k, p, budget_s=10.0, min_calls=3):
    """µs per call of the reference's CPU implementation on all host cores, on a bounded sample:
    as many calls on the workload's logits as fit in budget_s (at least min_calls)."""
    sys.path.insert(0, str(ROOT))
    from oracle import sampler_oracle as orc

    fn, kind, what = reference_cpu_impl()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    x = orc.anchor_logits(B=B, V=V, seed=1234) if B <= 64 else orc.zipf_logits(B, V, seed=7)
    fn(x, k, p, 0)  # warm-up
    n, t0 = 0, time.perf_counter()
    while n < min_calls or time.perf_counter() - t0 < budget_s:
        fn(x, k, p, n)
        n += 1
    dt = time.perf_counter() - t0
    return dt / n * 1e6, threads, n, kind, what


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------


def run_ours(args):
    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    sys.path.insert(0, str(ROOT))
    import llm_sampling_kernel_b200 as pkg
    from llm_sampling_kernel_b200 import fused

    ops = pkg.ops()
    result = {}
    launches = 0
    sampler = ClockSampler(local)
    with sampler:
        # ---- C1 anchor: per-rank B=1 row (weak scaling over ranks) ----
        per = C1["B"] * C1["V"] * 2
        nbuf = max(2, (2 * L2_BYTES) // per + 1)
        bufs = anchor_buffers(nbuf, C1["B"], C1["V"], device, seed=1234 + rank)

        def c1_step(i):
            ops.sample_fused(bufs[i % nbuf], C1["k"], C1["p"], 0x5EED, i, 0)

        ms = timed_steps(c1_step, args.steps, args.warmup, world)
        launches += args.steps
        c1_us = max_over_ranks(ms * 1000.0 / args.steps, world)
        # the same K calls issued into an idle GPU (host launch rate included)
        ms_nf = timed_steps(c1_step, args.steps, args.warmup, world, queue_fill=False)
        launches += args.steps
        c1_nofill_us = max_over_ranks(ms_nf * 1000.0 / args.steps, world)
        # hot L2 (one buffer), for reference
        ms_hot = timed_steps(lambda i: ops.sample_fused(bufs[0], C1["k"], C1["p"], 0x5EED, i, 0),
                             args.steps, args.warmup, world)
        c1_hot_us = max_over_ranks(ms_hot * 1000.0 / args.steps, world)
        launches += args.steps
        # the same calls replayed from a CUDA graph (how a serving engine issues a decode step):
        # 64 calls over 64 rotating buffers per graph; generator mode so replays advance the RNG
        per_graph = 64
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            for j in range(3):
                ops.sample_fused(bufs[j], C1["k"], C1["p"], 0x5EED, -1, 0)
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(g):
            for j in range(per_graph):
                ops.sample_fused(bufs[j % nbuf], C1["k"], C1["p"], 0x5EED, -1, 0)
        replays = max(3, args.steps // per_graph)
        ms_graph = timed_steps(lambda i: g.replay(), replays, 3, world)
        c1_graph_us = max_over_ranks(ms_graph * 1000.0 / (replays * per_graph), world)
        launches += replays * per_graph
        del g

        # ---- e2e through the public API with host buffers (pinned) ----
        # Each step samples a different pinned host buffer (as many as the device-resident anchor
        # rotates over, > 2x L2, so no step can reuse lines another step brought in): the call
        # reads the logits over PCIe in place and writes the id into a pinned host tensor. The
        # copy-engine variant (upload into a device buffer, the call, download of the id) is
        # timed beside it as `staged_us`.
        host = [b.cpu().pin_memory() for b in bufs]
        ids_host = torch.empty(C1["B"], dtype=torch.int64).pin_memory()
        dev_in = torch.empty_like(bufs[0])
        e2e_out = []

        def e2e_step(i):
            out = fused.sample_fused(host[i % len(host)], C1["k"], C1["p"], offset=i)
            if i == 0:
                e2e_out.append(out)

        ms_e2e = timed_steps(e2e_step, args.steps, args.warmup, world, queue_fill=False)
        e2e_us = max_over_ranks(ms_e2e * 1000.0 / args.steps, world)
        # the first step's id, read on the host, equals the device-resident call's
        e2e_ok = int(e2e_out[0][0]) == int(ops.sample_fused(bufs[0], C1["k"], C1["p"], 0x5EED, 0, 0).cpu()[0])
        launches += args.steps

        def staged_step(i):
            dev_in.copy_(host[i % len(host)], non_blocking=True)
            out = fused.sample_fused(dev_in, C1["k"], C1["p"], offset=i)
            ids_host.copy_(out, non_blocking=True)

        ms_staged = timed_steps(staged_step, args.steps, args.warmup, world, queue_fill=False)
        staged_us = max_over_ranks(ms_staged * 1000.0 / args.steps, world)
        launches += args.steps
        del bufs, host

        # ---- C3 B=1024 HBM-bound launch (roofline); rows sharded across ranks ----
        b_rank = C3["B"] // world
        big = zipf_buffers(2, b_rank, C3["V"], device, seed=7 + rank)
        c3_steps = max(3, min(args.steps, 50))

        def c3_step(i):
            ops.sample_fused(big[i % 2], C3["k"], C3["p"], 0x5EED, i, 0)

        ms3 = timed_steps(c3_step, c3_steps, max(3, args.warmup), world)
        # the streaming path launches a slice kernel and a row merge per call
        launches += c3_steps * (2 if ops.plan(b_rank, C3["V"], C3["k"], 0)[7] == 2 else 1)
        c3_us = max_over_ranks(ms3 * 1000.0 / c3_steps, world)
        del big
        torch.cuda.empty_cache()

        # ---- LM-head producer (one GPU): logits GEMM in L2-sized vocabulary chunks, each chunk's
        # top-k taken while it is in L2, one merge -- against the GEMM writing [B, V] logits to
        # HBM and the sampler reading them back ----
        lm_head = None
        if world == 1:
            lm_head = run_lm_head(ops, device, args)
            launches += lm_head.pop("launches")

        # ---- C5 adversarial cases (one GPU) ----
        adversarial = None
        if world == 1:
            adversarial = run_adversarial(ops, device, args)
            launches += adversarial.pop("launches")

        # ---- C4 vocab-sharded tensor parallel (N > 1) ----
        tp = None
        if world > 1:
            tp = run_tp(ops, world, rank, device, args)
            launches += tp.pop("launches")

    clocks = sampler.summary()
    hbm_peak, peak_src = measured_peaks()
    alg_bytes = b_rank * C3["V"] * 2 + b_rank * 8
    achieved = alg_bytes / (c3_us * 1e-6) / 1e9  # per rank
    plan1 = ops.plan(C1["B"], C1["V"], C1["k"], 0)
    plan3 = ops.plan(b_rank, C3["V"], C3["k"], 0)
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": round(c1_us, 3),
        "unit": "µs/call",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(c1_us / 1000.0, 6),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u16-key select + f32 softmax (bf16 logits)",
        "data": "synthetic (seeded, generated on device)",
        "config": {
            "workload": "C1 anchor: B=1 per GPU, V=151936, k=50, p=0.9, BF16 N(0,2^2) + 20 ids boosted by 8",
            "B_per_gpu": C1["B"], "V": C1["V"], "top_k": C1["k"], "top_p": C1["p"],
            "l2": f"cold: {nbuf} rotating input buffers ({nbuf * per / 2**20:.0f} MiB > 2x L2)",
            "plan": {"splits": plan1[0], "chunks": plan1[1], "threads": plan1[2], "capacity": plan1[3]},
            "parallelism": f"dp{world} (independent rows, no collective)",
        },
        "queue_fill": f"{QUEUE_FILL_US} us device spin before the start event (amortised device latency)",
        "no_queue_fill_us": round(c1_nofill_us, 3),
        "hot_l2_us": round(c1_hot_us, 3),
        "graph_replay_us": round(c1_graph_us, 3),
        "e2e": {"value": round(e2e_us, 3), "unit": "µs/call", "h2d_bytes_per_step": per,
                "d2h_bytes_per_step": C1["B"] * 8, "api": "llm_sampling_kernel_b200.fused.sample_fused",
                "transfer": "pinned host logits read in place over PCIe by the call's kernel, id written "
                            "to a pinned host tensor; one host buffer per step, rotating over > 2x L2",
                "ids_match_device_call": e2e_ok,
                "staged_us": round(staged_us, 3),
                "staged": "copy-engine upload to a device buffer, the call, copy-engine download of the id"},
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4),
            # the committed summary is a B=1024 call; a rank's call reads its rows' share
            "traffic": (None if committed_traffic() is None
                        else int(committed_traffic() * b_rank / C3["B"])),
            "kernel": (f"fs_slice_kernel<bf16,{plan3[1]}> + fs_rowmerge_kernel<bf16> (one call, both launches)"
                       if plan3[7] == 2 else f"fs_cluster_kernel<bf16,{plan3[1]}>"),
            "workload": f"C3 B={b_rank} per GPU, V=151936, k=50, p=0.95, Zipf(1.1)-biased N(0,3^2), "
                        f"2 rotating 311 MB buffers (> 2x L2)",
            "us_per_launch": round(c3_us, 3), "algorithmic_bytes_per_launch": alg_bytes,
            "peak_source": peak_src,
        },
        "b1024": {"us_per_call": round(c3_us, 3), "rows_per_gpu": b_rank,
                  "aggregate_hbm_gbs": round(achieved * world, 1), "scaling": "strong",
                  "plan": {"splits": plan3[0], "chunks": plan3[1], "path": plan3[7],
                           "workspace_bytes": plan3[8]}},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if tp is not None:
        line["tp"] = tp
    if lm_head is not None:
        line["lm_head"] = lm_head
    if adversarial is not None:
        line["adversarial"] = adversarial
    if world == 1 and not args.no_cpu:
        cpu_us, threads, n, kind, what = cpu_reference_time(C1["B"], C1["V"], C1["k"], C1["p"],
                                                            budget_s=args.cpu_budget)
        line["cpu_baseline"] = {"value": round(cpu_us, 1), "unit": "µs/call", "cores": threads, "kind": kind,
                                "sample": f"C1 row (B=1, V=151936, k=50, p=0.9) x {n} calls of {what}, "
                                          f"{threads} host threads"}
    print(json.dumps(line), flush=True)


def adversarial_buffers(case, n, B, V, device, seed):
    """C5 inputs, fp16: 1 = logits taking 16 distinct values; 2 = near-flat N(0, 0.1^2);
    3 = N(0, 2^2) (greedy); 4 = N(0, 2^2) with +-inf and the most negative finite value planted in
    some rows (a +inf row, a row with -inf entries, a row that is entirely the lowest value)."""
    g = torch.Generator(device=device).manual_seed(seed)
    if case == 1:
        levels = torch.linspace(-3.0, 3.0, 16, device=device)
        x = levels[torch.randint(0, 16, (n * B, V), generator=g, device=device)]
    elif case == 2:
        x = torch.randn(n * B, V, generator=g, device=device) * 0.1
    else:
        x = torch.randn(n * B, V, generator=g, device=device) * 2.0
    x = x.to(torch.float16)
    if case == 4:
        xv = x.view(n, B, V)
        xv[:, 0, 7] = float("inf")
        xv[:, 1, ::3] = float("-inf")
        xv[:, 2, :] = -65504.0
        xv[:, 3, 100] = -65504.0
    return [x[i * B:(i + 1) * B] for i in range(n)]


def run_adversarial(ops, device, args):
    """The four adversarial configurations at B=8, V=151936, FP16: 16 distinct values at k=1024,
    p=0.99; top-p only (k=V, p=0.5) on N(0, 0.1^2) (the wide path); greedy k=1; rows with +-inf and
    the most negative finite value (k=1024, p=0.9). Also the 16-value rows at k=50, p=0.9 (the tie
    fallback at small k). Each timed over rotating buffers > 2x L2."""
    B, V = 8, C1["V"]
    per = B * V * 2
    nbuf = max(2, (2 * L2_BYTES) // per + 1)
    steps = max(3, min(args.steps, 200))
    warm = max(3, args.warmup)
    cases = ((1, "case1_16_values_k1024_p099_us", 1024, 0.99), (2, "case2_top_p_only_k_eq_V_p05_us", V, 0.5),
             (3, "case3_greedy_k1_us", 1, 0.9), (4, "case4_inf_and_lowest_finite_k1024_us", 1024, 0.9),
             (1, "case1_16_values_k50_p09_us", 50, 0.9))
    out = {}
    launches = 0
    for case, name, k, p in cases:
        bufs = adversarial_buffers(case, nbuf, B, V, device, seed=40 + case)

        def step(i, bufs=bufs, k=k, p=p):
            ops.sample_fused(bufs[i % nbuf], k, p, 0x5EED, i, 0)

        out[name] = round(timed_steps(step, steps, warm, 1) * 1000.0 / steps, 3)
        launches += steps * (5 if ops.plan(B, V, k, 0)[7] == 3 else 1)
        del bufs
        torch.cuda.empty_cache()
    out.update({"B": B, "V": V, "dtype": "fp16", "launches": launches,
                "l2": f"cold: {nbuf} rotating buffers per case ({nbuf * per / 2**20:.0f} MiB > 2x L2)",
                "paths": {"case2": "wide (histogram clear, histogram, row, count, pick launches)",
                          "others": "cluster (one launch)"}})
    return out


def run_lm_head(ops, device, args):
    """B=1024 rows of H=4096 hidden states through a [151936, 4096] bf16 LM head: the GEMM alone,
    the GEMM writing [B, V] logits to HBM followed by the sampler (k=50, p=0.95), and the chunked
    pipeline (llm_sampling_kernel_b200.lm_head.LMHeadSampler). Synthetic random weights."""
    from llm_sampling_kernel_b200.lm_head import LMHeadSampler

    B, H, V, k, p = 1024, 4096, 151936, 50, 0.95
    g = torch.Generator(device=device).manual_seed(17)
    w = (torch.randn(V, H, generator=g, device=device) * 0.02).to(torch.bfloat16)
    h = (torch.randn(B, H, generator=g, device=device)).to(torch.bfloat16)
    logits = torch.empty(B, V, dtype=torch.bfloat16, device=device)
    lm = LMHeadSampler(w, k, max_batch=B)
    steps = max(3, min(args.steps, 20))
    warm = max(3, args.warmup)

    def gemm(i):
        torch.matmul(h, w.t(), out=logits)

    def unfused(i):
        torch.matmul(h, w.t(), out=logits)
        ops.sample_fused(logits, k, p, 0x5EED, i, 0)

    def pipelined(i):
        lm.sample(h, p, seed=0x5EED, offset=i)

    out = {}
    for name, fn in (("gemm_only_us", gemm), ("unfused_us", unfused), ("pipelined_us", pipelined)):
        out[name] = round(timed_steps(fn, steps, warm, 1) * 1000.0 / steps, 3)
    flops = 2.0 * B * H * V
    out.update({
        "B": B, "H": H, "V": V, "top_k": k, "top_p": p, "chunk": lm.chunk, "parts": lm.parts,
        "gemm_tflops": round(flops / (out["gemm_only_us"] * 1e-6) / 1e12, 1),
        "sampling_overhead_unfused_us": round(out["unfused_us"] - out["gemm_only_us"], 3),
        "sampling_overhead_pipelined_us": round(out["pipelined_us"] - out["gemm_only_us"], 3),
        "launches": steps * (2 + 1 + 3 * lm.parts + 1),
        "what": "bf16 GEMM (cuBLAS via torch.matmul) into L2-sized chunks, shard top-k per chunk, "
                "one candidate merge + draw; [B, V] logits never written to HBM",
    })
    del w, h, logits, lm
    torch.cuda.empty_cache()
    return out


def run_tp(ops, world, rank, device, args):
    """C4: vocab-sharded TP through llm_sampling_kernel_b200.sharded.VocabShardedSampler: local
    shard top-k -> exchange of packed candidates -> merge + sample on every rank. Two exchanges:
    the p2p kernel (pushes into every rank's buffers over NVLink, flags, bounded wait, merge in
    the same kernel) and an NCCL all-gather followed by the merge kernel."""
    import torch.distributed as dist

    from llm_sampling_kernel_b200.sharded import VocabShardedSampler

    B, V, k, p = C4["B"], C4["V"], C4["k"], C4["p"]
    out = {"B": B, "V": V, "top_k": k, "top_p": p, "exchange_bytes_per_rank": B * (k + 1) * 8}
    launches = 0
    results = {}
    for backend in ("p2p", "nccl"):
        sampler = VocabShardedSampler(vocab=V, top_k=k, ops=ops, backend=backend, max_batch=B)
        lo, hi = sampler.cols
        full = tp_logits(B, V, device)
        shard = full[:, lo:hi].contiguous()
        del full
        if backend == "p2p":
            try:  # set-up is collective and fails on every rank together
                sampler.sample(shard, p, seed=0x5EED, offset=0)
            except RuntimeError as e:
                out["p2p_error"] = str(e)[:200]
                continue

        def step(i):
            sampler.sample(shard, p, seed=0x5EED, offset=i)

        steps = max(3, min(args.steps, 200))
        ms = timed_steps(step, steps, max(3, args.warmup), world)
        us = max_over_ranks(ms * 1000.0 / steps, world)
        launches += 2 * steps
        if backend == "p2p":
            # the same step replayed from a CUDA graph (the exchange epoch lives on the device):
            # 32 steps per graph, no host work between them
            per_graph = 32
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(side):
                with torch.cuda.graph(g, stream=side):
                    for j in range(per_graph):
                        sampler.sample(shard, p, seed=0x5EED, offset=j)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            replays = max(3, min(args.steps, 200) // per_graph)
            msg = timed_steps(lambda i: g.replay(), replays, 3, world)
            out["graph_us_per_call"] = round(max_over_ranks(msg * 1000.0 / (replays * per_graph), world), 3)
            launches += 2 * per_graph * replays
            del g
        ids, status = sampler.sample(shard, p, seed=0x5EED, offset=0)
        all_ids = [torch.empty_like(ids) for _ in range(world)]
        dist.all_gather(all_ids, ids)
        results[backend] = (us, all(torch.equal(all_ids[0], t) for t in all_ids) and bool((status == 0).all()), ids)
        sampler.close()
        out["shard_vocab"] = hi - lo
    if "p2p" in results:
        out["us_per_call"] = round(results["p2p"][0], 3)
        out["backend"] = "p2p: shard top-k kernel + exchange-merge kernel over NVLink peer memory"
        out["backends_agree"] = bool(torch.equal(results["p2p"][2], results["nccl"][2]))
    else:
        out["us_per_call"] = round(results["nccl"][0], 3)
        out["backend"] = "nccl all_gather_into_tensor + merge kernel"
    out["nccl_us_per_call"] = round(results["nccl"][0], 3)
    out["ranks_agree"] = all(r[1] for r in results.values())
    out["launches"] = launches
    # per rank: its logit columns read once + the candidate blocks it sends and receives
    lo_hi = VocabShardedSampler(vocab=V, top_k=k, ops=ops).cols
    alg = B * (lo_hi[1] - lo_hi[0]) * 2 + B * (k + 1) * 8 * world * 2
    best = out.get("graph_us_per_call", out["us_per_call"])
    peak, _ = measured_peaks()
    out["roofline"] = {"algorithmic_bytes_per_rank": alg, "us": best,
                       "achieved_gbs": round(alg / (best * 1e-6) / 1e9, 1),
                       "frac_of_hbm": round(alg / (best * 1e-6) / 1e9 / peak, 4)}
    return out


# ---------------------------------------------------------------------------------------------
# reference arm
# ---------------------------------------------------------------------------------------------


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return
    cpu_us, threads, n, kind, what = cpu_reference_time(C1["B"], C1["V"], C1["k"], C1["p"],
                                                        budget_s=max(5.0, min(60.0, args.cpu_budget)))
    line = {
        "metric": METRIC,
        "value": round(cpu_us, 1),
        "unit": "µs/call",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(cpu_us / 1000.0, 4),
        "higher_is_better": False,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (torch CPU)",
        "data": "synthetic (seeded)",
        "impl": "reference",
        "config": {"workload": "C1 anchor: B=1 per GPU, V=151936, k=50, p=0.9, BF16 N(0,2^2) + 20 ids boosted by 8",
                   "B_per_gpu": C1["B"], "V": C1["V"], "top_k": C1["k"], "top_p": C1["p"],
                   "parallelism": f"dp{world} (rank 0 alone runs the host-CPU reference)"},
        "cpu_baseline": {"value": round(cpu_us, 1), "unit": "µs/call", "cores": threads, "kind": kind,
                         "sample": f"C1 row (B=1, V=151936, k=50, p=0.9) x {n} calls of {what}, "
                                   f"{threads} host threads"},
        "e2e": {"value": round(cpu_us, 1), "unit": "µs/call", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------------
# comparison rungs (B200): the reference's own CUDA kernel and FlashInfer's sampler
# ---------------------------------------------------------------------------------------------


def reference_kernel_module():
    """The reference's CUDA extension compiled unchanged for sm_100a into oracle/_ref by
    oracle/build_ref_kernel.py (None when it was not built)."""
    import glob
    import importlib.util

    found = sorted(glob.glob(str(ROOT / "oracle" / "_ref" / "fused_sampling_ref*.so")))
    if not found:
        return None
    spec = importlib.util.spec_from_file_location("fused_sampling_ref", found[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def flashinfer_sampling():
    """FlashInfer's sampling module, loaded from the JIT build kept in oracle/_ref/flashinfer
    (FLASHINFER_WORKSPACE_BASE), or None."""
    base = ROOT / "oracle" / "_ref" / "flashinfer"
    if not base.exists():
        return None
    os.environ.setdefault("FLASHINFER_WORKSPACE_BASE", str(base))
    os.environ.setdefault("FLASHINFER_CUDA_ARCH_LIST", "10.0")
    try:
        import flashinfer.sampling as fis

        fis.get_sampling_module()
        return fis
    except Exception as e:  # noqa: BLE001
        log(f"flashinfer unavailable: {e}")
        return None


def rungs(args, device):
    """µs per call of the comparison rungs at C1 (cold L2, rotating buffers) and C3 (B=1024):
    this repository's operator, the reference's own kernel (k <= 128; its semantics), and
    FlashInfer's top_k_top_p_sampling_from_probs on a precomputed full-vocabulary softmax
    ("from_probs", the reference's bar) and with that softmax inside the timed region. FlashInfer
    samples by rejection on the full-vocabulary distribution: a different rule from the
    reference's (exactly-k top-k, renormalised softmax, exclusive-prefix cut, inverse CDF), timed
    here as a rung, not compared for ids."""
    import llm_sampling_kernel_b200 as pkg

    ops = pkg.ops()
    out = {}
    steps = max(20, min(args.steps, 2000))
    warm = max(3, args.warmup)
    per = C1["V"] * 2
    nbuf = max(2, (2 * L2_BYTES) // per + 1)
    bufs = anchor_buffers(nbuf, 1, C1["V"], device, seed=4321)
    big = zipf_buffers(2, C3["B"], C3["V"], device, seed=9)

    def c1(fn):
        return timed_steps(lambda i: fn(bufs[i % nbuf]), steps, warm, 1) * 1000.0 / steps

    def c3(fn):
        n = max(3, min(steps, 50))
        return timed_steps(lambda i: fn(big[i % 2]), n, warm, 1) * 1000.0 / n

    out["ours"] = {"c1_us": round(c1(lambda x: ops.sample_fused(x, 50, 0.9, 0x5EED, 1, 0)), 3),
                   "c3_us": round(c3(lambda x: ops.sample_fused(x, 50, 0.95, 0x5EED, 1, 0)), 3)}
    ref = None
    try:
        ref = reference_kernel_module()
    except Exception as e:  # noqa: BLE001
        out["reference_kernel"] = {"unavailable": str(e)[:200]}
    if ref is not None:
        sys.path.insert(0, str(ROOT))
        from oracle import sampler_oracle as orc

        x = bufs[0]
        want = orc.topk_order(orc.bits16(x.cpu()), 50)
        same = bool(np.array_equal(ref.topk_fused(x, 50, 0).cpu().numpy(), want))
        out["reference_kernel"] = {
            "c1_us": round(c1(lambda x: ref.sample_fused(x, 50, 0.9, 0x5EED, 1, 0)), 3),
            "c3_us": round(c3(lambda x: ref.sample_fused(x, 50, 0.95, 0x5EED, 1, 0)), 3),
            "topk_matches_oracle_c1": same,
            "what": "the reference's csrc/ (topk_partial_kernel + merge_sample_kernel) compiled unchanged "
                    "for sm_100a by oracle/build_ref_kernel.py",
        }
    elif "reference_kernel" not in out:
        out["reference_kernel"] = {"unavailable": "oracle/_ref/fused_sampling_ref*.so not built"}
    fis = flashinfer_sampling()
    if fis is None:
        out["flashinfer"] = {"unavailable": "no FlashInfer sampling build in oracle/_ref/flashinfer"}
    else:
        probs1 = [torch.softmax(b.float(), dim=-1) for b in bufs[:64]]
        probs3 = [torch.softmax(b.float(), dim=-1) for b in big]

        def fp1(i):
            fis.top_k_top_p_sampling_from_probs(probs1[i % len(probs1)], 50, 0.9)

        def fp3(i):
            fis.top_k_top_p_sampling_from_probs(probs3[i % 2], 50, 0.95)

        n3 = max(3, min(steps, 50))
        out["flashinfer"] = {
            "from_probs_c1_us": round(timed_steps(fp1, steps, warm, 1) * 1000.0 / steps, 3),
            "from_probs_c3_us": round(timed_steps(fp3, n3, warm, 1) * 1000.0 / n3, 3),
            "from_logits_c1_us": round(c1(lambda x: fis.top_k_top_p_sampling_from_probs(
                torch.softmax(x.float(), dim=-1), 50, 0.9)), 3),
            "from_logits_c3_us": round(c3(lambda x: fis.top_k_top_p_sampling_from_probs(
                torch.softmax(x.float(), dim=-1), 50, 0.95)), 3),
            "version": getattr(sys.modules.get("flashinfer"), "__version__", "?"),
            "semantics": "rejection sampling over the full-vocabulary distribution (top_k_first); "
                         "from_probs: softmax precomputed outside the timed region (48 MB of fp32 probs "
                         "per C1 buffer set: L2-warm)",
        }
    del bufs, big
    torch.cuda.empty_cache()
    return out


def run_rungs(args):
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    line = {"rungs": rungs(args, device), "steps": args.steps, "warmup": args.warmup,
            "unit": "µs/call", "config": {"c1": "B=1, V=151936, k=50, p=0.9, BF16 (cold L2)",
                                          "c3": "B=1024, V=151936, k=50, p=0.95, BF16 Zipf rows"}}
    print(json.dumps(line), flush=True)


def run_sweep(args):
    """CTAs per row (S) against batch, vocabulary and k, on both the cluster and the streaming
    path: CUDA-event µs per call over rotating input buffers (> 2x L2), one JSON line. The plan's
    measured split table (make_plan) is read off these numbers."""
    import llm_sampling_kernel_b200 as pkg
    from llm_sampling_kernel_b200 import abi

    ops = pkg.ops()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    rows = []
    for V in (128256, 151936):
        for B in (1, 4, 16, 32, 64, 96, 128, 256):
            per = B * V * 2
            nbuf = max(2, (2 * L2_BYTES) // per + 1)
            g = torch.Generator(device=device).manual_seed(B + V)
            x = (torch.randn(nbuf * B, V, generator=g, device=device) * 2.0).to(torch.bfloat16)
            bufs = [x[i * B:(i + 1) * B] for i in range(nbuf)]
            for k in (1, 50, 256, 1024):
                for path in (abi.FS_PATH_CLUSTER, abi.FS_PATH_STREAM):
                    if path == abi.FS_PATH_STREAM and k > 256:
                        continue
                    for S in (4, 8, 16):
                        try:
                            pl = ops.plan(B, V, k, S)
                        except RuntimeError:
                            continue
                        if pl[0] != S:  # raised to hold the row in registers: not this split
                            continue
                        m_slots = max(64, 1 << max(0, (2 * k - 1).bit_length()))
                        if path == abi.FS_PATH_STREAM and S * m_slots > 4096:
                            continue  # the streaming plan would use fewer slices

                        def call(i, S=S, path=path, k=k):
                            ops.sample_ex(bufs[i % nbuf], k, 0.9, None, None, None, 0x5EED, i, S, 0, 0, False, path)

                        try:
                            n = 60
                            ms = timed_steps(call, n, 5, 1)
                        except RuntimeError as e:
                            rows.append({"V": V, "B": B, "k": k, "path": path, "S": S, "error": str(e)[:80]})
                            continue
                        rows.append({"V": V, "B": B, "k": k, "path": path, "S": S, "us": round(ms * 1000.0 / n, 3)})
            del x, bufs
            torch.cuda.empty_cache()
    print(json.dumps({"sweep": rows, "dtype": "bf16", "top_p": 0.9, "l2": "cold (rotating buffers > 2x L2)"}),
          flush=True)


def run_profile_case(args):
    """A few launches of one configuration, untimed: the target of the ncu captures in profiles/.
    c1 = the anchor (B=1), c3 = the B=1024 HBM-bound launch, c5w = the top-p-only wide path
    (B=8, k=V)."""
    sys.path.insert(0, str(ROOT))
    import llm_sampling_kernel_b200 as pkg

    ops = pkg.ops()
    device = torch.device("cuda", 0)
    if args.profile_case == "c1":
        x = anchor_buffers(1, C1["B"], C1["V"], device)[0]
        k, p = C1["k"], C1["p"]
    elif args.profile_case == "c5w":
        # the adversarial top-p-only case: B=8, V=151936 FP16 N(0, 0.1^2), k=V, p=0.5 (wide path)
        g = torch.Generator(device=device).manual_seed(2)
        x = (torch.randn(8, C1["V"], generator=g, device=device) * 0.1).to(torch.float16)
        k, p = C1["V"], 0.5
    else:
        x = zipf_buffers(1, C3["B"], C3["V"], device)[0]
        k, p = C3["k"], C3["p"]
    for i in range(3):
        ops.sample_fused(x, k, p, 0x5EED, i, 0)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": args.profile_case, "launches": 3}), flush=True)


def main():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU-baseline work")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--sweep", action="store_true",
                    help="time both paths over CTAs per row x batch x vocabulary x k and exit")
    ap.add_argument("--rungs", action="store_true",
                    help="time the comparison rungs (reference kernel, FlashInfer) and exit")
    ap.add_argument("--profile-case", choices=["c1", "c3", "c5w"], default=None,
                    help="run three untimed launches of one configuration (ncu target) and exit")
    args = ap.parse_args()
    if args.profile_case:
        run_profile_case(args)
        return
    if args.rungs:
        run_rungs(args)
        return
    if args.sweep:
        run_sweep(args)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)
    world, _, _ = dist_env()
    if world > 1 and args.impl == "ours":
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
