"""Benchmark: propose_with_update rows/s on benchmark config 2
(B=256, S=8192, k=16, P=32, R=128, 8 backoff candidates, factor 2.0,
min_token_prob 0.1) on 1..8 GPUs of one node.

One bench step is one propose_with_update over the B=256 rows of a decode
step. Steps run as CUDA-graph replays of the fused kernel; they rotate over
32 independent replicas of the [256, 8192] token buffer (256 MiB, above the
126 MB L2), each replica advancing through the config's 100-step decode
loop, so every step reads its rows from HBM. With N GPUs every rank drafts
its own 256 rows (weak scaling, no collective on the data path) and the
reported value is all rows of all ranks / max-over-ranks time.

``--impl reference`` times the reference algorithm's CPU path instead (the
numpy restatement in oracle/, parallel over rows on the host cores) on a
bounded sample of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

# Rank 0 prints exactly one JSON line on stdout; NCCL's version banner
# (NCCL_DEBUG=VERSION) would print another one there.
if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
    os.environ["NCCL_DEBUG"] = "WARN"

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

B, S, T, K = 256, 8192, 5, 16
DECODE_STEPS = 100
NREP = 32
METRIC = "propose_with_update rows/s (B=256,S=8192)"
CONFIG = {"workload": "config2: local-only propose_with_update, B=256, "
                      "S=8192, k=16, P=32, R=128, C=8, factor=2.0, "
                      "min_prob=0.1, 100-step decode loop",
          "global_batch": B, "seq_len": S,
          "l2": "inputs larger than L2: 32 rotating replicas x 8 MiB",
          "rows_per_gpu": "the same seeded 256 rows on every GPU"}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=12800)
    ap.add_argument("--warmup", type=int, default=320)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=400)
    ap.add_argument("--cpu-rows", type=int, default=256,
                    help="rows per step in the CPU sample")
    ap.add_argument("--cpu-steps", type=int, default=10,
                    help="timed decode steps of the CPU sample (about "
                         "10-30 s of CPU work over all workers)")
    ap.add_argument("--no-e2e", action="store_true",
                    help="skip the end-to-end API leg (profiling runs)")
    ap.add_argument("--no-cpu", action="store_true",
                    help="skip the CPU baseline leg (profiling runs)")
    ap.add_argument("--mode", default="draft",
                    choices=["draft", "sa", "global", "sharded", "vllm",
                             "rebuild"],
                    help="draft: config 2 (+ SA build, SA query and "
                         "global-path lines); sa: SA build + queries only "
                         "(config 4); global: config 3 only; sharded: "
                         "config 5 only (1..8 GPUs under torchrun); vllm: "
                         "config 2 through the vLLM adapter's call "
                         "sequence (1 GPU); rebuild: config-3 snapshot, "
                         "incremental vs full suffix-array build (1 GPU)")
    ap.add_argument("--vllm-steps", type=int, default=2000,
                    help="timed steps of --mode vllm")
    ap.add_argument("--sa-log2n", type=int, default=24,
                    help="SA build size (config 4: 2^24 tokens)")
    ap.add_argument("--sa-reps", type=int, default=5)
    ap.add_argument("--no-sa", action="store_true",
                    help="skip the SA build measurement in draft mode")
    ap.add_argument("--no-global", action="store_true",
                    help="skip the config 3 measurement in draft mode")
    ap.add_argument("--global-steps", type=int, default=60,
                    help="timed decode steps of config 3")
    ap.add_argument("--global-warmup", type=int, default=8)
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the config 5 measurement in draft mode")
    ap.add_argument("--sharded-log2-corpus", type=int, default=26,
                    help="config 5 corpus and index capacity 2^k tokens "
                         "(26 = the config; smaller for profiling captures)")
    ap.add_argument("--sharded-steps", type=int, default=512,
                    help="timed propose steps of config 5 per GPU")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def workload(rank: int):
    """Config 2's rows and decode steps. Every rank drafts the same seeded
    256 rows (weak scaling with identical per-GPU work: a step's time is
    its slowest row's, so rows drawn per rank would make the max over
    ranks measure sampling variance rather than the system)."""
    from suffixgpu_b200 import workloads as wl
    del rank
    return wl.config2(seed=2, steps=DECODE_STEPS)


def algorithmic_bytes(data, rep_shift) -> np.ndarray:
    """Per-decode-step algorithmic bytes for every replica: the committed
    row read once for drafting rows (4 * min(q, S)), the update (sampled
    ids, count in/out, appended ids) and the outputs (draft + num_valid).
    Returns [NREP, DECODE_STEPS]."""
    q0 = data["num_tokens"].astype(np.int64)
    samp = data["sampled"]
    out = np.zeros((NREP, DECODE_STEPS))
    for r in range(NREP):
        q = np.roll(q0, rep_shift * r)
        for j in range(DECODE_STEPS):
            sj = np.roll(samp[j], rep_shift * r, axis=0)
            cnt = (sj != -1).sum(axis=1)
            qn = q + cnt
            mask = (cnt > 0) & (qn < S)
            read = 4 * np.minimum(qn, S)[mask].sum()
            upd = (4 * T + 8 + 4 * cnt).sum()
            outb = B * (4 * K + 4)
            out[r, j] = read + upd + outb
            q = qn
    return out


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 f"--query-gpu={self.FIELDS}", "--format=csv,noheader",
                 "-lms", "50"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        time.sleep(0.15)

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["n/a"]}
        time.sleep(0.1)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        mhz, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                mhz.append(float(parts[0].split()[0]))
                mx = float(parts[1].split()[0])
            except ValueError:
                continue
            for nm, v in zip(names, parts[3:7]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(mhz) if mhz else None,
                "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz)}


# ---------------------------------------------------------------------------
# device-side timing
# ---------------------------------------------------------------------------
# Cycles of the spin kernel that keeps the stream busy while the host
# records the start event and issues the timed work (about 130 us at
# 1965 MHz, several times the host's launch latency).
SPIN_CYCLES = 1 << 18


def device_window(run, world: int) -> float:
    """Device time (ms) of the work ``run()`` enqueues on the current
    stream. A spin kernel is queued first, so the start event is recorded
    on a stream that is already busy and ``run()``'s first launch is queued
    before the spin ends: the host's event-record and launch latency stay
    outside the window. Barrier and synchronize on both sides."""
    import torch
    import torch.distributed as dist
    stream = torch.cuda.current_stream()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    torch.cuda._sleep(SPIN_CYCLES)
    e0.record(stream)
    run()
    e1.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    return e0.elapsed_time(e1)


def ranks_ms(ms: float, world: int, dev) -> list[float]:
    """Every rank's device time, gathered on all ranks (rank order)."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return [ms]
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist
    from suffixgpu_b200 import SuffixGPUDrafter
    from suffixgpu_b200 import workloads as wl

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev,
                                timeout=datetime.timedelta(seconds=120))

    data = workload(rank)
    shift = 7
    drafter = SuffixGPUDrafter(device=dev, **wl.CONFIG2_DRAFTER)
    tok0 = torch.from_numpy(data["token_ids"]).to(dev)
    q0 = torch.from_numpy(data["num_tokens"]).to(dev)
    samp0 = torch.from_numpy(data["sampled"]).to(dev)  # [100, B, T]
    reps = []
    for r in range(NREP):
        tok = torch.roll(tok0, shifts=shift * r, dims=0).contiguous()
        cnt0 = torch.roll(q0, shifts=shift * r, dims=0).contiguous()
        samp = torch.roll(samp0, shifts=shift * r, dims=1).contiguous()
        reps.append({"tok": tok, "cnt0": cnt0, "samp": samp})
    alg = algorithmic_bytes(data, shift)  # [NREP, 100]

    def step_seq(n):
        """(replica, decode step) of bench steps 0..n-1."""
        return [(i % NREP, (i // NREP) % DECODE_STEPS) for i in range(n)]

    cycle = NREP * DECODE_STEPS

    def run_seq(seq, marks=None, timed_from=0):
        """Each replica starts from its initial counts and chains the
        counts every call returns, so a sequence is self-contained (no
        copies between calls: one kernel launch per step). With marks =
        (start, end) events, start is recorded before step timed_from and
        end after the last step."""
        cur = [rp["cnt0"] for rp in reps]
        for i, (r, j) in enumerate(seq):
            if marks and i == timed_from:
                marks[0].record()
            rp = reps[r]
            if j == 0:
                cur[r] = rp["cnt0"]
            _, _, cur[r] = drafter.propose_with_update(
                cur[r], rp["tok"], rp["samp"][j])
        if marks:
            marks[1].record()

    def capture(seq, marks=None, timed_from=0):
        """A graph of the steps; with marks = (start, end) events, their
        records bracket steps timed_from.. of the graph."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run_seq(seq, marks, timed_from)
        return g

    def staggered(k):
        """Untimed lead-in, then k timed steps. The replicas are row
        permutations of one set of rows, so k steps of replicas all at the
        same decode step would each time the same slowest row; the lead-in
        advances replica r by r decode steps, so consecutive timed steps
        are at different points of the decode loop, as in a long run."""
        lead = [(r, j) for r in range(NREP) for j in range(r)]
        pos = list(range(NREP))
        timed = []
        for i in range(k):
            r = i % NREP
            timed.append((r, pos[r] % DECODE_STEPS))
            pos[r] += 1
        return lead, timed

    # warm-up: eager calls (exercise the API), then the graphs once
    run_seq(step_seq(max(args.warmup, 3)))
    torch.cuda.synchronize()
    # Up to one decode cycle the timed steps are one graph whose first and
    # last nodes record the timing events, so the window holds exactly the
    # K steps on the device (no graph launch latency); longer runs replay
    # cycle graphs inside a busy-stream window.
    marks = None
    timed_seq = step_seq(args.steps)
    if args.steps <= cycle:
        marks = tuple(torch.cuda.Event(enable_timing=True, external=True)
                      for _ in range(2))
        lead, timed_seq = staggered(args.steps)
        full, part = None, capture(lead + timed_seq, marks, len(lead))
    else:
        full = capture(step_seq(cycle))
        rem = args.steps % cycle
        part = capture(step_seq(rem)) if rem else None
    for g in (full, part):
        if g is not None:
            g.replay()
    torch.cuda.synchronize()

    # count our kernel launches per step (one fused launch per call)
    launches = args.steps  # one sg_local_draft per propose_with_update

    clock = ClockSampler(local)
    clock.start()

    def replays():
        if full is not None:
            for _ in range(args.steps // cycle):
                full.replay()
        if part is not None:
            part.replay()

    ms = device_window(replays, world)
    timing = "busy-stream window around the graph replays"
    if marks is not None:
        ms = marks[0].elapsed_time(marks[1])
        timing = ("events recorded by graph nodes around exactly the K "
                  "timed steps, after an untimed lead-in that staggers the "
                  "replicas' decode steps")
    clocks = clock.stop()
    ms_ranks = ranks_ms(ms, world, dev)
    ms_max = max(ms_ranks)

    # algorithmic bytes over the timed steps (the reset node is outside)
    alg_total = float(sum(alg[r, j] for (r, j) in timed_seq))
    per_launch_ms = ms / args.steps
    achieved = alg_total / args.steps / (per_launch_ms * 1e-3) / 1e9
    peaks = _peaks()
    rows_total = world * B * args.steps

    # end-to-end through the public API with host buffers
    e2e = None if args.no_e2e else run_e2e(args, drafter, reps, data, dev,
                                           world)

    res = None
    if rank == 0:
        res = {
            "metric": METRIC,
            "value": rows_total / (ms_max * 1e-3),
            "unit": "rows/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps,
            "ms_per_step_ranks": [m / args.steps for m in ms_ranks],
            "ms_per_step_median": statistics.median(ms_ranks) / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int32",
            "data": "synthetic (seeded copy/Zipf rows, benchmark config 2)",
            "config": dict(CONFIG, parallelism=f"dp{world}",
                           timing=timing),
            "impl": "ours",
            "gpu_launches": launches,
            "e2e": e2e,
            "roofline": {
                "bound": "hbm",
                "kernel": "local_draft_kernel",
                "achieved": achieved,
                "peak": peaks["hbm_gbs"],
                "peak_source": peaks["source"],
                "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"],
                "traffic": _traffic(),
                "alg_bytes_per_launch": alg_total / args.steps,
                "launch_us": per_launch_ms * 1e3,
            },
            "clocks": clocks,
        }
        res["cpu_baseline"] = None if (args.no_cpu or world > 1) \
            else cpu_baseline(args, data)
        if not args.no_sa:
            res["sa_build"] = run_sa(args, dev)
        if not args.no_global:
            res["global"] = run_global(args, dev)
    if not args.no_sharded:
        sh = run_sharded(args, dev, world, rank)  # every rank takes part
        if rank == 0:
            res["sharded"] = sh
    if world > 1:
        dist.barrier()
        del full, part
        dist.destroy_process_group()
    return res


def sa_alg_bytes(n: int, rounds: int) -> float:
    """Algorithmic bytes of one SA build: read the tokens and write the SA
    (8n) plus, per doubling round, gathering two ranks, writing a rank and
    LSD 8-bit passes over (key, u32 index) records with a 2*ceil(log2(n+1))
    bit key: h * n * (12 + 24 * ceil(2 * ceil(log2(n + 1)) / 8))."""
    import math
    kb = 2 * math.ceil(math.log2(n + 1))
    return 8 * n + rounds * n * (12 + 24 * math.ceil(kb / 8))


def run_rebuild(args, dev) -> dict:
    """The config-3 rebuild: the active corpus is 4 M tokens of template
    documents (each with its SEP) + PAD, the next snapshot evicts the
    oldest 32 documents and appends 32 finished 4096-token rows. Times the
    snapshot's suffix array built from scratch and merged from the
    previous one (sg_suffix_array_append), CUDA events around each call
    (both synchronise the stream once or twice per doubling round), and
    checks that the two arrays are identical."""
    import torch
    from suffixgpu_b200 import ops
    from suffixgpu_b200 import workloads as wl
    data = wl.config3(seed=3, steps=1)
    docs = data["corpus_docs"]
    sep = np.array([-2], dtype=np.int32)
    pad = np.array([2 ** 31 - 1], dtype=np.int32)
    n_docs = docs.shape[0]
    old = np.concatenate([np.concatenate([d, sep]) for d in docs]
                         + [pad]).astype(np.int32)
    evict = 32 * (docs.shape[1] + 1)
    rows = data["token_ids"][:32]
    new_part = np.concatenate([np.concatenate([r, sep]) for r in rows])
    kept = len(old) - 1 - evict
    snap = np.concatenate([old[evict:-1], new_part, pad]).astype(np.int32)
    t_old = torch.from_numpy(old).to(dev)
    t_new = torch.from_numpy(snap).to(dev)
    sa_old = torch.empty(len(old), dtype=torch.int32, device=dev)
    r_old = ops.build_suffix_array_into(t_old, sa_old)
    full = torch.empty(len(snap), dtype=torch.int32, device=dev)
    inc = torch.empty(len(snap), dtype=torch.int32, device=dev)

    def timed(fn):
        fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(max(3, args.sa_reps)):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ts.append(e0.elapsed_time(e1))
        return float(statistics.median(ts))
    ms_full = timed(lambda: ops.build_suffix_array_into(t_new, full))
    ms_inc = timed(lambda: ops.append_suffix_array_into(
        t_new, inc, sa_old, len(old), evict, kept, r_old))
    r_new = ops.append_suffix_array_into(t_new, inc, sa_old, len(old),
                                         evict, kept, r_old)
    if not torch.equal(full, inc):
        raise RuntimeError("incremental suffix array differs from the full "
                           "build")
    n = len(snap)
    return {"metric": "config-3 rebuild, suffix array of the next snapshot",
            "value": n / (ms_inc * 1e-3) / 1e6, "unit": "Mtok/s",
            "n_tokens": n, "ms_incremental": ms_inc, "ms_full": ms_full,
            "speedup": ms_full / ms_inc, "previous_rounds": r_old,
            "new_rounds": r_new, "tail_tokens": n - (kept - (1 << r_old)),
            "identical": True,
            "workload": f"config3 corpus ({n_docs} x {docs.shape[1]} "
                        "template documents + SEP + PAD), evict 32 "
                        "documents, append 32 rows of 4096 tokens"}


def run_sa(args, dev) -> dict:
    """benchmark config 4: suffix array of 2^24 tokens (50% i.i.d. Zipf,
    50% copies of earlier spans). Times whole builds with CUDA events; the
    build synchronises once per doubling round, so the time includes those
    host round trips."""
    import torch
    from suffixgpu_b200 import ops
    from suffixgpu_b200 import workloads as wl
    n = 1 << args.sa_log2n
    tok = torch.from_numpy(wl.config4(n=n, n_queries=1)["tokens"]).to(dev)
    out = torch.empty(n, dtype=torch.int32, device=dev)
    rounds = ops.build_suffix_array_into(tok, out)  # warm-up (+ workspace)
    ops.build_suffix_array_into(tok, out)
    torch.cuda.synchronize()
    times = []
    for _ in range(max(1, args.sa_reps)):
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        rounds = ops.build_suffix_array_into(tok, out)
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = float(statistics.median(times))
    alg = sa_alg_bytes(n, rounds)
    peaks = _peaks()
    achieved = alg / (ms * 1e-3) / 1e9
    queries = run_queries(args, tok, out, dev, peaks)
    dram = _sa_traffic()
    measured = None
    if dram is not None:
        # measured DRAM bytes of a 2^22 build, scaled by tokens x rounds
        scaled = dram["bytes"] * (n / (1 << 22)) * (rounds / dram["rounds"])
        gbs = scaled / (ms * 1e-3) / 1e9
        measured = {"traffic_bytes_per_build": scaled,
                    "achieved": gbs, "frac": gbs / peaks["hbm_gbs"],
                    "unit": "GB/s",
                    "source": "ncu dram__bytes_read.sum + dram__bytes_write.sum "
                              "of every launch of a 2^22 build "
                              "(profiles/sa_build_config4.txt), scaled to "
                              "this build by tokens x doubling rounds"}
    return {"metric": "SA build Mtok/s", "value": n / (ms * 1e-3) / 1e6,
            "unit": "Mtok/s", "n_tokens": n, "ms_per_build": ms,
            "doubling_rounds": rounds, "reps": len(times),
            "workload": "config4: 2^24 tokens, 50% Zipf(1.1) / 50% copies "
                        "U[32,1024], vocab 128256",
            "roofline": {"bound": "hbm", "achieved": achieved,
                         "peak": peaks["hbm_gbs"],
                         "peak_source": peaks["source"], "unit": "GB/s",
                         "frac": achieved / peaks["hbm_gbs"],
                         "alg_bytes_per_build": alg,
                         "measured_dram": measured},
            "sa_search": queries}


def run_queries(args, tok, sa, dev, peaks) -> dict:
    """benchmark config 4 queries: 1000 corpus substrings per capped length
    (32, 16, 8, 4, 2) against the built SA, all 5000 in one search_interval
    launch (rows padded to width 32, pattern length per row). Every pattern
    occurs in the corpus, so every interval must be non-empty: a
    size-independent check of the full-size search. Algorithmic bytes per
    query: 2 * ITERS * (4 + 4 * len) (an SA entry and the compared tokens
    per probe of both bounds)."""
    import math
    import torch
    from suffixgpu_b200 import ops
    n = tok.numel()
    rng = np.random.default_rng(44)
    caps = (32, 16, 8, 4, 2)
    nq = 1000
    host = tok.cpu().numpy()
    pats = np.zeros((nq * len(caps), 32), dtype=np.int32)
    plen = np.zeros(nq * len(caps), dtype=np.int64)
    for i, c in enumerate(caps):
        st = rng.integers(0, n - c, size=nq)
        pats[i * nq:(i + 1) * nq, :c] = host[st[:, None] + np.arange(c)]
        plen[i * nq:(i + 1) * nq] = c
    pat = torch.from_numpy(pats).to(dev)
    pl = torch.from_numpy(plen).to(dev)
    for _ in range(3):
        start, end = ops.search_interval(sa, tok, pat, pl)
    torch.cuda.synchronize()
    reps = 20
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        start, end = ops.search_interval(sa, tok, pat, pl)
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    found = int((end > start).sum().item())
    iters = math.ceil(math.log2(n + 1))
    alg = float(sum(2 * iters * (4 + 4 * c) * nq for c in caps))
    achieved = alg / (ms * 1e-3) / 1e9
    return {"metric": "sa_search queries/s", "value": len(plen) / (ms * 1e-3),
            "unit": "queries/s", "queries_per_launch": len(plen),
            "us_per_launch": ms * 1e3, "all_found": found == len(plen),
            "roofline": {"bound": "hbm (latency-bound probes)",
                         "achieved": achieved, "peak": peaks["hbm_gbs"],
                         "unit": "GB/s", "frac": achieved / peaks["hbm_gbs"],
                         "alg_bytes_per_launch": alg}}


NREP5, DECODE5 = 16, 32


def run_sharded(args, dev, world: int, rank: int) -> dict | None:
    """benchmark config 5: the global drafter on every GPU of the job, 128
    query rows (S=16384) per GPU, k=32, P=64, R=256, 8 backoff levels,
    factor 2.0, min_prob 0.1, over a 2^26-token template corpus (512
    templates x 512, vocab 128256) that every rank bulk-loads from the same
    seed. Two multi-GPU modes, both bit-exact to one index:
    ``shards`` (config 5 as specified: each rank queries its 2^26 / N
    positions' part of the suffix array, three collectives per step) and
    ``replicated`` (the whole suffix array on every rank, no collective).
    One step = one propose_with_update of the rank's rows over 16 rotating
    replicas of the token buffer (128 MiB > L2), each walking a 32-step
    decode loop; steps are replayed from a CUDA graph when capture works
    (eager otherwise). Value: all ranks' rows / max-over-ranks device time
    (weak scaling). The shards mode also reports per-phase device times of
    a few eager steps (rank 0 and the max over ranks)."""
    import torch
    from suffixgpu_b200 import workloads as wl
    lg = min(26, max(16, args.sharded_log2_corpus))
    # every rank drafts the same seeded 128 rows (identical per-GPU work)
    data = wl.config5(rank=0, steps=DECODE5, n_docs=1 << (lg - 10))
    docs = torch.from_numpy(data["corpus_docs"]).to(dev)
    res = {}
    for mode in ("shards", "replicated"):
        res[mode] = _run_config5_mode(args, dev, world, rank, mode, data,
                                      docs, lg)
        torch.cuda.empty_cache()
    if rank != 0:
        return None
    out = res["shards"]
    out["replicated"] = res["replicated"]
    return out


def _phase_times(d, run_seq, world, dev) -> dict:
    """Per-phase device times of the sharded step: 8 steps captured in a
    CUDA graph with an event-record node between phases (eager steps when
    capture is refused), averaged per phase, rank 0 and max over ranks.
    Phases are timed per stream: "chain" is the shard chain on the side
    stream (collectives included), "own" the rank's rows on the caller's
    stream (delta scan and local step overlap the chain)."""
    import torch
    d.phase_events = []
    how = "CUDA graph with event-record nodes"
    try:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            run_seq(8)
        evs = d.phase_events
        d.phase_events = None
        g.replay()
        torch.cuda.synchronize()
    except Exception as e:  # capture refused: eager steps
        d.phase_events = []
        run_seq(8)
        torch.cuda.synchronize()
        evs = d.phase_events
        how = f"eager steps ({type(e).__name__} in capture)"
        g = None
    d.phase_events = None
    acc: dict = {}
    last: dict = {}
    for lane, name, ev in evs:
        if name != "start" and lane in last:
            acc.setdefault(f"{lane}:{name}", []).append(
                last[lane].elapsed_time(ev))
        last[lane] = ev
    names = list(acc)
    mine = [1e3 * sum(acc[k]) / len(acc[k]) for k in names]
    allr = [max(ranks_ms(v, world, dev)) for v in mine]
    del g
    return {"order": names, "us_rank0": mine, "us_max_over_ranks": allr,
            "how": how}


def _length_search_probe(d, run_seq, steps, world, dev) -> dict:
    """Eager device time per step of the shards mode with each length
    search (every length in one round / longest match first)."""
    import torch
    out = {}
    keep = d.length_search
    for ls in ("all", "longest"):
        d.length_search = ls
        run_seq(min(steps, 16))
        torch.cuda.synchronize()
        ms = device_window(lambda: run_seq(steps), world)
        out[ls] = max(ranks_ms(ms, world, dev)) / steps * 1e3
    d.length_search = keep
    return {"us_per_step_eager": out,
            "used": "longest" if d._longest_first() else "all"}


def _run_config5_mode(args, dev, world, rank, mode, data, docs, lg):
    import torch
    from suffixgpu_b200 import SuffixGPUDrafter
    from suffixgpu_b200 import workloads as wl
    from suffixgpu_b200.distributed import (ReplicatedSuffixDrafter,
                                            ShardedSuffixDrafter)
    cfg = dict(wl.CONFIG5_DRAFTER)
    cfg["global_capacity"] = 1 << lg
    if mode == "shards":
        d = ShardedSuffixDrafter(device=dev, **cfg)
    elif world > 1:
        d = ReplicatedSuffixDrafter(device=dev, **cfg)
    else:
        d = SuffixGPUDrafter(device=dev, **cfg)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    d.load_documents(list(docs.unbind(0)))
    torch.cuda.synchronize()
    load_s = time.perf_counter() - t0
    b = data["token_ids"].shape[0]
    tok0 = torch.from_numpy(data["token_ids"]).to(dev)
    q0 = torch.from_numpy(data["num_tokens"]).to(dev)
    samp0 = torch.from_numpy(data["sampled"]).to(dev)
    reps = []
    for r in range(NREP5):
        reps.append({"tok": torch.roll(tok0, 5 * r, 0).contiguous(),
                     "cnt0": torch.roll(q0, 5 * r, 0).contiguous(),
                     "samp": torch.roll(samp0, 5 * r, 1).contiguous()})
    cycle = NREP5 * DECODE5

    def run_seq(n, marks=None):
        cur = [rp["cnt0"] for rp in reps]
        if marks:
            marks[0].record()
        for i in range(n):
            r, j = i % NREP5, (i // NREP5) % DECODE5
            if j == 0:
                cur[r] = reps[r]["cnt0"]
            _, _, cur[r] = d.propose_with_update(cur[r], reps[r]["tok"],
                                                 reps[r]["samp"][j])
        if marks:
            marks[1].record()

    run_seq(3 * NREP5)
    torch.cuda.synchronize()
    steps = max(1, min(args.sharded_steps, cycle))
    phases = None
    if mode == "shards":
        phases = _phase_times(d, run_seq, world, dev)
    probe = None
    if mode == "shards":
        probe = _length_search_probe(d, run_seq, 64, world, dev)
    marks = tuple(torch.cuda.Event(enable_timing=True, external=True)
                  for _ in range(2))
    graph = None
    timing = "events recorded by the timed graph's first and last nodes"
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            run_seq(steps, marks)
        graph.replay()
        torch.cuda.synchronize()
    except Exception as e:  # capture of the collectives refused: eager
        graph = None
        timing = f"eager steps in a busy-stream window ({type(e).__name__})"
        torch.cuda.synchronize()
    if graph is not None:
        ms = device_window(graph.replay, world)
        ms = marks[0].elapsed_time(marks[1])
    else:
        ms = device_window(lambda: run_seq(steps), world)
    ms_ranks = ranks_ms(ms, world, dev)
    ms_max = max(ms_ranks)
    load_max = max(ranks_ms(load_s, world, dev))
    del graph
    out = {"metric": "propose_with_update rows/s, global drafter "
                     f"(config 5, {mode} suffix array)",
           "value": world * b * steps / (ms_max * 1e-3), "unit": "rows/s",
           "n_gpus": world, "rows_per_gpu": b, "steps": steps,
           "ms_per_step": ms_max / steps, "scaling": "weak",
           "ms_per_step_ranks": [m / steps for m in ms_ranks],
           "timing": timing,
           "corpus_tokens": int(d.global_index.active_len),
           "load_s": load_max,
           "workload": "config5: 128 rows x S=16384 per GPU, k=32, P=64, "
                       "R=256, 8 backoff, factor 2.0, min_prob 0.1; "
                       f"2^{lg}-token corpus of 512 x 512 templates (5% "
                       "substitution, vocab 128256); "
                       + ("suffix array split into one shard per GPU by "
                          "corpus position (global ranks), tails "
                          "all-gathered, bounds all-reduced, samples "
                          "reduce-scattered" if mode == "shards" else
                          "whole suffix array on every GPU"),
           "l2": "16 rotating replicas x 8 MiB token buffer"}
    if phases is not None:
        out["phases"] = phases
    if probe is not None:
        out["length_search"] = probe
    del d
    return out


def _global_graph_loop(args, setup, data, samp, q_host, dev) -> dict:
    """The config-3 loop again on a fresh drafter, with propose_with_update
    captured once into a CUDA graph (static count and sampled-id buffers,
    the new counts written back into the count buffer) and replayed every
    step between the harvests and the poll: the host then issues one graph
    launch and one small copy per propose. Step 0 runs eagerly on the
    capture stream (it creates the side streams and buffers); the timed
    steps are the same as the eager loop's."""
    import torch
    d, gi, _ = setup()
    tok = torch.from_numpy(data["token_ids"]).to(dev)
    n = torch.from_numpy(data["num_tokens"]).to(dev)
    b = tok.shape[0]
    steps = args.global_warmup + args.global_steps
    warm = max(1, args.global_warmup)
    cap = torch.cuda.Stream(dev)

    def harvest(j):
        rows = [(4 * j + i) % b for i in range(4)]
        d.harvest_finished(rows, [q_host[r] for r in rows], tok)
        d.poll()

    harvest(0)
    cap.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(cap):
        _, _, n = d.propose_with_update(n, tok, samp[0])
    torch.cuda.synchronize()
    n_s = n.clone()
    samp_s = samp[0].clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap):
        _, _, g_n = d.propose_with_update(n_s, tok, samp_s)
        n_s.copy_(g_n)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    r0 = gi.rebuilds
    t1 = time.perf_counter()
    for j in range(1, steps):
        if j == warm:
            torch.cuda.synchronize()
            r0 = gi.rebuilds
            t1 = time.perf_counter()
            e0.record()
        harvest(j)
        samp_s.copy_(samp[j])
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t1
    timed = steps - warm
    ms = e0.elapsed_time(e1) / timed
    rebuilds = gi.rebuilds - r0
    gi.wait_rebuild()
    del graph
    return {"value": b / (ms * 1e-3), "unit": "rows/s", "ms_per_step": ms,
            "wall_ms_per_step": wall * 1e3 / timed, "steps": timed,
            "rebuilds_in_timed_steps": rebuilds,
            "mode": "same loop, propose_with_update replayed from one CUDA "
                    "graph (harvests, polls and background rebuilds "
                    "eager)"}


def run_global(args, dev) -> dict:
    """benchmark config 3: global memory enabled (capacity 2^22, delta
    2^16, rebuild threshold 32768), corpus of 4096 template documents x
    1024 tokens pre-filled through harvest_rows, then B=64 x S=4096 query
    rows decoded step by step. Every step harvests 4 finished rows of the
    batch into the delta, polls, and runs propose_with_update; rebuilds run
    on the side stream from the host worker thread and swap in at a poll.
    The loop is timed with CUDA events (the host's Python bookkeeping is
    inside). The propose step alone is also replayed from a CUDA graph."""
    import torch
    from suffixgpu_b200 import SuffixGPUDrafter
    from suffixgpu_b200 import workloads as wl
    steps = args.global_warmup + args.global_steps
    data = wl.config3(seed=3, steps=steps)
    b, s = data["token_ids"].shape
    docs = torch.from_numpy(data["corpus_docs"]).to(dev)

    def setup():
        """A config-3 drafter with the corpus pre-filled (harvests of 16
        documents; each rebuild waited for, so no document is dropped)."""
        d = SuffixGPUDrafter(k=16, device=dev, max_pattern_len=32,
                             max_occurrences=128, num_backoff=8,
                             enable_global=True, global_capacity=1 << 22,
                             delta_capacity=1 << 16, rebuild_threshold=32768,
                             rebuild_stream=torch.cuda.Stream(dev))
        gi = d.global_index
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        per = 16
        for i in range(0, docs.shape[0], per):
            d.harvest_rows([docs[j] for j in
                            range(i, min(i + per, docs.shape[0]))],
                           [docs.shape[1]] * min(per, docs.shape[0] - i))
            gi.wait_rebuild()
        gi.wait_rebuild()
        torch.cuda.synchronize()
        return d, gi, time.perf_counter() - t0

    d, gi, prefill_s = setup()
    prefill_rebuilds = gi.rebuilds
    prefill_builds = len(gi.build_log)
    tok = torch.from_numpy(data["token_ids"]).to(dev)
    n = torch.from_numpy(data["num_tokens"]).to(dev)
    q_host = data["num_tokens"].astype(int).tolist()
    samp = [torch.from_numpy(x).to(dev) for x in data["sampled"]]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    r0 = 0
    t1 = 0.0
    for j in range(steps):
        if j == args.global_warmup:
            torch.cuda.synchronize()
            r0 = gi.rebuilds
            t1 = time.perf_counter()
            e0.record()
        rows = [(4 * j + i) % b for i in range(4)]
        d.harvest_finished(rows, [q_host[r] for r in rows], tok)
        d.poll()
        draft, nv, n = d.propose_with_update(n, tok, samp[j])
    e1.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t1
    ms = e0.elapsed_time(e1) / args.global_steps
    rebuilds = gi.rebuilds - r0
    gi.wait_rebuild()
    log = list(gi.build_log)

    def build_stats(entries):
        out = {}
        for kind in ("append", "full"):
            ts = [t for k, t, _ in entries if k == kind]
            out[kind] = {"builds": len(ts),
                         "mean_ms": 1e3 * sum(ts) / len(ts) if ts else None}
        return out
    # one full build of the final snapshot, for comparison
    from suffixgpu_b200 import ops
    m_fin = min(gi.active_len + 1, gi.capacity)
    scratch = torch.empty(m_fin, dtype=torch.int32, device=dev)
    ops.build_suffix_array_into(gi.corpus[:m_fin], scratch)
    torch.cuda.synchronize()
    tf = time.perf_counter()
    ops.build_suffix_array_into(gi.corpus[:m_fin], scratch)
    torch.cuda.synchronize()
    full_same_ms = (time.perf_counter() - tf) * 1e3
    del scratch
    graph_loop = _global_graph_loop(args, setup, data, samp, q_host, dev)
    # the propose step alone, replayed from a CUDA graph (no harvest)
    n_g = torch.from_numpy(data["num_tokens"]).to(dev)
    tok_g = tok.clone()
    sg = torch.cuda.Stream(dev)
    sg.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(sg):
        for _ in range(3):
            d.propose(n_g, tok_g)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=sg):
        for _ in range(10):
            d.propose(n_g, tok_g)
    graph.replay()
    torch.cuda.synchronize()
    g0 = torch.cuda.Event(enable_timing=True)
    g1 = torch.cuda.Event(enable_timing=True)
    g0.record()
    for _ in range(10):
        graph.replay()
    g1.record()
    torch.cuda.synchronize()
    graph_us = g0.elapsed_time(g1) * 1e3 / 100
    del graph
    return {"metric": "propose_with_update rows/s, global enabled",
            "value": b / (ms * 1e-3), "unit": "rows/s",
            "ms_per_step": ms, "wall_ms_per_step":
                wall * 1e3 / args.global_steps,
            "steps": args.global_steps, "warmup": args.global_warmup,
            "rebuilds_in_timed_steps": rebuilds,
            "active_corpus_tokens": gi.active_len,
            "prefill_s": prefill_s, "prefill_rebuilds": prefill_rebuilds,
            "suffix_array_builds": {
                "prefill": build_stats(log[:prefill_builds]),
                "loop": build_stats(log[prefill_builds:]),
                "full_build_of_final_snapshot_ms": full_same_ms,
                "note": "append = incremental merge into the previous "
                        "suffix array (sg_suffix_array_append), full = "
                        "from-scratch build; host wall time of each build "
                        "on its stream (background thread in the loop)"},
            "graph_loop": graph_loop,
            "graph_propose_us": graph_us,
            "graph_propose_rows_per_s": b / (graph_us * 1e-6),
            "workload": "config3: 4096 x 1024 template corpus (64 templates "
                        "x 256, 5% substitution, vocab 32000), B=64, "
                        "S=4096, k=16, P=32, R=128, capacity 2^22, delta "
                        "2^16, threshold 32768, 4 harvests + poll per step"}


def run_vllm(args, dev) -> dict:
    """Config 2 through vLLM's ngram_gpu call sequence on the adapter
    (suffixgpu_b200.vllm_adapter.SuffixGPUProposer): per step vLLM's own
    update_token_ids_ngram (valid counts, next ids; torch ops) and the
    adapter's propose, eager, as the V1 model runner issues them, over the
    32 rotating replicas of the main bench. Beside it the same steps as one
    direct propose_with_update call each. Both loops are host-bound; the
    difference is the adapter's and vLLM's per-step overhead."""
    import torch
    from types import SimpleNamespace
    from suffixgpu_b200 import SuffixGPUDrafter
    from suffixgpu_b200 import workloads as wl
    from suffixgpu_b200.vllm_adapter import SuffixGPUProposer
    data = workload(0)
    cfg = wl.CONFIG2_DRAFTER
    spec = SimpleNamespace(
        num_speculative_tokens=cfg["k"],
        prompt_lookup_max=cfg["max_pattern_len"],
        prompt_lookup_min=cfg.get("min_match_len", 1),
        suffix_decoding_max_spec_factor=cfg.get("max_spec_factor"),
        suffix_decoding_min_token_prob=cfg.get("min_token_prob", 0.0),
        suffix_decoding_max_cached_requests=0)
    vcfg = SimpleNamespace(speculative_config=spec,
                           model_config=SimpleNamespace(max_model_len=S),
                           scheduler_config=SimpleNamespace(max_num_seqs=B))
    prop = SuffixGPUProposer(vcfg, dev,
                             max_occurrences=cfg["max_occurrences"],
                             num_backoff=cfg["num_backoff"])
    direct = SuffixGPUDrafter(device=dev, **cfg)
    shift = 7
    tok0 = torch.from_numpy(data["token_ids"]).to(dev)
    q0 = torch.from_numpy(data["num_tokens"]).to(dev)
    samp0 = torch.from_numpy(data["sampled"]).to(dev)
    reps = []
    for r in range(NREP):
        reps.append({"tok": torch.roll(tok0, shifts=shift * r,
                                       dims=0).contiguous(),
                     "cnt0": torch.roll(q0, shifts=shift * r,
                                        dims=0).contiguous(),
                     "samp": torch.roll(samp0, shifts=shift * r,
                                        dims=1).contiguous()})
    batch = SimpleNamespace(num_reqs=B, vocab_size=1 << 30)
    discard = torch.zeros(B, dtype=torch.bool, device=dev)
    n = args.vllm_steps

    from vllm.v1.spec_decode.ngram_proposer_gpu import NgramProposerGPU
    stock_update = NgramProposerGPU.update_token_ids_ngram

    def loop(via_vllm, steps: int) -> float:
        cur = [rp["cnt0"].clone() for rp in reps]
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        for i in range(steps):
            r, j = i % NREP, (i // NREP) % DECODE_STEPS
            rp = reps[r]
            if j == 0:
                cur[r] = rp["cnt0"].clone()
            # vLLM keeps every count below max_model_len (its
            # update_token_ids_ngram gathers token count - 1 from the row;
            # a count past the row is out of range there), so both loops
            # hold the config's overflowing rows at S - 1
            if via_vllm:
                update = (prop.update_token_ids_ngram if via_vllm != "stock"
                          else (lambda *a: stock_update(prop, *a)))
                _, counts, valid = update(rp["samp"][j], batch, rp["tok"],
                                          cur[r], discard)
                prop.propose(cur[r], rp["tok"], valid, counts)
                cur[r] = torch.clamp(cur[r] + counts, max=S - 1)
            else:
                _, _, nxt = direct.propose_with_update(
                    cur[r], rp["tok"], rp["samp"][j])
                cur[r] = torch.clamp(nxt, max=S - 1)
        e1.record()
        torch.cuda.synchronize()
        wall = time.perf_counter() - t0
        return e0.elapsed_time(e1) * 1e-3, wall

    for mode in (True, "stock", False):
        loop(mode, 3 * NREP)
    dev_v, wall_v = loop(True, n)
    dev_s, _ = loop("stock", n)
    dev_d, wall_d = loop(False, n)
    return {"metric": "propose rows/s through the vLLM ngram_gpu call "
                      "sequence (config 2)",
            "value": B * n / dev_v, "unit": "rows/s", "steps": n,
            "us_per_step": dev_v * 1e6 / n,
            "host_us_per_step": wall_v * 1e6 / n,
            "direct_propose_with_update": {
                "value": B * n / dev_d, "us_per_step": dev_d * 1e6 / n},
            "with_vllm_stock_update_token_ids_ngram": {
                "value": B * n / dev_s, "us_per_step": dev_s * 1e6 / n},
            "workload": "config2 rows (B=256, S=8192, k=16, P=32, R=128), "
                        "32 rotating replicas, eager, update_token_ids_ngram "
                        "+ SuffixGPUProposer.propose per step"}


def run_e2e(args, drafter, reps, data, dev, world):
    """Same metric through the public API with host buffers. Per step the
    step's sampled ids come from page-locked host memory and draft +
    num_valid go back to page-locked host memory, inside the timed region.

    Headline ("host buffers"): the host tensors go straight to
    propose_with_update (out=(draft, num_valid)); the kernel reads the ids
    and writes the results over the host link, one launch per step.
    Beside it ("copies"): an explicit H2D copy of the ids, the call on
    device tensors, and D2H copies of draft + num_valid."""
    import torch
    import torch.distributed as dist
    n = args.e2e_steps
    samp_host = [torch.from_numpy(np.roll(data["sampled"], 7 * r, axis=1))
                 .pin_memory() for r in range(NREP)]
    samp_dev = torch.empty(B, T, dtype=torch.int32, device=dev)
    out_draft = torch.empty(B, K, dtype=torch.int32).pin_memory()
    out_nv = torch.empty(B, dtype=torch.int32).pin_memory()
    seq = [(i % NREP, (i // NREP) % DECODE_STEPS) for i in range(n + 3)]

    def loop(one):
        cur = [rp["cnt0"] for rp in reps]

        def step(r, j):
            if j == 0:
                cur[r] = reps[r]["cnt0"]
            cur[r] = one(r, j, cur[r])

        for (r, j) in seq[:3]:  # warm-up
            step(r, j)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        for (r, j) in seq[3:]:
            step(r, j)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        tt = torch.tensor([dt], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        return world * B * n / float(tt.item())

    def host_buffers(r, j, cnt):
        _, _, cnt = drafter.propose_with_update(
            cnt, reps[r]["tok"], samp_host[r][j], out=(out_draft, out_nv))
        return cnt

    def copies(r, j, cnt):
        samp_dev.copy_(samp_host[r][j], non_blocking=True)
        d, nv, cnt = drafter.propose_with_update(cnt, reps[r]["tok"],
                                                 samp_dev)
        out_draft.copy_(d, non_blocking=True)
        out_nv.copy_(nv, non_blocking=True)
        return cnt

    v_host = loop(host_buffers)
    v_copy = loop(copies)
    return {"value": v_host, "unit": "rows/s",
            "h2d_bytes_per_step": B * T * 4,
            "d2h_bytes_per_step": B * K * 4 + B * 4,
            "steps": n,
            "mode": "eager public API with page-locked host buffers: "
                    "propose_with_update(num_tokens, token_ids, "
                    "sampled_host, out=(draft_host, num_valid_host)); the "
                    "kernel reads the sampled ids from and writes draft + "
                    "num_valid to host memory (one launch per step)",
            "copies": {"value": v_copy, "unit": "rows/s",
                       "mode": "eager public API on device tensors with "
                               "explicit copies: H2D sampled ids, D2H "
                               "draft + num_valid"}}


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return {"hbm_gbs": float(pk["hbm_gbs"]), "source": "measured"}
    except (OSError, KeyError, ValueError):
        return {"hbm_gbs": 6650.0, "source": "fallback"}


def _traffic():
    """DRAM bytes per launch of the kernel from the committed ncu summary
    (profiles/local_draft_config2.txt), or None."""
    path = os.path.join(ROOT, "profiles", "local_draft_config2.txt")
    try:
        for ln in open(path):
            if ln.startswith("traffic_bytes_per_launch:"):
                return float(ln.split(":")[1])
    except OSError:
        pass
    return None


# ---------------------------------------------------------------------------
# CPU baseline (oracle port of the reference's torch CPU path)
# ---------------------------------------------------------------------------
def _sa_traffic():
    """Measured DRAM bytes of one 2^22 suffix-array build and its rounds,
    from the committed ncu summary (profiles/sa_build_config4.txt)."""
    path = os.path.join(ROOT, "profiles", "sa_build_config4.txt")
    got = {}
    try:
        for ln in open(path):
            if ln.startswith("dram_bytes_per_build_2^22:"):
                got["bytes"] = float(ln.split(":")[1])
            elif ln.startswith("dram_rounds_2^22:"):
                got["rounds"] = float(ln.split(":")[1])
    except OSError:
        return None
    return got if len(got) == 2 else None


def _cpu_chunk(payload):
    rows, steps, warm, cfg = payload
    sys.path.insert(0, ROOT)
    from oracle import suffix_oracle as so
    tok, q, samp = rows
    d = so.SuffixDrafter(**cfg)
    for j in range(warm):  # untimed decode steps
        _, _, q = d.propose_with_update(q, tok, samp[j])
    t0 = time.perf_counter()
    for j in range(warm, warm + steps):
        _, _, q = d.propose_with_update(q, tok, samp[j])
    return time.perf_counter() - t0


def cpu_baseline(args, data, cores=None, warm: int = 1) -> dict:
    """Reference algorithm (numpy port) on a bounded sample: cpu_rows rows
    of config 2 for cpu_steps decode steps, rows split across one process
    per host core (rows are independent). Each worker times its own
    compute; the sample's time is the slowest worker's."""
    import multiprocessing as mp
    from concurrent.futures import ProcessPoolExecutor
    cores = cores or max(1, os.cpu_count() or 1)
    rows = min(args.cpu_rows, B)
    steps = args.cpu_steps
    warm = max(0, min(warm, data["sampled"].shape[0] - steps))
    tok = data["token_ids"][:rows].copy()
    q = data["num_tokens"][:rows].copy()
    samp = data["sampled"][:warm + steps, :rows].copy()
    nproc = min(cores, rows)
    bounds = np.linspace(0, rows, nproc + 1).astype(int)
    from suffixgpu_b200.workloads import CONFIG2_DRAFTER
    chunks = [((tok[a:b_].copy(), q[a:b_].copy(), samp[:, a:b_].copy()),
               steps, warm, dict(CONFIG2_DRAFTER))
              for a, b_ in zip(bounds[:-1], bounds[1:]) if b_ > a]
    t0 = time.perf_counter()
    with ProcessPoolExecutor(max_workers=len(chunks),
                             mp_context=mp.get_context("spawn")) as ex:
        times = list(ex.map(_cpu_chunk, chunks))
    wall = time.perf_counter() - t0
    slowest = max(times)
    return {"value": rows * steps / slowest, "unit": "rows/s",
            "cores": len(chunks), "kind": "port",
            "sample": f"{rows} rows of config 2 x {steps} timed decode "
                      f"steps after {warm} untimed, "
                      f"numpy restatement of the reference CPU path, "
                      f"{len(chunks)} worker processes; slowest worker "
                      f"{slowest:.2f} s compute, {wall:.2f} s wall with "
                      f"start-up"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    data = workload(0)
    warm = max(1, min(args.warmup, 5))
    cb = cpu_baseline(args, data, warm=warm)
    v = cb["value"]
    return {
        "metric": METRIC, "value": v, "unit": "rows/s", "n_gpus": 0,
        "steps": args.cpu_steps, "warmup": warm,
        "ms_per_step": 1e3 * min(args.cpu_rows, B) / v,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int32",
        "data": "synthetic (seeded copy/Zipf rows, benchmark config 2)",
        "config": dict(CONFIG, parallelism="host cores"),
        "impl": "reference", "cpu_baseline": cb,
        "e2e": {"value": v, "unit": "rows/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    if args.impl == "reference":
        res = run_reference(args)
    elif args.mode == "rebuild":
        import torch
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(dev)
        res = run_rebuild(args, dev)
    elif args.mode == "vllm":
        import torch
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(dev)
        res = run_vllm(args, dev)
    elif args.mode in ("sa", "global"):
        import torch
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(dev)
        res = run_sa(args, dev) if args.mode == "sa" else run_global(args, dev)
    elif args.mode == "sharded":
        import datetime
        import torch
        import torch.distributed as dist
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        torch.cuda.set_device(dev)
        if world > 1:
            dist.init_process_group("nccl", device_id=dev,
                                    timeout=datetime.timedelta(seconds=300))
        res = run_sharded(args, dev, world, rank)
        if world > 1:
            dist.destroy_process_group()
    else:
        res = run_ours(args)
    if res is not None:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
