#!/usr/bin/env python3
"""bench.py - decode tok/s of the speculative verify round (greedy, --guess 4).

Workload: the Gemma-4-E2B text stack with seeded random
weights (35 layers, hidden 1536, FFN 6144, 8 query heads / 1 KV head, head
256, vocab 262144, window 512, global every 5th, int4 g32 with f16 scales,
bf16 N(0,0.02) norms and embeddings), a 1024-id prompt (a 256-id passage,
uniform over the vocab, seed 0, repeated 4x with 10% substitutions), 256
tokens generated greedily in verify rounds of 4 lanes.

A step is one generation of those 256 tokens after the primed prompt: 64
verify rounds whose blocks come from the always-right proposer of the
reference's guess bracket (app_main.c:1235 main_guess_run), so every round
commits 4 tokens and the rate measures the verify round itself.

  value  device-resident: every block uploaded to HBM before the timed
         region, rounds chained on the stream, CUDA events (igc_session_bench)
  e2e    the same generation through the public round call
         (igc_session_round) with host ids in and host ids out each round

Also reported: the n-gram scout's own rate and acceptance, verify-round us
for K = 1, 2, 4, 8, 16, the projection kernels against the HBM roofline
(timed inside the timed graphed passes by launch stamps), and the reference
engine on the host cores.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
"""

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

TOKENS = 256
GUESS = 4
PROMPT_LEN = 1024
PREFILL_LEN = 4096
VOCAB = 262144
CKPT_DIR = os.environ.get("IGLLM_BENCH_CKPT", "/tmp/igllm_bench_e2b_s1")
METRIC = "decode tok/s (greedy, --guess 4)"


def make_prompt(seed=0):
    """A 256-id passage (uniform, seed 0 for config 0; a replica takes its
    rank as the seed) repeated 4x with 10% substitutions."""
    rng = np.random.default_rng(seed)
    passage = rng.integers(0, VOCAB, 256)
    prompt = np.tile(passage, 4)
    swap = rng.random(PROMPT_LEN) < 0.10
    prompt[swap] = rng.integers(0, VOCAB, int(swap.sum()))
    return prompt.astype(np.int32)


def oracle_blocks(last, cont, rounds, k):
    """Round r's block: the last committed id, then the next k-1 true ids."""
    seq = np.concatenate([[last], cont]).astype(np.int32)
    return np.stack([seq[r * k: r * k + k] for r in range(rounds)])


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock and throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def profiler_range(on):
    """cuProfilerStart/Stop around the timed rounds, so that a profiler run
    with --profile-from-start off sees exactly those launches."""
    import ctypes
    try:
        cu = ctypes.CDLL("libcuda.so.1")
        (cu.cuProfilerStart if on else cu.cuProfilerStop)()
    except OSError:
        pass


class Ranks:
    """One process a GPU under torchrun: its rank, the world size, and a host
    process group (None when alone).  Replicas share nothing on the device:
    the group is gloo over host sockets, used only for the barrier around the
    timed region and the maximum of the ranks' device times, so no NCCL
    communicator exists."""

    def __init__(self, backend="gloo"):
        self.rank = int(os.environ.get("RANK", "0"))
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dist = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=300))
            self.dist = dist

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max(self, x):
        """The largest of every rank's x (each rank gets it)."""
        if not self.dist:
            return float(x)
        import torch
        t = torch.tensor([float(x)], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.dist:
            self.dist.barrier()
            self.dist.destroy_process_group()


def aggregate(tokens_per_rank, slowest_seconds, world):
    """Whole-job throughput: every rank's tokens over the slowest rank's time."""
    return world * tokens_per_rank / slowest_seconds


# ---------------------------------------------------------------------------
# the reference engine on the host cores (oracle/_ref, built from app_core.c)

def host_cores():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def ensure_checkpoint():
    """The synthetic E2B checkpoint on disk for the reference engine.  It is
    written by a child process that exits before the reference runs, so the
    process that times the reference never maps this repository's CUDA
    library (the generator lives there, beside the in-HBM one)."""
    if not os.path.exists(os.path.join(CKPT_DIR, "model.safetensors")):
        code = ("import sys; sys.path.insert(0, %r); import igllm_b200 as ig; "
                "ig.synth_write(ig.spec_e2b(seed=1, window_limit=4096), %r, threads=%d)"
                % (ROOT, CKPT_DIR, min(32, host_cores())))
        subprocess.run([sys.executable, "-c", code], check=True)
    return CKPT_DIR


def reference_rounds(rounds_per_step, steps, warmup, cores):
    """The reference's own verify rounds on the host, over the positions the
    GPU arm covers: prime the 1024-id prompt, then session_guess(4) +
    keep(4) rounds from position 1024 to 1280 (64 rounds, every block kept,
    as the always-right proposer's would be; the cost of a round does not
    depend on which ids it verifies), `rounds_per_step` of them a step.
    When a step would run past position 1280 the session is primed again,
    untimed: the reference's session_hold refuses once its sliding ring has
    turned over (app_core.c:13935-13945), so it cannot wind back."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import igo
    folder = ensure_checkpoint()
    rm = igo.RefModel(folder, threads=cores, window_limit=4096)
    rs = igo.RefSession(rm)
    prompt = make_prompt()
    rounds_total = TOKENS // GUESS
    t0 = time.perf_counter()
    rs.prime(prompt)
    prime_s = time.perf_counter() - t0
    rng = np.random.default_rng(7)
    last = int(prompt[-1])
    done = 0
    times = []
    for it in range(warmup + steps):
        if done + rounds_per_step > rounds_total:
            rs.reset()
            rs.prime(prompt)
            last, done = int(prompt[-1]), 0
        t0 = time.perf_counter()
        for _ in range(rounds_per_step):
            blk = np.concatenate([[last], rng.integers(0, VOCAB, GUESS - 1)]).astype(np.int32)
            rs.guess(blk, want=False)
            top = rs.rows_argmax(GUESS)
            rs.keep(GUESS)
            last = int(top[-1])
        done += rounds_per_step
        if it >= warmup:
            times.append(time.perf_counter() - t0)
    rs.close()
    rm.close()
    return times, prime_s


def cpu_baseline_line(cores, rounds=8):
    times, prime_s = reference_rounds(rounds, 1, 0, cores)
    tok = rounds * GUESS / times[0]
    return {"value": round(tok, 3), "unit": "tok/s", "cores": cores, "kind": "reference",
            "sample": f"{rounds} verify rounds of {GUESS} lanes after the 1024-id prime "
                      f"(prime took {prime_s:.1f} s), reference engine app_core.c built with -O3 AVX-512, "
                      f"{cores} threads, same synthetic E2B weights read from safetensors"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = host_cores()
    rounds = 8
    times, prime_s = reference_rounds(rounds, args.steps, args.warmup, cores)
    total = sum(times)
    tok = rounds * GUESS * len(times) / total
    line = {
        "impl": "reference", "metric": METRIC, "value": round(tok, 3), "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1000 * total / len(times), 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "E2B int4 g32 greedy --guess 4 verify rounds, 1024-id prompt, 256 tokens (config 0)",
                   "sample": f"{rounds} rounds of 4 lanes a step, positions 1024-1280 as the GPU arm "
                             f"(re-primed untimed after every 64 rounds)",
                   "threads": cores},
        "cpu_baseline": {"value": round(tok, 3), "unit": "tok/s", "cores": cores, "kind": "reference",
                         "sample": f"{rounds} verify rounds of {GUESS} lanes a step after the 1024-id prime "
                                   f"({prime_s:.1f} s)"},
        "e2e": {"value": round(tok, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm

def run_ours(args):
    import igllm_b200 as ig

    local = int(os.environ.get("LOCAL_RANK", "0"))
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        import torch
        torch.cuda.set_device(local)
    ranks = Ranks("gloo")
    rank, world = ranks.rank, ranks.world
    barrier, max_over_ranks = ranks.barrier, ranks.max

    model = ig.Model(spec=ig.spec_e2b(seed=1, window_limit=4096), device=local, window_limit=4096)
    sess = ig.Session(model)
    prompt = make_prompt(rank)  # config 0's prompt on rank 0; each replica its own stream
    sess.prime(prompt)
    base = sess.fill
    # the true greedy continuation, by plain steps
    cont = []
    tok = int(prompt[-1])
    for _ in range(TOKENS + GUESS):
        tok, _ = sess.step(tok, want_logits=False)
        cont.append(tok)
    sess.hold(base)
    rounds = TOKENS // GUESS
    blocks = oracle_blocks(int(prompt[-1]), np.array(cont), rounds, GUESS)

    # device-resident rounds
    for _ in range(args.warmup):
        sess.bench(blocks, GUESS)
        sess.hold(base)
    ig.launch_count()
    sess.stamps(GUESS, reset=True)
    barrier()
    with ClockSampler(local) as clocks:
        dev_ms = []
        profiler_range(True)
        for _ in range(args.steps):
            ms, top = sess.bench(blocks, GUESS)
            dev_ms.append(ms)
            sess.hold(base)
        profiler_range(False)
    launches = ig.launch_count()
    stamps = sess.stamps(GUESS, reset=True)  # the timed passes' own launch spans
    total_s = max_over_ranks(sum(dev_ms) / 1000.0)
    value = aggregate(TOKENS * args.steps, total_s, world)
    check_ok = int(top[-1]) == int(cont[rounds * GUESS - 1])

    # end to end through the round call, host ids in and out each round
    for _ in range(1):
        for r in range(rounds):
            sess.round(blocks[r])
        sess.hold(base)
    barrier()
    e2e_s, takes = 0.0, 0
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for r in range(rounds):
            take, made = sess.round(blocks[r])
            takes += take
        e2e_s += time.perf_counter() - t0
        sess.hold(base)
    e2e_s = max_over_ranks(e2e_s)
    e2e = aggregate(TOKENS * args.steps, e2e_s, world)
    h2d = rounds * (1 + GUESS) * 4
    d2h = rounds * GUESS * 4

    # the shipped proposer: the n-gram scout, one generation
    scout = ig.Scout()
    scout.note(prompt)
    last, made_n, rounds_n, drawn, kept = int(prompt[-1]), 0, 0, 0, 0
    t0 = time.perf_counter()
    while made_n < TOKENS:
        d = scout.draw(min(GUESS - 1, TOKENS - made_n - 1)) if TOKENS - made_n > 1 else np.zeros(0, np.int32)
        if len(d) == 0:
            last, _ = sess.step(last, want_logits=False)
            new = [last]
        else:
            blk = np.concatenate([[last], d]).astype(np.int32)
            take, last = sess.round(blk)
            new = list(blk[1:1 + take]) + [last]
            drawn += len(d)
            kept += take
        rounds_n += 1
        made_n += len(new)
        scout.note(np.array(new, np.int32))
    ngram_s = time.perf_counter() - t0
    sess.hold(base)

    # verify-round cost against K
    per_k = {}
    for k in (1, 2, 4, 8, 16):
        r_k = 16
        blk_k = oracle_blocks(int(prompt[-1]), np.array(cont), r_k, k) if r_k * k <= len(cont) else \
            np.tile(blocks[:1, :1], (r_k, k))
        sess.bench(blk_k, k)
        sess.hold(base)
        ms, _ = sess.bench(blk_k, k)
        sess.hold(base)
        per_k[str(k)] = round(1000.0 * ms / r_k, 1)

    # prefill: 4096 uniform ids (seed 1) through the
    # prime call, then the first token; a warm-up prime captures the graphs
    psess = ig.Session(model)
    pids = np.random.default_rng(1).integers(0, VOCAB, PREFILL_LEN).astype(np.int32)
    psess.prime(pids)
    psess.reset()
    t0 = time.perf_counter()
    psess.prime(pids)
    t1 = time.perf_counter()
    psess.step(int(pids[-1]), want_logits=False)
    t2 = time.perf_counter()
    psess.close()
    prefill = {"tok_s": round((PREFILL_LEN - 1) / (t1 - t0), 1), "ttft_ms": round(1000 * (t2 - t0), 2),
               "prompt": f"{PREFILL_LEN} uniform ids, seed 1 (config 3), chunks of 512 lanes through the tcgen05 lane "
                         "GEMM; TTFT = the prime plus the first step"}

    # config 1: sampled verify rounds (heat 0.8, top-k 64, top-p 0.95,
    # --guess 8) through the round call; each block guesses the greedy
    # continuation from the session's current position
    sampled_rounds, sampled_tokens = 64, 0
    seq = np.concatenate([[int(prompt[-1])], cont]).astype(np.int32)
    sess.round(seq[:8], ig.Taste(0.8, 64, 0.95, 1.0, 64, 1))  # captures the 8-lane pass
    sess.hold(base)
    t0 = time.perf_counter()
    done = 0
    for r in range(sampled_rounds):
        at = min(done, len(seq) - 8)
        take, made = sess.round(seq[at: at + 8], ig.Taste(0.8, 64, 0.95, 1.0, 64, 1000 + r))
        sampled_tokens += take + 1
        done += take + 1 if take == 7 else 0  # a rejected guess leaves the session off the greedy path
        if take < 7:
            sess.hold(base + done)
    sampled_s = time.perf_counter() - t0
    sess.hold(base)
    sampled = {"round_ms": round(1000 * sampled_s / sampled_rounds, 3),
               "tok_s": round(sampled_tokens / sampled_s, 1), "tokens": sampled_tokens, "rounds": sampled_rounds,
               "workload": "config 1: heat 0.8, top-k 64, top-p 0.95, --guess 8, guesses from the greedy "
                           "continuation, through igc_session_round (host ids in and out)"}

    crowd = crowd_bench(ig, model) if not args.no_crowd else None
    long_ctx = long_context_bench(ig) if not args.no_crowd else None
    cache8 = cache8_bench(ig, model) if not args.no_crowd else None
    export = export_bench(ig) if not args.no_crowd else None

    # the projection kernels against the HBM roofline, from the timed
    # region's own graphed passes: every projection and attention launch
    # stamped its span (first block past its wait on the kernel ahead to the
    # last block's end) and the pass's last kernel summed them on the device
    passes = args.steps * rounds
    gemv = [(b, ns) for c, b, ns in stamps if c == 0]
    head = [(b, ns) for c, b, ns in stamps if c == 1]
    attn_ns = sum(ns for c, b, ns in stamps if c == 2)
    g_bytes = sum(b for b, _ in gemv)                      # per pass
    g_ms = sum(ns for _, ns in gemv) / 1e6 / passes       # per pass
    h_bytes = sum(b for b, _ in head)
    h_ms = sum(ns for _, ns in head) / 1e6 / passes
    attn_ms = attn_ns / 1e6 / passes
    pass_ms = sum(dev_ms) / passes  # this rank's device time a pass
    peak, peak_kind = peaks()
    achieved = g_bytes / (g_ms / 1000.0) / 1e9 if g_ms > 0 else None
    # DRAM bytes per projection launch: the algorithmic bytes times the
    # DRAM/algorithmic ratio ncu measured on the same kernels (profiles/).
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "gemv_e2b_layer0_k4_full.txt")) as f:
            for ln in f:
                if ln.startswith("dram_over_algorithmic:"):
                    traffic = round(float(ln.split()[1]) * g_bytes / max(1, len(gemv)))
    except OSError:
        traffic = None
    round_s = per_k[str(GUESS)] / 1e6
    bytes_round = model.decode_bytes()

    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1000.0 * total_s / args.steps, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int4 weights, f16 hi/lo activations, f32 accumulate",
        "data": "synthetic (seeded E2B-shaped weights, BASELINE config 0 prompt)",
        "weights": "BASELINE's distributions (int4 codes uniform in [-8,7], f16 scales |N(0,0.02)|, bf16 norms and "
                   "embeddings N(0,0.02)) drawn by a counter-based splitmix64 generator over a normal quantile "
                   "table, not numpy PCG64 (the same bits in HBM and in the reference's safetensors file)",
        "config": {"workload": "E2B int4 g32 greedy --guess 4 verify rounds, 1024-id prompt, 256 tokens (config 0)",
                   "proposer": "always-right (reference guess bracket's oracle); n-gram scout reported beside",
                   "l2": "weights 938 MB per round, larger than the 126 MB L2",
                   "parallelism": f"replicas x{world}"},
        "e2e": {"value": round(e2e, 1), "unit": "tok/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
        "gpu_launches": launches,
        "verify_round_us": per_k,
        "prefill": prefill,
        "ngram": {"tok_s": round(TOKENS / ngram_s, 1), "rounds": rounds_n, "guesses": drawn, "kept": kept},
        "sampled": sampled,
        "crowd": crowd,
        "long_context": long_ctx,
        "cache8": cache8,
        "export": export,
        "roofline": {"bound": "hbm", "kernel": "int4 skinny GEMM (layer projections)",
                     "achieved": round(achieved, 1) if achieved else None, "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4) if achieved else None, "traffic": traffic,
                     "peak_kind": peak_kind,
                     "timing": "launch stamps of the timed graphed passes (%globaltimer: first block past its "
                               "wait to last block's end), summed on the device over every timed pass",
                     "launches_per_pass": len(gemv), "algorithmic_bytes_per_launch": round(g_bytes / max(1, len(gemv))),
                     "bytes_per_pass": g_bytes, "ms_per_pass": round(g_ms, 4),
                     "head_ms_per_pass": round(h_ms, 4),
                     "head_gbs": round(h_bytes / (h_ms / 1000.0) / 1e9, 1) if h_ms else None,
                     "attention_ms_per_pass": round(attn_ms, 4),
                     "pass_ms": round(pass_ms, 4),
                     "stamped_share_of_pass": round((g_ms + h_ms + attn_ms) / pass_ms, 4) if pass_ms else None,
                     "round_frac": round(bytes_round / round_s / 1e9 / peak, 4)},
        "clocks": clocks.summary(),
        "check": {"last_round_argmax_matches_stepped_stream": check_ok, "e2e_kept": takes,
                  "e2e_kept_max": rounds * (GUESS - 1) * args.steps},
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            line["cpu_baseline"] = cpu_baseline_line(host_cores())
        except Exception as exc:  # the reference build is missing: say so
            line["cpu_baseline"] = {"value": None, "unit": "tok/s", "cores": host_cores(), "kind": "reference",
                                    "sample": f"unavailable: {exc}"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    ranks.close()


CROWD_STREAMS = 64
CROWD_TOKENS = 512  # config 4: 512 tokens a stream


def crowd_bench(ig, model):
    """BASELINE config 4 on one GPU: 64 independent streams, each primed with
    its own 1024-id prompt (built as config 0's, seeds 100..163), greedy
    --guess 4 verify rounds of all 64 streams at once through igc_crowd_round
    (256 lanes a weight sweep, the tcgen05 lane GEMM).  Blocks come from each
    stream's own greedy continuation (the always-right proposer, found first
    by one-lane crowd rounds), CROWD_TOKENS tokens a stream; the timed rounds
    take host ids in and host ids out each round."""
    sessions = [ig.Session(model) for _ in range(CROWD_STREAMS)]
    prompts = [make_prompt(100 + i) for i in range(CROWD_STREAMS)]
    t0 = time.perf_counter()
    for s_, p_ in zip(sessions, prompts):
        s_.prime(p_)
    prime_s = time.perf_counter() - t0
    base = [s_.fill for s_ in sessions]
    last = np.array([p_[-1] for p_ in prompts], np.int32)
    # each stream's greedy continuation, one lane a stream a round
    one = ig.Crowd(model, CROWD_STREAMS, 1)
    cont = np.zeros((CROWD_STREAMS, CROWD_TOKENS + GUESS), np.int32)
    cur = last.copy()
    for t in range(CROWD_TOKENS + GUESS):
        _, made, _ = one.round(sessions, cur.reshape(-1, 1))
        cont[:, t] = made
        cur = made
    one.close()
    for s_, b_ in zip(sessions, base):
        s_.hold(b_)
    crowd = ig.Crowd(model, CROWD_STREAMS, GUESS)
    seqs = np.concatenate([last[:, None], cont], axis=1)  # seqs[:, i] is the id at base + i

    def generation():
        done = np.zeros(CROWD_STREAMS, np.int64)
        rounds = 0
        while done.min() < CROWD_TOKENS:
            blocks = np.stack([seqs[j, done[j]: done[j] + GUESS] for j in range(CROWD_STREAMS)])
            take, made, _ = crowd.round(sessions, blocks)
            done += take + 1
            rounds += 1
        return int(done.sum()), rounds

    generation()  # captures the round's graph
    for s_, b_ in zip(sessions, base):
        s_.hold(b_)
    t0 = time.perf_counter()
    tokens, rounds = generation()
    wall = time.perf_counter() - t0
    crowd.close()
    for s_ in sessions:
        s_.close()
    flops = 2.0 * CROWD_STREAMS * GUESS * model.linear_params() * rounds
    tflops = flops / wall / 1e12
    return {"streams": CROWD_STREAMS, "k": GUESS, "tokens_per_stream": CROWD_TOKENS,
            "tok_s": round(tokens / wall, 1), "round_ms": round(1000 * wall / rounds, 3), "rounds": rounds,
            "tokens": tokens, "prime_s_all": round(prime_s, 2),
            "tensor": {"tflops": round(tflops, 1), "peak": 1388.0, "frac": round(tflops / 1388.0, 4),
                       "peak_kind": "measured sustained bf16 (MEASURED_PEAKS.json bf16_tflops_sustained); "
                                    "three f16 products a step (hi/lo split) counted once"},
            "workload": "config 4 on one GPU: 64 streams x 1024-id prompts (seeds 100-163), greedy --guess 4, "
                        f"{CROWD_TOKENS} tokens a stream, all streams in one crowd round; host ids in and out "
                        "every round (wall clock)"}


def cache8_bench(ig, float_model):
    """The --cache 8 storage (app_core.c:14270-14284) on config 0's shape and
    prompt: the same weights with every owner layer's key and value scales
    in the checkpoint, greedy --guess 4 rounds of always-right blocks through
    igc_session_bench (device-resident), beside the float cache's rounds."""
    spec = ig.spec_e2b(seed=1, window_limit=4096)
    spec.cache_scale_k, spec.cache_scale_v = 1.0 / 2048, 1.0 / 64
    model = ig.Model(spec=spec, device=0, window_limit=4096, cache_bits=8)
    prompt = make_prompt(0)
    blocks = np.random.default_rng(5).integers(0, VOCAB, (64, GUESS)).astype(np.int32)
    out = {}
    for name, m in (("bytes", model), ("float", float_model)):
        s = ig.Session(m)
        s.prime(prompt)
        base = s.fill
        s.bench(blocks[:2], GUESS)
        s.hold(base)
        ms, _ = s.bench(blocks, GUESS)
        out[name] = {"round_us": round(1000 * ms / len(blocks), 1), "tok_s": round(len(blocks) * GUESS / (ms / 1e3), 1),
                     "cache_mb_at_window": round(s.cache_room() / 1e6, 1)}
        s.close()
    model.close()
    out["workload"] = ("config 0's prompt and weights, --cache 8 (key scale 1/2048, value 1/64, x1-1.375 by layer), "
                       "64 always-right --guess 4 rounds on the device; owner layers write e4m3 codes, each layer "
                       "decodes the rows it reads, then attends")
    return out


def export_bench(ig):
    """The shipped export's form at full size (its config.json and
    quantization_config, app_core.c:7886): 512-wide global heads, the doubled
    feed-forward of the sharing layers (12288 wide) coded in 2 bits, the
    embedding a 2-bit table that is also the head, the per-layer table in 4
    bits.  Greedy --guess 4 rounds of always-right blocks after config 0's
    prompt, on the device.  Then the forms the tiles do not hold on top (8-bit
    per-layer input planes, a dense per-layer model projection, activation
    grids on every projection): that model runs its plain path, timed through
    igc_session_round (host ids in and out)."""
    out = {}
    prompt = make_prompt(0)
    blocks = np.random.default_rng(6).integers(0, VOCAB, (32, GUESS)).astype(np.int32)
    spec = ig.spec_e2b(seed=1, window_limit=4096)
    spec.global_head_dim, spec.double_wide, spec.late_mlp_bits = 512, 1, 2
    spec.embed_bits, spec.ple_embed_bits, spec.tied_head = 2, 4, 1
    model = ig.Model(spec=spec, device=0, window_limit=4096)
    s = ig.Session(model)
    s.prime(prompt)
    base = s.fill
    s.bench(blocks[:2], GUESS)
    s.hold(base)
    ms, _ = s.bench(blocks, GUESS)
    out["tiles"] = {"round_us": round(1000 * ms / len(blocks), 1), "tok_s": round(len(blocks) * GUESS / (ms / 1e3), 1),
                    "decode_mb": round(model.decode_bytes() / 1e6, 1)}
    s.close()
    model.close()
    spec.ple_bits8, spec.dense_ple_lift, spec.grid_in, spec.grid_out = 1, 1, 0.05, 0.02
    model = ig.Model(spec=spec, device=0, window_limit=4096)
    s = ig.Session(model)
    short = prompt[:128]  # the plain path primes slowly: a short prompt
    s.prime(short)
    base = s.fill
    seq = np.concatenate([[int(short[-1])], blocks.ravel()]).astype(np.int32)
    s.round(seq[:GUESS])  # captures the pass
    s.hold(base)
    rounds = 8
    t0 = time.perf_counter()
    for r in range(rounds):
        s.round(seq[r * GUESS: r * GUESS + GUESS])
    wall = time.perf_counter() - t0
    out["plain"] = {"round_ms": round(1000 * wall / rounds, 2), "rounds": rounds}
    s.close()
    model.close()
    out["workload"] = ("the export's form at E2B size, config 0's prompt, --guess 4: 'tiles' 32 always-right rounds on the "
                       "device (every lane counted); 'plain' adds 8-bit per-layer input planes, a dense per-layer model "
                       "projection and activation grids, a 128-id prompt, 8 rounds through igc_session_round")
    return out


def long_context_bench(ig):
    """an 8192-id prompt (a random 2048-id document x4 with
    5% edits, seed 2), greedy --guess 8 verify rounds at that depth, then a
    second prompt sharing the first 7680 ids by the --keep path (wind back to
    7680, prime the other 512; the reference re-primes all 8192 because its
    session_hold refuses once a sliding ring has turned over,
    app_core.c:13935-13945), beside a full re-prime for comparison."""
    rng = np.random.default_rng(2)
    doc = rng.integers(0, VOCAB, 2048)
    first = np.tile(doc, 4)
    edit = rng.random(8192) < 0.05
    first[edit] = rng.integers(0, VOCAB, int(edit.sum()))
    second = first.copy()
    second[7680:] = rng.integers(0, VOCAB, 512)
    first, second = first.astype(np.int32), second.astype(np.int32)
    model = ig.Model(spec=ig.spec_e2b(seed=1, window_limit=9216), device=0, window_limit=9216)
    s = ig.Session(model)
    s.prime(second)  # captures the chunk graphs
    s.reset()
    t0 = time.perf_counter()
    s.prime(first)
    prime_s = time.perf_counter() - t0
    base = s.fill
    blocks = np.random.default_rng(3).integers(0, VOCAB, (16, 8)).astype(np.int32)
    s.bench(blocks[:1], 8)
    s.hold(base)
    ms, _ = s.bench(blocks, 8)
    # the --keep file (app_core.c:14010 session_save / :14076 session_load):
    # the primed prompt written, then read into a fresh session that goes on
    # from it with no prime
    s.hold(base)
    keep_path = os.path.join(tempfile.mkdtemp(prefix="igllm_keep_"), "prompt.keep")
    t0 = time.perf_counter()
    s.save(keep_path, kind=ig.KEEP_PROMPT)
    save_s = time.perf_counter() - t0
    keep_mb = os.path.getsize(keep_path) / 1e6
    r = ig.Session(model)
    t0 = time.perf_counter()
    r.load(keep_path)
    load_s = time.perf_counter() - t0
    resumed = r.guess(blocks[0], want_logits=False) is None and r.fill == base + 8
    os.remove(keep_path)
    r.close()
    s.hold(7680)
    t0 = time.perf_counter()
    s.prime(second[7680:])
    keep_s = time.perf_counter() - t0
    s.reset()
    t0 = time.perf_counter()
    s.prime(second)
    full_s = time.perf_counter() - t0
    s.close()
    model.close()
    return {"prime_8192_ms": round(1000 * prime_s, 1), "prime_tok_s": round(8191 / prime_s, 1),
            "verify_round_us_k8_at_8192": round(1000 * ms / len(blocks), 1),
            "keep_prefix_7680_then_512_ms": round(1000 * keep_s, 1), "full_reprime_ms": round(1000 * full_s, 1),
            "keep_file": {"save_ms": round(1000 * save_s, 1), "load_ms": round(1000 * load_s, 1),
                          "mb": round(keep_mb, 1), "resumed": bool(resumed),
                          "what": "the 8191-id prompt's cache written in the reference's file layout and read "
                                  "into a fresh session, which then runs a block with no prime"},
            "workload": "config 2: 8192-id prompt (2048-id document x4, 5% edits, seed 2), greedy --guess 8 "
                        "rounds at depth 8192, second prompt sharing 7680 ids by the keep path"}


def run_profile_case(args):
    """A small verify-round case for kernel profilers (no JSON line): the E2B
    layer stack at full width with a vocabulary of `--case-vocab` ids, so the
    per-layer kernels are the benchmark's own while the device holds about
    1.3 GB (at 32768 ids).  The session is primed to `--case-context` ids,
    then `--case-rounds` verify rounds of `--case-k` lanes run between
    cuProfilerStart and cuProfilerStop: a profiler started with
    --profile-from-start off sees those launches only."""
    import igllm_b200 as ig
    spec = ig.spec_e2b(seed=1, window_limit=args.case_window)
    spec.vocab = args.case_vocab
    model = ig.Model(spec=spec, device=0, window_limit=args.case_window)
    rng = np.random.default_rng(0)
    if args.case_prime > 0:
        # one prime of `--case-prime` ids (the chunked tcgen05 path), captured
        # first by an identical prime outside the profiler range
        sess = ig.Session(model)
        ids = rng.integers(0, args.case_vocab, args.case_prime).astype(np.int32)
        sess.prime(ids)
        sess.reset()
        profiler_range(True)
        t0 = time.perf_counter()
        sess.prime(ids)
        wall = time.perf_counter() - t0
        profiler_range(False)
        print(f"profile case: prime of {args.case_prime} ids, vocab {args.case_vocab}: {1000 * wall:.1f} ms",
              flush=True)
        return
    if args.case_streams > 0:
        # crowd rounds: `--case-streams` sessions primed to `--case-context`
        # ids each, `--case-rounds` greedy rounds of `--case-k` lanes for all
        sessions = [ig.Session(model) for _ in range(args.case_streams)]
        for s_ in sessions:
            s_.prime(rng.integers(0, args.case_vocab, args.case_context).astype(np.int32))
        crowd = ig.Crowd(model, args.case_streams, args.case_k)
        blocks = rng.integers(0, args.case_vocab, (args.case_streams, args.case_k)).astype(np.int32)
        crowd.round(sessions, blocks)  # captures the round's graph
        profiler_range(True)
        t0 = time.perf_counter()
        for _ in range(args.case_rounds):
            crowd.round(sessions, blocks)
        wall = time.perf_counter() - t0
        profiler_range(False)
        print(f"profile case: {args.case_rounds} crowd rounds of {args.case_streams} x {args.case_k} lanes at "
              f"context {args.case_context}, vocab {args.case_vocab}: {1000 * wall / args.case_rounds:.2f} ms/round",
              flush=True)
        return
    sess = ig.Session(model)
    sess.prime(rng.integers(0, args.case_vocab, args.case_context).astype(np.int32))
    blocks = rng.integers(0, args.case_vocab, (args.case_rounds, args.case_k)).astype(np.int32)
    sess.bench(blocks[:1], args.case_k)  # captures the pass of this shape
    profiler_range(True)
    ms, _ = sess.bench(blocks, args.case_k)
    profiler_range(False)
    print(f"profile case: {args.case_rounds} rounds of {args.case_k} lanes at context {args.case_context}, "
          f"vocab {args.case_vocab}: {1000 * ms / args.case_rounds:.1f} us/round", flush=True)
    sess.close()
    model.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the host-core reference baseline")
    ap.add_argument("--no-crowd", action="store_true",
                    help="skip the 64-stream crowd and long-context measurements")
    ap.add_argument("--profile-case", action="store_true",
                    help="run the small profiler case instead of the benchmark (no JSON line)")
    ap.add_argument("--case-vocab", type=int, default=32768)
    ap.add_argument("--case-k", type=int, default=4)
    ap.add_argument("--case-rounds", type=int, default=3)
    ap.add_argument("--case-context", type=int, default=1024)
    ap.add_argument("--case-streams", type=int, default=0, help="profile crowd rounds of this many sessions")
    ap.add_argument("--case-window", type=int, default=4096, help="positions each session's caches hold")
    ap.add_argument("--case-prime", type=int, default=0, help="profile one prime of this many ids")
    args = ap.parse_args()
    if args.profile_case:
        run_profile_case(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
