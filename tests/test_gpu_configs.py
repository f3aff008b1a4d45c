"""The CUDA verify round at the benchmark's own configurations, against the
reference engine itself (GPU, sm_100a).

The checkpoint is the benchmark's: the Gemma-4-E2B shape with BASELINE's
literal distributions (norms N(0, 0.02) used as they are, no layer scalar),
written to a safetensors folder that both sides load - the reference engine
compiled from its own app_core.c (oracle/_ref, through oracle/ref_harness.c)
and this library through igc_model_load.

  config 0  the 1024-id prompt (a 256-id passage x4 with 10% substitutions,
            seed 0), greedy --guess 4: 64 tokens of the reference's own
            greedy stream (session_step), checked block by block against this
            library's four-lane rounds fed the same ids (logits within 2e-2,
            argmax equal wherever the reference's top-2 gap is above 2e-2),
            and this library's free-running n-gram-scout stream equal to the
            reference's up to its first excused step (app_main.c:1473-1480:
            a stream with guessing equals the stream without).
  depth     1536 ids primed, then blocks of 1, 4, 8 and 16 lanes: every
            sliding layer past its 512 window and the global layers at depth.
  config 1  heat 0.8, top-k 64, top-p 0.95, --guess 8: over 10,000 seeds the
            token a sampled round emits at its first lane is distributed as
            the reference's shaped distribution of that lane's row
            (chi-squared; app_test.c:4410-4520 tests the rule the same way).
  config 2  the 8192-id prompt and a second sharing its first 7680 ids: the
            --keep path (wind back, prime the rest) leaves exactly the caches
            a full prime leaves (this library only; the reference re-primes).

Tolerance: logits agree within 2e-2 absolute (the task's bar, fp32
accumulate).  Under these literal weights most steps have a top-2 gap below
that bar; the tests print the excused fraction.
"""

import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL = 2e-2
CKPT = os.environ.get("IGLLM_BENCH_CKPT", "/tmp/igllm_bench_e2b_s1")
VOCAB = 262144
WINDOW = 4096
STREAM = 64


def _threads():
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()


def _prompt():
    """BASELINE config 0's prompt: a 256-id passage (uniform, seed 0) x4 with 10% substitutions."""
    rng = np.random.default_rng(0)
    passage = rng.integers(0, VOCAB, 256)
    prompt = np.tile(passage, 4)
    swap = rng.random(1024) < 0.10
    prompt[swap] = rng.integers(0, VOCAB, int(swap.sum()))
    return prompt.astype(np.int32)


def _gap(row):
    top2 = np.partition(row, -2)[-2:]
    return float(abs(top2[1] - top2[0]))


def _shaped(row, heat, top_count, top_portion):
    """app_core.c:14572 pick_shape without echo penalty: top-k by logit,
    softmax of (x - max) / heat, the top-p prefix whose running mass first
    reaches the portion, renormalised.  Returns {id: probability}."""
    order = np.argsort(-row, kind="stable")[:top_count]
    w = np.exp((row[order].astype(np.float64) - row[order[0]]) / heat)
    w /= w.sum()
    keep = int(np.searchsorted(np.cumsum(w), top_portion) + 1)
    w = w[:keep] / w[:keep].sum()
    return dict(zip(order[:keep].tolist(), w.tolist()))


@pytest.fixture(scope="module")
def e2b(igc_lib, igo_mod):
    """The benchmark checkpoint on disk, the reference engine and this
    library on it, and the reference's results on config 0's prompt."""
    if not os.path.exists(os.path.join(CKPT, "model.safetensors")):
        igc_lib.synth_write(igc_lib.spec_e2b(seed=1, window_limit=WINDOW), CKPT, threads=min(32, _threads()))
    rm = igo_mod.RefModel(CKPT, threads=_threads(), window_limit=WINDOW)
    model = igc_lib.Model(folder=CKPT, window_limit=WINDOW)
    prompt = _prompt()
    rs = igo_mod.RefSession(rm)
    rs.prime(prompt)
    last = int(prompt[-1])
    # config 1's block: lane 0 verifies the likeliest-but-one id (accepted now
    # and then), the other lanes the next likeliest ids
    row0 = rs.guess(np.array([last], np.int32))[0]
    rs.keep(0)
    order = np.argsort(-row0, kind="stable")
    block8 = np.array([last] + order[1:8].tolist(), np.int32)
    rows8 = rs.guess(block8)
    rs.keep(0)
    # config 0: the reference's own greedy stream by plain steps
    ref_rows, ref_tokens = [], []
    tok = last
    for _ in range(STREAM):
        row = rs.step(tok)
        ref_rows.append(row)
        tok = int(row.argmax())
        ref_tokens.append(tok)
    rs.close()
    out = dict(model=model, rm=rm, prompt=prompt, rows8=rows8, block8=block8, ref_rows=ref_rows,
               ref_tokens=ref_tokens)
    yield out
    model.close()
    rm.close()


def test_config0_greedy_blocks_match_the_reference(igc_lib, e2b):
    s = igc_lib.Session(e2b["model"])
    s.prime(e2b["prompt"])
    ids = [int(e2b["prompt"][-1])] + e2b["ref_tokens"]
    excused = mism = 0
    worst = 0.0
    for r in range(STREAM // 4):
        block = np.array(ids[4 * r: 4 * r + 4], np.int32)
        rows = s.guess(block)
        s.guess_keep(4)
        for j in range(4):
            want = e2b["ref_rows"][4 * r + j]
            worst = max(worst, float(np.abs(rows[j] - want).max()))
            gap = _gap(want)
            if gap < ATOL:
                excused += 1
            elif int(rows[j].argmax()) != int(want.argmax()):
                mism += 1
    frac = excused / STREAM
    print(f"\nconfig 0: {STREAM} greedy steps at 1024-1088, max |logit diff| {worst:.2e}, "
          f"top-2 gap below {ATOL} at {excused} steps (excused fraction {frac:.3f})")
    assert worst <= ATOL, worst
    assert mism == 0


def test_config0_scout_stream_matches_the_reference(igc_lib, e2b):
    """The free-running stream: n-gram scout blocks of up to four lanes,
    greedy verify, keep - equal to the reference's plain greedy stream up to
    the first step whose top-2 gap is below the tolerance."""
    s = igc_lib.Session(e2b["model"])
    prompt = e2b["prompt"]
    s.prime(prompt)
    scout = igc_lib.Scout()
    scout.note(prompt)
    got, last, kept = [], int(prompt[-1]), 0
    while len(got) < STREAM:
        drawn = scout.draw(3)
        blk = np.concatenate([[last], drawn]).astype(np.int32)
        take, made = s.round(blk)
        new = [int(t) for t in blk[1:1 + take]] + [int(made)]
        kept += take
        got += new
        scout.note(np.array(new, np.int32))
        last = int(made)
    want = e2b["ref_tokens"]
    first = next((i for i in range(STREAM) if got[i] != want[i]), None)
    print(f"\nconfig 0 scout stream: {kept} guesses kept; "
          + ("equal to the reference's 64 tokens" if first is None else
             f"first difference at step {first}, reference top-2 gap {_gap(e2b['ref_rows'][first]):.2e}"))
    if first is not None:
        assert _gap(e2b["ref_rows"][first]) < ATOL, first


def test_depth_logits_match_the_reference(igc_lib, igo_mod, e2b):
    """1536 ids primed: every sliding layer masks past its 512 window and the
    global layers attend over the whole context; blocks of 1, 4, 8 and 16."""
    rng = np.random.default_rng(4)
    ids = rng.integers(0, VOCAB, 1536).astype(np.int32)
    rs = igo_mod.RefSession(e2b["rm"])
    rs.prime(ids)
    s = igc_lib.Session(e2b["model"])
    s.prime(ids)
    assert s.fill == rs.fill == len(ids) - 1
    last = int(ids[-1])
    worst = 0.0
    for k in (1, 4, 8, 16):
        block = np.array([last] + rng.integers(0, VOCAB, k - 1).tolist(), np.int32)
        want = rs.guess(block)
        rs.keep(0)
        got = s.guess(block)
        s.guess_keep(0)
        for g, w in zip(got, want):
            worst = max(worst, float(np.abs(g - w).max()))
            if _gap(w) > ATOL:
                assert int(g.argmax()) == int(w.argmax())
    rs.close()
    print(f"\ndepth 1535: blocks of 1/4/8/16 lanes, max |logit diff| {worst:.2e}")
    assert worst <= ATOL, worst


def test_config1_sampled_verify_matches_the_reference_distribution(igc_lib, e2b):
    """heat 0.8, top-k 64, top-p 0.95, --guess 8 after config 0's prompt:
    the token each sampled round emits at its first lane, over 10,000 seeds,
    against the reference's shaped distribution of that lane's row."""
    from scipy.stats import chi2
    heat, top_k, top_p = 0.8, 64, 0.95
    block = e2b["block8"]
    s = igc_lib.Session(e2b["model"])
    s.prime(e2b["prompt"])
    base = s.fill
    rows = s.guess(block)
    s.guess_keep(0)
    assert float(np.abs(rows - e2b["rows8"]).max()) <= ATOL
    q = _shaped(e2b["rows8"][0], heat, top_k, top_p)
    assert set(_shaped(rows[0], heat, top_k, top_p)) == set(q)
    n = 10000
    counts, accepted = {}, 0
    for seed in range(1, n + 1):
        take, made = s.round(block, igc_lib.Taste(heat, top_k, top_p, 1.0, 64, seed))
        token = int(block[1]) if take >= 1 else int(made)
        accepted += take >= 1
        counts[token] = counts.get(token, 0) + 1
        s.hold(base)
    assert set(counts) <= set(q), "a token outside the reference's shaped support"
    big = [t for t in q if q[t] * n >= 5]
    obs = [counts.get(t, 0) for t in big] + [n - sum(counts.get(t, 0) for t in big)]
    exp = [q[t] * n for t in big] + [n - sum(q[t] * n for t in big)]
    if exp[-1] < 5:  # fold a thin remainder into the last big bin
        obs[-2] += obs.pop()
        exp[-2] += exp.pop()
    stat = sum((o - e) ** 2 / e for o, e in zip(obs, exp))
    p = chi2.sf(stat, len(obs) - 1)
    g1 = int(block[1])
    print(f"\nconfig 1: {n} seeds, {len(q)} ids in the shaped support, chi-squared {stat:.1f} on "
          f"{len(obs) - 1} dof (p {p:.3f}); lane-0 guess accepted {accepted / n:.4f}, reference q {q.get(g1, 0):.4f}")
    assert p > 1e-3, (stat, len(obs), p)
    # the acceptance rate of the guess is its probability under q
    sd = np.sqrt(q[g1] * (1 - q[g1]) / n)
    assert abs(accepted / n - q[g1]) < 5 * sd


def _config2_prompts():
    """a random 2048-id document repeated 4x with 5% edits
    (8192 ids), and a second prompt sharing its first 7680 ids."""
    rng = np.random.default_rng(2)
    doc = rng.integers(0, VOCAB, 2048)
    first = np.tile(doc, 4)
    edit = rng.random(8192) < 0.05
    first[edit] = rng.integers(0, VOCAB, int(edit.sum()))
    second = first.copy()
    second[7680:] = rng.integers(0, VOCAB, 512)
    return first.astype(np.int32), second.astype(np.int32)


def test_config2_keep_prefix_matches_a_full_prime(igc_lib):
    """The --keep path at depth: after the 8192-id prompt, winding back to the
    7680 ids the second prompt shares and priming only its last 512 leaves
    the caches a full prime of the second prompt leaves, to the bit (the
    reference re-primes in full here, because its session_hold refuses once
    a sliding ring has turned over, app_core.c:13935-13945); then greedy
    --guess 8 blocks verify at depth 8192 on every layer kind."""
    spec = igc_lib.spec_e2b(seed=1, window_limit=9216)
    m = igc_lib.Model(spec=spec, window_limit=9216)
    first, second = _config2_prompts()
    a, b = igc_lib.Session(m), igc_lib.Session(m)
    a.prime(first)
    a.step(first[-1], want_logits=False)
    a.hold(7680)
    a.prime(second[7680:])
    b.prime(second)
    assert a.fill == b.fill == 8191
    top_a, row_a = a.step(second[-1])
    top_b, row_b = b.step(second[-1])
    assert np.array_equal(row_a, row_b) and top_a == top_b
    rng = np.random.default_rng(9)
    blk = np.array([top_a] + rng.integers(0, VOCAB, 7).tolist(), np.int32)
    assert np.array_equal(a.guess(blk), b.guess(blk))
    a.guess_keep(8)
    b.guess_keep(8)
    assert a.fill == b.fill == 8200
