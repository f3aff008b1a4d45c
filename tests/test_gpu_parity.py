"""The CUDA verify round against the CPU oracle (GPU, sm_100a).

Every check goes through the C ABI of libigllm_cuda (include/igllm_cuda.h).
Tolerance: logits agree within 2e-2 absolute (fp32 accumulate), the bar the
task states; the same runs are also held to a much tighter relative bar so a
precision regression shows long before it reaches 2e-2.  Greedy tokens must
agree wherever the oracle's top-2 gap is above the tolerance.
"""

import numpy as np
import pytest

from conftest import LITERAL, SMALL, TINY, WIDE

pytestmark = pytest.mark.gpu

ATOL = 2e-2      # the task's logit tolerance
TIGHT = 2e-4     # relative to the row's largest magnitude


def _check_rows(gpu, cpu):
    err = np.abs(gpu - cpu).max()
    scale = max(1.0, float(np.abs(cpu).max()))
    assert err <= ATOL, err
    assert err <= TIGHT * scale, (err, scale)
    for g, c in zip(np.atleast_2d(gpu), np.atleast_2d(cpu)):
        top2 = np.sort(c)[-2:]
        if top2[1] - top2[0] > ATOL:
            assert g.argmax() == c.argmax()


def _pair(igc, igo, folder, cfg):
    m = igc.Model(folder=folder, window_limit=cfg["window_limit"])
    om = igo.OracleModel(folder, window_limit=cfg["window_limit"])
    return m, om


@pytest.mark.parametrize("which", ["tiny", "small", "literal", "wide"])
def test_pass_parity(igc_lib, igo_mod, which, tiny_dir, small_dir, literal_dir, wide_dir):
    folder = {"tiny": tiny_dir, "small": small_dir, "literal": literal_dir, "wide": wide_dir}[which]
    cfg = {"tiny": TINY, "small": SMALL, "literal": LITERAL, "wide": WIDE}[which]
    m, om = _pair(igc_lib, igo_mod, folder, cfg)
    s, o = igc_lib.Session(m), igo_mod.OracleSession(om, threads=8)
    rng = np.random.default_rng(2)
    ids = rng.integers(0, cfg["vocab"], 53).astype(np.int32)  # 3 prime chunks + a ragged one
    s.prime(ids)
    o.prime(ids)
    assert s.fill == o.fill == len(ids) - 1
    top, row = s.step(ids[-1])
    orow = o.step(ids[-1])
    _check_rows(row, orow)
    for k in (1, 2, 4, 7, 8, 9, 16):
        blk = np.array([top] + list(rng.integers(0, cfg["vocab"], k - 1)), np.int32)
        rows = s.guess(blk)
        orows = o.guess(blk)
        _check_rows(rows, orows)
        keep = min(k, 2)
        s.guess_keep(keep)
        o.guess_keep(keep)
        assert s.fill == o.fill
        top, row = s.step(blk[keep - 1] if keep else blk[0])
        _check_rows(row, o.step(blk[keep - 1] if keep else blk[0]))


def test_guess_argmax_and_refusals(igc_lib, igo_mod, small_dir):
    m = igc_lib.Model(folder=small_dir, window_limit=SMALL["window_limit"])
    s = igc_lib.Session(m)
    s.prime(np.arange(5, 40, dtype=np.int32))
    top, _ = s.step(40)
    blk = np.array([top, 3, 4, 5], np.int32)
    rows = s.guess(blk)
    assert list(s.guess_top()) == list(rows.argmax(axis=1))
    # mid-block: every mover refuses (app_core.c:12144, :14449, :14477)
    with pytest.raises(igc_lib.IgcError) as e:
        s.step(3)
    assert e.value.code == igc_lib.FAIL_STATE
    with pytest.raises(igc_lib.IgcError):
        s.prime(np.arange(3, dtype=np.int32))
    with pytest.raises(igc_lib.IgcError):
        s.guess(blk)
    with pytest.raises(igc_lib.IgcError):
        s.hold(3)
    s.guess_keep(0)
    with pytest.raises(igc_lib.IgcError):
        s.guess_keep(0)
    with pytest.raises(igc_lib.IgcError):
        s.guess(np.zeros(17, np.int32))
    with pytest.raises(igc_lib.IgcError):
        s.step(m.vocab)


def test_dropped_block_is_bit_identical(igc_lib, small_dir):
    """app_test.c:4392: the same block after a drop gives the same logits to the bit."""
    m = igc_lib.Model(folder=small_dir, window_limit=SMALL["window_limit"])
    s = igc_lib.Session(m)
    s.prime(np.arange(1, 30, dtype=np.int32))
    s.step(29)
    blk = np.array([12, 13, 7, 8], np.int32)
    first = s.guess(blk)
    s.guess_keep(0)
    again = s.guess(blk)
    s.guess_keep(0)
    assert np.array_equal(first, again)
    assert s.fill == 29


def test_keep_matches_stepping(igc_lib, small_dir):
    """app_test.c:4600: a kept block leaves the state stepping would, within 1e-3."""
    m = igc_lib.Model(folder=small_dir, window_limit=SMALL["window_limit"])
    a, b = igc_lib.Session(m), igc_lib.Session(m)
    seed = np.array([1, 7, 8, 9, 10, 11, 12, 13, 7, 8, 9, 10, 11], np.int32)
    want = np.array([12, 13, 7, 8], np.int32)
    for s in (a, b):
        s.prime(seed)
        s.step(seed[-1])
    rows = a.guess(want)
    a.guess_keep(2)
    for t in want[:2]:
        _, last = b.step(t)
    assert np.abs(rows[1] - last).max() <= 1e-3
    _, ra = a.step(5)
    _, rb = b.step(5)
    assert np.abs(ra - rb).max() <= 1e-3


def test_hold_rewinds_past_the_window(igc_lib, igo_mod, tiny_dir):
    """app_core.c:13935 session_hold, which the reference refuses once a ring
    has wrapped; full-length caches wind back anywhere."""
    m = igc_lib.Model(folder=tiny_dir, window_limit=TINY["window_limit"])
    s = igc_lib.Session(m)
    ids = np.arange(2, 60, dtype=np.int32)
    s.prime(ids)
    _, first = s.step(ids[-1])
    s.hold(20)
    assert s.fill == 20
    s.prime(ids[20:])
    _, again = s.step(ids[-1])
    assert np.array_equal(first, again)


def test_taste_parity(igc_lib, igo_mod, small_dir):
    """The tempered verify on the device rows draws what the oracle draws on
    its own rows for the same seeds (ties aside, which these rows do not have)."""
    m, om = _pair(igc_lib, igo_mod, small_dir, SMALL)
    s, o = igc_lib.Session(m), igo_mod.OracleSession(om, threads=8)
    ids = np.arange(3, 40, dtype=np.int32)
    s.prime(ids)
    o.prime(ids)
    s.step(ids[-1])
    o.step(ids[-1])
    blk = np.array([5, 9, 11, 4], np.int32)
    s.guess(blk, want_logits=False)
    orows = o.guess(blk)
    agree = total = 0
    for case in range(3):
        for seed in range(60):
            kw = [(0.8, 64, 0.95, 1.0), (1.0, 12, 0.9, 1.4), (1.2, 32, 1.0, 1.0)][case]
            t = igc_lib.Taste(kw[0], kw[1], kw[2], kw[3], 64, seed * 2654435761 + 12345)
            ot = igo_mod.Taste(kw[0], kw[1], kw[2], kw[3], 64, seed * 2654435761 + 12345)
            total += 1
            agree += s.guess_taste(blk, t) == o.guess_taste(orows, blk, ot)
    assert agree >= total - 2, (agree, total)
    s.guess_keep(0)


def test_sampled_step_pick(igc_lib, igo_mod, small_dir):
    m, om = _pair(igc_lib, igo_mod, small_dir, SMALL)
    s, o = igc_lib.Session(m), igo_mod.OracleSession(om, threads=8)
    ids = np.arange(3, 30, dtype=np.int32)
    s.prime(ids)
    o.prime(ids)
    s.step(ids[-1])
    orow = o.step(ids[-1])
    t = igc_lib.Taste(0.8, 64, 0.95, 1.0, 64, 77)
    ot = igo_mod.Taste(0.8, 64, 0.95, 1.0, 64, 77)
    assert s.pick(t) == o.pick(orow, ot)
    greedy = igc_lib.Taste(0.0, 64, 0.95, 1.0, 64, 0)
    assert s.pick(greedy) == int(orow.argmax())


def test_greedy_guess_stream_matches_plain(igc_lib, small_dir):
    """app_main.c:1473: rounds driven by the n-gram scout produce the plain
    greedy stream."""
    m = igc_lib.Model(folder=small_dir, window_limit=SMALL["window_limit"])
    plain, spec = igc_lib.Session(m), igc_lib.Session(m)
    prompt = np.tile(np.array([11, 22, 33, 44, 55, 66], np.int32), 5)
    plain.prime(prompt)
    spec.prime(prompt)
    tok = prompt[-1]
    want = []
    for _ in range(24):
        tok, _ = plain.step(tok, want_logits=False)
        want.append(tok)
    scout = igc_lib.Scout()
    scout.note(prompt)
    got = []
    last = prompt[-1]
    while len(got) < 24:
        drawn = scout.draw(3)
        blk = np.concatenate([[last], drawn]).astype(np.int32)
        take, made = spec.round(blk)
        new = list(blk[1:1 + take]) + [made]
        got += new
        scout.note(np.array(new, np.int32))
        last = made
    assert got[:24] == want


def test_desk_entries(igc_lib, igo_mod):
    """The backend table (app_core.c:5222) on the GPU against the oracle's kernels."""
    import ctypes
    igo = igo_mod
    lib = igo.igo_lib()
    desk = igc_lib.Desk(0)
    rng = np.random.default_rng(9)
    for rows, cols, lanes in [(37, 96, 5), (300, 1536, 16), (64, 6144, 3), (16, 32, 1)]:
        code = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
        sc16 = np.abs(rng.normal(0, 0.02, (rows, cols // 32))).astype(np.float16)
        plane = igc_lib.IgcPlane(form=2, row_count=rows, col_count=cols, code_data=code.ctypes.data,
                                 row_stride=cols // 2, gain_data=sc16.ctypes.data, gain_type=2, bit_count=4,
                                 code_bias=8, code_flip=0, group_size=32, group_count=cols // 32)
        act = rng.normal(0, 1, (lanes, cols)).astype(np.float32)
        got = desk.mat_mat(plane, act, lanes, rows)
        sc32 = sc16.astype(np.float32)
        op = igo.make_plane(code, sc32)
        want = np.zeros((lanes, rows), np.float32)
        lib.igo_mat_mat(ctypes.byref(op), igo.fptr(act), cols, lanes, igo.fptr(want), rows, 1)
        assert np.abs(got - want).max() <= 1e-4 * max(1.0, np.abs(want).max())
    x = rng.normal(0, 3, 1536).astype(np.float32)
    w = rng.normal(1, 0.1, 1536).astype(np.float32)
    want = np.zeros_like(x)
    lib.igo_norm_rms(igo.fptr(x), igo.fptr(w), 1536, 1e-6, igo.fptr(want))
    np.testing.assert_allclose(desk.norm_rms(x, w, 1e-6), want, rtol=1e-5, atol=1e-6)
    v = rng.normal(0, 4, 999).astype(np.float32)
    want = v.copy()
    lib.igo_soft_max(igo.fptr(want), len(want))
    np.testing.assert_allclose(desk.soft_max(v), want, rtol=1e-5, atol=1e-8)
    g, r = rng.normal(0, 2, 6144).astype(np.float32), rng.normal(0, 1, 6144).astype(np.float32)
    want = np.array([lib.igo_gelu_tanh(float(a)) * b for a, b in zip(g, r)], np.float32)
    np.testing.assert_allclose(desk.gelu_gate(g, r), want, rtol=1e-5, atol=1e-6)
    h = rng.normal(0, 1, 256).astype(np.float32)
    cs, sn = np.cos(np.arange(128) * 0.1).astype(np.float32), np.sin(np.arange(128) * 0.1).astype(np.float32)
    want = h.copy()
    lib.igo_rope_turn(igo.fptr(want), 256, igo.fptr(cs), igo.fptr(sn))
    np.testing.assert_allclose(desk.rope_turn(h, cs, sn), want, rtol=1e-6, atol=1e-6)
    desk.close()


def test_e2b_shape_against_oracle(igc_lib, igo_mod):
    """The benchmark's full Gemma-4-E2B shape (35 layers, 262144 vocab), built
    straight into HBM from the synthetic spec, against the oracle fed the same
    tensors in host memory: one prime, one step and one block of four."""
    spec = igc_lib.spec_e2b(norm_offset=1.0, seed=5, window_limit=1024)
    m = igc_lib.Model(spec=spec, window_limit=1024)
    om = igo_mod.OracleModel(tensors=igc_lib.synth_tensors(spec), config=igc_lib.synth_config(spec),
                             window_limit=1024)
    s, o = igc_lib.Session(m), igo_mod.OracleSession(om, threads=16)
    rng = np.random.default_rng(4)
    ids = rng.integers(0, 262144, 40).astype(np.int32)
    s.prime(ids)
    o.prime(ids)
    top, row = s.step(ids[-1])
    _check_rows(row, o.step(ids[-1]))
    blk = np.array([top, 17, 99, 1234], np.int32)
    _check_rows(s.guess(blk), o.guess(blk))
    s.guess_keep(1)
    o.guess_keep(1)


def test_e2b_lane_batches_are_bit_identical(igc_lib):
    """At the benchmark's size the wider lane counts run their projections
    in side-by-side batches of four or eight lanes (q|k|v and gate|up in
    batches of four held to one wave of the SMs, some warp groups taking two
    row blocks): single steps, an eight-lane block, a nine-lane block and a
    sixteen-lane block give the same bits."""
    spec = igc_lib.spec_e2b(norm_offset=1.0, seed=6, window_limit=1024)
    m = igc_lib.Model(spec=spec, window_limit=1024)
    rng = np.random.default_rng(8)
    ids = rng.integers(0, 262144, 40).astype(np.int32)
    block = rng.integers(0, 262144, 16).astype(np.int32)
    a = igc_lib.Session(m)
    a.prime(ids)
    stepped = np.stack([a.step(t)[1] for t in block[:9]])
    b = igc_lib.Session(m)
    b.prime(ids)
    assert np.array_equal(stepped, b.guess(block[:9]))
    c = igc_lib.Session(m)
    c.prime(ids)
    assert np.array_equal(stepped, c.guess(block)[:9])
    d = igc_lib.Session(m)
    d.prime(ids)
    assert np.array_equal(stepped[:8], d.guess(block[:8]))


def test_lane_batching_is_bit_identical(igc_lib, small_dir):
    """A position's logits do not depend on how many lanes shared its pass:
    one lane at a time (the packed four-lane mode), one nine-lane block (two
    8-lane tiles, 8-warp blocks) and blocks of four and five lanes (16-warp
    blocks) give the same bits, which is what lets a greedy stream with
    guessing equal the stream without it exactly."""
    m = igc_lib.Model(folder=small_dir, window_limit=SMALL["window_limit"])
    ids = np.array([3, 17, 29, 5, 8, 41, 77, 90, 12, 13, 14, 15, 16, 7, 9, 100, 200, 300, 11, 2, 4, 6, 8, 10,
                    12, 14, 16, 18, 20], np.int32)
    block = ids[19:28]
    a = igc_lib.Session(m)
    a.prime(ids[:20])
    stepped = np.stack([a.step(t)[1] for t in block])
    b = igc_lib.Session(m)
    b.prime(ids[:20])
    nine = b.guess(block)
    c = igc_lib.Session(m)
    c.prime(ids[:20])
    four = c.guess(block[:4])
    c.guess_keep(4)
    five = c.guess(block[4:])
    assert np.array_equal(stepped, nine)
    assert np.array_equal(stepped, np.concatenate([four, five]))


def test_wide_lane_batches_are_bit_identical(igc_lib, wide_dir):
    """The same for a down projection wide enough to run in side-by-side
    batches of four lanes: a nine-lane block (three batches), blocks of four
    and five, and single steps give the same bits."""
    m = igc_lib.Model(folder=wide_dir, window_limit=WIDE["window_limit"])
    ids = np.array([3, 17, 29, 5, 8, 41, 77, 90, 12, 13, 14, 15, 16, 7, 9, 100, 200, 300, 11, 2, 4, 6, 8, 10,
                    12, 14, 16, 18, 20], np.int32)
    block = ids[19:28]
    a = igc_lib.Session(m)
    a.prime(ids[:20])
    stepped = np.stack([a.step(t)[1] for t in block])
    b = igc_lib.Session(m)
    b.prime(ids[:20])
    nine = b.guess(block)
    c = igc_lib.Session(m)
    c.prime(ids[:20])
    four = c.guess(block[:4])
    c.guess_keep(4)
    five = c.guess(block[4:])
    assert np.array_equal(stepped, nine)
    assert np.array_equal(stepped, np.concatenate([four, five]))


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


def test_sampled_verify_matches_the_shaped_distribution(igc_lib, tiny_dir):
    """The single-token rejection rule (app_core.c:14762 session_guess_taste:
    accept the guess t with probability q(t), else draw from q without t)
    emits tokens distributed as q itself.  Over 4000 seeds, the token a
    two-lane sampled round emits after its first id matches q (heat 0.8,
    top-k 64, top-p 0.95) by a chi-squared test."""
    from scipy.stats import chi2
    m = igc_lib.Model(folder=tiny_dir, window_limit=TINY["window_limit"])
    s = igc_lib.Session(m)
    ids = np.arange(3, 40, dtype=np.int32)
    s.prime(ids)
    last = int(ids[-1])
    base = s.fill
    row = s.guess(np.array([last], np.int32))[0]
    s.guess_keep(0)
    q = _shaped(row, 0.8, 64, 0.95)
    guess = sorted(q, key=lambda t: -q[t])[1]  # the second likeliest: accepted now and then
    counts = {}
    n = 4000
    for seed in range(1, n + 1):
        take, made = s.round(np.array([last, guess], np.int32), igc_lib.Taste(0.8, 64, 0.95, 1.0, 64, seed))
        token = guess if take >= 1 else made
        counts[token] = counts.get(token, 0) + 1
        s.hold(base)
    assert set(counts) <= set(q), "a token outside the shaped support"
    big = [t for t in q if q[t] * n >= 5]
    obs = [counts.get(t, 0) for t in big] + [n - sum(counts.get(t, 0) for t in big)]
    exp = [q[t] * n for t in big] + [n - sum(q[t] * n for t in big)]
    if exp[-1] < 5:  # fold a thin remainder into the last big bin
        obs[-2] += obs.pop()
        exp[-2] += exp.pop()
    stat = sum((o - e) ** 2 / e for o, e in zip(obs, exp))
    p = chi2.sf(stat, len(obs) - 1)
    assert p > 1e-3, (stat, len(obs), p)
    assert 0.0 < counts.get(guess, 0) / n < 1.0
