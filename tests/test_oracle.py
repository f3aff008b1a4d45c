"""The CPU oracle, pinned to the reference.

Two kinds of pin, both on the CPU:

* the known-answer values of the reference's own unit tests (app_test.c:
  test_gemma :579, test_kernel :1114, test_scout :4654, test_guess :4350),
  restated here as data; and
* the reference engine itself, compiled from its own app_core.c into
  oracle/_ref, run side by side with the restatement on seeded synthetic
  checkpoints.
"""

import ctypes
import math

import numpy as np
import pytest

from conftest import LITERAL, SMALL, TINY


# ---- app_test.c:579 test_gemma: the U8 4-bit layout -----------------------------

def test_gemma_four_bit_decode(igo_mod):
    igo = igo_mod
    lib = igo.igo_lib()
    # four codes a row pair: 0, 1, 2, 3, -7, -6, 7, -8 (low nibble first, offset 8)
    code = np.tile(np.array([0x98, 0xBA, 0x21, 0x0F], np.uint8), (3, 1))
    scale = np.array([[0.5], [1.0], [2.0]], np.float32)
    plane = igo.make_plane(code, scale)
    row = np.zeros(8, np.float32)
    lib.igo_plane_row(ctypes.byref(plane), 0, igo.fptr(row))
    assert row[0] == 0.0 and row[3] == 1.5 and row[4] == -3.5 and row[7] == -4.0
    lib.igo_plane_row(ctypes.byref(plane), 2, igo.fptr(row))
    assert row[6] == 14.0
    # kern_row_code over the same row: sum code * act * scale with act = 1..8
    act = np.arange(1, 9, dtype=np.float32)
    got = lib.igo_row_code(ctypes.byref(plane), 0, igo.fptr(act))
    assert got == pytest.approx((0 + 2 + 6 + 12 - 35 - 36 + 49 - 64) * 0.5, abs=1e-5)


def test_mat_mat_against_plain_loop(igo_mod):
    igo = igo_mod
    lib = igo.igo_lib()
    rng = np.random.default_rng(5)
    rows, cols, lanes = 37, 96, 5
    code = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    scale = np.abs(rng.normal(0, 0.02, (rows, cols // 32))).astype(np.float32)
    plane = igo.make_plane(code, scale)
    act = rng.normal(0, 1, (lanes, cols)).astype(np.float32)
    out = np.zeros((lanes, rows), np.float32)
    lib.igo_mat_mat(ctypes.byref(plane), igo.fptr(act), cols, lanes, igo.fptr(out), rows, 1)
    nib = np.stack([code & 15, code >> 4], axis=-1).reshape(rows, cols).astype(np.float64) - 8.0
    w = nib * np.repeat(scale.astype(np.float64), 32, axis=1)
    want = act.astype(np.float64) @ w.T
    np.testing.assert_allclose(out, want, atol=1e-5)


# ---- app_test.c:1114 test_kernel ------------------------------------------------

def test_logit_cap_against_tanh(igo_mod):
    lib = igo_mod.igo_lib()
    cap = 30.0
    have = (-200.0 + 400.0 * np.arange(4001, dtype=np.float32) / np.float32(4000)).astype(np.float32)
    want = np.tanh(have.astype(np.float64) / cap) * cap
    lib.igo_logit_cap(igo_mod.fptr(have), len(have), cap)
    assert np.abs(have - want).max() <= 5e-7 * cap
    assert np.all(np.diff(have) >= 0)
    edge = np.array([0.0, 300.0, -300.0, 1e30, -1e30], np.float32)
    lib.igo_logit_cap(igo_mod.fptr(edge), 5, cap)
    assert edge[0] == 0.0 and edge[1] == cap and edge[2] == -cap and edge[3] == cap and edge[4] == -cap


def test_gelu_closed_form(igo_mod):
    lib = igo_mod.igo_lib()
    for v in (-3.0, -0.5, 0.0, 0.7, 2.5):
        inner = 0.7978845608028654 * (v + 0.044715 * v ** 3)
        assert lib.igo_gelu_tanh(v) == pytest.approx(0.5 * v * (1 + math.tanh(inner)), abs=1e-5)
    for v in np.linspace(-20, 20, 501, dtype=np.float32):
        vd = float(v)
        inner = 0.7978845608028654 * (vd + 0.044715 * vd ** 3)
        assert abs(lib.igo_gelu_tanh(float(v)) - 0.5 * vd * (1 + math.tanh(inner))) < 1e-5
    assert lib.igo_gelu_tanh(0.0) == 0.0
    assert lib.igo_gelu_tanh(-40.0) == 0.0 and lib.igo_gelu_tanh(-1e30) == 0.0
    assert lib.igo_gelu_tanh(40.0) == 40.0 and lib.igo_gelu_tanh(1e30) == pytest.approx(1e30, rel=1e-7)
    g = lib.igo_gelu_tanh(-6.0)
    assert -1e-8 < g <= 0.0


def test_soft_max_properties(igo_mod):
    lib = igo_mod.igo_lib()
    a = np.array([1, 2, 3, 4, 5], np.float32)
    b = a + 100
    lib.igo_soft_max(igo_mod.fptr(a), 5)
    lib.igo_soft_max(igo_mod.fptr(b), 5)
    assert abs(a.sum() - 1.0) < 1e-6
    np.testing.assert_allclose(a, b, atol=1e-6)
    w = np.array([1000, 1000, 1000], np.float32)
    lib.igo_soft_max(igo_mod.fptr(w), 3)
    assert abs(w[0] - 1 / 3) < 1e-6


def test_rope_rotate_half_and_inverse(igo_mod):
    lib = igo_mod.igo_lib()
    v = np.arange(1, 9, dtype=np.float32)
    keep = v.copy()
    cs = np.cos(0.3 * np.arange(1, 5)).astype(np.float32)
    sn = np.sin(0.3 * np.arange(1, 5)).astype(np.float32)
    lib.igo_rope_turn(igo_mod.fptr(v), 8, igo_mod.fptr(cs), igo_mod.fptr(sn))
    np.testing.assert_allclose(v[:4], keep[:4] * cs - keep[4:] * sn, atol=1e-5)
    np.testing.assert_allclose(v[4:], keep[4:] * cs + keep[:4] * sn, atol=1e-5)
    back = -sn
    lib.igo_rope_turn(igo_mod.fptr(v), 8, igo_mod.fptr(cs), igo_mod.fptr(back))
    np.testing.assert_allclose(v, keep, atol=1e-4)


def test_norm_weight_used_directly(igo_mod):
    lib = igo_mod.igo_lib()
    x = np.array([1, 2, 3, 4], np.float32)
    w = np.array([0.5, -1, 2, 0.25], np.float32)
    out = np.zeros(4, np.float32)
    lib.igo_norm_rms(igo_mod.fptr(x), igo_mod.fptr(w), 4, 1e-6, igo_mod.fptr(out))
    turn = 1 / math.sqrt((1 + 4 + 9 + 16) / 4 + 1e-6)
    np.testing.assert_allclose(out, x * turn * w, atol=1e-5)
    lib.igo_norm_rms(igo_mod.fptr(x), None, 4, 1e-6, igo_mod.fptr(out))
    assert out[0] == pytest.approx(turn, abs=1e-5)


def test_proportional_rope_turns_a_quarter(igo_mod):
    lib = igo_mod.igo_lib()
    steps = np.zeros(128, np.float32)
    turn = ctypes.c_int()
    lib.igo_rope_steps(1e6, 0.25, 1, 256, igo_mod.fptr(steps), ctypes.byref(turn))
    assert turn.value == 32
    assert np.all(steps[32:] == 0) and np.all(steps[:32] > 0)
    assert steps[1] == np.float32(1.0 / 1e6 ** (2 / 256))


# ---- app_test.c:4654 test_scout (the oracle's and the product's) ----------------

SCOUT_CASES = [
    ([1, 2, 3, 4, 5, 6, 7, 8, 9], 4, []),
    ([1, 2, 3, 4, 5, 6, 7, 8, 9, 4, 5, 6], 4, [7, 8, 9, 4]),
    ([1, 2, 3, 4, 5, 6, 7, 8, 9, 4, 5, 6], 2, [7, 8]),
    ([7, 8, 9, 1], 3, []),
    ([5, 9, 3, 3, 4, 9, 7, 7, 7, 9], 2, []),
    ([5, 8, 9, 3, 4, 8, 9, 7, 1, 8, 9], 2, [7, 1]),
    ([7, 1, 2, 3, 5, 9, 2, 3, 6, 4, 1, 2, 3], 1, [5]),
    (list(np.arange(5000) % 977), 4, list((np.arange(5000) % 977)[5000 - 977:5000 - 977 + 4])),
]


@pytest.mark.parametrize("stream,want,expect", SCOUT_CASES)
def test_scout_known_answers(igo_mod, igc_lib, stream, want, expect):
    lib = igo_mod.igo_lib()
    s = lib.igo_scout_open()
    a = np.array(stream, np.int32)
    assert lib.igo_scout_note(s, igo_mod.iptr(a), len(a)) == 0
    out = np.zeros(8, np.int32)
    n = lib.igo_scout_draw(s, igo_mod.iptr(out), want)
    assert list(out[:n]) == list(expect)
    lib.igo_scout_close(s)
    # the product's host-C scout answers the same
    sc = igc_lib.Scout()
    sc.note(a)
    assert list(sc.draw(want)) == list(expect)
    assert sc.span == len(a)


def test_scout_edges(igc_lib):
    sc = igc_lib.Scout()
    assert len(sc.draw(4)) == 0
    assert len(sc.draw(0)) == 0
    sc.note([1, 2, 3, 1, 2, 3])
    sc.clear()
    assert sc.span == 0


# ---- the restatement against the reference itself ---------------------------------

def _pair(igo, folder, window=256):
    rm = igo.RefModel(folder, threads=4)
    om = igo.OracleModel(folder, window_limit=window)
    return rm, om


@pytest.mark.parametrize("which", ["tiny", "small", "literal"])
def test_oracle_matches_reference_engine(igo_mod, which, tiny_dir, small_dir, literal_dir):
    igo = igo_mod
    folder = {"tiny": tiny_dir, "small": small_dir, "literal": literal_dir}[which]
    cfg = {"tiny": TINY, "small": SMALL, "literal": LITERAL}[which]
    rm, om = _pair(igo, folder, cfg["window_limit"])
    rs, os_ = igo.RefSession(rm), igo.OracleSession(om, threads=4)
    rng = np.random.default_rng(1)
    ids = rng.integers(0, cfg["vocab"], 45).astype(np.int32)  # laps the sliding window
    rs.prime(ids)
    os_.prime(ids)
    r = rs.step(ids[-1])
    o = os_.step(ids[-1])
    scale = max(1.0, float(np.abs(r).max()))
    assert np.abs(r - o).max() <= 1e-4 * scale
    assert r.argmax() == o.argmax()
    limit = min(4, cfg["slide_span"])
    blk = np.array([r.argmax()] + list(rng.integers(0, cfg["vocab"], limit - 1)), np.int32)
    rr, oo = rs.guess(blk), os_.guess(blk)
    assert np.abs(rr - oo).max() <= 1e-4 * scale
    assert rs.keep(2) == 0 and os_.guess_keep(2) == 0
    assert rs.fill == os_.fill == len(ids) + 2
    r2, o2 = rs.step(7), os_.step(7)
    assert np.abs(r2 - o2).max() <= 1e-4 * scale
    rm.close()


def test_partial_keep_matches_stepping(igo_mod, small_dir):
    """app_test.c:4600: a kept block equals the same ids stepped, within 1e-3."""
    igo = igo_mod
    om = igo.OracleModel(small_dir, window_limit=512)
    a, b = igo.OracleSession(om, threads=4), igo.OracleSession(om, threads=4)
    seed = np.array([1, 7, 8, 9, 10, 11, 12, 13, 7, 8, 9, 10, 11], np.int32)
    want = np.array([12, 13, 7, 8], np.int32)
    for s in (a, b):
        s.prime(seed)
        s.step(seed[-1])
    rows = a.guess(want)
    assert a.guess_keep(2) == 0
    for t in want[:2]:
        last = b.step(t)
    assert np.abs(rows[1] - last).max() <= 1e-3
    assert a.fill == b.fill


def test_dropped_block_reruns_bit_identical(igo_mod, tiny_dir):
    igo = igo_mod
    om = igo.OracleModel(tiny_dir, window_limit=256)
    s = igo.OracleSession(om, threads=4)
    s.prime(np.arange(1, 30, dtype=np.int32))
    s.step(29)
    blk = np.array([12, 13, 7, 8], np.int32)
    first = s.guess(blk)
    assert s.guess_keep(0) == 0
    again = s.guess(blk)
    assert np.array_equal(first, again)
    assert s.guess_keep(0) == 0


def test_taste_matches_reference_engine(igo_mod, tiny_dir):
    """The rejection rule is the reference's arithmetic: same rows, same seed,
    same kept count and same drawn token."""
    igo = igo_mod
    rm, om = _pair(igo, tiny_dir)
    rs, os_ = igo.RefSession(rm), igo.OracleSession(om, threads=4)
    ids = np.arange(3, 33, dtype=np.int32)
    rs.prime(ids)
    os_.prime(ids)
    rs.step(ids[-1])
    os_.step(ids[-1])
    blk = np.array([5, 9, 11], np.int32)
    rows = rs.guess(blk)
    os_.guess(blk)
    for case in range(3):
        t = igo.Taste(0.8, 64, 0.95, 1.0, 64, 0)
        if case == 1:
            t = igo.Taste(1.0, 12, 0.9, 1.4, 64, 0)
        if case == 2:
            t = igo.Taste(1.2, 0, 1.0, 1.0, 64, 0)
        for seed in range(200):
            t.seed = seed * 2654435761 + 12345
            assert rs.taste(rows, blk, t) == os_.guess_taste(rows, blk, t)
    rm.close()


def test_rejection_rule_draws_the_plain_distribution(igo_mod, tiny_dir):
    """app_test.c:4410: the token committed at position 0 over many seeds is
    distributed as the plain sampler's shaped row (bar 0.01, >4 sigma)."""
    igo = igo_mod
    lib = igo.igo_lib()
    om = igo.OracleModel(tiny_dir, window_limit=256)
    s = igo.OracleSession(om, threads=4)
    s.prime(np.arange(1, 14, dtype=np.int32))
    s.step(13)
    look = igo.Taste(1.0, 12, 0.9, 1.0, 64, 1)
    rows = s.guess(np.array([12], np.int32))
    ids_room = np.zeros(512, np.int32)
    w_room = np.zeros(512, np.float32)
    echo = np.zeros(1, np.int32)
    keep = lib.igo_pick_shape(igo.fptr(rows[0]), 512, ctypes.byref(look), igo.iptr(echo), 0,
                              igo.iptr(ids_room), igo.fptr(w_room))
    guess_id = int(ids_room[keep // 2])
    s.guess_keep(0)
    blk = np.array([12, guess_id, 3], np.int32)
    rows = s.guess(blk)
    n = 40000
    for case, rule in enumerate([igo.Taste(1.0, 0, 1.0, 1.0, 64, 0), igo.Taste(1.0, 12, 0.9, 1.4, 64, 0)]):
        # the history lane 0 is judged against: every id fed before the block
        # (the prompt 1..12 and the stepped 13), plus the block's own first id
        e = np.concatenate([np.arange(1, 14), [12]]).astype(np.int32)
        keep = lib.igo_pick_shape(igo.fptr(rows[0]), 512, ctypes.byref(rule), igo.iptr(e), len(e),
                                  igo.iptr(ids_room), igo.fptr(w_room))
        want = np.zeros(512)
        want[ids_room[:keep]] = w_room[:keep]
        tally = np.zeros(512)
        takes = 0
        for r in range(n):
            rule.seed = r * 2654435761 + 12345
            take, made = s.guess_taste(rows, blk, rule)
            assert 0 <= take <= 2
            takes += take
            tally[blk[1] if take >= 1 else made] += 1
        assert 0 < takes < 2 * n
        assert np.abs(tally / n - want).max() < 0.01, case
    s.guess_keep(0)


def test_rejection_rule_edges(igo_mod, tiny_dir):
    """app_test.c:4522-4598: a cut guess is never kept, a whole-mass guess
    always is, and greedy is refused."""
    igo = igo_mod
    lib = igo.igo_lib()
    om = igo.OracleModel(tiny_dir, window_limit=256)
    s = igo.OracleSession(om, threads=4)
    s.prime(np.arange(1, 14, dtype=np.int32))
    s.step(13)
    rule = igo.Taste(1.0, 1, 1.0, 1.0, 64, 0)
    rows = s.guess(np.array([12], np.int32))
    best = int(rows[0].argmax())
    other = 1 if best == 0 else 0
    s.guess_keep(0)
    rows = s.guess(np.array([12, other], np.int32))
    total = 0
    for r in range(256):
        rule.seed = r * 6364136223846793005 + 1
        total += s.guess_taste(rows, np.array([12, other], np.int32), rule)[0]
    assert total == 0
    s.guess_keep(0)
    blk = np.array([12, best], np.int32)
    rows = s.guess(blk)
    for r in range(256):
        rule.seed = r * 6364136223846793005 + 1
        take, made = s.guess_taste(rows, blk, rule)
        assert take == 1
    greedy = igo.Taste(0.0, 64, 0.95, 1.0, 64, 0)
    assert s.guess_taste(rows, blk, greedy)[0] < 0
    s.guess_keep(0)


def test_dropin_build_exports_the_shim():
    """oracle/_ref/libref_cuda.so, the reference with its backend table on
    libigllm_cuda (oracle/app_cuda.c), loads here and exports the reference's
    wrappers plus the CUDA load entry (nothing is called without a GPU)."""
    import os
    import igo
    if not os.path.exists(igo.REF_CUDA_PATH):
        pytest.skip("built only where the reference source and the CUDA library are both present")
    lib = ctypes.CDLL(igo.REF_CUDA_PATH)
    for name in ("ref_model_load_cuda", "ref_cuda_status", "ref_cuda_close", "ref_desk_name", "ref_model_load",
                 "ref_session_guess", "ref_session_keep"):
        assert hasattr(lib, name), name
