"""The batched-lane path (igc_lanes.cu) on the GPU: the tcgen05 int4 GEMM.

A product of 64 or more lanes through the backend table's mat_mat runs as the
tcgen05 GEMM: staged activations and (code - 8) * scale weights, each split
into f16 hi and lo parts, in shared memory, three tcgen05.mma products a
16-column step into f32 accumulators in tensor memory, K slices added in a
fixed order.  Checked against the CPU checker's igo_mat_mat (the restatement
of app_core.c:3688 kern_row_code, fp32).  Tolerance: 2e-4 of each lane's
largest output magnitude (the hi/lo split keeps about 22 bits of every
activation and every weight exactly; the rest is f32 summation order), the
same relative bar the decode path's tests hold; the verify round's logits
are held to 2e-2 absolute.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL = 2e-4


def _plane(igc_lib, rng, rows, cols):
    code = rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8)
    sc16 = np.abs(rng.normal(0, 0.02, (rows, cols // 32))).astype(np.float16)
    plane = igc_lib.IgcPlane(form=2, row_count=rows, col_count=cols, code_data=code.ctypes.data,
                             row_stride=cols // 2, gain_data=sc16.ctypes.data, gain_type=2, bit_count=4,
                             code_bias=8, code_flip=0, group_size=32, group_count=cols // 32)
    return plane, code, sc16


@pytest.mark.parametrize("rows,cols,lanes", [
    (37, 96, 200),      # one partial row tile, a partial last column step, a partial second lane tile
    (300, 1536, 64),    # the fewest lanes the path takes
    (2560, 1536, 256),  # q|k|v of the E2B shape, two full lane tiles
    (1536, 6144, 130),  # the down projection: eight K slices
    (256, 1536, 512),   # the per-layer-embedding gate: one row tile, four lane tiles
])
def test_lane_gemm_matches_the_checker(igc_lib, igo_mod, rows, cols, lanes):
    rng = np.random.default_rng(rows + cols + lanes)
    plane, code, sc16 = _plane(igc_lib, rng, rows, cols)
    act = rng.normal(0, 1, (lanes, cols)).astype(np.float32)
    act[3] *= 1000.0  # lanes of very different magnitude each take their own staging scale
    act[5] *= 1e-3
    desk = igc_lib.Desk(0)
    try:
        got = desk.mat_mat(plane, act, lanes, rows)
        again = desk.mat_mat(plane, act, lanes, rows)
    finally:
        desk.close()
    lib = igo_mod.igo_lib()
    sc32 = sc16.astype(np.float32)  # kept alive: the plane holds its pointer
    op = igo_mod.make_plane(code, sc32)
    want = np.zeros((lanes, rows), np.float32)
    lib.igo_mat_mat(ctypes.byref(op), igo_mod.fptr(act), cols, lanes, igo_mod.fptr(want), rows, 8)
    assert np.array_equal(got, again)  # fixed-order sums: the same bits every call
    for j in range(lanes):  # each lane against its own magnitude
        err = float(np.abs(got[j] - want[j]).max())
        assert err <= REL * max(1e-30, float(np.abs(want[j]).max())), (j, err)


@pytest.mark.parametrize("which", ["tiny", "small", "wide"])
def test_chunked_prime_matches_the_checker(igc_lib, igo_mod, which, tiny_dir, small_dir, wide_dir):
    """A prompt of 64 or more ids primes in chunks of up to 512 lanes through
    the tcgen05 path (every projection a lane GEMM, attention in 16-lane
    groups in position order); what it leaves in the caches must give the
    checker's logits on the step, the block and the step after a keep that
    follow it, within 2e-2 (and 2e-4 of the row's magnitude)."""
    from conftest import SMALL, TINY, WIDE
    folder, cfg = {"tiny": (tiny_dir, TINY), "small": (small_dir, SMALL), "wide": (wide_dir, WIDE)}[which]
    m = igc_lib.Model(folder=folder, window_limit=cfg["window_limit"])
    om = igo_mod.OracleModel(folder, window_limit=cfg["window_limit"])
    s, o = igc_lib.Session(m), igo_mod.OracleSession(om, threads=8)
    rng = np.random.default_rng(31)
    n = min(cfg["window_limit"] - 40, 300)
    ids = rng.integers(0, cfg["vocab"], n).astype(np.int32)
    # a chunk of n - 41 lanes, then 40 lanes by 16-lane passes (a second
    # prime continuing from the first one's last id)
    for part in (ids[:n - 40], ids[n - 41:]):
        s.prime(part)
        o.prime(part)
    assert s.fill == o.fill == n - 1

    def close(got, want):
        err = float(np.abs(got - want).max())
        assert err <= 2e-2 and err <= 2e-4 * max(1.0, float(np.abs(want).max())), err

    top, row = s.step(ids[-1])
    close(row, o.step(ids[-1]))
    blk = np.array([top] + rng.integers(0, cfg["vocab"], 3).tolist(), np.int32)
    close(s.guess(blk), o.guess(blk))
    s.guess_keep(2)
    o.guess_keep(2)
    _, row = s.step(9)
    close(row, o.step(9))


def test_prime_attention_at_every_cluster_size(igc_lib, igo_mod, small_dir, monkeypatch):
    """A prime chunk's attention splits each 16-row block's positions over a
    cluster of 1, 2, 4, 8 or 16 blocks (the light layout, two blocks an SM,
    at up to 4); every size must leave caches that give the checker's logits
    within 2e-2 and 2e-4 of the row's magnitude.  Only the split of the sums
    over positions changes with the size."""
    from conftest import SMALL
    cfg = SMALL
    m = igc_lib.Model(folder=small_dir, window_limit=cfg["window_limit"])
    om = igo_mod.OracleModel(small_dir, window_limit=cfg["window_limit"])
    o = igo_mod.OracleSession(om, threads=8)
    rng = np.random.default_rng(47)
    n = min(cfg["window_limit"] - 8, 300)
    ids = rng.integers(0, cfg["vocab"], n).astype(np.int32)
    o.prime(ids)
    want = o.step(ids[-1])
    for cx in (1, 2, 4, 8, 16):
        monkeypatch.setenv("IGC_CHUNK_CLUSTER", str(cx))
        monkeypatch.setenv("IGC_CHUNK_CLUSTER_GLOBAL", str(cx))
        s = igc_lib.Session(m)  # the sizes are read when a session opens
        s.prime(ids)
        _, row = s.step(ids[-1])
        err = float(np.abs(row - want).max())
        assert err <= 2e-2 and err <= 2e-4 * max(1.0, float(np.abs(want).max())), (cx, err)
        s.close()


def test_crowd_round_matches_each_session_alone(igc_lib, small_dir):
    """Five sessions at different positions verify a block of four in one
    crowd round: every lane's logits agree with the session's own guess (the
    16-lane path) within 2e-2 and 2e-4 of the row's magnitude, the argmax ids
    agree wherever the top-2 gap is above 2e-2, each session keeps its
    leading matches as igc_session_round would, and a session's results do
    not depend on how many sessions share the round."""
    from conftest import SMALL
    m = igc_lib.Model(folder=small_dir, window_limit=SMALL["window_limit"])
    rng = np.random.default_rng(41)
    prompts = [rng.integers(0, SMALL["vocab"], n).astype(np.int32) for n in (20, 33, 70, 90, 131)]
    crowd_s = [igc_lib.Session(m) for _ in prompts]
    alone_s = [igc_lib.Session(m) for _ in prompts]
    for s, t, p in zip(crowd_s, alone_s, prompts):
        s.prime(p)
        t.prime(p)
    blocks = []
    for t, p in zip(alone_s, prompts):
        top, _ = t.step(p[-1], want_logits=False)
        blocks.append([p[-1], top] + rng.integers(0, SMALL["vocab"], 2).tolist())  # the first guess is right
        t.hold(t.fill - 1)
    blocks = np.array(blocks, np.int32)
    crowd = igc_lib.Crowd(m, 8, 4)
    takes, mades, rows = crowd.round(crowd_s, blocks, want_logits=True)
    for j, (t, blk) in enumerate(zip(alone_s, blocks)):
        want = t.guess(blk)
        got = rows[4 * j: 4 * j + 4]
        err = float(np.abs(got - want).max())
        assert err <= 2e-2 and err <= 2e-4 * max(1.0, float(np.abs(want).max())), (j, err)
        top = want.argmax(1)
        take = 0
        while take + 1 < 4 and top[take] == blk[take + 1]:
            take += 1
        gaps = np.sort(want, 1)[:, -2:]
        if (gaps[:, 1] - gaps[:, 0] > 2e-2).all():
            assert takes[j] == take and mades[j] == top[take], (j, takes[j], take)
        t.guess_keep(int(takes[j]) + 1)
        assert crowd_s[j].fill == t.fill
    assert (takes >= 1).all()
    # the same sessions one at a time through the crowd: the same bits
    for s, t in zip(crowd_s, alone_s):
        s.hold(t.fill - int(takes[crowd_s.index(s)]) - 1)
    solo = np.concatenate([crowd.round([s], blocks[j:j + 1], want_logits=True)[2] for j, s in enumerate(crowd_s)])
    assert np.array_equal(solo, rows)
    crowd.close()


def test_crowd_refuses_what_it_cannot_run(igc_lib, small_dir, tiny_dir):
    """A crowd round refuses, before anything runs and leaving every session
    as it was: a session named twice, a session with a block in flight, a
    session of another model, a full window and more sessions than the crowd
    holds; a crowd is refused blocks past 16 lanes or 512 lanes in all."""
    from conftest import SMALL, TINY
    m = igc_lib.Model(folder=small_dir, window_limit=SMALL["window_limit"])
    other = igc_lib.Model(folder=tiny_dir, window_limit=TINY["window_limit"])
    a, b = igc_lib.Session(m), igc_lib.Session(m)
    for s in (a, b):
        s.prime(np.arange(3, 30, dtype=np.int32))
    crowd = igc_lib.Crowd(m, 2, 4)
    blk = np.array([[29, 1, 2, 3], [29, 4, 5, 6]], np.int32)

    def refused(sessions, blocks, code):
        fills = [s.fill for s in sessions]
        with pytest.raises(igc_lib.IgcError) as e:
            crowd.round(sessions, blocks)
        assert e.value.code == code
        assert [s.fill for s in sessions] == fills

    refused([a, a], blk, igc_lib.FAIL_ARGUMENT)
    refused([a, igc_lib.Session(other)], blk, igc_lib.FAIL_ARGUMENT)
    refused([a, b, igc_lib.Session(m)], np.tile(blk[:1], (3, 1)), igc_lib.FAIL_ARGUMENT)
    b.guess(np.array([29, 7], np.int32), want_logits=False)
    refused([a, b], blk, igc_lib.FAIL_STATE)
    b.guess_keep(0)
    full = igc_lib.Session(m)
    full.prime(np.arange(SMALL["window_limit"] - 2, dtype=np.int32) % SMALL["vocab"])
    refused([a, full], blk, igc_lib.FAIL_STATE)
    take, made, _ = crowd.round([a, b], blk)  # the same sessions, unrefused, still run
    assert a.fill == 26 + take[0] + 1 and b.fill == 26 + take[1] + 1  # primed to 26, then take + 1 kept
    crowd.close()
    for limit, k in ((4, 17), (64, 16), (0, 4)):  # a block past 16 lanes, past 512 lanes in all, no room
        with pytest.raises(igc_lib.IgcError) as e:
            igc_lib.Crowd(m, limit, k)
        assert e.value.code == igc_lib.FAIL_ARGUMENT


def test_crowd_of_any_size(igc_lib, small_dir):
    """Crowds whose lane and session counts put their tables at odd offsets
    (3 sessions of 5 lanes, 5 of 3) run, and each session's rows are the same
    bits shared or alone."""
    from conftest import SMALL
    m = igc_lib.Model(folder=small_dir, window_limit=SMALL["window_limit"])
    rng = np.random.default_rng(7)
    for n, k in ((3, 5), (5, 3)):
        prompts = [rng.integers(0, SMALL["vocab"], 30 + 11 * j).astype(np.int32) for j in range(n)]
        shared = [igc_lib.Session(m) for _ in range(n)]
        alone = [igc_lib.Session(m) for _ in range(n)]
        for a, b, p in zip(shared, alone, prompts):
            a.prime(p)
            b.prime(p)
        blocks = np.stack([np.concatenate([p[-1:], rng.integers(0, SMALL["vocab"], k - 1)]) for p in prompts])
        crowd = igc_lib.Crowd(m, n, k)
        _, _, rows = crowd.round(shared, blocks.astype(np.int32), want_logits=True)
        for j in range(n):
            _, _, one = crowd.round([alone[j]], blocks[j:j + 1].astype(np.int32), want_logits=True)
            assert np.array_equal(one, rows[j * k:(j + 1) * k])
        crowd.close()
        for x in shared + alone:
            x.close()
    m.close()
