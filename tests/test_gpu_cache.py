"""The 8-bit cache and cache files on the GPU, against the reference engine.

  * model_memory_bytes and each layer's cache scales equal the reference's;
  * with cache_bits 8, a prime through the tcgen05 chunk path leaves layer
    0's codes exactly the reference's and layer 1's but at rounding ties of
    the grid; over the same cache, blocks of 1, 4 and 16 lanes match the
    reference's own 8-bit engine within 2e-2, and the peaks match;
  * the codes this library stores are the reference's grid of the float
    rows: a float session and a byte session primed alike, layer 0's codes
    equal cache_code8(row / scale) of the float rows, bit for bit;
  * files cross both ways: the reference loads this library's file and this
    library loads the reference's, at a fill where the 64-row rings have
    turned over, float and byte, and each side's continuation matches the
    other's; a file loaded back into this library continues bit-identically;
  * refusals: other shapes or storage (IGC_FAIL_STATE), damage
    (IGC_FAIL_FORMAT, session cleared), a missing file, a block in flight,
    a bad kind or note, and hold below the rows a turned-over file carried;
  * a block undone whole leaves the peaks as they were; crowd rounds over
    byte caches agree with lone rounds within the bar, and a session's crowd
    results are the same bits shared or alone.
"""

import numpy as np
import pytest

from conftest import CACHED
from test_cache_files import parse_cache_file

pytestmark = pytest.mark.gpu

ATOL = 2e-2
WINDOW = CACHED["window_limit"]
VOCAB = CACHED["vocab"]
FILL = 300  # past every 64-row ring


def _ids(n, seed):
    return np.random.default_rng(seed).integers(0, VOCAB, n).astype(np.int32)


@pytest.fixture(scope="module")
def models(igc_lib, igo_mod, cached_dir):
    out = {}
    for bits in (0, 8):
        out[bits] = (igc_lib.Model(folder=cached_dir, window_limit=WINDOW, cache_bits=bits),
                     igo_mod.RefModel(cached_dir, threads=8, window_limit=WINDOW, cache_bits=bits))
    yield out
    for m, rm in out.values():
        m.close()
        rm.close()


def test_memory_bytes_and_scales_match_reference(models):
    m, rm = models[8]
    assert m.memory_bytes() == rm.memory_bytes()
    for l in range(CACHED["layers"]):
        for side in (0, 1):
            assert m.cache_scale(l, side) == rm.cache_scale(l, side)
    assert m.cache_scale(0, 0) > 0 and m.cache_scale(9, 0) == 0  # owners only
    s = __import__("igllm_b200").Session(m)
    float_room = s.cache_room(0)
    assert s.cache_room() < float_room  # six owners' sides in bytes
    s.close()


def _grid_rank(codes):
    """A code's place on the signed grid (code 0x80, minus zero, ranks with 0)."""
    c = codes.astype(np.int32)
    mag = c & 0x7F
    return np.where(c & 0x80, -mag, mag)


def test_byte_cache_matches_reference(igc_lib, igo_mod, models, tmp_path):
    """Primed alike (this library through the tcgen05 chunk path), the two
    engines' byte caches differ only at rounding ties of the grid: their float
    rows differ in the last bits (products summed in different orders), so a
    value that close to a boundary between two codes can land on either.
    Layer 0's rows come from the embedding alone and their codes are the
    reference's exactly; layer 1's differ, where they do, by one step and
    rarely.  From there a tie flipped in one layer moves the next layer's
    inputs by more than float rounding would, and deeper codes drift further
    apart, in the reference's own engine just as much: the reference run over
    this library's cache lands where this library does (within 2e-2), and its
    distance from the reference over its own cache is reported beside.  Blocks
    of 1, 4 and 16 lanes from the same cache agree within 2e-2, and the peaks
    agree."""
    m, rm = models[8]
    ids = _ids(FILL + 1, 1)
    s = igc_lib.Session(m)
    rs = igo_mod.RefSession(rm)
    s.prime(ids)
    rs.prime(ids)
    for l in range(CACHED["layers"]):
        for side in (0, 1):
            a, b = s.cache_peak(l, side), rs.cache_peak(l, side)
            assert abs(a - b) <= 1e-3 * max(1.0, abs(b)), (l, side, a, b)
    mine, theirs = str(tmp_path / "mine.keep"), str(tmp_path / "theirs.keep")
    s.save(mine)
    assert rs.save(theirs) == 0
    fm, fr = parse_cache_file(mine, CACHED, WINDOW, 8), parse_cache_file(theirs, CACHED, WINDOW, 8)
    for side in (0, 1):
        assert np.array_equal(fm["rows"][0][side], fr["rows"][0][side])
        d = np.abs(_grid_rank(fm["rows"][1][side]) - _grid_rank(fr["rows"][1][side]))
        assert d.max() <= 1 and (d > 0).sum() <= 1e-3 * d.size, (side, int(d.max()), int((d > 0).sum()))
    # every engine and cache over the same blocks
    over_mine = igo_mod.RefSession(rm)
    assert over_mine.load(mine)[0] == 0
    worst = drift = 0.0
    tok = int(ids[-1])
    for k in (1, 4, 16):
        block = np.concatenate([[tok], _ids(k - 1, 100 + k)]).astype(np.int32)
        got = s.guess(block)
        same_cache = over_mine.guess(block)
        own_cache = rs.guess(block)
        worst = max(worst, float(np.abs(got - same_cache).max()))
        drift = max(drift, float(np.abs(same_cache - own_cache).max()))
        s.guess_keep(k)
        assert over_mine.keep(k) == 0 and rs.keep(k) == 0
        tok = int(own_cache[-1].argmax())
    print(f"8-bit cache: worst |logit diff| vs the reference over this library's cache {worst:.3e}; "
          f"the reference over its own cache vs over this library's {drift:.3e}")
    assert worst < ATOL
    s.close()
    over_mine.close()
    rs.close()


def test_codes_are_the_grid_of_float_rows(igc_lib, igo_mod, models, tmp_path):
    """Layer 0's rows depend only on the embedding, so a float session and a
    byte session hold the same rows there; the byte session's codes must be
    the reference's cache_code8 of row / scale (float32 division)."""
    ids = _ids(FILL + 1, 2)
    files = {}
    for bits in (0, 8):
        s = igc_lib.Session(models[bits][0])
        s.prime(ids)
        files[bits] = str(tmp_path / f"b{bits}.keep")
        s.save(files[bits])
        s.close()
    f0 = parse_cache_file(files[0], CACHED, WINDOW, 0)
    f8 = parse_cache_file(files[8], CACHED, WINDOW, 8)
    m8 = models[8][0]
    for side in (0, 1):
        rows = f0["rows"][0][side].astype(np.float32)
        scale = np.float32(m8.cache_scale(0, side))
        want = igo_mod.ref_cache_code8((rows / scale).ravel())
        got = f8["rows"][0][side].ravel()
        assert np.array_equal(got, want), int((got != want).sum())


@pytest.mark.parametrize("bits", [0, 8])
@pytest.mark.parametrize("fill", [40, FILL])
def test_files_cross_both_ways(igc_lib, igo_mod, models, tmp_path, bits, fill):
    m, rm = models[bits]
    ids = _ids(fill + 1, 3 + fill)
    block = np.concatenate([ids[-1:], _ids(3, 7)]).astype(np.int32)
    note = igc_lib.KeepNote()
    note.run_count = 1
    note.from_list[0], note.till_list[0], note.mark_list[0] = 2, 6, 12345
    # this library writes, the reference reads and continues
    s = igc_lib.Session(m)
    s.prime(ids)
    mine = str(tmp_path / "mine.keep")
    s.save(mine, stamp=42, note=note, kind=igc_lib.KEEP_TALK)
    rs = igo_mod.RefSession(rm)
    code, stamp, back, kind = rs.load(mine)
    assert (code, stamp, kind, rs.fill) == (0, 42, 1, fill)
    assert back.run_count == 1 and back.mark_list[0] == 12345
    assert np.array_equal(rs.ids(), ids[:-1])
    want = rs.guess(block)
    got = s.guess(block)
    print(f"bits {bits} fill {fill}: reference continuing this library's file, worst {np.abs(got - want).max():.3e}")
    assert np.abs(got - want).max() < ATOL
    s.guess_keep(0)
    rs.keep(0)
    # the reference writes, this library reads and continues
    rs2 = igo_mod.RefSession(rm)
    rs2.prime(ids)
    theirs = str(tmp_path / "theirs.keep")
    assert rs2.save(theirs, stamp=7, kind=0) == 0
    s2 = igc_lib.Session(m)
    stamp, back, kind = s2.load(theirs)
    assert (stamp, kind, s2.fill, back.run_count) == (7, 0, fill, 0)
    assert np.array_equal(s2.ids(), ids[:-1])
    for l in range(CACHED["layers"]):
        assert s2.cache_peak(l, 0) == rs2.cache_peak(l, 0)
        assert s2.cache_peak(l, 1) == rs2.cache_peak(l, 1)
    want = rs2.guess(block)
    got = s2.guess(block)
    print(f"bits {bits} fill {fill}: this library continuing the reference's file, worst "
          f"{np.abs(got - want).max():.3e}")
    assert np.abs(got - want).max() < ATOL
    # this library's own file back into a fresh session continues exactly
    s3 = igc_lib.Session(m)
    s3.load(mine)
    again = s3.guess(block)
    s.hold(fill)
    direct = s.guess(block)
    assert np.array_equal(again, direct)
    for x in (s, s2, s3):
        x.close()
    for x in (rs, rs2):
        x.close()


def test_refusals(igc_lib, models, cached_dir, tmp_path):
    m, _ = models[8]
    ids = _ids(FILL + 1, 9)
    s = igc_lib.Session(m)
    s.prime(ids)
    path = str(tmp_path / "a.keep")
    s.save(path)
    with pytest.raises(igc_lib.IgcError) as e:
        s.save(str(tmp_path / "b.keep"), kind=2)
    assert e.value.code == igc_lib.FAIL_ARGUMENT
    bad = igc_lib.KeepNote()
    bad.run_count = 1
    bad.from_list[0], bad.till_list[0] = 5, 5  # an empty run
    with pytest.raises(igc_lib.IgcError) as e:
        s.save(str(tmp_path / "b.keep"), note=bad)
    assert e.value.code == igc_lib.FAIL_ARGUMENT
    # a block in flight
    s.guess(np.array([1, 2], np.int32), want_logits=False)
    for call in (lambda: s.save(path), lambda: s.load(path)):
        with pytest.raises(igc_lib.IgcError) as e:
            call()
        assert e.value.code == igc_lib.FAIL_STATE
    s.guess_keep(0)
    # other storage, other window
    for other in (models[0][0], None):
        close = other is None
        if close:
            other = igc_lib.Model(folder=cached_dir, window_limit=512, cache_bits=8)
        t = igc_lib.Session(other)
        with pytest.raises(igc_lib.IgcError) as e:
            t.load(path)
        assert e.value.code == igc_lib.FAIL_STATE
        t.close()
        if close:
            other.close()
    # damage: cut short, bad text; missing
    with open(path, "rb") as f:
        data = f.read()
    t = igc_lib.Session(m)
    t.prime(_ids(20, 1))
    for name, blob in (("cut", data[:-9]), ("text", b"x" + data[1:])):
        p = str(tmp_path / f"{name}.keep")
        with open(p, "wb") as f:
            f.write(blob)
        with pytest.raises(igc_lib.IgcError) as e:
            t.load(p)
        assert e.value.code == igc_lib.FAIL_FORMAT
    assert t.fill == 0  # the cut file's read stopped half way: cleared
    with pytest.raises(igc_lib.IgcError) as e:
        t.load(str(tmp_path / "none.keep"))
    assert e.value.code == igc_lib.FAIL_MISSING
    # a turned-over file carries the last 64 rows of the sliding owners
    t.load(path)
    t.hold(FILL - 1)  # its window still lies inside what the file carried
    with pytest.raises(igc_lib.IgcError) as e:
        t.hold(FILL - 2)
    assert e.value.code == igc_lib.FAIL_SUPPORT
    t.hold(0)
    t.prime(_ids(30, 2))
    t.hold(10)  # a fresh start has every row again
    s.close()
    t.close()


def test_undone_block_restores_peaks(igc_lib, igo_mod, models):
    m, rm = models[8]
    ids = _ids(120, 11)
    s = igc_lib.Session(m)
    rs = igo_mod.RefSession(rm)
    s.prime(ids)
    rs.prime(ids)
    before = [(s.cache_peak(l, 0), s.cache_peak(l, 1)) for l in range(6)]
    block = (np.arange(16) * 131 % VOCAB).astype(np.int32)
    s.guess(block, want_logits=False)
    rs.guess(block, want=False)
    grew = [(s.cache_peak(l, 0), s.cache_peak(l, 1)) for l in range(6)]
    assert all(g[0] >= b[0] and g[1] >= b[1] for g, b in zip(grew, before))
    s.guess_keep(0)
    rs.keep(0)
    assert [(s.cache_peak(l, 0), s.cache_peak(l, 1)) for l in range(6)] == before
    for l in range(6):
        assert abs(s.cache_peak(l, 0) - rs.cache_peak(l, 0)) <= 1e-4 * max(1.0, rs.cache_peak(l, 0))
    s.close()
    rs.close()


def test_crowd_over_byte_caches(igc_lib, models):
    """Crowd rounds over byte caches: each session's lanes agree with its own
    16-lane guess within the bar, its peaks with the lone session's, and a
    session's results are the same bits whether its round is shared or not."""
    m, _ = models[8]
    k = 4
    prompts = [_ids(150 + 37 * j, 20 + j) for j in range(3)]
    lone, shared, single = [], [], []
    for p in prompts:
        trio = [igc_lib.Session(m) for _ in range(3)]
        for t in trio:
            t.prime(p)
        lone.append(trio[0])
        shared.append(trio[1])
        single.append(trio[2])
    blocks = np.stack([np.concatenate([p[-1:], _ids(k - 1, 40 + j)]) for j, p in enumerate(prompts)]).astype(np.int32)
    cr = igc_lib.Crowd(m, 3, k)
    _, _, rows = cr.round(shared, blocks, want_logits=True)
    for j in range(3):
        want = lone[j].guess(blocks[j])
        err = float(np.abs(rows[j * k:(j + 1) * k] - want).max())
        assert err <= ATOL and err <= 2e-4 * max(1.0, float(np.abs(want).max())), (j, err)
        for l in range(6):
            for side in (0, 1):
                a, b = shared[j].cache_peak(l, side), lone[j].cache_peak(l, side)
                assert abs(a - b) <= 1e-4 * max(1.0, b), (j, l, side, a, b)
        _, _, one = cr.round([single[j]], blocks[j:j + 1], want_logits=True)
        assert np.array_equal(one, rows[j * k:(j + 1) * k])
    cr.close()
    for x in lone + shared + single:
        x.close()
