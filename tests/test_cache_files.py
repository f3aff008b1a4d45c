"""The byte cache's grid and the cache file format, on the CPU.

The oracle's restatement of the e4m3 grid (oracle/igo.c igo_cache_code8 /
igo_cache_real8) is pinned against the reference's own conversions
(app_core.c:10980-11035, through oracle/ref_harness.c) on every code and
on a sweep of floats, ties and special values.  The cache file layout this
library writes (igllm_b200/csrc/igc_runtime.cu, "cache files") is pinned
against files the reference engine itself saves: header, runs, ids, the
rows of each owner's ring and the peaks, byte for byte in size and order.
keep_note_share is this library's host C against the reference's.
"""

import os
import struct

import numpy as np
import pytest

from conftest import CACHED, make_checkpoint

KEEP_TEXT = b"igllm cache 4\n\x00\x00"


def layer_layout(cfg, window, cache_bits):
    """Per layer (span, key bytes a value, value bytes a value, row width) as
    the reference lays out its rings (app_core.c:8553-8562, :8723-8731)."""
    L, share = cfg["layers"], cfg["share_count"]
    first_share = L - share
    kinds = [1 if (l == L - 1 or (cfg["global_every"] > 0 and (l + 1) % cfg["global_every"] == 0)) else 0
             for l in range(L)]
    out = []
    for l in range(L):
        if share > 0 and l >= first_share:
            out.append((0, 4, 4, 0))
            continue
        last = max(q for q in range(first_share) if kinds[q] == kinds[l])
        keep_full = share > 0 and last == l
        span = window if (kinds[l] == 1 or keep_full) else min(cfg["slide_span"], window)
        kb = 1 if cache_bits == 8 and cfg.get("cache_scale_k", 0) > 0 else 4
        vb = 1 if cache_bits == 8 and cfg.get("cache_scale_v", 0) > 0 else 4
        out.append((span, kb, vb, cfg["kv_heads"] * cfg["head_dim"]))
    return out


def parse_cache_file(path, cfg, window, cache_bits):
    """The fields of a cache file, split by the layout above."""
    with open(path, "rb") as f:
        data = f.read()
    assert data[:16] == KEEP_TEXT
    head = struct.unpack_from("<7Q", data, 16)
    runs = struct.unpack_from("<Q", data, 72)[0]
    at = 80
    run_list = [struct.unpack_from("<3Q", data, at + 24 * i) for i in range(runs)]
    at += 24 * runs
    fill, held = head[2], head[3]
    ids = np.frombuffer(data, np.int32, held, at)
    at += 4 * held
    rows = {}
    for l, (span, kb, vb, width) in enumerate(layer_layout(cfg, window, cache_bits)):
        n = min(fill, span)
        if span == 0 or n < 1:
            continue
        kdt, vdt = (np.uint8 if kb == 1 else np.float32), (np.uint8 if vb == 1 else np.float32)
        k = np.frombuffer(data, kdt, n * width, at).reshape(n, width)
        at += n * width * kb
        v = np.frombuffer(data, vdt, n * width, at).reshape(n, width)
        at += n * width * vb
        rows[l] = (k, v)
    L = cfg["layers"]
    kpk = np.frombuffer(data, np.float32, L, at)
    vpk = np.frombuffer(data, np.float32, L, at + 4 * L)
    at += 8 * L
    assert at == len(data), (at, len(data))
    return dict(mark=head[0], stamp=head[1], fill=fill, held=held, layers=head[4], bits=head[5], kind=head[6],
                runs=run_list, ids=ids, rows=rows, key_peak=kpk, value_peak=vpk)


def test_cache_grid_matches_reference(igo_mod):
    lib = igo_mod.igo_lib()
    codes = np.arange(256, dtype=np.uint8)
    ref = igo_mod.ref_cache_real8(codes)
    mine = np.array([lib.igo_cache_real8(int(c)) for c in codes], np.float32)
    assert np.array_equal(ref.view(np.uint32), mine.view(np.uint32))
    grid = np.unique(np.abs(ref))
    mids = ((grid[1:] + grid[:-1]) / 2).astype(np.float32)
    rng = np.random.default_rng(0)
    parts = [rng.standard_normal(20000).astype(np.float32) * s for s in (1e-4, 1e-3, 0.02, 1, 30, 300, 3000)]
    parts += [mids, -mids, np.nextafter(mids, np.float32(1e9)), np.nextafter(mids, np.float32(0)),
              np.array([np.nan, -np.nan, np.inf, -np.inf, 0.0, -0.0, 448, -448, 464, 463.99, 1 / 64, 1 / 512,
                        1 / 1024, -1 / 1024, 3 / 1024, 2 ** -126, -2 ** -149], np.float32)]
    x = np.concatenate(parts)
    want = igo_mod.ref_cache_code8(x)
    got = np.array([lib.igo_cache_code8(float(v)) for v in x], np.uint8)
    bad = np.nonzero(want != got)[0]
    assert bad.size == 0, [(float(x[i]), int(want[i]), int(got[i])) for i in bad[:8]]
    # the round trip through the grid lands on the grid (app_core.c:11020)
    back = igo_mod.ref_cache_real8(want)
    again = igo_mod.ref_cache_code8(back)
    finite = np.isfinite(x)
    assert np.array_equal(again[finite], want[finite])


def _note(rng, window):
    from igllm_b200 import KeepNote
    n = KeepNote()
    count = int(rng.integers(0, 5))
    at = 0
    for i in range(count):
        start = at + int(rng.integers(0, 6))
        end = start + 1 + int(rng.integers(0, 6))
        if end > window:
            break
        n.from_list[i], n.till_list[i], n.mark_list[i] = start, end, int(rng.integers(0, 3))
        n.run_count = i + 1
        at = end
    return n


def test_keep_note_share_matches_reference(igc_lib, igo_mod):
    import ctypes
    rng = np.random.default_rng(3)
    ref = igo_mod.ref_lib()
    for _ in range(3000):
        a, b = _note(rng, 64), _note(rng, 64)
        if rng.random() < 0.5:  # often the same runs, now and then one fold apart
            ctypes.memmove(ctypes.byref(b), ctypes.byref(a), ctypes.sizeof(a))
            if b.run_count and rng.random() < 0.5:
                b.mark_list[int(rng.integers(0, b.run_count))] += 1
        same = int(rng.integers(0, 40))
        want = ref.ref_keep_note_share(ctypes.byref(igo_mod.KeepNote.from_buffer_copy(bytes(a))),
                                       ctypes.byref(igo_mod.KeepNote.from_buffer_copy(bytes(b))), same)
        assert igc_lib.keep_note_share(a, b, same) == want


@pytest.fixture(scope="module")
def cached_ref(tmp_path_factory, igc_lib, igo_mod):
    d = str(tmp_path_factory.mktemp("cached_cpu"))
    make_checkpoint(igc_lib, d, CACHED)
    return d


@pytest.mark.parametrize("bits", [0, 8])
@pytest.mark.parametrize("fill", [40, 150])
def test_reference_files_have_the_layout(cached_ref, igo_mod, tmp_path, bits, fill):
    """The layout parse_cache_file assumes, and this library writes, is the
    one the reference's session_save writes: 64-row rings turned over at
    fill 150, the global owner and the last sliding owner full length."""
    window = CACHED["window_limit"]
    rm = igo_mod.RefModel(cached_ref, threads=8, window_limit=window, cache_bits=bits)
    rs = igo_mod.RefSession(rm)
    ids = np.random.default_rng(fill).integers(0, CACHED["vocab"], fill + 1).astype(np.int32)
    rs.prime(ids)
    note = igo_mod.KeepNote()
    note.run_count = 2
    note.from_list[0], note.till_list[0], note.mark_list[0] = 3, 9, 0xABCDEF
    note.from_list[1], note.till_list[1], note.mark_list[1] = 12, 20, 5
    path = str(tmp_path / "r.keep")
    assert rs.save(path, stamp=991, note=note, kind=1) == 0
    f = parse_cache_file(path, CACHED, window, bits)
    assert (f["fill"], f["held"], f["layers"], f["bits"], f["kind"], f["stamp"]) == (fill, fill, 10, bits, 1, 991)
    assert f["runs"] == [(3, 9, 0xABCDEF), (12, 20, 5)]
    assert np.array_equal(f["ids"], ids[:-1])
    assert sorted(f["rows"]) == [0, 1, 2, 3, 4, 5]
    for l in range(10):
        assert f["key_peak"][l] == np.float32(rs.cache_peak(l, 0))
        assert f["value_peak"][l] == np.float32(rs.cache_peak(l, 1))
    # a byte side holds codes of values / scale: every one decodes inside the peak
    if bits == 8:
        k0 = f["rows"][0][0]
        assert k0.dtype == np.uint8
        dec = igo_mod.ref_cache_real8(k0.ravel()) * np.float32(rm.cache_scale(0, 0))
        assert np.abs(dec).max() <= f["key_peak"][0] * 1.07
    # the reference reads its own file back, and refuses it when damaged
    rs2 = igo_mod.RefSession(rm)
    code, stamp, back, kind = rs2.load(path)
    assert (code, stamp, kind, rs2.fill) == (0, 991, 1, fill)
    with open(path, "rb") as fh:
        data = fh.read()
    cut = str(tmp_path / "cut.keep")
    with open(cut, "wb") as fh:
        fh.write(data[:-5])
    assert rs2.load(cut)[0] == -4 and rs2.fill == 0  # APP_FAIL_FORMAT, cleared
    rs.close()
    rs2.close()
    rm.close()
