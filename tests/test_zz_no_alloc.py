"""igc_norm_rms_fixed, the norm entry that allocates nothing.

Some callers of this library may not allocate device memory once they run:
a token loop that promised a fixed footprint, or code holding no desk (whose
norm_rms grows device buffers as longer vectors arrive).  The entry keeps its
vectors in one fixed array of the library's device image instead.

Checked here, through the C ABI, on two calls in a row: the result against
the desk's norm_rms (the existing entry) and against the CPU checker's
igo_norm_rms (an independent restatement of app_core.c:4667 kern_norm_rms,
which sums the squares in double); and, after one warm-up call, that further
calls leave the device's free memory unchanged.  Collected last, so that a
run that stops at the first failure has already run every other test; it
passes alone in a fresh process too.
"""

import ctypes

import numpy as np
import pytest

TOL = 1e-5  # relative to the row's largest magnitude (float sum vs double sum)


def _close(a, b):
    return float(np.abs(a - b).max()) <= TOL * max(1.0, float(np.abs(b).max()))


def _free_bytes():
    """Free device memory of the calling thread's current context (driver API)."""
    cu = ctypes.CDLL("libcuda.so.1")
    ctx = ctypes.c_void_p()
    assert cu.cuCtxGetCurrent(ctypes.byref(ctx)) == 0 and ctx.value, "no current context"
    free, total = ctypes.c_size_t(), ctypes.c_size_t()
    assert cu.cuMemGetInfo_v2(ctypes.byref(free), ctypes.byref(total)) == 0
    return free.value


def _oracle_norm(igo_mod, x, w, eps):
    lib = igo_mod.igo_lib()
    out = np.zeros_like(x)
    wp = igo_mod.fptr(w) if w is not None else None
    lib.igo_norm_rms(igo_mod.fptr(x), wp, len(x), eps, igo_mod.fptr(out))
    return out


@pytest.mark.gpu
def test_fixed_norm_matches_the_desk_and_the_checker_twice_in_a_row(igc_lib, igo_mod):
    desk = igc_lib.Desk(0)
    rng = np.random.default_rng(21)
    try:
        for n, with_gain in ((1536, True), (8960, True), (256, False), (igc_lib.FIXED_NORM_LIMIT, True)):
            x = (rng.standard_normal(n) * 3.0).astype(np.float32)
            w = rng.standard_normal(n).astype(np.float32) if with_gain else None
            from_desk = desk.norm_rms(x, w, 1e-6)
            from_checker = _oracle_norm(igo_mod, x, w, 1e-6)
            first = igc_lib.norm_rms_fixed(x, w, 1e-6, device=0)
            second = igc_lib.norm_rms_fixed(x, w, 1e-6, device=0)
            for got in (first, second):
                assert _close(got, from_desk), n
                assert _close(got, from_checker), n
            assert np.array_equal(first, second)
    finally:
        desk.close()


@pytest.mark.gpu
def test_fixed_norm_allocates_nothing_after_its_first_call(igc_lib):
    rng = np.random.default_rng(22)
    x = rng.standard_normal(igc_lib.FIXED_NORM_LIMIT).astype(np.float32)
    w = rng.standard_normal(igc_lib.FIXED_NORM_LIMIT).astype(np.float32)
    igc_lib.norm_rms_fixed(x, w, 1e-6, device=0)  # may create the context and load the module
    before = _free_bytes()
    for _ in range(8):
        igc_lib.norm_rms_fixed(x, w, 1e-6, device=0)
    assert _free_bytes() == before


@pytest.mark.gpu
def test_fixed_norm_refuses_what_the_array_cannot_hold(igc_lib):
    x = np.ones(igc_lib.FIXED_NORM_LIMIT + 1, np.float32)
    with pytest.raises(igc_lib.IgcError) as err:
        igc_lib.norm_rms_fixed(x, None, 1e-6, device=0)
    assert "exceed" in str(err.value)
    with pytest.raises(ValueError):
        igc_lib.norm_rms_fixed(np.ones(8, np.float32), np.ones(7, np.float32), 1e-6, device=0)
    # the refusals copied nothing and left the entry usable
    y = np.arange(1, 65, dtype=np.float32)
    got = igc_lib.norm_rms_fixed(y, None, 1e-6, device=0)
    want = y / np.sqrt(np.mean(y.astype(np.float64) ** 2) + 1e-6)
    assert _close(got, want.astype(np.float32))
