"""igc_norm_rms_fixed, the norm entry that allocates nothing, against the
desk's norm_rms (which grows device buffers as it goes).  Collected last, so
it also runs after every other GPU test has used the device."""

import numpy as np
import pytest

TOL = 1e-6  # relative to the row's largest magnitude; both run the same kernel


def _close(a, b):
    return float(np.abs(a - b).max()) <= TOL * max(1.0, float(np.abs(b).max()))


@pytest.mark.gpu
def test_fixed_norm_matches_the_desk_twice_in_a_row(igc_lib):
    desk = igc_lib.Desk(0)
    rng = np.random.default_rng(21)
    try:
        for n, with_gain in ((1536, True), (8960, True), (256, False), (igc_lib.FIXED_NORM_LIMIT, True)):
            x = (rng.standard_normal(n) * 3.0).astype(np.float32)
            w = rng.standard_normal(n).astype(np.float32) if with_gain else None
            want = desk.norm_rms(x, w, 1e-6)
            first = igc_lib.norm_rms_fixed(x, w, 1e-6, device=0)
            second = igc_lib.norm_rms_fixed(x, w, 1e-6, device=0)
            assert _close(first, want), n
            assert _close(second, want), n
            assert np.array_equal(first, second)
    finally:
        desk.close()


@pytest.mark.gpu
def test_fixed_norm_refuses_what_the_array_cannot_hold(igc_lib):
    x = np.ones(igc_lib.FIXED_NORM_LIMIT + 1, np.float32)
    with pytest.raises(igc_lib.IgcError) as err:
        igc_lib.norm_rms_fixed(x, None, 1e-6, device=0)
    assert "exceed" in str(err.value)
    # the refusal copied nothing and left the entry usable
    y = np.arange(1, 65, dtype=np.float32)
    got = igc_lib.norm_rms_fixed(y, None, 1e-6, device=0)
    want = y / np.sqrt(np.mean(y.astype(np.float64) ** 2) + 1e-6)
    assert _close(got, want.astype(np.float32))
