"""The C ABI library on the CPU: it loads, exports every entry the header
declares, and its host-side parts (synthetic checkpoints) behave."""

import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_entries():
    text = open(os.path.join(ROOT, "include", "igllm_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = set(re.findall(r"\b(igc_[a-z0-9_]+)\s*\(", text))
    return sorted(n for n in names if not n.startswith("igc_desk_t"))


def test_library_exports_every_declared_entry(igc_lib):
    lib = ctypes.CDLL(igc_lib.LIB_PATH)
    missing = [n for n in declared_entries() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(igc_lib.exported_symbols()) <= set(declared_entries())


def test_synth_values_are_a_pure_function_of_seed_name_index(igc_lib):
    a = igc_lib.synth_fill(3, "x.weight", 0, 100000)
    b = igc_lib.synth_fill(3, "x.weight", 0, 100000, threads=4)
    assert np.array_equal(a, b)
    c = igc_lib.synth_fill(4, "x.weight", 0, 100000)
    assert not np.array_equal(a, c)
    # codes are uniform over both nibbles
    lo, hi = a & 15, a >> 4
    for nib in (lo, hi):
        counts = np.bincount(nib, minlength=16) / len(nib)
        assert np.abs(counts - 1 / 16).max() < 0.01
    # scales are |N(0, 0.02)| in f16, norms N(0, 0.02) in bf16
    s = igc_lib.synth_fill(3, "x.weight_scale", 1, 200000).view(np.float16).astype(np.float64)
    assert np.all(s >= 0) and abs(s.mean() - 0.02 * np.sqrt(2 / np.pi)) < 5e-4
    n = igc_lib.synth_fill(3, "n.weight", 2, 200000)
    nv = (n.astype(np.uint32) << 16).view(np.float32)
    assert abs(nv.mean()) < 5e-4 and abs(nv.std() - 0.02) < 5e-4


def test_synth_checkpoint_is_what_the_reference_reads(igc_lib, igo_mod, tiny_dir):
    t = igo_mod.read_folder(tiny_dir)
    assert t["lm_head.weight"][0] == "U8" and t["lm_head.weight_scale"][0] == "F16"
    assert t["lm_head.weight"][1].shape == (512, 64)
    rm = igo_mod.RefModel(tiny_dir, threads=2)
    assert rm.vocab == 512
    rm.close()


def test_synth_tensors_match_the_written_file(igc_lib, tiny_dir):
    from conftest import TINY
    import igo
    spec = igc_lib.SynthSpec(**TINY)
    mem = igc_lib.synth_tensors(spec)
    disk = igo.read_folder(tiny_dir)
    assert set(mem) == set(disk)
    for name, (dt, arr) in mem.items():
        assert disk[name][0] == dt
        assert np.array_equal(np.asarray(disk[name][1]).view(arr.dtype).reshape(arr.shape), arr), name


def test_crowd_and_stamps_refuse_bad_arguments_before_any_device_call(igc_lib):
    """The crowd entries and the stamp reader check their arguments first, as
    every session entry does (a refused call changes nothing)."""
    lib = igc_lib._lib()
    out = ctypes.c_void_p()
    assert lib.igc_crowd_open(None, 4, 4, ctypes.byref(out)) == igc_lib.FAIL_ARGUMENT
    assert not out.value
    assert lib.igc_crowd_round(None, None, 1, None, None, None, None) == igc_lib.FAIL_ARGUMENT
    assert lib.igc_session_stamps(None, 4, None, None, None, 0, 0) == igc_lib.FAIL_ARGUMENT
    assert lib.igc_model_weight_count(None) == 0
