"""igllm_b200 - the B200 backend of the speculative verify round.

Python face of libigllm_cuda (include/igllm_cuda.h), mirroring the reference
engine's public API (iamhaymc/igllm app_core.c:158-425): the same entry
names (model_load, session_open, prime, step, guess, guess_keep,
guess_taste, pick, hold, scout_*), the same argument meaning and the same
refusals.  A refused call raises IgcError carrying the reference's app_code.

The library is built in-tree by igllm_b200/build.py; importing this module
does not build it, and every entry fails loudly if it is missing.
"""

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libigllm_cuda.so")

OKAY = 0
FAIL_ARGUMENT = -1
FAIL_MEMORY = -2
FAIL_FILE = -3
FAIL_FORMAT = -4
FAIL_MISSING = -5
FAIL_SUPPORT = -6
FAIL_STATE = -7
FAIL_DEVICE = -8
LANE_LIMIT = 16

_CODE_TEXT = {  # app_core.c:12406 app_code_text
    0: "okay", -1: "bad argument", -2: "out of memory", -3: "file not readable",
    -4: "malformed data", -5: "required piece missing", -6: "unsupported configuration",
    -7: "invalid state", -8: "device failure",
}


class IgcError(RuntimeError):
    def __init__(self, code, where=""):
        self.code = code
        detail = _lib().igc_last_error().decode() if code == FAIL_DEVICE else ""
        super().__init__(f"{where}: {_CODE_TEXT.get(code, code)} ({code}) {detail}".strip())


class Setup(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("window_limit", ctypes.c_int),
                ("verbose_level", ctypes.c_int), ("cache_bits", ctypes.c_int)]


class Taste(ctypes.Structure):  # app_core.c:60-67 app_taste
    _fields_ = [("heat_value", ctypes.c_float), ("top_count", ctypes.c_int),
                ("top_portion", ctypes.c_float), ("echo_penalty", ctypes.c_float),
                ("echo_window", ctypes.c_int), ("seed_value", ctypes.c_uint64)]


def taste_plain():
    """app_core.c:12426 app_taste_plain."""
    return Taste(1.0, 64, 0.95, 1.0, 64, 0x2545F4914F6CDD1D)


class SynthSpec(ctypes.Structure):
    _fields_ = [("vocab", ctypes.c_int), ("hidden", ctypes.c_int), ("layers", ctypes.c_int),
                ("heads", ctypes.c_int), ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int),
                ("inner", ctypes.c_int), ("ple_dim", ctypes.c_int), ("slide_span", ctypes.c_int),
                ("share_count", ctypes.c_int), ("global_every", ctypes.c_int),
                ("window_limit", ctypes.c_int), ("norm_offset", ctypes.c_float),
                ("with_layer_scalar", ctypes.c_int), ("seed", ctypes.c_uint64),
                ("cache_scale_k", ctypes.c_float), ("cache_scale_v", ctypes.c_float),
                ("double_wide", ctypes.c_int), ("global_head_dim", ctypes.c_int),
                ("late_mlp_bits", ctypes.c_int), ("group", ctypes.c_int), ("bf16_scales", ctypes.c_int),
                ("embed_bits", ctypes.c_int), ("ple_embed_bits", ctypes.c_int), ("tied_head", ctypes.c_int),
                ("ple_bits8", ctypes.c_int), ("dense_ple_lift", ctypes.c_int), ("grid_in", ctypes.c_float),
                ("grid_out", ctypes.c_float)]


def spec_e2b(norm_offset=0.0, seed=1, window_limit=32768):
    """The benchmark shape: Gemma-4-E2B text stack with BASELINE's overrides
    (global head 256, single-width feed-forward)."""
    return SynthSpec(vocab=262144, hidden=1536, layers=35, heads=8, kv_heads=1, head_dim=256,
                     inner=6144, ple_dim=256, slide_span=512, share_count=20, global_every=5,
                     window_limit=window_limit, norm_offset=norm_offset, with_layer_scalar=0,
                     seed=seed)


class IgcPlane(ctypes.Structure):  # app_core.c:1775 plane
    _fields_ = [("form", ctypes.c_int), ("row_count", ctypes.c_int), ("col_count", ctypes.c_int),
                ("real_data", ctypes.c_void_p), ("real_type", ctypes.c_int),
                ("code_data", ctypes.c_void_p), ("row_stride", ctypes.c_size_t),
                ("gain_data", ctypes.c_void_p), ("gain_type", ctypes.c_int),
                ("bias_data", ctypes.c_void_p), ("bit_count", ctypes.c_int),
                ("code_bias", ctypes.c_int), ("code_flip", ctypes.c_int),
                ("group_size", ctypes.c_int), ("group_count", ctypes.c_int),
                ("enter_gain", ctypes.c_float), ("leave_gain", ctypes.c_float)]


KEEP_PROMPT = 0  # app_core.c:367
KEEP_TALK = 1    # app_core.c:368
KEEP_RUNS = 16   # app_core.c:385


class KeepNote(ctypes.Structure):  # app_core.c:387-392 app_keep_note
    _fields_ = [("run_count", ctypes.c_int), ("from_list", ctypes.c_int32 * KEEP_RUNS),
                ("till_list", ctypes.c_int32 * KEEP_RUNS), ("mark_list", ctypes.c_uint64 * KEEP_RUNS)]


class _Desk(ctypes.Structure):
    pass


_P = ctypes.POINTER
_f = _P(ctypes.c_float)
_MATVEC = ctypes.CFUNCTYPE(None, _P(_Desk), _P(IgcPlane), _f, _f)
_MATMAT = ctypes.CFUNCTYPE(None, _P(_Desk), _P(IgcPlane), _f, ctypes.c_int, ctypes.c_int, _f, ctypes.c_int)
_NORM = ctypes.CFUNCTYPE(None, _P(_Desk), _f, _f, ctypes.c_int, ctypes.c_float, _f)
_SOFT = ctypes.CFUNCTYPE(None, _P(_Desk), _f, ctypes.c_int)
_GELU = ctypes.CFUNCTYPE(None, _P(_Desk), _f, _f, ctypes.c_int)
_ROPE = ctypes.CFUNCTYPE(None, _P(_Desk), _f, ctypes.c_int, _f, _f)
_Desk._fields_ = [("name_text", ctypes.c_char_p), ("state", ctypes.c_void_p), ("mat_vec", _MATVEC),
                  ("mat_mat", _MATMAT), ("norm_rms", _NORM), ("soft_max", _SOFT), ("gelu_gate", _GELU),
                  ("rope_turn", _ROPE)]

_LIB = None


def _lib():
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python igllm_b200/build.py`")
    lib = ctypes.CDLL(LIB_PATH)
    vp, i, i32p, fp = ctypes.c_void_p, ctypes.c_int, _P(ctypes.c_int32), _f
    sig = {
        "igc_model_load": (i, [ctypes.c_char_p, _P(Setup), _P(vp)]),
        "igc_model_synth": (i, [_P(SynthSpec), _P(Setup), _P(vp)]),
        "igc_model_free": (None, [vp]),
        "igc_model_vocab_count": (i, [vp]),
        "igc_model_layer_count": (i, [vp]),
        "igc_model_state_size": (i, [vp]),
        "igc_model_window_limit": (i, [vp]),
        "igc_model_decode_bytes": (ctypes.c_size_t, [vp]),
        "igc_model_device_bytes": (ctypes.c_size_t, [vp]),
        "igc_model_weight_count": (ctypes.c_size_t, [vp]),
        "igc_session_open": (i, [vp, _P(vp)]),
        "igc_session_close": (None, [vp]),
        "igc_session_reset": (None, [vp]),
        "igc_session_hold": (i, [vp, i]),
        "igc_session_prime": (i, [vp, i32p, i]),
        "igc_session_step": (i, [vp, ctypes.c_int32, fp, i32p]),
        "igc_session_guess": (i, [vp, i32p, i, fp]),
        "igc_session_guess_top": (i, [vp, i32p]),
        "igc_session_guess_keep": (i, [vp, i]),
        "igc_session_guess_taste": (i, [vp, i32p, i, _P(Taste), i32p]),
        "igc_session_pick": (ctypes.c_int32, [vp, _P(Taste)]),
        "igc_session_fill": (i, [vp]),
        "igc_session_guess_span": (i, [vp]),
        "igc_session_guess_limit": (i, [vp]),
        "igc_session_round": (i, [vp, i32p, i, _P(Taste), i32p, i32p]),
        "igc_session_serve_seconds": (ctypes.c_double, [vp]),
        "igc_session_serve_tokens": (ctypes.c_size_t, [vp]),
        "igc_session_bench": (i, [vp, i32p, i, i, fp, i32p]),
        "igc_session_profile": (i, [vp, i32p, i, _P(ctypes.c_int), _P(ctypes.c_double), fp, i]),
        "igc_session_stamps": (i, [vp, i, _P(ctypes.c_int), _P(ctypes.c_double), _P(ctypes.c_double), i, i]),
        "igc_scout_open": (i, [_P(vp)]),
        "igc_scout_close": (None, [vp]),
        "igc_scout_clear": (None, [vp]),
        "igc_scout_note": (i, [vp, i32p, i]),
        "igc_scout_span": (i, [vp]),
        "igc_scout_draw": (i, [vp, i32p, i]),
        "igc_synth_fill": (i, [ctypes.c_uint64, ctypes.c_uint64, i, ctypes.c_float, ctypes.c_size_t, vp, i]),
        "igc_synth_write": (i, [_P(SynthSpec), ctypes.c_char_p, i]),
        "igc_synth_stream": (ctypes.c_uint64, [ctypes.c_char_p]),
        "igc_back_open": (i, [_P(_Desk), i]),
        "igc_back_close": (None, [_P(_Desk)]),
        "igc_desk_status": (i, [_P(_Desk)]),
        "igc_last_error": (ctypes.c_char_p, []),
        "igc_launch_count": (ctypes.c_long, []),
        "igc_norm_rms_fixed": (i, [i, fp, fp, i, ctypes.c_float, fp]),
        "igc_crowd_open": (i, [vp, i, i, _P(vp)]),
        "igc_crowd_close": (None, [vp]),
        "igc_crowd_round": (i, [vp, _P(vp), i, i32p, i32p, i32p, fp]),
        "igc_session_save": (i, [vp, ctypes.c_char_p, ctypes.c_uint64, _P(KeepNote), i]),
        "igc_session_load": (i, [vp, ctypes.c_char_p, _P(ctypes.c_uint64), _P(KeepNote), _P(ctypes.c_int)]),
        "igc_session_ids": (i, [vp, i32p, i]),
        "igc_keep_note_share": (i, [_P(KeepNote), _P(KeepNote), i]),
        "igc_model_cache_scale": (ctypes.c_float, [vp, i, i]),
        "igc_session_cache_peak": (ctypes.c_float, [vp, i, i]),
        "igc_session_cache_room": (ctypes.c_size_t, [vp]),
        "igc_session_cache_room_at": (ctypes.c_size_t, [vp, i]),
        "igc_model_memory_bytes": (ctypes.c_size_t, [vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _LIB = lib
    return lib


def exported_symbols():
    """Names the library must export (every entry of include/igllm_cuda.h)."""
    return [
        "igc_back_open", "igc_back_close", "igc_desk_status", "igc_model_load", "igc_model_free",
        "igc_model_vocab_count", "igc_model_layer_count", "igc_model_state_size",
        "igc_model_window_limit", "igc_model_decode_bytes", "igc_model_device_bytes", "igc_model_weight_count",
        "igc_session_open", "igc_session_close", "igc_session_reset", "igc_session_hold",
        "igc_session_prime", "igc_session_step", "igc_session_guess", "igc_session_guess_top",
        "igc_session_guess_keep", "igc_session_guess_taste", "igc_session_pick", "igc_session_fill",
        "igc_session_guess_span", "igc_session_guess_limit", "igc_session_round",
        "igc_session_serve_seconds", "igc_session_serve_tokens", "igc_session_bench", "igc_session_profile",
        "igc_session_stamps",
        "igc_scout_open", "igc_scout_close",
        "igc_scout_clear", "igc_scout_note", "igc_scout_span", "igc_scout_draw", "igc_synth_fill",
        "igc_synth_write", "igc_model_synth", "igc_last_error", "igc_launch_count", "igc_norm_rms_fixed",
        "igc_crowd_open", "igc_crowd_close", "igc_crowd_round",
        "igc_session_save", "igc_session_load", "igc_session_ids", "igc_keep_note_share",
        "igc_model_cache_scale", "igc_session_cache_peak", "igc_session_cache_room", "igc_session_cache_room_at",
        "igc_model_memory_bytes",
    ]


def _check(code, where):
    if code != OKAY:
        raise IgcError(code, where)


def _ids(ids):
    a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32))
    return a, a.ctypes.data_as(_P(ctypes.c_int32))


def launch_count():
    """Kernels this library launched on this thread since the last call."""
    return _lib().igc_launch_count()


class Model:
    """app_core.c:12439 model_load (or a synthetic spec built straight in HBM)."""

    def __init__(self, folder=None, spec=None, device=0, window_limit=0, cache_bits=0):
        lib = _lib()
        self._h = ctypes.c_void_p()
        setup = Setup(device, window_limit, 0, int(cache_bits))
        if spec is not None:
            _check(lib.igc_model_synth(ctypes.byref(spec), ctypes.byref(setup), ctypes.byref(self._h)),
                   "model_synth")
        else:
            _check(lib.igc_model_load(str(folder).encode(), ctypes.byref(setup), ctypes.byref(self._h)),
                   "model_load")

    @property
    def vocab(self):
        return _lib().igc_model_vocab_count(self._h)

    @property
    def layers(self):
        return _lib().igc_model_layer_count(self._h)

    @property
    def window_limit(self):
        return _lib().igc_model_window_limit(self._h)

    def decode_bytes(self):
        return _lib().igc_model_decode_bytes(self._h)

    def device_bytes(self):
        return _lib().igc_model_device_bytes(self._h)

    def linear_params(self):
        """Weights of the int4 projections one lane multiplies (head included)."""
        return _lib().igc_model_weight_count(self._h)

    def memory_bytes(self):
        """app_core.c:12667 model_memory_bytes."""
        return _lib().igc_model_memory_bytes(self._h)

    def cache_scale(self, layer, value_side):
        """app_core.c:14515 model_cache_scale."""
        return _lib().igc_model_cache_scale(self._h, int(layer), int(value_side))

    def close(self):
        if self._h:
            _lib().igc_model_free(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """app_core.c:14219 session_open and the calls on a session."""

    def __init__(self, model):
        self.model = model
        self._h = ctypes.c_void_p()
        _check(_lib().igc_session_open(model._h, ctypes.byref(self._h)), "session_open")

    def close(self):
        if self._h:
            _lib().igc_session_close(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        _lib().igc_session_reset(self._h)

    @property
    def fill(self):
        return _lib().igc_session_fill(self._h)

    def hold(self, keep):
        _check(_lib().igc_session_hold(self._h, int(keep)), "session_hold")

    def save(self, path, stamp=0, note=None, kind=KEEP_PROMPT):
        """app_core.c:14010 session_save."""
        _check(_lib().igc_session_save(self._h, str(path).encode(), int(stamp),
                                       ctypes.byref(note) if note is not None else None, int(kind)),
               "session_save")

    def load(self, path):
        """app_core.c:14076 session_load; returns (stamp, note, kind)."""
        stamp, note, kind = ctypes.c_uint64(), KeepNote(), ctypes.c_int()
        _check(_lib().igc_session_load(self._h, str(path).encode(), ctypes.byref(stamp), ctypes.byref(note),
                                       ctypes.byref(kind)), "session_load")
        return stamp.value, note, kind.value

    def ids(self):
        """app_core.c:14183 session_ids."""
        n = _lib().igc_session_ids(self._h, None, 0)
        a = np.zeros(max(n, 1), np.int32)
        _lib().igc_session_ids(self._h, a.ctypes.data_as(_P(ctypes.c_int32)), len(a))
        return a[:n]

    def cache_peak(self, layer, value_side):
        """app_core.c:14540 session_cache_peak."""
        return _lib().igc_session_cache_peak(self._h, int(layer), int(value_side))

    def cache_room(self, cache_bits=None):
        """Bytes the caches occupy (at `cache_bits` storage when given)."""
        if cache_bits is None:
            return _lib().igc_session_cache_room(self._h)
        return _lib().igc_session_cache_room_at(self._h, int(cache_bits))

    def prime(self, ids):
        a, p = _ids(ids)
        _check(_lib().igc_session_prime(self._h, p, len(a)), "session_prime")

    def step(self, id_value, want_logits=True):
        """One id; returns (argmax id, logit row or None)."""
        top = ctypes.c_int32()
        row = np.empty(self.model.vocab, np.float32) if want_logits else None
        rp = row.ctypes.data_as(_f) if want_logits else None
        _check(_lib().igc_session_step(self._h, int(id_value), rp, ctypes.byref(top)), "session_step")
        return top.value, row

    def guess(self, ids, want_logits=True):
        """A block of ids; returns the rows (K x vocab) or None."""
        a, p = _ids(ids)
        rows = np.empty((len(a), self.model.vocab), np.float32) if want_logits else None
        rp = rows.ctypes.data_as(_f) if want_logits else None
        _check(_lib().igc_session_guess(self._h, p, len(a), rp), "session_guess")
        return rows

    def guess_top(self):
        out = np.empty(_lib().igc_session_guess_span(self._h), np.int32)
        _check(_lib().igc_session_guess_top(self._h, out.ctypes.data_as(_P(ctypes.c_int32))), "guess_top")
        return out

    def guess_keep(self, keep):
        _check(_lib().igc_session_guess_keep(self._h, int(keep)), "session_guess_keep")

    def guess_taste(self, ids, taste):
        a, p = _ids(ids)
        made = ctypes.c_int32()
        take = _lib().igc_session_guess_taste(self._h, p, len(a), ctypes.byref(taste), ctypes.byref(made))
        if take < 0:
            raise IgcError(FAIL_STATE, "session_guess_taste")
        return take, made.value

    def pick(self, taste):
        return _lib().igc_session_pick(self._h, ctypes.byref(taste))

    def round(self, ids, taste=None):
        """guess + verify + keep; returns (take, made)."""
        a, p = _ids(ids)
        take, made = ctypes.c_int32(), ctypes.c_int32()
        tp = ctypes.byref(taste) if taste is not None else None
        n = _lib().igc_session_round(self._h, p, len(a), tp, ctypes.byref(take), ctypes.byref(made))
        if n < 0:
            raise IgcError(n, "session_round")
        return take.value, made.value

    def bench(self, blocks, k):
        """Verify rounds with every block resident in HBM (see igc_session_bench);
        returns (device ms, last round's argmax ids)."""
        a, p = _ids(np.asarray(blocks, np.int32).reshape(-1))
        ms = ctypes.c_float()
        top = np.zeros(k, np.int32)
        _check(_lib().igc_session_bench(self._h, p, len(a) // k, k, ctypes.byref(ms),
                                        top.ctypes.data_as(_P(ctypes.c_int32))), "session_bench")
        return ms.value, top

    def profile(self, ids):
        """One kept pass with per-launch device times: list of (class, bytes, ms)."""
        a, p = _ids(ids)
        cap = 4096
        cls = np.zeros(cap, np.int32)
        byt = np.zeros(cap, np.float64)
        ms = np.zeros(cap, np.float32)
        n = _lib().igc_session_profile(self._h, p, len(a), cls.ctypes.data_as(_P(ctypes.c_int)),
                                       byt.ctypes.data_as(_P(ctypes.c_double)), ms.ctypes.data_as(_f), cap)
        if n < 0:
            raise IgcError(n, "session_profile")
        return list(zip(cls[:n].tolist(), byt[:n].tolist(), ms[:n].tolist()))

    def stamps(self, k, reset=False):
        """Launch stamps of the graphed k-lane passes with a head since the last
        reset: list of (class, weight bytes, total ns)."""
        cap = 4096
        cls = np.zeros(cap, np.int32)
        byt = np.zeros(cap, np.float64)
        ns = np.zeros(cap, np.float64)
        n = _lib().igc_session_stamps(self._h, int(k), cls.ctypes.data_as(_P(ctypes.c_int)),
                                      byt.ctypes.data_as(_P(ctypes.c_double)),
                                      ns.ctypes.data_as(_P(ctypes.c_double)), cap, 1 if reset else 0)
        if n < 0:
            raise IgcError(n, "session_stamps")
        return list(zip(cls[:n].tolist(), byt[:n].tolist(), ns[:n].tolist()))

    def serve_seconds(self):
        return _lib().igc_session_serve_seconds(self._h)

    def serve_tokens(self):
        return _lib().igc_session_serve_tokens(self._h)


CROWD_LANE_LIMIT = 512  # include/igllm_cuda.h IGC_CROWD_LANE_LIMIT


class Crowd:
    """igc_crowd: one greedy verify round for many sessions of one model in
    one pass (the lanes of every session's block share each weight sweep)."""

    def __init__(self, model, session_limit, lanes_per_session):
        self.model = model
        self.k = int(lanes_per_session)
        self.limit = int(session_limit)
        self._h = ctypes.c_void_p()
        _check(_lib().igc_crowd_open(model._h, self.limit, self.k, ctypes.byref(self._h)), "crowd_open")

    def close(self):
        if self._h:
            _lib().igc_crowd_close(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def round(self, sessions, blocks, want_logits=False):
        """blocks: (len(sessions), k) ids.  Returns (takes, mades, logits or None)."""
        n = len(sessions)
        a, p = _ids(np.asarray(blocks, np.int32).reshape(-1))
        if len(a) != n * self.k:
            raise ValueError(f"crowd round: {len(a)} ids for {n} sessions of {self.k}")
        hs = (ctypes.c_void_p * n)(*[s._h.value for s in sessions])
        take = np.zeros(n, np.int32)
        made = np.zeros(n, np.int32)
        rows = np.empty((n * self.k, self.model.vocab), np.float32) if want_logits else None
        rp = rows.ctypes.data_as(_f) if want_logits else None
        c = _lib().igc_crowd_round(self._h, hs, n, p, take.ctypes.data_as(_P(ctypes.c_int32)),
                                   made.ctypes.data_as(_P(ctypes.c_int32)), rp)
        if c < 0:
            raise IgcError(c, "crowd_round")
        return take, made, rows


class Scout:
    """app_core.c:12277-12361 the n-gram proposer (host C)."""

    def __init__(self):
        self._h = ctypes.c_void_p()
        _check(_lib().igc_scout_open(ctypes.byref(self._h)), "scout_open")

    def __del__(self):
        try:
            if self._h:
                _lib().igc_scout_close(self._h)
        except Exception:
            pass

    def clear(self):
        _lib().igc_scout_clear(self._h)

    def note(self, ids):
        a, p = _ids(ids)
        _check(_lib().igc_scout_note(self._h, p, len(a)), "scout_note")

    @property
    def span(self):
        return _lib().igc_scout_span(self._h)

    def draw(self, want):
        out = np.zeros(max(int(want), 1), np.int32)
        n = _lib().igc_scout_draw(self._h, out.ctypes.data_as(_P(ctypes.c_int32)), int(want))
        return out[:n]


class Desk:
    """app_core.c:5222 back_desk on the GPU: host pointers in and out."""

    def __init__(self, device=0):
        self._d = _Desk()
        _check(_lib().igc_back_open(ctypes.byref(self._d), device), "back_open")

    def close(self):
        if self._d.state:
            _lib().igc_back_close(ctypes.byref(self._d))

    def status(self):
        return _lib().igc_desk_status(ctypes.byref(self._d))

    def mat_mat(self, plane, act, lanes, out_rows):
        act = np.ascontiguousarray(act, np.float32)
        out = np.zeros((lanes, out_rows), np.float32)
        self._d.mat_mat(ctypes.byref(self._d), ctypes.byref(plane), act.ctypes.data_as(_f),
                        act.shape[-1], lanes, out.ctypes.data_as(_f), out_rows)
        _check(self.status(), "desk.mat_mat")
        return out

    def norm_rms(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros_like(x)
        wa = np.ascontiguousarray(w, np.float32) if w is not None else None
        if wa is not None and wa.size != x.size:
            raise ValueError(f"norm_rms: gain has {wa.size} values for {x.size}")
        wp = wa.ctypes.data_as(_f) if wa is not None else None
        self._d.norm_rms(ctypes.byref(self._d), x.ctypes.data_as(_f), wp, len(x), eps, out.ctypes.data_as(_f))
        _check(self.status(), "desk.norm_rms")
        return out

    def soft_max(self, x):
        x = np.array(x, np.float32)
        self._d.soft_max(ctypes.byref(self._d), x.ctypes.data_as(_f), len(x))
        _check(self.status(), "desk.soft_max")
        return x

    def gelu_gate(self, gate, rise):
        g = np.array(gate, np.float32)
        r = np.ascontiguousarray(rise, np.float32)
        self._d.gelu_gate(ctypes.byref(self._d), g.ctypes.data_as(_f), r.ctypes.data_as(_f), len(g))
        _check(self.status(), "desk.gelu_gate")
        return g

    def rope_turn(self, x, cs, sn):
        x = np.array(x, np.float32)
        c = np.ascontiguousarray(cs, np.float32)
        s = np.ascontiguousarray(sn, np.float32)
        self._d.rope_turn(ctypes.byref(self._d), x.ctypes.data_as(_f), len(x), c.ctypes.data_as(_f),
                          s.ctypes.data_as(_f))
        _check(self.status(), "desk.rope_turn")
        return x


FIXED_NORM_LIMIT = 65536  # include/igllm_cuda.h IGC_FIXED_NORM_LIMIT


def norm_rms_fixed(x, w, eps, device=0):
    """igc_norm_rms_fixed: the desk's norm_rms through a fixed device array,
    with no allocation on the device (vectors up to FIXED_NORM_LIMIT floats;
    overlapping calls on one device race)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    wa = np.ascontiguousarray(w, np.float32) if w is not None else None
    if wa is not None and wa.size != x.size:
        raise ValueError(f"norm_rms_fixed: gain has {wa.size} values for {x.size}")
    wp = wa.ctypes.data_as(_f) if wa is not None else None
    code = _lib().igc_norm_rms_fixed(int(device), x.ctypes.data_as(_f), wp, len(x), float(eps),
                                     out.ctypes.data_as(_f))
    if code == FAIL_ARGUMENT and len(x) > FIXED_NORM_LIMIT:
        raise IgcError(code, f"norm_rms_fixed: {len(x)} floats exceed the fixed array's {FIXED_NORM_LIMIT}")
    _check(code, "norm_rms_fixed")
    return out


def synth_write(spec, folder, threads=8):
    """Writes config.json, tokenizer.json and model.safetensors for `spec`."""
    os.makedirs(folder, exist_ok=True)
    _check(_lib().igc_synth_write(ctypes.byref(spec), str(folder).encode(), int(threads)), "synth_write")


class SynthTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 128), ("dtype", ctypes.c_int), ("rank", ctypes.c_int),
                ("shape", ctypes.c_int64 * 2), ("kind", ctypes.c_int), ("offset", ctypes.c_float),
                ("bytes", ctypes.c_size_t)]


_DTYPE_NAME = {1: "F32", 2: "F16", 3: "BF16", 5: "I8", 6: "U8"}


def synth_tensors(spec, threads=8):
    """Every tensor of a synthetic checkpoint, generated in memory:
    name -> (dtype name, numpy array of the stored bits)."""
    lib = _lib()
    lib.igc_synth_list.restype = ctypes.c_int
    lib.igc_synth_list.argtypes = [_P(SynthSpec), ctypes.c_void_p, ctypes.c_int]
    lib.igc_synth_tensor_fill.restype = ctypes.c_int
    lib.igc_synth_tensor_fill.argtypes = [_P(SynthSpec), _P(SynthTensor), ctypes.c_void_p, ctypes.c_int]
    n = lib.igc_synth_list(ctypes.byref(spec), None, 0)
    room = (SynthTensor * n)()
    lib.igc_synth_list(ctypes.byref(spec), room, n)
    out = {}
    for t in room:
        shape = [t.shape[0], t.shape[1]] if t.rank == 2 else [t.shape[0]]
        arr = np.empty(shape, {6: np.uint8, 5: np.int8, 1: np.float32}.get(t.dtype, np.uint16))
        _check(lib.igc_synth_tensor_fill(ctypes.byref(spec), ctypes.byref(t), arr.ctypes.data_as(ctypes.c_void_p),
                                         threads), "synth_tensor_fill")
        out[t.name.decode()] = (_DTYPE_NAME[t.dtype], arr)
    return out


def synth_config(spec):
    """The config.json a synthetic checkpoint carries, parsed."""
    import json
    lib = _lib()
    lib.igc_synth_config_text.restype = ctypes.c_void_p
    lib.igc_synth_config_text.argtypes = [_P(SynthSpec)]
    p = lib.igc_synth_config_text(ctypes.byref(spec))
    text = ctypes.string_at(p).decode()
    ctypes.CDLL(None).free(ctypes.c_void_p(p))
    return json.loads(text)


def synth_fill(seed, name, kind, count, offset=0.0, threads=1):
    """The values of one synthetic tensor stream (kind 0 bytes, else u16 bits)."""
    lib = _lib()
    out = np.empty(count, np.uint8 if kind == 0 else np.uint16)
    stream = lib.igc_synth_stream(name.encode())
    _check(lib.igc_synth_fill(seed, stream, kind, offset, count, out.ctypes.data_as(ctypes.c_void_p), threads),
           "synth_fill")
    return out


def keep_note_share(held, now, same_count):
    """app_core.c:13991 keep_note_share."""
    return _lib().igc_keep_note_share(ctypes.byref(held), ctypes.byref(now), int(same_count))
