"""ctypes face of the CPU checkers (TEST INFRASTRUCTURE).

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm load this module.  It binds

  * oracle/_build/libigo.so - the plain-C restatement of the reference's verify
    round (oracle/igo.c), fed from a safetensors folder read here; and
  * oracle/_ref/libref_*.so - the reference engine itself, compiled from its
    own app_core.c by oracle/Makefile, driven through oracle/ref_harness.c.
"""

import ctypes
import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
IGO_LIB = os.path.join(HERE, "_build", "libigo.so")
REF_DIR = os.path.join(HERE, "_ref")

LANE_LIMIT = 16


def build():
    """Builds libigo.so and, where the reference source is present, libref_*.so."""
    subprocess.run(["make", "-s", "-C", HERE, "all"], check=True, stdout=subprocess.PIPE)


# ---- safetensors --------------------------------------------------------------

_DT = {"F32": np.float32, "F16": np.uint16, "BF16": np.uint16, "U8": np.uint8, "I8": np.int8,
       "I32": np.int32, "I64": np.int64, "F64": np.float64}


def read_safetensors(path):
    """name -> (dtype string, numpy view) for one file, memory-mapped."""
    with open(path, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
        head = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    base = 8 + n
    out = {}
    for name, d in head.items():
        if name == "__metadata__":
            continue
        a, b = d["data_offsets"]
        raw = mm[base + a: base + b]
        out[name] = (d["dtype"], raw.view(_DT[d["dtype"]]).reshape(d["shape"]))
    return out


def read_folder(folder):
    idx = os.path.join(folder, "model.safetensors.index.json")
    tensors = {}
    if os.path.exists(idx):
        files = sorted(set(json.load(open(idx))["weight_map"].values()))
        for f in files:
            tensors.update(read_safetensors(os.path.join(folder, f)))
    else:
        tensors.update(read_safetensors(os.path.join(folder, "model.safetensors")))
    return tensors


def to_f32(dtype, arr):
    """bf16/f16/f32 tensor values as float32 (bf16 exactly by bit shift)."""
    a = np.asarray(arr)
    if dtype == "BF16":
        return (a.astype(np.uint32) << 16).view(np.float32).reshape(a.shape)
    if dtype == "F16":
        return a.view(np.float16).astype(np.float32)
    return a.astype(np.float32)


# ---- the restatement ----------------------------------------------------------


class IgoPlane(ctypes.Structure):
    _fields_ = [("code", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("rows", ctypes.c_int),
                ("cols", ctypes.c_int), ("row_stride", ctypes.c_int), ("groups", ctypes.c_int),
                ("group_size", ctypes.c_int)]


class IgoLayer(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int), ("share", ctypes.c_int), ("source", ctypes.c_int),
                ("gain", ctypes.c_float)] + \
               [(n, IgoPlane) for n in ("q", "k", "v", "o", "gate", "up", "down", "ple_gate", "ple_proj")] + \
               [("has_v", ctypes.c_int)] + \
               [(n, ctypes.c_void_p) for n in ("q_norm", "k_norm", "enter_norm", "after_attn_norm",
                                                "before_feed_norm", "after_feed_norm", "after_ple_norm")]


class IgoModel(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int) for n in ("vocab", "hidden", "layers", "heads", "kv_heads", "head_dim",
                                            "inner", "ple_dim", "ple_vocab", "slide_span", "window_limit")] + \
               [("eps", ctypes.c_float), ("softcap", ctypes.c_float),
                ("rope_theta", ctypes.c_double * 2), ("rope_share", ctypes.c_double * 2),
                ("rope_proportional", ctypes.c_int * 2),
                ("embed", ctypes.c_void_p), ("ple_embed", ctypes.c_void_p), ("ple_lift", IgoPlane),
                ("ple_norm", ctypes.c_void_p), ("final_norm", ctypes.c_void_p), ("head", IgoPlane),
                ("layer", ctypes.POINTER(IgoLayer))]


class KeepNote(ctypes.Structure):  # app_core.c:387-392 app_keep_note
    _fields_ = [("run_count", ctypes.c_int), ("from_list", ctypes.c_int32 * 16), ("till_list", ctypes.c_int32 * 16),
                ("mark_list", ctypes.c_uint64 * 16)]


class Taste(ctypes.Structure):  # app_core.c:60-67
    _fields_ = [("heat", ctypes.c_float), ("top_count", ctypes.c_int), ("top_portion", ctypes.c_float),
                ("echo_penalty", ctypes.c_float), ("echo_window", ctypes.c_int), ("seed", ctypes.c_uint64)]


_IGO = None


def igo_lib():
    global _IGO
    if _IGO is None:
        if not os.path.exists(IGO_LIB):
            build()
        lib = ctypes.CDLL(IGO_LIB)
        vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)
        i32p = ctypes.POINTER(ctypes.c_int32)
        for name, res, args in [
            ("igo_session_open", vp, [ctypes.POINTER(IgoModel), i]),
            ("igo_session_close", None, [vp]),
            ("igo_session_fill", i, [vp]),
            ("igo_session_prime", i, [vp, i32p, i]),
            ("igo_session_step", i, [vp, ctypes.c_int32, f]),
            ("igo_session_guess", i, [vp, i32p, i, f]),
            ("igo_session_guess_keep", i, [vp, i]),
            ("igo_session_hold", i, [vp, i]),
            ("igo_session_guess_taste", i, [vp, f, i32p, i, ctypes.POINTER(Taste), i32p]),
            ("igo_session_pick", ctypes.c_int32, [vp, f, ctypes.POINTER(Taste)]),
            ("igo_session_echo", i, [vp, i32p, i]),
            ("igo_row_code", ctypes.c_float, [ctypes.POINTER(IgoPlane), i, f]),
            ("igo_mat_mat", None, [ctypes.POINTER(IgoPlane), f, i, i, f, i, i]),
            ("igo_norm_rms", None, [f, f, i, ctypes.c_float, f]),
            ("igo_gelu_tanh", ctypes.c_float, [ctypes.c_float]),
            ("igo_logit_cap", None, [f, i, ctypes.c_float]),
            ("igo_soft_max", None, [f, i]),
            ("igo_rope_turn", None, [f, i, f, f]),
            ("igo_rope_steps", None, [ctypes.c_double, ctypes.c_double, i, i, f, ctypes.POINTER(ctypes.c_int)]),
            ("igo_plane_row", None, [ctypes.POINTER(IgoPlane), i, f]),
            ("igo_scout_open", vp, []),
            ("igo_scout_close", None, [vp]),
            ("igo_scout_clear", None, [vp]),
            ("igo_scout_note", i, [vp, i32p, i]),
            ("igo_scout_span", i, [vp]),
            ("igo_scout_draw", i, [vp, i32p, i]),
            ("igo_pick_shape", i, [f, i, ctypes.POINTER(Taste), i32p, i, i32p, f]),
            ("igo_guess_draw_state", ctypes.c_uint64, [ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64]),
            ("igo_draw_unit", ctypes.c_float, [ctypes.POINTER(ctypes.c_uint64)]),
            ("igo_cache_code8", ctypes.c_uint8, [ctypes.c_float]),
            ("igo_cache_real8", ctypes.c_float, [ctypes.c_uint8]),
        ]:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _IGO = lib
    return _IGO


def fptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def iptr(a):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))


def make_plane(code, scale_f32):
    """An IgoPlane over U8 codes [rows][bytes] and f32 scales [rows][groups]."""
    rows, stride = code.shape
    groups = scale_f32.shape[1]
    cols = stride * 2
    p = IgoPlane(code.ctypes.data, scale_f32.ctypes.data, rows, cols, stride, groups, cols // groups)
    return p


class OracleModel:
    """The restatement's model over a checkpoint folder (configuration read
    the way app_core.c:8325 config_read reads it), or over tensors already in
    memory (`tensors` name -> (dtype, array), `config` the parsed json)."""

    def __init__(self, folder=None, window_limit=4096, tensors=None, config=None):
        self.keep = []  # arrays the C struct points into
        cfg = config if config is not None else json.load(open(os.path.join(folder, "config.json")))
        tc = cfg.get("text_config", cfg)
        t = tensors if tensors is not None else read_folder(folder)
        P = next(p for p in ("model.language_model.", "language_model.model.", "model.", "")
                 if p + "embed_tokens.weight" in t)
        L = int(tc["num_hidden_layers"])
        heads = int(tc["num_attention_heads"])
        m = IgoModel()
        emb = t[P + "embed_tokens.weight"][1]
        m.vocab, m.hidden = emb.shape
        m.layers = L
        m.heads = heads
        m.kv_heads = int(tc.get("num_key_value_heads", 1))
        m.ple_dim = int(tc.get("hidden_size_per_layer_input", 0))
        m.slide_span = int(tc.get("sliding_window", 512))
        m.window_limit = int(min(window_limit, tc.get("max_position_embeddings", 131072)))
        m.eps = float(tc.get("rms_norm_eps", 1e-6))
        m.softcap = float(tc.get("final_logit_softcapping", 0.0))
        rp = tc.get("rope_parameters", {})
        for k, name, theta in ((0, "sliding_attention", 10000.0), (1, "full_attention", 1e6)):
            r = rp.get(name, {})
            m.rope_theta[k] = float(r.get("rope_theta", theta))
            m.rope_share[k] = float(r.get("partial_rotary_factor", 1.0))
            m.rope_proportional[k] = 1 if r.get("rope_type", "default") == "proportional" else 0
        self.keep.append(np.ascontiguousarray(emb))
        m.embed = self.keep[-1].ctypes.data

        def plane(stem):
            code = np.ascontiguousarray(t[stem + ".weight"][1])
            dt, sc = t[stem + ".weight_scale"]
            sc = np.ascontiguousarray(to_f32(dt, sc))
            self.keep += [code, sc]
            return make_plane(code, sc)

        def vec(stem):
            dt, v = t[stem + ".weight"] if stem + ".weight" in t else t[stem]
            a = np.ascontiguousarray(to_f32(dt, v).reshape(-1))
            self.keep.append(a)
            return a.ctypes.data

        if m.ple_dim:
            pe = np.ascontiguousarray(t[P + "embed_tokens_per_layer.weight"][1])
            self.keep.append(pe)
            m.ple_embed = pe.ctypes.data
            m.ple_vocab = pe.shape[0]
            m.ple_lift = plane(P + "per_layer_model_projection")
            m.ple_norm = vec(P + "per_layer_projection_norm")
        m.final_norm = vec(P + "norm")
        m.head = plane("lm_head")
        kinds = tc.get("layer_types")
        share = int(tc.get("num_kv_shared_layers", 0))
        first_share = L - share
        layers = (IgoLayer * L)()
        kind_of = []
        for li in range(L):
            if li == L - 1:
                kind = 1
            elif kinds:
                kind = 0 if kinds[li] == "sliding_attention" else 1
            else:
                kind = 0 if (li + 1) % 6 else 1
            kind_of.append(kind)
        for li in range(L):
            lw = layers[li]
            s = f"{P}layers.{li}."
            lw.kind = kind_of[li]
            lw.share = 1 if share > 0 and li >= first_share else 0
            lw.source = -1
            if lw.share:
                lw.source = max(p for p in range(first_share) if kind_of[p] == kind_of[li])
            lw.q = plane(s + "self_attn.q_proj")
            lw.q_norm = vec(s + "self_attn.q_norm")
            if not lw.share:
                lw.k = plane(s + "self_attn.k_proj")
                lw.v = plane(s + "self_attn.v_proj")
                lw.has_v = 1
                lw.k_norm = vec(s + "self_attn.k_norm")
            lw.o = plane(s + "self_attn.o_proj")
            lw.gate = plane(s + "mlp.gate_proj")
            lw.up = plane(s + "mlp.up_proj")
            lw.down = plane(s + "mlp.down_proj")
            lw.enter_norm = vec(s + "input_layernorm")
            lw.after_attn_norm = vec(s + "post_attention_layernorm")
            lw.before_feed_norm = vec(s + "pre_feedforward_layernorm")
            lw.after_feed_norm = vec(s + "post_feedforward_layernorm")
            if m.ple_dim:
                lw.ple_gate = plane(s + "per_layer_input_gate")
                lw.ple_proj = plane(s + "per_layer_projection")
                lw.after_ple_norm = vec(s + "post_per_layer_input_norm")
            if s + "layer_scalar" in t:
                dt, v = t[s + "layer_scalar"]
                lw.gain = float(to_f32(dt, v).reshape(-1)[0])
            else:
                lw.gain = 1.0
        m.head_dim = layers[0].q.rows // heads
        m.inner = layers[0].gate.rows
        self.layers = layers
        m.layer = layers
        self.m = m


class OracleSession:
    """app_core.c session API over the restatement."""

    def __init__(self, model, threads=8):
        self.model = model
        self.lib = igo_lib()
        self.h = self.lib.igo_session_open(ctypes.byref(model.m), threads)

    def close(self):
        if self.h:
            self.lib.igo_session_close(self.h)
            self.h = None

    def __del__(self):
        self.close()

    @property
    def fill(self):
        return self.lib.igo_session_fill(self.h)

    def prime(self, ids):
        a = np.ascontiguousarray(ids, np.int32)
        assert self.lib.igo_session_prime(self.h, iptr(a), len(a)) == 0

    def step(self, id_value):
        row = np.empty(self.model.m.vocab, np.float32)
        assert self.lib.igo_session_step(self.h, int(id_value), fptr(row)) == 0
        return row

    def guess(self, ids):
        a = np.ascontiguousarray(ids, np.int32)
        rows = np.empty((len(a), self.model.m.vocab), np.float32)
        assert self.lib.igo_session_guess(self.h, iptr(a), len(a), fptr(rows)) == 0
        return rows

    def guess_keep(self, keep):
        return self.lib.igo_session_guess_keep(self.h, int(keep))

    def hold(self, keep):
        return self.lib.igo_session_hold(self.h, int(keep))

    def guess_taste(self, rows, ids, taste):
        a = np.ascontiguousarray(ids, np.int32)
        r = np.ascontiguousarray(rows, np.float32)
        made = ctypes.c_int32()
        take = self.lib.igo_session_guess_taste(self.h, fptr(r), iptr(a), len(a), ctypes.byref(taste),
                                                ctypes.byref(made))
        return take, made.value

    def pick(self, row, taste):
        r = np.ascontiguousarray(row, np.float32)
        return self.lib.igo_session_pick(self.h, fptr(r), ctypes.byref(taste))


# ---- the reference itself ------------------------------------------------------


def _cpu_flags():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def ref_lib_path():
    flags = _cpu_flags()
    wide = {"avx512f", "avx512bw", "avx512dq", "avx512vl"} <= flags
    name = "libref_wide.so" if wide else "libref_avx2.so"
    return os.path.join(REF_DIR, name)


_REF = None
_REF_CUDA = None
REF_CUDA_PATH = os.path.join(REF_DIR, "libref_cuda.so")


def ref_cuda_lib():
    """The reference engine with its backend table served by libigllm_cuda
    (oracle/app_cuda.c), built by oracle/Makefile where the reference source
    and the CUDA library were both present."""
    global _REF_CUDA
    if _REF_CUDA is None:
        if not os.path.exists(REF_CUDA_PATH):
            raise RuntimeError(f"{REF_CUDA_PATH} is missing: run `make -C oracle all` after building the library")
        lib = _bind_ref(ctypes.CDLL(REF_CUDA_PATH))
        vp, i = ctypes.c_void_p, ctypes.c_int
        lib.ref_model_load_cuda.restype = i
        lib.ref_model_load_cuda.argtypes = [ctypes.c_char_p, i, i, i, ctypes.POINTER(vp)]
        lib.ref_desk_name.restype = ctypes.c_char_p
        lib.ref_desk_name.argtypes = [vp]
        lib.ref_cuda_status.restype = i
        lib.ref_cuda_status.argtypes = []
        lib.ref_cuda_close.restype = None
        lib.ref_cuda_close.argtypes = []
        _REF_CUDA = lib
    return _REF_CUDA


def ref_lib():
    global _REF
    if _REF is None:
        path = ref_lib_path()
        if not os.path.exists(path):
            build()
        _REF = _bind_ref(ctypes.CDLL(path))
    return _REF


def _bind_ref(lib):
    """Argument and result types of the ref_* wrappers (oracle/ref_harness.c)."""
    vp, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_float)
    i32p = ctypes.POINTER(ctypes.c_int32)
    for name, res, args in [
        ("ref_model_load", i, [ctypes.c_char_p, i, i, ctypes.POINTER(vp)]),
        ("ref_model_free", None, [vp]),
        ("ref_model_vocab", i, [vp]),
        ("ref_model_decode_bytes", ctypes.c_size_t, [vp]),
        ("ref_model_window", i, [vp]),
        ("ref_session_open", i, [vp, ctypes.POINTER(vp)]),
        ("ref_session_close", None, [vp]),
        ("ref_session_reset", None, [vp]),
        ("ref_session_fill", i, [vp]),
        ("ref_session_hold", i, [vp, i]),
        ("ref_session_prime", i, [vp, i32p, i]),
        ("ref_session_step", i, [vp, ctypes.c_int32, f]),
        ("ref_session_guess", i, [vp, i32p, i, f]),
        ("ref_session_rows", vp, [vp]),
        ("ref_session_keep", i, [vp, i]),
        ("ref_session_taste", i, [vp, f, i32p, i, ctypes.POINTER(Taste), i32p]),
        ("ref_session_pick", ctypes.c_int32, [vp, f, ctypes.POINTER(Taste)]),
        ("ref_session_serve_seconds", ctypes.c_double, [vp]),
        ("ref_session_serve_tokens", ctypes.c_size_t, [vp]),
        ("ref_model_load_bits", i, [ctypes.c_char_p, i, i, i, ctypes.POINTER(vp)]),
        ("ref_model_memory_bytes", ctypes.c_size_t, [vp]),
        ("ref_model_cache_scale", ctypes.c_float, [vp, i, i]),
        ("ref_session_cache_peak", ctypes.c_float, [vp, i, i]),
        ("ref_session_cache_room", ctypes.c_size_t, [vp]),
        ("ref_session_save", i, [vp, ctypes.c_char_p, ctypes.c_uint64, ctypes.POINTER(KeepNote), i]),
        ("ref_session_load", i, [vp, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(KeepNote),
                                 ctypes.POINTER(ctypes.c_int)]),
        ("ref_session_ids", i, [vp, i32p, i]),
        ("ref_keep_note_share", i, [ctypes.POINTER(KeepNote), ctypes.POINTER(KeepNote), i]),
        ("ref_cache_code8", None, [f, i, ctypes.POINTER(ctypes.c_uint8)]),
        ("ref_cache_real8", None, [ctypes.POINTER(ctypes.c_uint8), i, f]),
    ]:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


class RefModel:
    """The reference's model_load; with `cuda_device` set, the build whose
    backend table is libigllm_cuda's (its products on that GPU)."""

    def __init__(self, folder, threads=8, window_limit=0, cuda_device=None, cache_bits=0):
        self.h = ctypes.c_void_p()
        if cuda_device is None:
            self.lib = ref_lib()
            code = self.lib.ref_model_load_bits(str(folder).encode(), threads, window_limit, int(cache_bits),
                                                ctypes.byref(self.h))
        else:
            self.lib = ref_cuda_lib()
            code = self.lib.ref_model_load_cuda(str(folder).encode(), threads, window_limit, int(cuda_device),
                                                ctypes.byref(self.h))
        if code != 0:
            raise RuntimeError(f"reference model_load failed: {code}")
        self.vocab = self.lib.ref_model_vocab(self.h)

    def decode_bytes(self):
        return self.lib.ref_model_decode_bytes(self.h)

    def memory_bytes(self):
        return self.lib.ref_model_memory_bytes(self.h)

    def cache_scale(self, layer, value_side):
        return self.lib.ref_model_cache_scale(self.h, int(layer), int(value_side))

    def close(self):
        if self.h:
            self.lib.ref_model_free(self.h)
            self.h = ctypes.c_void_p()


class RefSession:
    def __init__(self, model):
        self.model = model
        self.lib = model.lib
        self.h = ctypes.c_void_p()
        assert self.lib.ref_session_open(model.h, ctypes.byref(self.h)) == 0

    def close(self):
        if self.h:
            self.lib.ref_session_close(self.h)
            self.h = ctypes.c_void_p()

    @property
    def fill(self):
        return self.lib.ref_session_fill(self.h)

    def reset(self):
        self.lib.ref_session_reset(self.h)

    def prime(self, ids):
        a = np.ascontiguousarray(ids, np.int32)
        assert self.lib.ref_session_prime(self.h, iptr(a), len(a)) == 0

    def step(self, id_value, want=True):
        row = np.empty(self.model.vocab, np.float32) if want else None
        assert self.lib.ref_session_step(self.h, int(id_value), fptr(row) if want else None) == 0
        return row

    def guess(self, ids, want=True):
        a = np.ascontiguousarray(ids, np.int32)
        rows = np.empty((len(a), self.model.vocab), np.float32) if want else None
        code = self.lib.ref_session_guess(self.h, iptr(a), len(a), fptr(rows) if want else None)
        if code != 0:
            raise RuntimeError("reference session_guess refused")
        return rows

    def rows_argmax(self, k):
        """Argmax of each row the last guess left in the session (app_main.c:482)."""
        p = self.lib.ref_session_rows(self.h)
        rows = np.ctypeslib.as_array(ctypes.cast(p, ctypes.POINTER(ctypes.c_float)), shape=(k * self.model.vocab,))
        return rows.reshape(k, self.model.vocab).argmax(axis=1)

    def keep(self, n):
        return self.lib.ref_session_keep(self.h, int(n))

    def hold(self, n):
        return self.lib.ref_session_hold(self.h, int(n))

    def taste(self, rows, ids, taste):
        a = np.ascontiguousarray(ids, np.int32)
        r = np.ascontiguousarray(rows, np.float32)
        made = ctypes.c_int32()
        take = self.lib.ref_session_taste(self.h, fptr(r), iptr(a), len(a), ctypes.byref(taste), ctypes.byref(made))
        return take, made.value

    def pick(self, row, taste):
        r = np.ascontiguousarray(row, np.float32)
        return self.lib.ref_session_pick(self.h, fptr(r), ctypes.byref(taste))

    def serve_seconds(self):
        return self.lib.ref_session_serve_seconds(self.h)

    def cache_peak(self, layer, value_side):
        return self.lib.ref_session_cache_peak(self.h, int(layer), int(value_side))

    def save(self, path, stamp=0, note=None, kind=0):
        return self.lib.ref_session_save(self.h, str(path).encode(), int(stamp),
                                         ctypes.byref(note) if note is not None else None, int(kind))

    def load(self, path):
        """(code, stamp, note, kind) of app_core.c:14076 session_load."""
        stamp, note, kind = ctypes.c_uint64(), KeepNote(), ctypes.c_int()
        code = self.lib.ref_session_load(self.h, str(path).encode(), ctypes.byref(stamp), ctypes.byref(note),
                                         ctypes.byref(kind))
        return code, stamp.value, note, kind.value

    def ids(self):
        n = self.lib.ref_session_ids(self.h, None, 0)
        out = np.zeros(max(n, 1), np.int32)
        self.lib.ref_session_ids(self.h, iptr(out), len(out))
        return out[:n]


def ref_cache_code8(x):
    """The reference's own cache_code8 (app_core.c:11008) over an array."""
    a = np.ascontiguousarray(x, np.float32)
    out = np.zeros(len(a), np.uint8)
    ref_lib().ref_cache_code8(fptr(a), len(a), out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)))
    return out


def ref_cache_real8(codes):
    c = np.ascontiguousarray(codes, np.uint8)
    out = np.zeros(len(c), np.float32)
    ref_lib().ref_cache_real8(c.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)), len(c), fptr(out))
    return out
