"""Python binding of libneedle_b200.so, the B200 Needle-3 engine.

The reference's Python callers reach its engine through the C ABI with
ctypes/cffi (`examples/python-via-cffi/infer.py`, `crates/needle-python`);
this module does the same over `include/needle.h`:

    eng = V3Engine.load("needle3.cact")          # or V3Engine.from_bytes(raw)
    s = eng.session(hint=320, kv_int8=True)
    logits = s.prefill(prompt_ids)                # last-position logits
    logits = s.decode_step(token)

plus batched sessions, device-resident decode batches and single-kernel entry
points on device pointers. Every failure raises NeedleError carrying
`needle_last_error()`. There is no CPU fallback: without the built library the
import of `lib()` fails loudly.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libneedle_b200.so")

_lib = None


class NeedleError(RuntimeError):
    pass


STREAM_CB = C.CFUNCTYPE(None, C.c_char_p, C.c_void_p)


def _take_str(p) -> str | None:
    """A char* the library allocated, as text (freed); None for NULL."""
    if not p:
        return None
    try:
        return C.string_at(p).decode("utf-8")
    finally:
        lib().needle_free_str(p)


class Tokenizer:
    """The container's SentencePiece tokenizer from its RAW blob
    (SpTokenizer, sp_tokenizer.rs:116-414); host only."""

    def __init__(self, blob: bytes):
        self._t = lib().needle_tokenizer_new(blob, len(blob))
        if not self._t:
            _fail("needle_tokenizer_new")

    def encode(self, text: str) -> list[int]:
        raw = text.encode("utf-8")
        n = lib().needle_tokenizer_encode(self._t, raw, None, 0)
        if n == C.c_size_t(-1).value:
            _fail("needle_tokenizer_encode")
        out = np.zeros(max(n, 1), np.uint32)
        lib().needle_tokenizer_encode(self._t, raw, out.ctypes.data, n)
        return [int(x) for x in out[:n]]

    def decode(self, ids) -> str:
        a = np.ascontiguousarray(ids, np.uint32)
        r = _take_str(lib().needle_tokenizer_decode(self._t, a.ctypes.data, len(a)))
        if r is None:
            _fail("needle_tokenizer_decode")
        return r

    def tool_mask(self, tools_json: str, written: bytes, vocab: int, unique_keys: bool = True) -> np.ndarray:
        """The grammar mask after the tool-call bytes `written` (constrained.rs:431-461)."""
        out = np.zeros(vocab, np.float32)
        if not lib().needle_tokenizer_tool_mask(self._t, tools_json.encode(), written, len(written), unique_keys,
                                                out.ctypes.data, vocab):
            _fail("needle_tokenizer_tool_mask")
        return out

    def __del__(self):
        try:
            if self._t:
                lib().needle_tokenizer_free(self._t)
                self._t = None
        except Exception:
            pass


def lib() -> C.CDLL:
    """Load (once) and declare the C ABI."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise NeedleError(f"{LIB_PATH} is missing: build it with `python needle-rs_b200/build.py`")
    L = C.CDLL(LIB_PATH)
    vp, sz, u32p, f32p, b = C.c_void_p, C.c_size_t, C.POINTER(C.c_uint32), C.c_void_p, C.c_bool
    sig = {
        "needle_v3_load": (vp, [C.c_char_p]),
        "needle_v3_load_bytes": (vp, [C.c_char_p, sz]),
        "needle_v3_load_with_depth": (vp, [C.c_char_p, sz]),
        "needle_v3_load_bytes_with_depth": (vp, [C.c_char_p, sz, sz]),
        "needle_v3_num_layers": (sz, [vp]),
        "needle_v3_run": (vp, [vp, C.c_char_p, C.c_char_p]),
        "needle_v3_run_json": (vp, [vp, C.c_char_p, C.c_char_p]),
        "needle_v3_reasoning": (vp, [vp, C.c_char_p]),
        "needle_v3_generate": (vp, [vp, C.c_char_p, C.c_char_p, sz, C.c_float, C.c_uint64, b, b]),
        "needle_v3_run_stream": (vp, [vp, C.c_char_p, C.c_char_p, STREAM_CB, vp]),
        "needle_tokenizer_new": (vp, [C.c_char_p, sz]),
        "needle_tokenizer_free": (None, [vp]),
        "needle_tokenizer_encode": (sz, [vp, C.c_char_p, vp, sz]),
        "needle_tokenizer_decode": (vp, [vp, vp, sz]),
        "needle_tokenizer_tool_mask": (b, [vp, C.c_char_p, C.c_char_p, sz, b, vp, sz]),
        "needle_v3_has_confidence": (b, [vp]),
        "needle_v3_confidence_for": (b, [vp, C.c_char_p, C.c_char_p, C.c_char_p, vp]),
        "needle_v3_kv_bytes": (sz, [vp, sz, b]),
        "needle_v3_max_seq_len": (sz, [vp]),
        "needle_v3_free": (None, [vp]),
        "needle_free_str": (None, [vp]),
        "needle_last_error": (C.c_char_p, []),
        "needle_v3_session_new": (vp, [vp, sz, b]),
        "needle_v3_session_free": (None, [vp]),
        "needle_v3_session_pos": (sz, [vp]),
        "needle_v3_session_bytes": (sz, [vp]),
        "needle_v3_session_slots": (sz, [vp, sz]),
        "needle_v3_session_kv": (b, [vp, sz, vp, vp, vp, vp]),
        "needle_v3_prefill": (b, [vp, vp, vp, sz, f32p]),
        "needle_v3_decode_step": (b, [vp, vp, C.c_uint32, f32p]),
        "needle_v3_prefill_batch": (b, [vp, vp, vp, vp, sz, f32p, vp]),
        "needle_v3_decode_batch": (b, [vp, vp, vp, sz, f32p, vp]),
        "needle_v3_generate_ids": (sz, [vp, vp, sz, sz, C.c_float, C.c_uint64, b, C.c_uint32, vp]),
        "needle_v3_sample": (C.c_uint32, [vp, sz, C.c_float, vp]),
        "needle_v3_batch_new": (vp, [vp, vp, sz]),
        "needle_v3_batch_free": (None, [vp]),
        "needle_v3_batch_tokens": (vp, [vp]),
        "needle_v3_batch_next": (vp, [vp]),
        "needle_v3_batch_step": (b, [vp, vp, vp, b]),
        "needle_v3_batch_feed_next": (b, [vp, vp]),
        "needle_v3_batch_set_tokens": (b, [vp, vp]),
        "needle_v3_batch_profile": (b, [vp, vp, vp]),
        "needle_v3_batch_get_next": (b, [vp, vp]),
        "needle_v3_geometry": (b, [vp, vp]),
        "needle_v3_device": (C.c_int, [vp]),
        "nd_cq_project": (C.c_int, [vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, C.c_int, C.c_int, vp,
                                    C.c_int, C.c_int, C.c_int, C.c_int, vp]),
        "nd_cq_project_grouped": (C.c_int, [C.c_int, vp, vp, vp, C.c_int, C.c_int, vp, vp, C.c_int, C.c_int, vp,
                                            C.c_int, C.c_int, vp]),
        "nd_cq_prepare": (C.c_int, [vp, C.c_int, C.c_int, vp, C.c_int, vp]),
        "nd_kv_quant": (C.c_int, [vp, C.c_int, C.c_int, vp, vp, vp]),
        "nd_attend_step": (C.c_int, [vp, vp, vp, vp, vp, C.c_int, C.c_int, vp, vp, C.c_int, C.c_int,
                                     C.c_int, C.c_int, C.c_int, vp, vp]),
        "nd_last_error": (C.c_char_p, []),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def last_error() -> str | None:
    e = lib().needle_last_error()
    return e.decode() if e else None


def _fail(what: str):
    raise NeedleError(f"{what}: {last_error()}")


def _ptr(a: np.ndarray | None):
    return None if a is None else a.ctypes.data


GEOM_KEYS = ("vocab", "out_vocab", "d_model", "heads", "kv_heads", "layers", "qk_head_dim",
             "v_head_dim", "max_seq_len", "hada_n", "lanes", "window", "conv_taps", "logit_rows")


class V3Engine:
    """A loaded container on the current CUDA device (V3Engine, v3_engine.rs:29-385)."""

    def __init__(self, handle: int):
        self._h = handle
        g = np.zeros(14, np.int64)
        if not lib().needle_v3_geometry(self._h, g.ctypes.data):
            _fail("geometry")
        self.geometry = dict(zip(GEOM_KEYS, (int(x) for x in g)))
        self.logit_rows = self.geometry["logit_rows"]

    @classmethod
    def from_bytes(cls, raw: bytes, depth: int | None = None) -> "V3Engine":
        """`depth` loads that rung of the intelligence ladder
        (from_bytes_with_depth, v3_engine.rs:140-143)."""
        if depth is None:
            h = lib().needle_v3_load_bytes(raw, len(raw))
            if not h:
                _fail("needle_v3_load_bytes")
        else:
            h = lib().needle_v3_load_bytes_with_depth(raw, len(raw), depth)
            if not h:
                _fail("needle_v3_load_bytes_with_depth")
        return cls(h)

    @classmethod
    def load(cls, path: str, depth: int | None = None) -> "V3Engine":
        """`depth` as in load_with_depth (v3_engine.rs:132-138)."""
        if depth is None:
            h = lib().needle_v3_load(path.encode())
            if not h:
                _fail("needle_v3_load")
        else:
            h = lib().needle_v3_load_with_depth(path.encode(), depth)
            if not h:
                _fail("needle_v3_load_with_depth")
        return cls(h)

    def close(self):
        if self._h:
            lib().needle_v3_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def handle(self):
        return self._h

    def kv_bytes(self, seq_len: int, kv_int8: bool = False) -> int:
        return lib().needle_v3_kv_bytes(self._h, seq_len, kv_int8)

    def max_seq_len(self) -> int:
        return lib().needle_v3_max_seq_len(self._h)

    def num_layers(self) -> int:
        return lib().needle_v3_num_layers(self._h)

    # ---- text level (V3Engine::run / run_json / generate / generate_with)
    def _text(self, p, what):
        r = _take_str(p)
        if r is None:
            _fail(what)
        return r

    def run(self, query: str, tools_json: str) -> str:
        return self._text(lib().needle_v3_run(self._h, query.encode(), tools_json.encode()), "needle_v3_run")

    def run_json(self, query: str, tools_json: str) -> str:
        return self._text(lib().needle_v3_run_json(self._h, query.encode(), tools_json.encode()),
                          "needle_v3_run_json")

    def generate(self, query: str, tools_json: str, max_new_tokens: int = 0, temperature: float = 0.0,
                 seed: int = 0, constrain: bool = False, kv_int8: bool = False) -> str:
        return self._text(lib().needle_v3_generate(self._h, query.encode(), tools_json.encode(), max_new_tokens,
                                                   temperature, seed, constrain, kv_int8), "needle_v3_generate")

    def run_stream(self, query: str, tools_json: str, on_piece) -> str:
        cb = STREAM_CB(lambda piece, _ud: on_piece(piece.decode("utf-8")))
        return self._text(lib().needle_v3_run_stream(self._h, query.encode(), tools_json.encode(), cb, None),
                          "needle_v3_run_stream")

    def has_confidence(self) -> bool:
        return bool(lib().needle_v3_has_confidence(self._h))

    def confidence_for(self, query: str, tools_json: str, completion: str) -> float:
        """Probability from the confidence head (V3Engine::confidence_for, v3_engine.rs:351-368)."""
        out = np.zeros(1, np.float32)
        if not lib().needle_v3_confidence_for(self._h, query.encode(), tools_json.encode(), completion.encode(),
                                              out.ctypes.data):
            _fail("needle_v3_confidence_for")
        return float(out[0])

    def reasoning(self, text: str) -> str | None:
        return _take_str(lib().needle_v3_reasoning(self._h, text.encode()))

    def session(self, hint: int = 1, kv_int8: bool = False) -> "Session":
        s = lib().needle_v3_session_new(self._h, hint, kv_int8)
        if not s:
            _fail("needle_v3_session_new")
        return Session(self, s, kv_int8)

    def prefill_batch(self, sessions, prompts, logits: bool = True):
        """Prefill fresh sessions; returns (last logits [n, rows] or None, picks [n])."""
        n = len(sessions)
        arr = (C.c_void_p * n)(*[s._s for s in sessions])
        ids = np.concatenate([np.asarray(p, np.uint32) for p in prompts]) if n else np.zeros(0, np.uint32)
        lens = np.array([len(p) for p in prompts], np.uint64)
        out = np.zeros((n, self.logit_rows), np.float32) if logits else None
        picks = np.zeros(n, np.uint32)
        if not lib().needle_v3_prefill_batch(self._h, arr, ids.ctypes.data, lens.ctypes.data, n,
                                             _ptr(out), picks.ctypes.data):
            _fail("needle_v3_prefill_batch")
        return out, picks

    def group(self, sessions) -> "SessionGroup":
        """The sessions as a group for repeated batched calls (decode_batch)."""
        return SessionGroup(sessions)

    def decode_batch(self, sessions, tokens, logits: bool = True):
        """One decode step of every session (a list or a SessionGroup) with host
        tokens in; returns (logits [n, rows] or None, picks [n])."""
        n = len(sessions)
        arr = sessions._arr if isinstance(sessions, SessionGroup) else (C.c_void_p * n)(*[s._s for s in sessions])
        tok = np.ascontiguousarray(tokens, np.uint32)
        out = np.zeros((n, self.logit_rows), np.float32) if logits else None
        picks = np.zeros(n, np.uint32)
        if not lib().needle_v3_decode_batch(self._h, arr, tok.ctypes.data, n, _ptr(out), picks.ctypes.data):
            _fail("needle_v3_decode_batch")
        return out, picks

    def generate_ids(self, prompt, max_new_tokens: int, temperature: float = 0.0, seed: int = 0,
                     kv_int8: bool = False, eos_id: int | None = None) -> np.ndarray:
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(1, max_new_tokens), np.uint32)
        n = lib().needle_v3_generate_ids(self._h, p.ctypes.data, len(p), max_new_tokens, temperature,
                                         seed, kv_int8, 0xFFFFFFFF if eos_id is None else eos_id,
                                         out.ctypes.data)
        if n == C.c_size_t(-1).value:
            _fail("needle_v3_generate_ids")
        return out[:n].copy()

    def batch(self, sessions) -> "Batch":
        n = len(sessions)
        arr = (C.c_void_p * n)(*[s._s for s in sessions])
        b = lib().needle_v3_batch_new(self._h, arr, n)
        if not b:
            _fail("needle_v3_batch_new")
        return Batch(self, b, list(sessions))


class SessionGroup:
    """A fixed list of one engine's sessions whose handle array is built once,
    for repeated batched calls (building it from a list of thousands of
    sessions costs about as much as a decode step's host work). Holds the
    sessions; they must stay open while the group is used."""

    def __init__(self, sessions):
        self.sessions = list(sessions)
        self._arr = (C.c_void_p * len(self.sessions))(*[s._s for s in self.sessions])

    def __len__(self):
        return len(self.sessions)


class Session:
    """A device KV cache (V3Cache, cache.rs:148-527)."""

    def __init__(self, eng: V3Engine, s: int, kv_int8: bool):
        self.eng, self._s, self.kv_int8 = eng, s, kv_int8

    def close(self):
        if self._s:
            lib().needle_v3_session_free(self._s)
            self._s = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def pos(self) -> int:
        return lib().needle_v3_session_pos(self._s)

    def bytes(self) -> int:
        return lib().needle_v3_session_bytes(self._s)

    def slots(self, layer: int) -> int:
        return lib().needle_v3_session_slots(self._s, layer)

    def kv(self, layer: int):
        """Layer `layer`'s ring in the reference's layout (V3Cache::kv,
        cache.rs:382-393), flattened: (k, v) f32 [slots * kv_heads * dim], or
        for int8 (kq, k_scale, vq, v_scale) with scales [slots * kv_heads]."""
        g = self.eng.geometry
        n, kvh = self.slots(layer), g["kv_heads"]
        dt = np.int8 if self.kv_int8 else np.float32
        k = np.zeros(n * kvh * g["qk_head_dim"], dt)
        v = np.zeros(n * kvh * g["v_head_dim"], dt)
        ks = np.zeros(n * kvh, np.float32) if self.kv_int8 else None
        vs = np.zeros(n * kvh, np.float32) if self.kv_int8 else None
        if not lib().needle_v3_session_kv(self._s, layer, k.ctypes.data, v.ctypes.data, _ptr(ks), _ptr(vs)):
            _fail("needle_v3_session_kv")
        return (k, ks, v, vs) if self.kv_int8 else (k, v)

    def prefill(self, ids) -> np.ndarray:
        a = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros(self.eng.logit_rows, np.float32)
        if not lib().needle_v3_prefill(self.eng._h, self._s, a.ctypes.data, len(a), out.ctypes.data):
            _fail("needle_v3_prefill")
        return out

    def decode_step(self, token: int) -> np.ndarray:
        out = np.zeros(self.eng.logit_rows, np.float32)
        if not lib().needle_v3_decode_step(self.eng._h, self._s, int(token), out.ctypes.data):
            _fail("needle_v3_decode_step")
        return out


class Batch:
    """Sessions decoded together from device-resident tokens (graph-replayed)."""

    def __init__(self, eng: V3Engine, b: int, sessions):
        self.eng, self._b, self.sessions = eng, b, sessions

    def close(self):
        if self._b:
            lib().needle_v3_batch_free(self._b)
            self._b = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def tokens_ptr(self) -> int:
        return lib().needle_v3_batch_tokens(self._b)

    @property
    def next_ptr(self) -> int:
        return lib().needle_v3_batch_next(self._b)

    def step(self, d_logits: int | None = None, stream: int | None = None, use_graph: bool = True):
        if not lib().needle_v3_batch_step(self._b, d_logits, stream, use_graph):
            _fail("needle_v3_batch_step")

    def feed_next(self, stream: int | None = None):
        if not lib().needle_v3_batch_feed_next(self._b, stream):
            _fail("needle_v3_batch_feed_next")

    def set_tokens(self, tokens):
        t = np.ascontiguousarray(tokens, np.uint32)
        assert len(t) == len(self.sessions)
        if not lib().needle_v3_batch_set_tokens(self._b, t.ctypes.data):
            _fail("needle_v3_batch_set_tokens")

    PROFILE_KINDS = ("engram", "embed", "layer_pre", "qkvg_proj", "qkv_post", "attention", "attn_finish",
                     "out_proj", "layer_post", "final", "lm_head", "bookkeeping")

    def profile(self):
        """One eager step with per-kernel-group timing: ({kind: ms}, launches)."""
        ms = np.zeros(12, np.float32)
        n = C.c_int(0)
        if not lib().needle_v3_batch_profile(self._b, ms.ctypes.data, C.addressof(n)):
            _fail("needle_v3_batch_profile")
        return dict(zip(self.PROFILE_KINDS, (float(x) for x in ms))), n.value

    def get_next(self) -> np.ndarray:
        out = np.zeros(len(self.sessions), np.uint32)
        if not lib().needle_v3_batch_get_next(self._b, out.ctypes.data):
            _fail("needle_v3_batch_get_next")
        return out


def sample(logits, temperature: float, state: int) -> tuple[int, int]:
    """One temperature draw (sample + SplitMix64, v3_engine.rs:422-464):
    returns (token id, the generator's next state)."""
    lg = np.ascontiguousarray(logits, np.float32)
    st = C.c_uint64(state)
    pick = lib().needle_v3_sample(lg.ctypes.data, len(lg), temperature, C.byref(st))
    if pick == 0xFFFFFFFF:
        _fail("needle_v3_sample")
    return int(pick), int(st.value)


# ------------------------------------------------------------------ kernels
def _check(rc: int, what: str):
    if rc != 0:
        raise NeedleError(f"{what}: {lib().nd_last_error().decode()}")


def cq_project(packed_ptr, norms_ptr, rows, in_feat, bits, levels, xh_ptr, ldx, M, y_ptr, ldy,
               row0=0, nrows=None, path=0, stream=None):
    lv = np.zeros(16, np.float32)
    lv[: 1 << bits] = np.asarray(levels, np.float32)[: 1 << bits]
    _check(lib().nd_cq_project(packed_ptr, norms_ptr, rows, in_feat, bits, lv.ctypes.data, xh_ptr, ldx,
                               M, y_ptr, ldy, row0, rows - row0 if nrows is None else nrows, path, stream),
           "nd_cq_project")


def cq_project_grouped(mats, in_feat, bits, levels, xh_ptr, ldx, M, y_ptr, ldy, path=0, stream=None):
    """mats: [(packed_ptr, norms_ptr, rows)], up to four matrices sharing
    in_feat, bits and levels; y [M][ldy] receives their rows side by side."""
    n = len(mats)
    packed = (C.c_void_p * n)(*[m[0] for m in mats])
    norms = (C.c_void_p * n)(*[m[1] for m in mats])
    rows = (C.c_int * n)(*[m[2] for m in mats])
    lv = np.zeros(16, np.float32)
    lv[: 1 << bits] = np.asarray(levels, np.float32)[: 1 << bits]
    _check(lib().nd_cq_project_grouped(n, C.cast(packed, C.c_void_p), C.cast(norms, C.c_void_p),
                                       C.cast(rows, C.c_void_p), in_feat, bits, lv.ctypes.data, xh_ptr, ldx, M,
                                       y_ptr, ldy, path, stream),
           "nd_cq_project_grouped")


def cq_prepare(x_ptr, M, in_feat, xh_ptr, ld_out, stream=None):
    _check(lib().nd_cq_prepare(x_ptr, M, in_feat, xh_ptr, ld_out, stream), "nd_cq_prepare")


def kv_quant(x_ptr, rows, dim, q_ptr, scales_ptr, stream=None):
    _check(lib().nd_kv_quant(x_ptr, rows, dim, q_ptr, scales_ptr, stream), "nd_kv_quant")


def attend_step(q_ptr, k_ptr, v_ptr, ks_ptr, vs_ptr, int8, slots, lo_ptr, hi_ptr, B, heads, kv_heads,
                qk, vh, out_ptr, stream=None):
    _check(lib().nd_attend_step(q_ptr, k_ptr, v_ptr, ks_ptr, vs_ptr, int(int8), slots, lo_ptr, hi_ptr, B,
                                heads, kv_heads, qk, vh, out_ptr, stream), "nd_attend_step")
