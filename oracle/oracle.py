"""TEST INFRASTRUCTURE — ctypes wrapper of the CPU oracle (_build/libneedle_oracle.so).

The oracle restates the reference's needle-core v3 path in C++ (see
oracle.hpp). Only the test suite, `__graft_entry__.smoke()` and bench.py's
cpu_baseline leg load it, as the checker; product code never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libneedle_oracle.so")
_lib = None


def build():
    r = subprocess.run(["make", "-C", HERE, "-s"], capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH) or os.environ.get("NEEDLE_ORACLE_REBUILD", "1") == "1":
            build()  # make is incremental: a no-op when the library is current
        _lib = C.CDLL(LIB_PATH)
        vp, sz = C.c_void_p, C.c_size_t
        for name, res, args in [
            ("orc_cq_new", vp, [vp, sz, sz, sz, sz, C.c_int, vp, C.c_char_p, sz]),
            ("orc_model_load", vp, [C.c_char_p, sz, C.c_char_p, sz]),
            ("orc_model_load_depth", vp, [C.c_char_p, sz, sz, C.c_char_p, sz]),
            ("orc_ladder_order", None, [sz, vp]),
            ("orc_ladder_layers", C.c_int, [sz, sz, vp]),
            ("orc_model_layer_roles", C.c_int, [vp, vp, C.c_int]),
            ("orc_model_has_confidence", C.c_int, [vp]),
            ("orc_confidence_logit", C.c_int, [vp, vp, sz, vp]),
            ("orc_probe_forward", None, [vp, sz, sz, vp, vp, vp, vp, vp, vp, sz, sz, sz, sz, vp]),
            ("orc_session_new", vp, [vp, sz, C.c_int]),
            ("orc_session_clone", vp, [vp]),
            ("orc_quant_into", C.c_float, [vp, vp, sz]),
            ("orc_f16_to_f32", C.c_float, [C.c_uint16]),
            ("orc_cq_in_padded", sz, [vp]),
            ("orc_session_pos", sz, [vp]),
            ("orc_session_bytes", sz, [vp]),
            ("orc_session_slots", sz, [vp, sz]),
            ("orc_session_saturated", C.c_int, [vp]),
            ("orc_prefill", sz, [vp, vp, vp, sz, vp]),
            ("orc_decode_step", sz, [vp, vp, C.c_uint32, vp]),
            ("orc_model_kv_bytes", sz, [vp, sz, C.c_int]),
            ("orc_max_threads", C.c_int, []),
            ("orc_ngram_valid", C.c_int, [sz, sz, vp, sz, sz]),
            ("orc_splitmix64_next", C.c_uint64, [vp]),
            ("orc_splitmix64_next_f64", C.c_double, [vp]),
            ("orc_sample", C.c_uint32, [vp, sz, C.c_float, vp]),
        ]:
            f = getattr(_lib, name)
            f.restype, f.argtypes = res, args
        for name in ["orc_cq_free", "orc_model_free", "orc_session_free"]:
            getattr(_lib, name).argtypes = [vp]
            getattr(_lib, name).restype = None
    return _lib


def set_threads(n: int):
    lib().orc_set_threads(C.c_int(n))


def P(a):
    return C.c_void_p(a.ctypes.data)


class CqWeight:
    def __init__(self, blob: bytes, out: int, inp: int, bits: int, codebook, group: int = 128):
        self.blob = np.frombuffer(blob, np.uint8).copy()
        cb = np.ascontiguousarray(codebook, np.float32)
        err = C.create_string_buffer(256)
        self.h = lib().orc_cq_new(P(self.blob), len(self.blob), out, inp, group, bits, P(cb), err, 256)
        if not self.h:
            raise ValueError(err.value.decode())
        self.out, self.inp, self.bits = out, inp, bits
        self.in_pad = lib().orc_cq_in_padded(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_cq_free(self.h)

    def prepare(self, x):
        x = np.ascontiguousarray(x, np.float32)
        xh = np.zeros(self.in_pad, np.float32)
        lib().orc_cq_prepare(C.c_void_p(self.h), P(x), P(xh))
        return xh

    def matvec(self, x):
        x = np.ascontiguousarray(x, np.float32)
        y = np.zeros(self.out, np.float32)
        lib().orc_cq_matvec(C.c_void_p(self.h), P(x), P(y))
        return y

    def matvec_prepared(self, xh, row_start=0, rows=None):
        rows = self.out - row_start if rows is None else rows
        xh = np.ascontiguousarray(xh, np.float32)
        y = np.zeros(rows, np.float32)
        lib().orc_cq_matvec_rows_prepared(C.c_void_p(self.h), P(xh), C.c_size_t(row_start), C.c_size_t(rows), P(y))
        return y

    def matvec_reference(self, xh):
        xh = np.ascontiguousarray(xh, np.float32)
        y = np.zeros(self.out, np.float32)
        lib().orc_cq_matvec_reference(C.c_void_p(self.h), P(xh), P(y))
        return y

    def matmul_prepared(self, xh, row_start=0, rows=None):
        xh = np.ascontiguousarray(xh, np.float32)
        batch = xh.shape[0]
        rows = self.out - row_start if rows is None else rows
        y = np.zeros((batch, rows), np.float32)
        lib().orc_cq_matmul_prepared(C.c_void_p(self.h), P(xh), C.c_size_t(batch), C.c_size_t(row_start),
                                     C.c_size_t(rows), P(y))
        return y

    def dequant_row(self, o):
        out = np.zeros(self.inp, np.float32)
        lib().orc_cq_dequant_row(C.c_void_p(self.h), C.c_size_t(o), P(out))
        return out

    def row_indices(self, o):
        out = np.zeros(self.in_pad, np.uint8)
        lib().orc_cq_row_indices(C.c_void_p(self.h), C.c_size_t(o), P(out))
        return out


def fwht_normalized(x):
    x = np.array(x, np.float32)
    lib().orc_fwht_normalized(P(x), C.c_size_t(len(x)))
    return x


def fake_quant(x, bits=8):
    x = np.array(x, np.float32)
    lib().orc_fake_quant(P(x), C.c_size_t(len(x)), C.c_uint32(bits))
    return x


def quant_into(x):
    x = np.ascontiguousarray(x, np.float32)
    q = np.zeros(len(x), np.int8)
    s = lib().orc_quant_into(P(x), P(q), len(x))
    return q, np.float32(s)


def attend_step(q, slots, lo, hi, heads, kv_heads, qk, vh, k=None, v=None, kq=None, ks=None, vq=None, vs=None):
    out = np.zeros(heads * vh, np.float32)
    f = lambda a, dt: None if a is None else np.ascontiguousarray(a, dt)
    q, k, v, kq, ks, vq, vs = (f(q, np.float32), f(k, np.float32), f(v, np.float32), f(kq, np.int8),
                               f(ks, np.float32), f(vq, np.int8), f(vs, np.float32))
    p = lambda a: None if a is None else P(a)
    lib().orc_attend_step(P(q), p(k), p(v), p(kq), p(ks), p(vq), p(vs), C.c_size_t(slots), C.c_size_t(lo),
                          C.c_size_t(hi), C.c_size_t(heads), C.c_size_t(kv_heads), C.c_size_t(qk),
                          C.c_size_t(vh), P(out))
    return out


def attend(q, seq, heads, kv_heads, qk, vh, window, k=None, v=None, kq=None, ks=None, vq=None, vs=None):
    out = np.zeros(seq * heads * vh, np.float32)
    f = lambda a, dt: None if a is None else np.ascontiguousarray(a, dt)
    q, k, v, kq, ks, vq, vs = (f(q, np.float32), f(k, np.float32), f(v, np.float32), f(kq, np.int8),
                               f(ks, np.float32), f(vq, np.int8), f(vs, np.float32))
    p = lambda a: None if a is None else P(a)
    lib().orc_attend(P(q), p(k), p(v), p(kq), p(ks), p(vq), p(vs), C.c_size_t(seq), C.c_size_t(heads),
                     C.c_size_t(kv_heads), C.c_size_t(qk), C.c_size_t(vh), C.c_size_t(window), P(out))
    return out


class SplitMix64:
    """The reference's sampling RNG (v3_engine.rs:446-464), in the oracle."""

    def __init__(self, seed: int):
        self.state = C.c_uint64(seed)

    def next_u64(self) -> int:
        return int(lib().orc_splitmix64_next(C.byref(self.state)))

    def next_f64(self) -> float:
        return float(lib().orc_splitmix64_next_f64(C.byref(self.state)))


def sample(logits, temperature: float, rng: SplitMix64) -> int:
    """sample (v3_engine.rs:422-443): one draw from softmax(logits / T)."""
    lg = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_sample(P(lg), len(lg), C.c_float(temperature), C.byref(rng.state)))


def engram_indices(tokens, orders, heads, slots, seed_heads=0):
    t = np.ascontiguousarray(tokens, np.uint32)
    o = np.ascontiguousarray(orders, np.uint64)
    out = np.zeros(len(t) * len(orders) * heads, np.uint32)
    lib().orc_engram_indices(P(t), C.c_size_t(len(t)), P(o), C.c_size_t(len(o)), C.c_size_t(heads),
                             C.c_uint32(slots), C.c_size_t(seed_heads), P(out))
    return out.reshape(len(t), len(orders) * heads)


def ngram_valid(p, table, orders, heads):
    o = np.ascontiguousarray(orders, np.uint64)
    return bool(lib().orc_ngram_valid(p, table, P(o), len(o), heads))


def probe_forward(cells, probes, gain, query, row_bias, proj, bias):
    """ProbeHead::forward (heads.rs:65-118) on explicit weights; cells (seq, ncells, d)."""
    cells = np.ascontiguousarray(cells, np.float32)
    seq, ncells, d = cells.shape
    probes = np.ascontiguousarray(probes, np.float32)
    k = probes.shape[0] // ncells
    query = np.ascontiguousarray(query, np.float32)
    proj = np.ascontiguousarray(proj, np.float32)
    out_dim = proj.shape[0]
    out = np.zeros(out_dim, np.float32)
    arrs = [np.ascontiguousarray(a, np.float32) for a in (gain, row_bias, bias)]
    lib().orc_probe_forward(P(cells), seq, d, P(probes), P(arrs[0]), P(query), P(arrs[1]), P(proj), P(arrs[2]),
                            ncells, k, query.shape[0], out_dim, P(out))
    return out


def ladder_order(num_layers: int):
    """ladder.rs:28: the order blocks join the ladder."""
    out = np.zeros(max(num_layers, 1), np.int64)
    lib().orc_ladder_order(C.c_size_t(num_layers), P(out))
    return [int(x) for x in out[:num_layers]]


def ladder_layers(num_layers: int, depth: int):
    """ladder.rs:67: the blocks a rung keeps, ascending, or None outside 2..=num_layers."""
    out = np.zeros(max(depth, 1), np.int64)
    if not lib().orc_ladder_layers(num_layers, depth, P(out)):
        return None
    return [int(x) for x in out[:depth]]


class Model:
    def __init__(self, raw: bytes, depth: int | None = None):
        """The full model, or the `depth`-block rung sliced at load (v3.rs:656)."""
        err = C.create_string_buffer(256)
        self.raw = raw
        if depth is None:
            self.h = lib().orc_model_load(raw, len(raw), err, 256)
        else:
            self.h = lib().orc_model_load_depth(raw, len(raw), depth, err, 256)
        if not self.h:
            raise ValueError(err.value.decode())
        g = np.zeros(14, np.int64)
        lib().orc_model_geom(C.c_void_p(self.h), P(g))
        keys = ("vocab", "out_vocab", "d_model", "heads", "kv_heads", "layers", "qk_head_dim", "v_head_dim",
                "max_seq_len", "hada_n", "lanes", "window", "conv_taps", "logit_rows")
        self.geometry = dict(zip(keys, (int(x) for x in g)))
        self.rows = self.geometry["logit_rows"]

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_free(self.h)

    def forward_sequence(self, ids):
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros((len(ids), self.rows), np.float32)
        lib().orc_forward_sequence(C.c_void_p(self.h), P(ids), C.c_size_t(len(ids)), P(out))
        return out

    def has_confidence(self) -> bool:
        return bool(lib().orc_model_has_confidence(C.c_void_p(self.h)))

    def confidence_logit(self, ids) -> float:
        """The confidence head's logit over `ids` (v3_engine.rs:351-368 before the sigmoid)."""
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros(1, np.float32)
        if not lib().orc_confidence_logit(C.c_void_p(self.h), P(ids), C.c_size_t(len(ids)), P(out)):
            raise ValueError("no confidence head or empty input")
        return float(out[0])

    def layer_roles(self):
        """(global-attention layers, Engram sites) of this model's stack."""
        out = np.zeros(64, np.int64)
        lib().orc_model_layer_roles(C.c_void_p(self.h), P(out), 64)
        ng, ns = int(out[0]), int(out[1])
        return [int(x) for x in out[2:2 + ng]], [int(x) for x in out[2 + ng:2 + ng + ns]]

    def kv_bytes(self, seq_len, int8):
        return lib().orc_model_kv_bytes(self.h, seq_len, int(int8))

    def session(self, hint=1, int8=False):
        return Session(self, hint, int8)

    def mlp(self, layer, x):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(self.geometry["d_model"], np.float32)
        lib().orc_model_mlp(C.c_void_p(self.h), C.c_size_t(layer), P(x), P(out))
        return out


class Session:
    def __init__(self, m: Model, hint: int, int8: bool, handle=None):
        self.m = m
        self.h = handle if handle is not None else lib().orc_session_new(m.h, hint, int(int8))

    def clone(self):
        return Session(self.m, 0, False, handle=lib().orc_session_clone(self.h))

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_session_free(self.h)

    @property
    def pos(self):
        return lib().orc_session_pos(self.h)

    def bytes(self):
        return lib().orc_session_bytes(self.h)

    def slots(self, li):
        return lib().orc_session_slots(self.h, li)

    def saturated(self):
        return bool(lib().orc_session_saturated(self.h))

    def prefill(self, ids):
        ids = np.ascontiguousarray(ids, np.uint32)
        out = np.zeros(self.m.rows, np.float32)
        n = lib().orc_prefill(self.m.h, self.h, P(ids), len(ids), P(out))
        return out if n else np.zeros(0, np.float32)

    def decode_step(self, tok):
        out = np.zeros(self.m.rows, np.float32)
        lib().orc_decode_step(self.m.h, self.h, int(tok), P(out))
        return out

    def kv(self, li, int8, kd, vd, kvh):
        slots = self.slots(li)
        if int8:
            kq = np.zeros(slots * kd, np.int8)
            vq = np.zeros(slots * vd, np.int8)
            ks = np.zeros(slots * kvh, np.float32)
            vs = np.zeros(slots * kvh, np.float32)
            lib().orc_session_kv(C.c_void_p(self.h), C.c_size_t(li), None, None, P(kq), P(ks), P(vq), P(vs))
            return kq, ks, vq, vs
        k = np.zeros(slots * kd, np.float32)
        v = np.zeros(slots * vd, np.float32)
        lib().orc_session_kv(C.c_void_p(self.h), C.c_size_t(li), P(k), P(v), None, None, None, None)
        return k, v


def greedy(model: Model, prompt, n_new: int, int8: bool = False):
    """Greedy continuation as V3Engine::generate_with runs it at temperature 0
    (v3_engine.rs:193-315), without EOS handling: returns (tokens, per-step logits)."""
    s = model.session(len(prompt) + n_new, int8)
    lg = s.prefill(prompt)
    toks, logs = [], [lg]
    for _ in range(n_new):
        t = int(np.argmax(lg))
        toks.append(t)
        lg = s.decode_step(t)
        logs.append(lg)
    return np.array(toks, np.uint32), np.stack(logs)
