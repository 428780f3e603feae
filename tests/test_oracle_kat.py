"""Known-answer tests of the reference's inline unit tests, run against the CPU
oracle (each cites the reference test it ports), plus the reference's
self-consistency invariants (decode == prefill, int8 stepping == int8 prefill)."""
import numpy as np
import pytest
from conftest import cact_pack, orc

# ------------------------------------------------------------------ hadamard.rs:102-172


def test_fwht_matches_dense_walsh_and_is_an_involution():
    rng = np.random.default_rng(0)
    for n in (8, 128, 1024):
        x = rng.normal(size=n).astype(np.float32)
        y = orc.fwht_normalized(x)
        dense = (cact_pack.walsh(n) @ x.astype(np.float64)).astype(np.float32)
        assert np.max(np.abs(y - dense)) < 1e-5
        assert np.max(np.abs(orc.fwht_normalized(y) - x)) < 1e-5


def test_f16_round_trip_over_all_halves():
    # math.rs:74-104: exact for every binary16 value.
    h = np.arange(65536, dtype=np.uint16)
    want = h.view(np.float16).astype(np.float32)
    got = np.array([orc.lib().orc_f16_to_f32(int(v)) for v in h[::97]], np.float32)
    w = want[::97]
    same = (got == w) | (np.isnan(got) & np.isnan(w))
    assert same.all()


# ------------------------------------------------------------------ cq.rs:1094-1420
def _case(out, inp, bits, seed=0):
    rng = np.random.default_rng(seed)
    cb = cact_pack.lloyd_codebook()
    idx, norms = cact_pack.random_cq(rng, out, inp, bits)
    blob = cact_pack.cq_blob(idx, norms, bits)
    return cb, idx, norms, blob


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("inp", [256, 200])
def test_dequant_and_matvec_match_dense_reconstruction(bits, inp):
    cb, idx, norms, blob = _case(12, inp, bits)
    w = orc.CqWeight(blob, 12, inp, bits, cb)
    dense = cact_pack.dequantize(idx, norms, bits, cb, inp)
    for o in range(12):
        assert np.max(np.abs(w.dequant_row(o) - dense[o])) < 1e-5
        assert np.array_equal(w.row_indices(o), idx[o])  # LSB-first unpack, bit-exact
    x = np.random.default_rng(1).normal(size=inp).astype(np.float32)
    y = w.matvec(x)
    assert np.max(np.abs(y - dense @ x)) < 1e-4 * max(1.0, np.abs(dense @ x).max())
    # The lane-split LUT path agrees with the single-accumulator reference (cq.rs:381).
    xh = w.prepare(x)
    assert np.max(np.abs(w.matvec_prepared(xh) - w.matvec_reference(xh))) < 1e-5


@pytest.mark.parametrize("bits", [2, 4])
def test_matmul_is_bit_identical_to_repeated_matvec(bits):
    # cq.rs:1198 — the batched path decodes once per group and sums in the same lane order.
    cb, idx, norms, blob = _case(300, 768, bits)
    w = orc.CqWeight(blob, 300, 768, bits, cb)
    xh = np.stack([w.prepare(np.random.default_rng(i).normal(size=768).astype(np.float32)) for i in range(40)])
    mm = w.matmul_prepared(xh, 5, 290)
    mv = np.stack([w.matvec_prepared(x, 5, 290) for x in xh])
    assert np.array_equal(mm, mv)


def test_bad_geometry_is_rejected():
    cb, idx, norms, blob = _case(4, 128, 2)
    with pytest.raises(ValueError):
        orc.CqWeight(blob, 4, 128, 2, cb, group=96)  # not a power of two
    with pytest.raises(ValueError):
        orc.CqWeight(blob[:-3], 4, 128, 2, cb)  # short blob
    with pytest.raises(ValueError):
        orc.CqWeight(blob, 4, 128, 7, cb)  # unsupported width


# ------------------------------------------------------------------ v3/attention.rs:383-456
def test_conv_is_causal_and_zero_padded():
    buf = np.array([1.0, 2.0, 3.0], np.float32)
    orc.lib().orc_causal_conv(orc.P(buf), orc.P(np.array([10.0, 100.0], np.float32)), 3, 1, 2)
    assert list(buf) == [10.0, 120.0, 230.0]


def test_attend_step_wraps_the_ring():
    out = orc.attend_step([0.0], 3, 2, 4, 1, 1, 1, 1, k=[1.0, 1.0, 1.0], v=[30.0, 40.0, 20.0])
    assert abs(out[0] - 30.0) < 1e-5


def test_a_window_of_one_attends_only_to_itself():
    out = orc.attend([1.0, 1.0], 2, 1, 1, 1, 1, 1, k=[1.0, 1.0], v=[5.0, 9.0])
    assert list(out) == [5.0, 9.0]
    out2 = orc.attend([1.0, 1.0], 2, 1, 1, 1, 1, 0, k=[1.0, 1.0], v=[5.0, 9.0])
    assert out2[0] == 5.0 and abs(out2[1] - 7.0) < 1e-6


# ------------------------------------------------------------------ v3/kernels.rs:195-225
def test_hada_blocks_and_kron():
    import ctypes as C
    for n, want in ((1024, (32, 32)), (512, (16, 32)), (256, (16, 16))):
        ba, bb = C.c_size_t(), C.c_size_t()
        orc.lib().orc_hada_blocks(C.c_size_t(n), C.byref(ba), C.byref(bb))
        assert (ba.value, bb.value) == want
    out = np.zeros(4, np.float32)
    z = np.array([1, 2, 3, 4], np.float32)
    a = np.array([1, 2, 3, 4], np.float32)
    b = np.array([0, 1, 1, 0], np.float32)
    orc.lib().orc_kron_apply(orc.P(z), orc.P(a), orc.P(b), C.c_size_t(2), C.c_size_t(2), orc.P(out))
    assert list(out) == [14.0, 10.0, 20.0, 14.0]


# ------------------------------------------------------------------ v3/engram.rs:139-172
def test_engram_hash_known_answers():
    a = orc.engram_indices([10, 20, 30], [2], 1, 18432)
    b = orc.engram_indices([10, 99, 30], [2], 1, 18432)
    assert a[0, 0] == b[0, 0] and a[1, 0] != b[1, 0] and a[2, 0] != b[2, 0]
    row = orc.engram_indices([7, 8, 9], [2, 3], 3, 18432)[2]
    assert len(set(row.tolist())) > 1
    assert not orc.ngram_valid(0, 0, [2, 3], 1) and orc.ngram_valid(1, 0, [2, 3], 1)
    assert not orc.ngram_valid(1, 1, [2, 3], 1) and orc.ngram_valid(2, 1, [2, 3], 1)


def test_engram_hash_matches_an_independent_restatement():
    # u32 FNV-style mix of engram.rs:31-61, written out in numpy.
    toks = np.random.default_rng(3).integers(0, 8192, 40).astype(np.uint32)
    got = orc.engram_indices(toks, [2, 3], 3, 18432)
    for oi, order in enumerate((2, 3)):
        for h in range(3):
            seed = np.uint32((0x9E3779B9 * (oi * 3 + h + 1)) & 0xFFFFFFFF)
            for p in range(40):
                acc = int(seed)
                for j in range(order):
                    t = 0 if j > p else int(toks[p - j])
                    acc = ((acc ^ t) * 0x01000193) & 0xFFFFFFFF
                acc ^= acc >> 15
                assert got[p, oi * 3 + h] == acc % 18432


# ------------------------------------------------------------------ v3/mhc.rs:154-238
def test_mhc_mix_down_and_scatter():
    import ctypes as C
    lanes = np.array([1.0, 2.0, 10.0, 20.0], np.float32)
    rows = np.zeros(2, np.float32)
    u = np.zeros(2, np.float32)
    orc.lib().orc_mix_down(orc.P(lanes), orc.P(rows), C.c_float(0.0), orc.P(np.zeros(2, np.float32)),
                           C.c_size_t(0), C.c_size_t(2), C.c_size_t(2), orc.P(u))
    hi, lo = 1 / (1 + np.exp(-4.0)), 1 / (1 + np.exp(4.0))
    assert abs(u[0] - (hi + lo * 10)) < 1e-6 and abs(u[1] - (hi * 2 + lo * 20)) < 1e-6
    buf = np.arange(1, 7, dtype=np.float32)
    before = buf.sum()
    post = np.zeros(3, np.float32)
    res = np.full(9, 0.3, np.float32)
    y = np.array([7.0, 8.0], np.float32)
    orc.lib().orc_scatter_up(orc.P(buf), orc.P(post), orc.P(res), orc.P(y), C.c_float(1.0), C.c_float(1.0),
                             orc.P(np.full(3, -100.0, np.float32)), orc.P(np.zeros(9, np.float32)),
                             C.c_size_t(0), C.c_size_t(3), C.c_size_t(2))
    assert abs(buf.sum() - before) < 1e-3


# ------------------------------------------------------------------ cache.rs + kv quant parity
def test_kv_quant_edge_cases():
    assert np.all(orc.fake_quant(np.zeros(48, np.float32)) == 0)
    x = (np.sin(np.arange(64) * 0.37) * 3).astype(np.float32)
    step = np.abs(x).max() / 127
    assert np.all(np.abs(orc.fake_quant(x) - x) <= step * 0.5 + 1e-6)
    q, s = orc.quant_into(x)
    assert np.array_equal(q.astype(np.float32) * s, orc.fake_quant(x))


def test_requantising_a_fake_quantised_vector_is_stable():
    # The prefill path quantises fake-quantised K/V again (model.rs:785-829); the
    # codes and scale must equal those of quantising the raw vector once.
    rng = np.random.default_rng(5)
    for _ in range(2000):
        x = (rng.normal(size=48) * 10 ** rng.uniform(-3, 3)).astype(np.float32)
        q1, s1 = orc.quant_into(x)
        q2, s2 = orc.quant_into(orc.fake_quant(x))
        assert np.array_equal(q1, q2) and s1 == s2


def test_hoisted_scale_reader_matches_dequantised_buffer():
    # v3_kv_quant_parity.rs:102-218.
    rng = np.random.default_rng(7)
    H, KVH, QK, V, S = 4, 2, 48, 64, 17
    q = rng.uniform(-1, 1, H * QK).astype(np.float32)
    k = np.concatenate([rng.uniform(-1, 1, QK) * (1 if r % 2 == 0 else 40) for r in range(S * KVH)]).astype(np.float32)
    v = np.concatenate([rng.uniform(-1, 1, V) * (0.01 if r % 2 == 0 else 3) for r in range(S * KVH)]).astype(np.float32)
    kd = np.concatenate([orc.fake_quant(c) for c in k.reshape(-1, QK)])
    vd = np.concatenate([orc.fake_quant(c) for c in v.reshape(-1, V)])
    kq, ks = zip(*[orc.quant_into(c) for c in k.reshape(-1, QK)])
    vq, vs = zip(*[orc.quant_into(c) for c in v.reshape(-1, V)])
    for lo, hi in ((0, 0), (0, 9), (3, 16), (5, 5)):
        a = orc.attend_step(q, S, lo, hi, H, KVH, QK, V, k=kd, v=vd)
        b = orc.attend_step(q, S, lo, hi, H, KVH, QK, V, kq=np.concatenate(kq), ks=np.array(ks),
                            vq=np.concatenate(vq), vs=np.array(vs))
        rms = np.sqrt(np.mean(a ** 2))
        assert np.max(np.abs(a - b)) < 1e-5 * max(rms, 1.0)


def test_kv_bytes_match_config_rs(full_oracle):
    # config.rs:311-374
    assert full_oracle.kv_bytes(512, False) == 512 * 20 * 224 * 4
    assert full_oracle.kv_bytes(512, True) == 512 * 20 * (224 + 16)


# ------------------------------------------------------------------ model-level invariants
@pytest.mark.parametrize("int8", [False, True])
def test_decode_steps_equal_prefill_bit_for_bit(tiny_oracle, int8):
    # v3_forward_parity.rs:133-199 and v3_kv_int8.rs:190-302: stepping a prompt equals
    # prefilling it, exactly, in f32 and in int8 - including through the window ring.
    m = tiny_oracle
    toks = np.random.default_rng(2).integers(1, 512, 30).astype(np.uint32)
    s = m.session(4, int8)
    outs = [s.prefill(toks[:3])]
    for t in toks[3:]:
        outs.append(s.decode_step(t))
    for n in (3, 11, 30):
        p = m.session(30, int8)
        assert np.array_equal(p.prefill(toks[:n]), outs[n - 3])


def test_prefilled_cache_continues_like_a_stepped_one(tiny_oracle):
    # v3_forward_parity.rs:259-328: 24-token continuation after a batched prefill.
    m = tiny_oracle
    toks = np.random.default_rng(4).integers(1, 512, 14).astype(np.uint32)
    a, b = m.session(64), m.session(64)
    a.prefill(toks)
    b.prefill(toks[:1])
    for t in toks[1:]:
        b.decode_step(t)
    rng = np.random.default_rng(5)
    for t in rng.integers(1, 512, 24):
        assert np.array_equal(a.decode_step(t), b.decode_step(t))


def test_cache_growth_and_window(tiny_oracle):
    m = tiny_oracle  # window 8, global layers 1 and 3, max_seq 96
    s = m.session(2)
    s.prefill(np.arange(1, 21, dtype=np.uint32))
    assert s.slots(0) == 8 and s.slots(2) == 8  # local layers cap at the window
    assert s.slots(1) >= 20 and s.slots(3) >= 20  # global layers grow
