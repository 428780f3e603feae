"""The confidence probe head on the CPU: the oracle's ProbeHead against the
reference's own cases (crates/needle-core/src/v3/heads.rs:284-313) and a numpy
restatement of heads.rs:65-177, and its ladder slice against a rung written as
a container of its own (v3.rs:745-787)."""
import numpy as np
import pytest
from conftest import cact_pack, orc
from rung_container import header_layers, write_rung


def test_a_zero_probe_averages_the_sequence():
    d = 4
    out = orc.probe_forward(np.array([[[1, 0, 0, 0]], [[3, 0, 0, 0]]], np.float32), np.zeros((1, d)), [1.0],
                            np.zeros((1, d)), [0.0], np.ones((1, d)), [0.5])
    assert abs(out[0] - (2.0 / np.sqrt(4.0 / 4.0) + 0.5)) < 1e-5


def test_the_gain_scales_the_summary():
    d = 4
    args = (np.zeros((1, d)),)
    cells = np.array([[[2, 0, 0, 0]]], np.float32)
    base = orc.probe_forward(cells, *args, [1.0], np.zeros((1, d)), [0.0], np.ones((1, d)), [0.5])[0] - 0.5
    scaled = orc.probe_forward(cells, *args, [3.0], np.zeros((1, d)), [0.0], np.ones((1, d)), [0.5])[0] - 0.5
    assert abs(scaled - 3 * base) < 1e-4


def numpy_head(cells, probes, gain, query, row_bias, proj, bias):
    seq, l1, d = cells.shape
    k = probes.shape[0] // l1
    q = query.shape[0]
    c = cells.astype(np.float64)
    r = np.zeros((l1 * k, d))
    for pair in range(l1 * k):
        s = c[:, pair // k, :] @ probes[pair] / np.sqrt(d)
        w = np.exp(s - s.max())
        w /= w.sum()
        v = w @ c[:, pair // k, :]
        r[pair] = v / np.sqrt(np.mean(v * v) + 1e-6) * gain[pair]
    pooled = np.zeros((q, d))
    for qi in range(q):
        u = r @ query[qi] / np.sqrt(d) + row_bias[qi]
        w = np.exp(u - u.max())
        w /= w.sum()
        pooled[qi] = w @ r
    return proj @ pooled.reshape(-1) + bias


def test_random_head_against_numpy():
    rng = np.random.default_rng(0)
    seq, l1, k, q, d = 37, 5, 3, 2, 64
    cells = rng.normal(0, 1, (seq, l1, d)).astype(np.float32)
    w = dict(probes=rng.normal(0, 0.2, (l1 * k, d)), gain=1 + rng.normal(0, 0.1, l1 * k),
             query=rng.normal(0, 0.2, (q, d)), row_bias=rng.normal(0, 0.3, (q, l1 * k)),
             proj=rng.normal(0, 0.1, (2, q * d)), bias=rng.normal(0, 0.1, 2))
    w = {a: np.asarray(v, np.float32) for a, v in w.items()}
    got = orc.probe_forward(cells, w["probes"], w["gain"], w["query"], w["row_bias"], w["proj"], w["bias"])
    want = numpy_head(cells, **{a: v.astype(np.float64) for a, v in w.items()})
    assert np.allclose(got, want, rtol=1e-4, atol=1e-5), (got, want)


@pytest.fixture(scope="module")
def head_raw():
    return cact_pack.build_container(cact_pack.tiny(), seed=1, confidence_head=True)


def test_container_head_loads_and_scores(head_raw, tiny_raw):
    m = orc.Model(head_raw)
    assert m.has_confidence() and not orc.Model(tiny_raw).has_confidence()
    ids = np.random.default_rng(3).integers(1, 512, 40).astype(np.uint32)
    assert np.isfinite(m.confidence_logit(ids))
    # the head does not change the forward
    assert np.array_equal(m.session(40, False).prefill(ids), orc.Model(tiny_raw).session(40, False).prefill(ids))


@pytest.mark.parametrize("depth", [2, 3])
def test_rung_head_equals_a_rung_container(head_raw, depth):
    kept = orc.ladder_layers(header_layers(head_raw), depth)
    built, sliced = orc.Model(write_rung(head_raw, kept)), orc.Model(head_raw, depth)
    ids = np.random.default_rng(depth).integers(1, 512, 25).astype(np.uint32)
    assert built.has_confidence() and sliced.has_confidence()
    assert built.confidence_logit(ids) == sliced.confidence_logit(ids)
    assert sliced.confidence_logit(ids) != orc.Model(head_raw).confidence_logit(ids)


def test_c_abi_reads_the_head_records_before_any_gpu_work(head_raw):
    from conftest import nb
    lib = nb.lib()
    h = lib.needle_v3_load_bytes(head_raw, len(head_raw))
    if h:  # a machine with a GPU loads it
        lib.needle_v3_free(h)
    else:
        assert b"head" not in lib.needle_last_error()
    # A manifest naming the router (code 3, seven tensors) where only six follow.
    _, _, recs = cact_pack.read_directory(head_raw)
    man = [r for r in recs if r["shape"] == [1] and r["dtype"] == 1][-2]
    bad = bytearray(head_raw)
    bad[man["offset"]:man["offset"] + 2] = np.float16(3.0).tobytes()
    assert lib.needle_v3_load_bytes(bytes(bad), len(bad)) is None
    assert b"head tensors ran out" in lib.needle_last_error()
