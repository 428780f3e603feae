"""Ladder rungs on the GPU: needle_v3_load_with_depth / the bytes form slice the
container at load (v3.rs:656-745) and the engine's forward matches the oracle's
rung, and is bit-identical to the same rung written as a container of its own
(the mHC lane-matrix rows are then addressed through the container's block
numbers on one side and the rung's on the other)."""
import numpy as np
import pytest
from conftest import nb, orc
from rung_container import header_layers, write_rung
from test_gpu_model import rel_err, tol

pytestmark = pytest.mark.gpu


def _run(model, ids, steps, int8, tokens=None):
    s = model.session(len(ids) + steps, int8)
    out = [s.prefill(ids)]
    for i in range(steps):
        t = int(np.argmax(out[-1])) if tokens is None else int(tokens[i])
        out.append(s.decode_step(t))
    return np.stack(out)


@pytest.mark.parametrize("geom,depth", [("tiny", 2), ("tiny", 3), ("shipped", 6), ("shipped", 8)])
@pytest.mark.parametrize("int8", [False, True])
def test_rung_matches_oracle(cuda, tiny_raw, full_raw, geom, depth, int8):
    raw = tiny_raw if geom == "tiny" else full_raw
    g, o = nb.V3Engine.from_bytes(raw, depth), orc.Model(raw, depth)
    try:
        assert g.geometry == o.geometry and g.num_layers() == depth
        for n in (1, 100, 1025):
            assert g.kv_bytes(n, int8) == o.kv_bytes(n, int8)
        vocab = 512 if geom == "tiny" else 8192
        ids = np.random.default_rng(depth).integers(1, vocab, 40).astype(np.uint32)
        want = _run(o, ids, 16, int8)
        toks = [int(np.argmax(x)) for x in want[:-1]]
        got = _run(g, ids, 16, int8, toks)
        worst = max(rel_err(a, b) for a, b in zip(got, want))
        assert worst < tol(int8, geom == "tiny"), worst
        assert [int(np.argmax(x)) for x in got] == [int(np.argmax(x)) for x in want]
    finally:
        g.close()


@pytest.mark.parametrize("depth", [6, 12])
def test_rung_is_bit_identical_to_a_rung_container(cuda, full_raw, depth):
    rung = write_rung(full_raw, orc.ladder_layers(header_layers(full_raw), depth))
    a, b = nb.V3Engine.from_bytes(full_raw, depth), nb.V3Engine.from_bytes(rung)
    try:
        ids = np.random.default_rng(5).integers(1, 8192, 300).astype(np.uint32)
        for int8 in (False, True):
            assert np.array_equal(_run(a, ids, 8, int8), _run(b, ids, 8, int8))
    finally:
        a.close()
        b.close()


def test_full_depth_and_bad_depths(cuda, full_raw):
    g = nb.V3Engine.from_bytes(full_raw, 20)
    assert g.num_layers() == 20
    g.close()
    for bad in (0, 1, 21):
        with pytest.raises(nb.NeedleError, match="outside the ladder"):
            nb.V3Engine.from_bytes(full_raw, bad)
