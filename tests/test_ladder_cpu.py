"""Ladder rungs on the CPU: the oracle's ladder against the reference's own
fixture (tests/golden/ladder_rungs.json, gated upstream by
crates/needle-infer/tests/v3_ladder_slice.rs:39-68), the load-time slice
against a rung written as a container of its own, and the C ABI's rejection of
depths outside 2..num_layers (crates/needle-c/tests/v3_ffi_smoke.rs:199-240)
before any GPU work."""
import json
import os

import numpy as np
import pytest
from conftest import GOLDEN, nb, orc
from rung_container import header_layers, write_rung

FIX = json.load(open(os.path.join(GOLDEN, "ladder_rungs.json")))


def test_ladder_order_matches_the_reference_fixture():
    assert orc.ladder_order(FIX["parent_layers"]) == FIX["ladder_order"]
    for r in FIX["rungs"]:
        assert orc.ladder_layers(FIX["parent_layers"], r["depth"]) == r["selected"]
    assert orc.ladder_order(1) == [0] and orc.ladder_order(0) == []
    for bad in (0, 1, FIX["parent_layers"] + 1):
        assert orc.ladder_layers(FIX["parent_layers"], bad) is None


def test_sliced_roles_match_every_rung_of_the_fixture(full_oracle, full_raw):
    assert full_oracle.layer_roles() == (FIX["parent_global"], FIX["parent_engram_sites"])
    for r in FIX["rungs"]:
        m = orc.Model(full_raw, r["depth"])
        assert m.geometry["layers"] == r["depth"]
        assert m.layer_roles() == (r["global_layers"], r["engram_sites"]), r["depth"]


@pytest.mark.parametrize("depth,globals_,sites", [
    (6, [1, 3, 4, 5], [5]), (8, [1, 3, 5, 7], [4, 7]),
    (12, [2, 5, 8, 11], [4, 6, 11]), (16, [4, 9, 12, 15], [3, 7, 10, 15])])
def test_known_rungs(full_raw, depth, globals_, sites):
    """v3_ladder_slice.rs:44-49."""
    m = orc.Model(full_raw, depth)
    assert m.layer_roles() == (globals_, sites)
    assert m.kv_bytes(512, True) < orc.Model(full_raw).kv_bytes(512, True)


def test_full_depth_loads_unchanged(full_raw, full_oracle):
    m = orc.Model(full_raw, 20)
    assert m.layer_roles() == full_oracle.layer_roles()
    ids = np.arange(1, 9, dtype=np.uint32)
    assert np.array_equal(m.session(8, False).prefill(ids), full_oracle.session(8, False).prefill(ids))


def _run(model, ids, steps, int8):
    s = model.session(len(ids) + steps, int8)
    out = [s.prefill(ids)]
    for _ in range(steps):
        out.append(s.decode_step(int(np.argmax(out[-1]))))
    return np.stack(out)


@pytest.mark.parametrize("geom,depth", [("tiny", 2), ("tiny", 3), ("shipped", 6), ("shipped", 8)])
def test_slice_equals_a_rung_container(tiny_raw, full_raw, geom, depth):
    """The load-time slice and a rung written as its own container are the same
    model (v3.rs:644-655): identical logits from the oracle, f32 and int8 KV.
    The tiny rungs move blocks to other mHC lanes and drop an Engram site."""
    raw = tiny_raw if geom == "tiny" else full_raw
    kept = orc.ladder_layers(header_layers(raw), depth)
    rung = write_rung(raw, kept)
    built, sliced = orc.Model(rung), orc.Model(raw, depth)
    assert built.geometry == sliced.geometry and built.layer_roles() == sliced.layer_roles()
    ids = np.random.default_rng(depth).integers(1, 256, 12).astype(np.uint32)
    for int8 in (False, True):
        assert np.array_equal(_run(built, ids, 4, int8), _run(sliced, ids, 4, int8))


def test_tiny_rung_differs_from_the_full_stack(tiny_raw, tiny_oracle):
    ids = np.arange(1, 11, dtype=np.uint32)
    a = _run(orc.Model(tiny_raw, 3), ids, 0, False)
    b = _run(tiny_oracle, ids, 0, False)
    assert not np.allclose(a, b)


def test_c_abi_rejects_depths_outside_the_ladder(tiny_raw):
    lib = nb.lib()
    for bad in (0, 1, 5, 99):
        assert lib.needle_v3_load_bytes_with_depth(tiny_raw, len(tiny_raw), bad) is None
        assert b"outside the ladder" in lib.needle_last_error(), bad
    assert lib.needle_v3_load_bytes_with_depth(None, 0, 3) is None
    assert lib.needle_last_error() == b"data was null"
    assert lib.needle_v3_load_with_depth(None, 8) is None
    assert b"null" in lib.needle_last_error()
    assert lib.needle_v3_load_with_depth(b"/nonexistent/needle3.cact", 8) is None
    err = lib.needle_last_error()
    assert b"at 8 layers" in err and b"cannot read" in err
