"""Pin the CPU oracle (and the container packer) against the reference's own
fixtures and its own numpy model. These are the anchors every GPU parity test
inherits: the GPU path is compared with the oracle, and the oracle is compared
here with what the reference itself produces."""
import json
import os

import numpy as np
import pytest
from conftest import GOLDEN, cact_pack, orc, sha256


def test_fake_quant_matches_upstream_vectors():
    # crates/needle-core/tests/v3_kv_quant_parity.rs:18-65: tolerance max(|b|,1)*1e-5.
    with open(os.path.join(GOLDEN, "kv_quant_vectors.json")) as f:
        v = json.load(f)
    assert v["bits"] == 8
    for case in v["cases"]:
        dim = case["dim"]
        x = np.array(case["in"], np.float32)
        want = np.array(case["out"], np.float32)
        got = np.concatenate([orc.fake_quant(c, 8) for c in x.reshape(-1, dim)])
        tol = np.maximum(np.abs(want), 1.0) * 1e-5
        assert np.all(np.abs(got - want) <= tol), case["name"]


@pytest.mark.parametrize("name", ["tiny", "full"])
def test_oracle_matches_reference_numpy_model(name, tiny_raw, full_raw):
    g = np.load(os.path.join(GOLDEN, f"numpy_ref_{name}.npz"))
    raw = tiny_raw if name == "tiny" else full_raw
    assert str(g["container_sha256"]) == sha256(raw), "packer output changed; regenerate golden"
    m = orc.Model(raw)
    logits = m.forward_sequence(g["tokens"])
    want = g["logits"]
    got = logits[g["rows"]]
    rms = np.sqrt(np.mean(want.astype(np.float64) ** 2))
    # The reference's parity gate is rel < 5e-3 of RMS (v3_forward_parity.rs:61-131);
    # the restatement agrees to ~3e-6.
    assert np.max(np.abs(got - want)) / rms < 1e-4
    assert np.array_equal(logits.argmax(-1), g["argmax"])


def test_packer_reproduces_shipped_directory():
    """The packer's canon, shapes, widths and byte sizes equal the shipped
    needle3.cact directory for every tensor before the probe heads."""
    with open(os.path.join(GOLDEN, "cact_v3_directory.json")) as f:
        ref = json.load(f)
    geom = cact_pack.shipped()
    # Rebuild only the directory cheaply: header words from the geometry, records from a
    # tiny-valued container would change shapes, so check the shipped-geometry writer by
    # parsing a real build (cached by conftest).
    from conftest import container
    raw = container("shipped", 0)
    words, cb, recs = cact_pack.read_directory(raw)
    gj = ref["geometry"]
    assert words[2] == ref["codebook_len"] == 28
    for k in ("vocab_size", "out_vocab", "d_model", "num_heads", "num_kv_heads", "num_layers", "qk_head_dim",
              "v_head_dim", "max_seq_len", "hada_n", "mhc_lanes", "sliding_window", "qkv_conv_taps",
              "engram_slots", "engram_sub_dim", "num_engram_tables", "engram_conv_taps",
              "engram_conv_dilation", "engram_seed_heads", "kv_window", "kv_bits"):
        idx = {"kv_window": 3, "kv_bits": 4, "vocab_size": 5, "out_vocab": 6, "d_model": 7, "num_heads": 8,
               "num_kv_heads": 9, "num_layers": 10, "qk_head_dim": 11, "v_head_dim": 12, "max_seq_len": 13,
               "hada_n": 14, "mhc_lanes": 15, "sliding_window": 16, "qkv_conv_taps": 19, "engram_slots": 20,
               "engram_sub_dim": 21, "num_engram_tables": 22, "engram_conv_taps": 23,
               "engram_conv_dilation": 24, "engram_seed_heads": 25}[k]
        assert words[idx] == gj[k], k
    gmask = words[17] | (words[18] << 32)
    assert [i for i in range(words[10]) if gmask >> i & 1] == gj["global_layers"]
    assert list(words[27:27 + words[26]]) == gj["engram_orders"]
    assert list(words[32:32 + words[31]]) == gj["engram_layers"]
    assert np.float32(words[48]) == np.float32(gj["rope_theta"])
    n = len(recs)
    assert n == 573  # canon up to final_norm; heads (7) and tokenizer (1) follow in the shipped file
    for mine, theirs in zip(recs, ref["records"][:n]):
        for k in ("dtype", "ndim", "shape", "nbytes", "group", "bits"):
            assert mine[k] == theirs[k], (mine["index"], k)
        assert mine["offset"] % 64 == 0
    # The first blob sits where the shipped one does once the directory length is equal.
    assert recs[0]["offset"] == -(-(196 + 112 + 44 * n) // 64) * 64


def test_shipped_row_bytes():
    # cq.rs:1275-1300 row byte arithmetic for shipped shapes.
    assert 576 * 768 * 2 // 8 + 576 * 6 * 2 == 117504
    assert 8192 * 768 * 4 // 8 + 8192 * 6 * 2 == 3244032
    assert 110592 * 128 * 2 // 8 + 110592 * 2 == 3760128
