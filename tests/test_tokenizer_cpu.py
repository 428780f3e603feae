"""The container tokenizer on the CPU (needle_tokenizer_*, host code): the
reference's own known answers on its toy vocabulary
(crates/needle-infer/src/sp_tokenizer.rs:449-620), malformed blobs, and the
encoder and decoder against real SentencePiece (the gate of
crates/needle-infer/tests/tokenizer_v3_parity.rs) on a BPE model trained with
the `sentencepiece` package: the committed fixture, and random texts against
the live library when it is importable."""
import random
import struct

import pytest
from conftest import GOLDEN, cact_pack, nb

NORMAL, UNKNOWN, CONTROL, USER, BYTE = 0, 1, 2, 3, 4


def blob(pieces, dummy=True, byte_fallback=True, specials=(0, 1, 2, 3)):
    out = struct.pack("<5I", len(pieces), *specials) + bytes([int(dummy), int(byte_fallback)]) + b"\0\0"
    for surface, score, ty in pieces:
        b = surface.encode() if isinstance(surface, str) else surface
        out += struct.pack("<fBH", score, ty, len(b)) + b
    return out


@pytest.fixture(scope="module")
def toy():
    p = [("<pad>", 0, CONTROL), ("</s>", 0, CONTROL), ("<s>", 0, CONTROL), ("<unk>", 0, UNKNOWN),
         ("<tool_call>", 0, USER), ("<tool>", 0, USER), ("▁", -1, NORMAL), ("a", -2, NORMAL),
         ("b", -3, NORMAL), ("c", -4, NORMAL), ("ab", -0.5, NORMAL), ("abc", -0.25, NORMAL),
         ("▁a", -0.75, NORMAL)]
    p += [(f"<0x{b:02X}>", -50.0, BYTE) for b in range(256)]
    return nb.Tokenizer(blob(p))


def test_toy_known_answers(toy):
    assert toy.encode("<tool_call>") == [6, 4]  # longest marker first
    assert toy.encode("a") == [12]  # dummy prefix merges into "▁a"
    assert toy.encode("b") == [6, 8]
    assert toy.encode("abc") == [6, 11]  # ab, then ab + c
    assert toy.encode("z") == [6, 13 + 0x7A]  # byte fallback
    assert toy.encode("€") == [6, 13 + 0xE2, 13 + 0x82, 13 + 0xAC]
    for s in ["a", "ab", "abc", "a b", "z", "€", "abc abc"]:
        assert toy.decode(toy.encode(s)) == s
    assert toy.decode([2, 6, 11, 1, 3]) == "abc"  # control and unknown pieces vanish
    assert toy.encode("") == [] and toy.decode([]) == ""
    assert toy.decode([99999]) == ""  # ids past the table are skipped


def test_decode_replaces_ill_formed_bytes(toy):
    e2, x82 = 13 + 0xE2, 13 + 0x82
    assert toy.decode([e2, x82]) == "�"  # truncated 3-byte sequence: one replacement
    assert toy.decode([13 + 0xFF, 7]) == "�a"
    assert toy.decode([13 + 0xC3, 13 + 0xA9]) == "é"


@pytest.mark.parametrize("bad,msg", [
    (blob([("a", 0, NORMAL)])[:10], "truncated"),
    (blob([("a", 0, NORMAL)])[:-1], "truncated"),
    (blob([]), "zero pieces"),
    (blob([("a", 0, NORMAL)], specials=(0, 9, 0, 0)), "eos id 9"),
    (blob([("nope", 0, BYTE)], specials=(0, 0, 0, 0)), "byte piece 0"),
    (blob([(b"a\xff", 0, NORMAL)], specials=(0, 0, 0, 0)), "not valid UTF-8"),
])
def test_malformed_blobs_are_rejected(bad, msg):
    with pytest.raises(nb.NeedleError, match=msg):
        nb.Tokenizer(bad)


def test_sentencepiece_fixture(sp_fixture):
    t = nb.Tokenizer(sp_fixture["blob"])
    assert len(sp_fixture["cases"]) >= 20
    for c in sp_fixture["cases"]:
        assert t.encode(c["text"]) == c["ids"], c["text"]
        assert t.decode(c["ids"]) == c["decoded"], c["text"]


def test_random_texts_against_live_sentencepiece():
    spm = pytest.importorskip("sentencepiece")
    import os
    import sys
    import tempfile
    sys.path.insert(0, GOLDEN)
    import make_tokenizer_golden as g
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "c.txt"), "w") as f:
            f.write("\n".join(g.corpus(random.Random(0))))
        spm.SentencePieceTrainer.train(
            input=os.path.join(d, "c.txt"), model_prefix=os.path.join(d, "m"), vocab_size=600, model_type="bpe",
            byte_fallback=True, user_defined_symbols=g.MARKERS, normalization_rule_name="identity",
            remove_extra_whitespaces=False, add_dummy_prefix=True, pad_id=0, eos_id=1, bos_id=2, unk_id=3,
            character_coverage=1.0, minloglevel=2, num_threads=1)
        sp = spm.SentencePieceProcessor(model_file=os.path.join(d, "m.model"))
    t = nb.Tokenizer(g.blob_of(sp))
    alpha = list("abcdefghijklmnopqrstuvwxyz ABCXYZ  .,!?{}[]\":\n\t0123456789") + \
        ["é", "ü", "—", "日", "本", "\U0001F600", "€"] + g.MARKERS
    r = random.Random(1)
    for _ in range(1500):
        s = "".join(r.choice(alpha) if r.random() < 0.7 else " " + r.choice(g.WORDS) for _ in range(r.randint(0, 30)))
        ids = sp.encode(s)
        assert t.encode(s) == ids, s
        assert t.decode(ids) == sp.decode(ids), s


def test_text_calls_check_arguments_before_any_gpu_work(tiny_raw):
    lib = nb.lib()
    assert lib.needle_v3_run(None, b"q", b"[]") is None
    assert lib.needle_last_error() == b"handle was null"
    assert lib.needle_v3_generate(None, b"q", b"[]", 0, 0.0, 0, True, False) is None
    assert lib.needle_tokenizer_new(None, 0) is None
    assert lib.needle_last_error() == b"blob was null"
    # A container whose tokenizer record is malformed fails at load, before
    # the device is touched.
    raw = cact_pack.build_container(cact_pack.tiny(), seed=1, tokenizer=blob([]))
    assert lib.needle_v3_load_bytes(raw, len(raw)) is None
    assert b"bad tokenizer record" in lib.needle_last_error()


def test_tokenizer_encode_reports_bad_text(toy):
    lib = nb.lib()
    assert lib.needle_tokenizer_encode(toy._t, b"a\xffb", None, 0) == (1 << 64) - 1
    assert b"not UTF-8" in lib.needle_last_error()
