"""Writes tests/golden/sp_bpe_tokenizer.json: a SentencePiece BPE model trained
here with the `sentencepiece` package (seeded synthetic corpus), exported in
the container's RAW tokenizer blob layout (sp_tokenizer.rs:8-15), together with
the ids and decoded text that real SentencePiece produces for a set of texts.

The reference's own tokenizer gate (crates/needle-infer/tests/
tokenizer_v3_parity.rs) checks its encoder against real `sentencepiece` output
on the shipped model, whose blob travels only inside the weights (absent
here). This fixture applies the same gate to a model trained with the same
settings the shipped vocabulary shows: BPE, byte fallback, the chat markers as
user-defined pieces, no normalisation, whitespace kept, a dummy prefix.

Run from the repo root: python tests/golden/make_tokenizer_golden.py
"""
import base64
import json
import os
import random
import struct
import tempfile

import sentencepiece as spm

HERE = os.path.dirname(os.path.abspath(__file__))
MARKERS = ["<|im_start|>", "<|im_end|>", "<think>", "</think>", "<tools>", "</tools>", "<tool_call>",
           "</tool_call>", "<tool_result>", "</tool_result>"]
WORDS = ("the a of to in on for with from by at is are was be call tool weather city country light room "
         "door music play stop send email message note time date today tomorrow flight book hotel price "
         "open close turn off set timer alarm minute hour name arguments value list search find result "
         "model token layer cache batch prompt answer query user assistant system json string number true "
         "false null paris london tokyo berlin kitchen bedroom garage volume brightness temperature").split()
TEXTS = [
    "What's the weather in Paris?", "Turn off the bedroom lights", "Book a flight from London to JFK tomorrow",
    "Email alice@example.com saying the build is green",
    "<|im_start|>user\n<tools>[]</tools>\nhi<|im_end|>\n<|im_start|>assistant\n",
    '{"name":"get_weather","arguments":{"city":"Paris"}}', "set(x) := {1, 2, 3}", "   leading and trailing   ",
    "naive cafe -- resume", "naïve café — résumé", "日本語のテキスト",
    "emoji \U0001F600 and \U0001F680!", "tabs\tand\nnewlines\r\n", "<tool_call>{\"name\":\"x\"}</tool_call>",
    "<think>plan</think>answer", "a", " ", "  ", "", "x" * 40, "12345 67.890", "</tool_call><tool_call>",
    "<tools><tool_call>", "The quick brown fox jumps over the lazy dog.",
]


def corpus(rng: random.Random) -> list[str]:
    lines = []
    for _ in range(4000):
        n = rng.randint(3, 14)
        words = [rng.choice(WORDS) for _ in range(n)]
        if rng.random() < 0.3:
            words[0] = words[0].capitalize()
        line = " ".join(words)
        if rng.random() < 0.2:
            line = '{"name":"' + rng.choice(WORDS) + '","arguments":{"' + rng.choice(WORDS) + '":"' + \
                   rng.choice(WORDS) + '"}}'
        if rng.random() < 0.1:
            line = "<tool_call>" + line + "</tool_call>"
        lines.append(line + rng.choice([".", "?", "!", ""]))
    return lines


def blob_of(sp: spm.SentencePieceProcessor) -> bytes:
    out = struct.pack("<5I", sp.get_piece_size(), sp.pad_id(), sp.eos_id(), sp.bos_id(), sp.unk_id())
    out += bytes([1, 1]) + b"\0\0"  # add_dummy_prefix, byte_fallback
    for i in range(sp.get_piece_size()):
        ty = 2 if sp.is_control(i) else 1 if sp.is_unknown(i) else 4 if sp.is_byte(i) else \
            3 if sp.id_to_piece(i) in MARKERS else 0
        s = sp.id_to_piece(i).encode("utf-8")
        out += struct.pack("<fBH", sp.get_score(i), ty, len(s)) + s
    return out


def main():
    rng = random.Random(0)
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "corpus.txt"), "w") as f:
            f.write("\n".join(corpus(rng)))
        spm.SentencePieceTrainer.train(
            input=os.path.join(d, "corpus.txt"), model_prefix=os.path.join(d, "m"), vocab_size=600,
            model_type="bpe", byte_fallback=True, user_defined_symbols=MARKERS,
            normalization_rule_name="identity", remove_extra_whitespaces=False, add_dummy_prefix=True,
            pad_id=0, eos_id=1, bos_id=2, unk_id=3, character_coverage=1.0, minloglevel=2, seed_sentencepiece_size=100000,
            num_threads=1)
        sp = spm.SentencePieceProcessor(model_file=os.path.join(d, "m.model"))
    cases = [{"text": t, "ids": sp.encode(t), "decoded": sp.decode(sp.encode(t))} for t in TEXTS]
    fixture = {"generator": "tests/golden/make_tokenizer_golden.py", "sentencepiece": spm.__version__,
               "pieces": sp.get_piece_size(), "blob_b64": base64.b64encode(blob_of(sp)).decode(), "cases": cases}
    with open(os.path.join(HERE, "sp_bpe_tokenizer.json"), "w") as f:
        json.dump(fixture, f, indent=1, ensure_ascii=True)
        f.write("\n")
    print(f"{len(cases)} cases, {sp.get_piece_size()} pieces")


if __name__ == "__main__":
    main()
