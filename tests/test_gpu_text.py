"""Text-level calls on the GPU engine (needle_v3_run / run_json / generate /
run_stream, V3Engine::generate_with, v3_engine.rs:193-401) on a shipped-geometry
container carrying a SentencePiece tokenizer record: the completion equals the
oracle's greedy continuation of [bos] + encode(chat prompt), cut at </s> or
<|im_end|> and decoded. The prompt is restated here from prompt.rs."""
import json

import numpy as np
import pytest
from conftest import nb, orc

pytestmark = pytest.mark.gpu

BOS, EOS = 2, 1
TOOLS = json.dumps([{"name": "get_weather", "description": "Get current weather for a city",
                     "parameters": {"type": "object", "properties": {"city": {"type": "string"}},
                                    "required": ["city"]}}], indent=2)
QUERY = "What's the weather in Paris?"


def compact_json(s: str) -> str:
    out, in_str, esc = [], False, False
    for c in s:
        if in_str:
            out.append(c)
            if esc:
                esc = False
            elif c == "\\":
                esc = True
            elif c == '"':
                in_str = False
        elif c == '"':
            in_str = True
            out.append(c)
        elif c not in " \t\n\r":
            out.append(c)
    return "".join(out)


def build_prompt(query: str, tools: str) -> str:
    return f"<|im_start|>user\n<tools>{compact_json(tools)}</tools>\n{query}<|im_end|>\n<|im_start|>assistant\n"


def between(text: str, a: str, b: str):
    i = text.find(a)
    if i < 0:
        return None
    rest = text[i + len(a):]
    j = rest.find(b)
    return rest if j < 0 else rest[:j]


@pytest.fixture(scope="module")
def text_gpu(cuda, text_raw):
    return nb.V3Engine.from_bytes(text_raw)


@pytest.fixture(scope="module")
def text_oracle(text_raw):
    return orc.Model(text_raw)


def oracle_text(model, tok, query, tools, n, int8):
    im_end = tok.encode("<|im_end|>")[-1]
    ids = np.array([BOS] + tok.encode(build_prompt(query, tools)), np.uint32)
    toks, _ = orc.greedy(model, ids, n, int8)
    out = []
    for t in toks:
        if int(t) in (EOS, im_end):
            break
        out.append(int(t))
    return tok.decode(out), out


@pytest.mark.parametrize("int8", [False, True])
def test_generate_matches_the_oracle(text_gpu, text_oracle, sp_fixture, int8):
    tok = nb.Tokenizer(sp_fixture["blob"])
    want, toks = oracle_text(text_oracle, tok, QUERY, TOOLS, 48, int8)
    got = text_gpu.generate(QUERY, TOOLS, max_new_tokens=48, kv_int8=int8)
    assert got == want, (toks, got, want)


def test_run_stream_json_and_defaults(text_gpu):
    text = text_gpu.run(QUERY, TOOLS)
    assert text == text_gpu.generate(QUERY, TOOLS, max_new_tokens=0)  # 0 means the default budget
    pieces = []
    assert text_gpu.run_stream(QUERY, TOOLS, pieces.append) == text
    assert "".join(pieces) == text and all(pieces)
    call = between(text, "<tool_call>", "</tool_call>")
    assert text_gpu.run_json(QUERY, TOOLS) == ("" if call is None else call.strip())


def test_sampling_is_seeded(text_gpu):
    a = text_gpu.generate(QUERY, TOOLS, max_new_tokens=24, temperature=0.8, seed=7)
    assert a == text_gpu.generate(QUERY, TOOLS, max_new_tokens=24, temperature=0.8, seed=7)


def test_constrained_generate(text_gpu):
    """The grammar only acts inside a <tool_call> span (its masks are checked
    on the CPU against constrained.rs's own cases); outside one, constrained
    greedy decoding (host argmax over the step's logits) picks exactly what
    the engine's device argmax picks."""
    a = text_gpu.generate(QUERY, TOOLS, max_new_tokens=48, constrain=True)
    b = text_gpu.generate(QUERY, TOOLS, max_new_tokens=48)
    assert "<tool_call>" in b or a == b


def test_text_errors(text_gpu, full_gpu):
    with pytest.raises(nb.NeedleError, match="no tokenizer record"):
        full_gpu.run(QUERY, TOOLS)
    assert text_gpu.reasoning("<think> plan it </think>answer") == "plan it"
    assert text_gpu.reasoning("no markers") is None
