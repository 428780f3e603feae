"""Grammar-constrained decoding on the CPU (needle_tokenizer_tool_mask): the
reference's own unit tests of constrained.rs (:774-916) restated as known
answers on masks, with one token per byte so a mask entry is a character."""
import struct

import pytest
from conftest import nb

NORMAL = 0


def blob(surfaces):
    out = struct.pack("<5I", len(surfaces), 0, 0, 0, 0) + bytes([0, 0]) + b"\0\0"
    for s in surfaces:
        b = s.encode()
        out += struct.pack("<fBH", 0.0, NORMAL, len(b)) + b
    return out


@pytest.fixture(scope="module")
def bytes_tok():
    return nb.Tokenizer(blob([chr(i) for i in range(128)]))


def allowed(mask):
    return {chr(i) for i in range(len(mask)) if mask[i] == 0.0}


TWO_KEYS = ('[{"name":"t","description":"x","parameters":'
            '{"alpha":{"type":"string"},"beta":{"type":"string"}}}]')


def test_unique_arg_keys_exclude_a_written_key(bytes_tok):
    m = bytes_tok.tool_mask(TWO_KEYS, b'[{"name":"t","arguments":{"', 128)
    assert allowed(m) == {"a", "b"}
    m = bytes_tok.tool_mask(TWO_KEYS, b'[{"name":"t","arguments":{"alpha":"x","', 128)
    assert m[ord("a")] < -1.0 and m[ord("b")] == 0.0
    # without the flag a written key stays available
    m = bytes_tok.tool_mask(TWO_KEYS, b'[{"name":"t","arguments":{"alpha":"x","', 128, unique_keys=False)
    assert m[ord("a")] == 0.0


def test_unique_arg_keys_reset_between_calls(bytes_tok):
    tools = '[{"name":"t","description":"x","parameters":{"alpha":{"type":"string"}}}]'
    m = bytes_tok.tool_mask(tools, b'[{"name":"t","arguments":{"alpha":"x"},{"name":"t","arguments":{"', 128)
    assert m[ord("a")] == 0.0


def test_every_key_written_lifts_the_filter(bytes_tok):
    tools = '[{"name":"t","parameters":{"alpha":{"type":"string"}}}]'
    m = bytes_tok.tool_mask(tools, b'[{"name":"t","arguments":{"alpha":"x","', 128)
    assert m[ord("a")] == 0.0  # the full key trie again rather than nothing


def test_name_mask_follows_the_declared_names():
    t = nb.Tokenizer(blob(["get", "▁get", "set"]))
    tools = '[{"name":"get_weather","parameters":{"location":{},"unit":{}}}]'
    m = t.tool_mask(tools, b'[{"name":"', 3)
    assert m[0] == 0.0 and m[1] < 0 and m[2] < 0  # " get" and "set" leave the trie


def test_quote_closes_only_a_complete_name(bytes_tok):
    tools = '[{"name":"get_weather"},{"name":"get_time"}]'
    assert allowed(bytes_tok.tool_mask(tools, b'[{"name":"get_', 128)) == {"w", "t"}
    assert allowed(bytes_tok.tool_mask(tools, b'[{"name":"get_weather', 128)) == {'"'}
    # a name off the trie: no constraint
    assert len(allowed(bytes_tok.tool_mask(tools, b'[{"name":"x', 128))) == 128


@pytest.mark.parametrize("tools", [
    '[{"name":"get_weather","description":"Get weather","parameters":{"location":{"type":"string"},'
    '"unit":{"type":"string"}}}]',
    '[{"name":"get_weather","parameters":{"type":"object","properties":{"location":{"type":"string"},'
    '"unit":{"type":"string"}},"required":["location"]}}]',
])
def test_argument_keys_flat_and_json_schema(bytes_tok, tools):
    m = bytes_tok.tool_mask(tools, b'[{"name":"get_weather","arguments":{"', 128)
    assert allowed(m) == {"l", "u"}  # never "type" or "required"
    m = bytes_tok.tool_mask(tools, b'[{"name":"get_weather","arguments":{"location":"Paris","', 128)
    assert allowed(m) == {"u"}


def test_value_strings_are_not_constrained(bytes_tok):
    tools = '[{"name":"get_weather","parameters":{"location":{}}}]'
    m = bytes_tok.tool_mask(tools, b'[{"name":"get_weather","arguments":{"location":"Pa', 128)
    assert len(allowed(m)) == 128
    m = bytes_tok.tool_mask(tools, b'[{"name":"get_weather","arguments":{"location":"P,\\"x","', 128)
    assert allowed(m) == {"l"}  # an escaped quote does not end the value


@pytest.mark.parametrize("name,snake", [("getWeather", "get_weather"), ("GetWeather", "get_weather"),
                                        ("get-weather", "get_weather"), ("get.weather", "get_weather"),
                                        ("HTMLParser", "html_parser"), ("already_snake", "already_snake")])
def test_tool_names_are_matched_in_snake_case(bytes_tok, name, snake):
    """tokenizer.rs:426-431: the grammar expects the snake_case form."""
    tools = '[{"name":"%s"}]' % name
    for k in range(len(snake)):
        m = bytes_tok.tool_mask(tools, b'[{"name":"' + snake[:k].encode(), 128)
        assert allowed(m) == {snake[k]}, (snake, k)
    assert allowed(bytes_tok.tool_mask(tools, b'[{"name":"' + snake.encode(), 128)) == {'"'}


def test_no_tools_no_mask(bytes_tok):
    assert len(allowed(bytes_tok.tool_mask("[]", b'[{"name":"', 128))) == 128
    assert len(allowed(bytes_tok.tool_mask("not json", b'[{"name":"', 128))) == 128
