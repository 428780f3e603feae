"""The confidence probe head on the GPU engine (needle_v3_confidence_for,
v3_engine.rs:351-368): cells captured by the forward, pooled and projected by
the head kernels, against the oracle's head over the same ids, at full depth
and on a ladder rung."""
import numpy as np
import pytest
from conftest import nb, orc
from test_gpu_text import QUERY, TOOLS, build_prompt

pytestmark = pytest.mark.gpu

BOS = 2
COMPLETIONS = ["", '<tool_call>[{"name":"get_weather","arguments":{"city":"Paris"}}]</tool_call>',
               "No tool applies here."]


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


@pytest.mark.parametrize("depth", [None, 6])
def test_confidence_matches_the_oracle(cuda, head_text_raw, sp_fixture, depth):
    g = nb.V3Engine.from_bytes(head_text_raw, depth)
    o = orc.Model(head_text_raw, depth)
    tok = nb.Tokenizer(sp_fixture["blob"])
    try:
        assert g.has_confidence()
        for c in COMPLETIONS:
            ids = np.array([BOS] + tok.encode(build_prompt(QUERY, TOOLS) + c), np.uint32)
            logit = o.confidence_logit(ids)
            p = g.confidence_for(QUERY, TOOLS, c)
            assert abs(p - sigmoid(logit)) < 5e-4, (c, p, sigmoid(logit), logit)
            assert 0.0 < p < 1.0
    finally:
        g.close()


def test_no_head_is_reported(full_gpu):
    assert not full_gpu.has_confidence()
    with pytest.raises(nb.NeedleError, match="no confidence head"):
        full_gpu.confidence_for(QUERY, TOOLS, "")
