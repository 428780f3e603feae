"""Temperature sampling without a GPU: the SplitMix64 generator and `sample`
(crates/needle-infer/src/v3_engine.rs:422-464) of the product's host code
(needle_v3_sample) against the oracle's restatement and against the
generator's definition computed here in exact integer arithmetic."""
import numpy as np
import pytest
from conftest import nb, orc

MASK = (1 << 64) - 1


def splitmix64(seed, n):
    """next_u64 (v3_engine.rs:452-459) in Python integers: exact mod 2^64."""
    s, out = seed, []
    for _ in range(n):
        s = (s + 0x9E3779B97F4A7C15) & MASK
        z = s
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & MASK
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & MASK
        out.append(z ^ (z >> 31))
    return out, s


def test_splitmix64_known_answers():
    # The published SplitMix64 test sequence for seed 1234567.
    want = [6457827717110365317, 3203168211198807973, 9817491932198370423, 4593380528125082431,
            16408922859458223821]
    assert splitmix64(1234567, 5)[0] == want
    r = orc.SplitMix64(1234567)
    assert [r.next_u64() for _ in range(5)] == want
    for seed in (0, 1, 42, 2**63 + 11, MASK):
        vals, _ = splitmix64(seed, 64)
        r = orc.SplitMix64(seed)
        assert [r.next_u64() for _ in range(64)] == vals
        r = orc.SplitMix64(seed)
        assert [r.next_f64() for _ in range(64)] == [(v >> 11) / float(1 << 53) for v in vals]


def test_product_sample_matches_the_oracle():
    """Chained draws on seeded logits: the same ids and the same generator
    state after every draw (one next_f64 per draw), at several temperatures,
    with masked (-1e9) entries as constrained decoding adds them."""
    rng = np.random.default_rng(7)
    for trial in range(40):
        n = int(rng.choice([2, 3, 17, 512, 8192]))
        logits = (rng.standard_normal(n) * rng.choice([0.5, 3.0, 12.0])).astype(np.float32)
        if trial % 3 == 0:
            logits[rng.integers(0, n, max(1, n // 4))] -= np.float32(1e9)
        temp = float(rng.choice([0.2, 0.7, 1.0, 2.5]))
        seed = int(rng.integers(0, 2**63))
        state = seed
        ref = orc.SplitMix64(seed)
        for _ in range(8):
            pick, state = nb.sample(logits, temp, state)
            assert pick == orc.sample(logits, temp, ref)
            assert state == ref.state.value
        assert state == (seed + 8 * 0x9E3779B97F4A7C15) & MASK


def test_sample_edges():
    one = np.array([3.5], np.float32)
    assert nb.sample(one, 1.0, 5)[0] == 0
    flat = np.zeros(10, np.float32)
    # Equal weights: the pick is floor(u * 10) (up to the running subtraction).
    vals, _ = splitmix64(99, 1)
    u = (vals[0] >> 11) / float(1 << 53)
    pick, _ = nb.sample(flat, 0.9, 99)
    assert pick == orc.sample(flat, 0.9, orc.SplitMix64(99))
    assert abs(pick - int(u * 10)) <= 1
    # One finite entry among masked ones always wins.
    masked = np.full(64, -1e9, np.float32)
    masked[37] = 0.0
    assert nb.sample(masked, 1.0, 1)[0] == 37
    with pytest.raises(nb.NeedleError, match="temperature"):
        nb.sample(flat, 0.0, 1)
    lib = nb.lib()
    assert lib.needle_v3_sample(None, 4, 1.0, None) == 0xFFFFFFFF
    assert b"null" in lib.needle_last_error()
