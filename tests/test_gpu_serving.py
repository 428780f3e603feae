"""Parity in the regime the benchmark times: thousands of
sessions on the shipped geometry, prompts around the 1024-position window, and
batched decode steps replayed from CUDA graphs and through the host API.

At 4096 int8 sessions the step takes the large-batch kernel shapes (warp-per-row
Q/K/V post-processing, 14-row mHC tiles, 7-row block-tail CTAs, the attention
split count of that batch). Prompt lengths 1016..1060 put some sessions past
the local layers' 1024-slot window during prefill and wrap the others' rings
during decode; half the sessions start with rings no larger than their prompt,
so the global layers' rings grow past 1024 at the first decode step. A sample
of sessions is replayed on the CPU oracle: logits at every step within the bars
of test_gpu_model (1e-3 of the logit RMS for f32 KV, 1e-2 for int8 KV), greedy
tokens exact, and the int8 rings equal the oracle's up to single-step code
flips (crates/needle-core/src/v3/cache.rs:68-122, 346-377).

test_engine_quantiser_is_bit_exact pins the forward's own int8 quantiser: the
same prompts in an f32 and an int8 batch give layer 0 identical pre-quantisation
keys and values (nothing upstream of layer 0's attention depends on the KV
precision), so the int8 ring must equal quant_into (cache.rs:100-106) of the f32
ring, code for code and scale bit for scale bit.
"""
import os
import threading

import numpy as np
import pytest
from conftest import nb, orc
from test_gpu_model import REL, REL_INT8, rel_err

pytestmark = pytest.mark.gpu

STEPS = 6  # 4 steps through Batch.step (graph replay), 2 through decode_batch


def prompt(i, n):
    return np.random.default_rng(1000 + i).integers(1, 8192, n).astype(np.uint32)


def plen(i):
    return 1016 + (i * 7) % 45


def hint(i):
    """Ring hint of session i: half the sessions hold rings sized for the whole
    run, half start at their prompt length and grow at the first decode step."""
    return plen(i) + 136 if i % 2 == 0 else plen(i)


def oracle_thread(model, samples, int8):
    """Prefill and greedy-decode the sampled sessions on the oracle in a
    background thread (the ctypes calls release the GIL, so this overlaps the
    GPU work). Returns (thread, results dict)."""
    res = {}

    def run():
        orc.set_threads(os.cpu_count() or 1)
        for i in samples:
            p = prompt(i, plen(i))
            s = model.session(hint(i), int8)
            lg = [s.prefill(p)]
            toks = []
            for _ in range(STEPS):
                t = int(np.argmax(lg[-1]))
                toks.append(t)
                lg.append(s.decode_step(t))
            res[i] = (np.stack(lg), np.array(toks, np.uint32), s)

    th = threading.Thread(target=run)
    th.start()
    return th, res


def run_serving(eng, cuda, n, int8, samples, model):
    torch = cuda
    geo = eng.geometry
    th, ref = oracle_thread(model, samples, int8)
    sessions = [eng.session(hint(i), int8) for i in range(n)]
    got_logits = {i: [] for i in samples}
    picks = np.zeros(n, np.uint32)
    for g0 in range(0, n, 64):
        ss = sessions[g0:g0 + 64]
        lg, pk = eng.prefill_batch(ss, [prompt(g0 + j, plen(g0 + j)) for j in range(len(ss))])
        picks[g0:g0 + len(ss)] = pk
        for i in samples:
            if g0 <= i < g0 + len(ss):
                got_logits[i].append(lg[i - g0].copy())
    got_picks = {i: [int(picks[i])] for i in samples}
    stream = torch.cuda.Stream()
    batch = eng.batch(sessions)
    batch.set_tokens(picks)
    d_logits = torch.zeros(n, eng.logit_rows, device="cuda")
    idx = torch.tensor(samples, device="cuda")
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(4):
            batch.step(d_logits.data_ptr(), stream=stream.cuda_stream, use_graph=True)
            batch.feed_next(stream=stream.cuda_stream)
            stream.synchronize()
            rows = d_logits.index_select(0, idx).cpu().numpy()
            nxt = batch.get_next()
            for k, i in enumerate(samples):
                got_logits[i].append(rows[k].copy())
                got_picks[i].append(int(nxt[i]))
    toks = batch.get_next()
    for _ in range(2):
        lg, toks = eng.decode_batch(sessions, toks)
        for i in samples:
            got_logits[i].append(lg[i].copy())
            got_picks[i].append(int(toks[i]))
    batch.close()
    assert all(s.pos == plen(i) + STEPS for i, s in enumerate(sessions))
    th.join()
    bar = REL_INT8 if int8 else REL
    worst, big = 0.0, 0
    flips = np.zeros(geo["layers"], np.int64)
    codes = np.zeros(geo["layers"], np.int64)
    sdev = np.zeros(geo["layers"])
    for i in samples:
        want_lg, want_tok, o = ref[i]
        g = np.stack(got_logits[i])
        assert g.shape == want_lg.shape
        for step in range(STEPS + 1):
            e = rel_err(g[step], want_lg[step])
            worst = max(worst, e)
            assert e < bar, (i, step, e)
        # picks after prefill and after steps 1..STEPS-1 are the tokens fed next
        assert np.array_equal(np.array(got_picks[i][:STEPS], np.uint32), want_tok), i
        assert got_picks[i][STEPS] == int(np.argmax(want_lg[STEPS]))
        s = sessions[i]
        for li in range(geo["layers"]):
            assert s.slots(li) == o.slots(li)
            if not int8:
                continue
            kq, ks, vq, vs = s.kv(li)
            okq, oks, ovq, ovs = o.kv(li, True, geo["kv_heads"] * geo["qk_head_dim"],
                                      geo["kv_heads"] * geo["v_head_dim"], geo["kv_heads"])
            for a, b in ((kq, okq), (vq, ovq)):
                d = np.abs(a.astype(np.int32) - b.astype(np.int32))
                big += int((d > 1).sum())
                flips[li] += int((d == 1).sum())
                codes[li] += d.size
            for a, b in ((ks, oks), (vs, ovs)):
                sdev[li] = max(sdev[li], float(np.max(np.abs(a / b - 1.0))))
    print(f"\nserving parity n={n} int8={int8}: worst logit rel err {worst:.3e}")
    if int8:
        frac = flips / np.maximum(codes, 1)
        print("int8 code flips per layer: " + " ".join(f"{x:.2e}" for x in frac))
        print("max relative scale deviation per layer: " + " ".join(f"{x:.1e}" for x in sdev))
        print(f"all layers: {flips.sum()}/{codes.sum()} = {flips.sum() / codes.sum():.2e}; larger than one step: {big}")
        # Every difference is exactly one quantisation step. At layer 0 the
        # inputs of the quantiser differ from the oracle's by f32 rounding only
        # (summation order), so flips are rare there (measured 7.6e-6 of the
        # codes at this scale); deeper layers add the drift of the earlier
        # layers' flips (measured up to 1.3e-2 of the codes).
        assert big == 0
        assert frac[0] < 1e-4
        assert frac.max() < 3e-2
        assert sdev.max() < 1e-2
    for s in sessions:
        s.close()
    return worst


def test_serving_scale_int8(full_gpu, full_oracle, cuda):
    """4096 int8 sessions: the benchmark's batch."""
    run_serving(full_gpu, cuda, 4096, True, [0, 5, 7, 1023, 2048, 2101, 3333, 4095], full_oracle)


def test_serving_scale_f32(full_gpu, full_oracle, cuda):
    """2048 f32 sessions (the warp-per-row and large-tile shapes start here)."""
    run_serving(full_gpu, cuda, 2048, False, [0, 9, 1500, 2047], full_oracle)


def test_engine_quantiser_is_bit_exact(full_gpu, cuda):
    """Layer 0's int8 ring equals quant_into of the f32 ring of the same
    prompts, after a batched prefill (two forwards of up to 16384 rows) and two
    batched decode steps of 2100 sessions (warp-per-row Q/K/V post-processing),
    and for one single session (one CTA per row)."""
    geo = full_gpu.geometry
    kvh, qk, vh = geo["kv_heads"], geo["qk_head_dim"], geo["v_head_dim"]

    def check(n, plens):
        prompts = [prompt(50 + i, plens[i]) for i in range(n)]
        f = [full_gpu.session(plens[i] + 4, False) for i in range(n)]
        q = [full_gpu.session(plens[i] + 4, True) for i in range(n)]
        _, pf = full_gpu.prefill_batch(f, prompts, logits=False)
        full_gpu.prefill_batch(q, prompts, logits=False)
        toks = pf
        for _ in range(2):
            _, nf = full_gpu.decode_batch(f, toks, logits=False)
            full_gpu.decode_batch(q, toks, logits=False)  # the same tokens: identical layer-0 inputs
            toks = nf
        checked = 0
        for i in range(0, n, max(1, n // 150)):
            k, v = f[i].kv(0)
            kq, ks, vq, vs = q[i].kv(0)
            live = min(plens[i] + 2, f[i].slots(0))
            k = k.reshape(-1, kvh, qk)[:live]
            v = v.reshape(-1, kvh, vh)[:live]
            kq, vq = kq.reshape(-1, kvh, qk)[:live], vq.reshape(-1, kvh, vh)[:live]
            ks, vs = ks.reshape(-1, kvh)[:live], vs.reshape(-1, kvh)[:live]
            for t in range(live):
                for h in range(kvh):
                    c, sc = orc.quant_into(k[t, h])
                    assert np.array_equal(kq[t, h], c) and ks[t, h].view(np.uint32) == sc.view(np.uint32), (i, t, h)
                    c, sc = orc.quant_into(v[t, h])
                    assert np.array_equal(vq[t, h], c) and vs[t, h].view(np.uint32) == sc.view(np.uint32), (i, t, h)
                    checked += 1
        for s in f + q:
            s.close()
        return checked

    assert check(1, [300]) == 302 * kvh
    assert check(2100, [8] * 2100) >= 150 * 10 * kvh
