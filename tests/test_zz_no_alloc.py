"""The allocation-free attention entry point, nd_attend_step_noalloc.

Callers such as a serving runtime that reserved the GPU's memory for its own
pool, or a latency-critical path that may not call an allocator, cannot let the
library allocate scratch. This entry point keeps the attention's split
partials in a fixed device array inside the library. These tests call it
through the C ABI twice in a row, with different shapes and precisions, and
compare each result with the allocating entry point nd_attend_step on the same
inputs, at the tolerance the attention parity tests use. The file is named so
pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest
from conftest import nb

pytestmark = pytest.mark.gpu

TOL = 1e-4  # as tests/test_gpu_kernels.py compares decode attention


def _fn():
    f = nb.lib().nd_attend_step_noalloc
    f.restype = C.c_int
    f.argtypes = [C.c_void_p] * 5 + [C.c_int, C.c_int, C.c_void_p, C.c_void_p] + [C.c_int] * 5 + [C.c_void_p] * 2
    return f


def _case(torch, B, S, H, KVH, QK, VH, int8, ranges, seed):
    rng = np.random.default_rng(seed)
    q = rng.normal(size=(B, H, QK)).astype(np.float32)
    if int8:
        k = rng.integers(-128, 128, size=(B, S, KVH, QK), dtype=np.int8)
        v = rng.integers(-128, 128, size=(B, S, KVH, VH), dtype=np.int8)
        ks = rng.uniform(0.001, 0.05, size=(B, S, KVH)).astype(np.float32)
        vs = rng.uniform(0.001, 0.05, size=(B, S, KVH)).astype(np.float32)
    else:
        k = rng.normal(size=(B, S, KVH, QK)).astype(np.float32)
        v = rng.normal(size=(B, S, KVH, VH)).astype(np.float32)
        ks = vs = None
    lo = np.array([r[0] for r in ranges], np.int32)
    hi = np.array([r[1] for r in ranges], np.int32)
    dev = {name: (torch.from_numpy(np.ascontiguousarray(a)).cuda() if a is not None else None)
           for name, a in dict(q=q, k=k, v=v, ks=ks, vs=vs, lo=lo, hi=hi).items()}
    return dev


def _run(torch, fn, d, B, S, H, KVH, QK, VH, int8):
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    out_a = torch.full((B, H * VH), float("nan"), device="cuda")
    out_b = torch.full((B, H * VH), float("nan"), device="cuda")
    args = (ptr(d["q"]), ptr(d["k"]), ptr(d["v"]), ptr(d["ks"]), ptr(d["vs"]), int(int8), S, ptr(d["lo"]),
            ptr(d["hi"]), B, H, KVH, QK, VH)
    nb.attend_step(*args, out_a.data_ptr())
    rc = fn(*args, out_b.data_ptr(), None)
    assert rc == 0, nb.lib().nd_last_error()
    torch.cuda.synchronize()
    return out_a.cpu().numpy(), out_b.cpu().numpy()


def test_noalloc_matches_the_allocating_entry_on_two_calls_in_a_row(cuda):
    torch, fn = cuda, _fn()
    # Call 1: BASELINE config 2 shape, int8 rings, full ranges.
    d1 = _case(torch, 64, 512, 12, 2, 48, 64, True, [(0, 511)] * 64, 0)
    a1, b1 = _run(torch, fn, d1, 64, 512, 12, 2, 48, 64, True)
    # Call 2: a different shape and precision reusing the same scratch: f32,
    # ranges that wrap a 17-slot ring and one single-position range.
    ranges = [(0, 0), (0, 9), (3, 16), (20, 36), (5, 5)]
    d2 = _case(torch, 5, 17, 4, 2, 48, 64, False, ranges, 1)
    a2, b2 = _run(torch, fn, d2, 5, 17, 4, 2, 48, 64, False)
    for a, b in ((a1, b1), (a2, b2)):
        assert np.isfinite(b).all()
        scale = max(1.0, float(np.abs(a).max()))
        assert float(np.abs(a - b).max()) <= TOL * scale


def test_noalloc_rejects_requests_beyond_its_fixed_scratch(cuda):
    torch, fn = cuda, _fn()
    B, H, KVH, QK, VH, S = 8192, 12, 2, 48, 64, 16  # 8192 * 12 * 66 floats > 2^20
    q = torch.zeros(B, H, QK, device="cuda")
    k = torch.zeros(B, S, KVH, QK, device="cuda")
    v = torch.zeros(B, S, KVH, VH, device="cuda")
    lo = torch.zeros(B, dtype=torch.int32, device="cuda")
    hi = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.zeros(B, H * VH, device="cuda")
    rc = fn(q.data_ptr(), k.data_ptr(), v.data_ptr(), None, None, 0, S, lo.data_ptr(), hi.data_ptr(), B, H, KVH,
            QK, VH, out.data_ptr(), None)
    assert rc != 0
    assert b"4 MiB" in nb.lib().nd_last_error()
