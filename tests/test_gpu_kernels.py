"""GPU parity of the single kernels, through the C ABI (nd_* entry points),
against the CPU oracle on identical seeded inputs.

Tolerances: index unpacking and int8 quantisation are bit-exact; f32 dot
products are compared at max|diff| <= 2e-5 * max(1, max|y|) because the GPU
sums in a different order than the reference's 8-lane loop.
"""
import numpy as np
import pytest
from conftest import cact_pack, nb, orc

pytestmark = pytest.mark.gpu


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def make_weight(torch, out, inp, bits, seed, codebook):
    rng = np.random.default_rng(seed)
    idx, norms = cact_pack.random_cq(rng, out, inp, bits)
    blob = cact_pack.cq_blob(idx, norms, bits)
    d = dev(torch, np.frombuffer(blob, np.uint8).copy())
    in_pad = idx.shape[1]
    packed_ptr = d.data_ptr()
    norms_ptr = packed_ptr + out * in_pad * bits // 8
    w = orc.CqWeight(blob, out, inp, bits, codebook)
    return d, packed_ptr, norms_ptr, w, idx, norms


def close(a, b, tol=2e-5):
    scale = max(1.0, float(np.abs(b).max()))
    return float(np.abs(a - b).max()) <= tol * scale


@pytest.mark.parametrize("bits", [2, 4])
def test_cq_prepare_is_bit_exact(cuda, bits):
    torch = cuda
    rng = np.random.default_rng(0)
    for inp in (768, 3072, 200):
        x = rng.normal(size=(3, inp)).astype(np.float32)
        in_pad = -(-inp // 128) * 128
        xg = dev(torch, x)
        xh = torch.zeros(3, in_pad, device="cuda")
        nb.cq_prepare(xg.data_ptr(), 3, inp, xh.data_ptr(), in_pad)
        cb = cact_pack.lloyd_codebook()
        _, _, _, w, _, _ = make_weight(torch, 4, inp, bits, 0, cb)
        want = np.stack([w.prepare(r) for r in x])
        assert np.array_equal(xh.cpu().numpy(), want)  # same butterflies, same order


@pytest.mark.parametrize("bits", [2, 4])
def test_cq_index_unpacking_is_bit_exact(cuda, bits):
    """With one-hot rotated inputs the kernel returns norm * level[idx[r, k]]
    for every row: the recovered indices must equal the packed ones."""
    torch = cuda
    cb = cact_pack.lloyd_codebook()
    out, inp = 300, 768
    d, pp, npp, w, idx, norms = make_weight(torch, out, inp, bits, 1, cb)
    levels = cact_pack.codebook_levels(cb, bits)
    ks = np.arange(0, inp, 7)[:8]
    for path in (1, 2):
        xh = np.zeros((8, inp), np.float32)
        xh[np.arange(8), ks] = 1.0
        y = torch.zeros(8, out, device="cuda")
        xd = dev(torch, xh)
        nb.cq_project(pp, npp, out, inp, bits, levels, xd.data_ptr(), inp, 8, y.data_ptr(), out,
                      path=path)
        torch.cuda.synchronize()
        yn = y.cpu().numpy()
        for m, k in enumerate(ks):
            want = (norms[:, k // 128].astype(np.float32) * levels[idx[:, k]]).astype(np.float32)
            assert np.array_equal(yn[m], want), (path, k)


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("shape", [(3072, 768), (1568, 768), (768, 768), (8192, 768), (24, 3072), (1000, 300),
                                   (20000, 768), (40003, 768)])
@pytest.mark.parametrize("levels_kind,path", [("f16", 1), ("f16", 5), ("f32", 1)])
def test_cq_gemv_matches_oracle(cuda, bits, shape, levels_kind, path):
    """Path 1 chooses: f16 codebook entries (the packer's
    codebooks) take the tensor-core GEMV past 9472 rows ((20000, 768) and
    (40003, 768): more tiles than the grid's warps, warps loop over tiles) and
    the SIMT kernels below; plain f32 entries are not f16 values and always
    take the SIMT kernels (the partial-sum table kernel for one row from 16384
    rows, the latency-ordered GEMV otherwise). Path 5 forces the tensor-core
    GEMV, so small matrices run its split-group form. One and two 16-column MMA
    tiles (M <= 4, M <= 8). Row 1 of every batch is zero."""
    torch = cuda
    out, inp = shape
    if levels_kind == "f16":
        cb = cact_pack.random_codebook(np.random.default_rng(9))  # BASELINE config 0 codebook
    else:
        cb = (np.random.default_rng(9).normal(0.0, 0.02, 28) / np.sqrt(128)).astype(np.float32)
    d, pp, npp, w, _, _ = make_weight(torch, out, inp, bits, 2, cb)
    levels = cact_pack.codebook_levels(cb, bits)
    rng = np.random.default_rng(3)
    for M in (1, 2, 3, 4, 5, 8):
        x = rng.normal(size=(M, inp)).astype(np.float32) * rng.choice([1e-3, 1.0, 40.0])
        if M > 1:
            x[1] = 0.0
        xh = np.stack([w.prepare(r) for r in x])
        y = torch.zeros(M, out, device="cuda")
        xd = dev(torch, xh)
        nb.cq_project(pp, npp, out, inp, bits, levels, xd.data_ptr(), xh.shape[1], M, y.data_ptr(),
                      out, path=path)
        torch.cuda.synchronize()
        want = w.matmul_prepared(xh)
        assert close(y.cpu().numpy(), want), (M, float(np.abs(y.cpu().numpy() - want).max()))


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("n_out", [768, 2304, 3072])
def test_cq_gemm_matches_oracle_config1(cuda, bits, n_out):
    """X [512, 768], W [N, 768]."""
    torch = cuda
    cb = cact_pack.random_codebook(np.random.default_rng(9))
    d, pp, npp, w, _, _ = make_weight(torch, n_out, 768, bits, 4, cb)
    levels = cact_pack.codebook_levels(cb, bits)
    x = np.random.default_rng(5).normal(size=(512, 768)).astype(np.float32)
    xg = dev(torch, x)
    xh = torch.zeros(512, 768, device="cuda")
    nb.cq_prepare(xg.data_ptr(), 512, 768, xh.data_ptr(), 768)
    y = torch.zeros(512, n_out, device="cuda")
    nb.cq_project(pp, npp, n_out, 768, bits, levels, xh.data_ptr(), 768, 512, y.data_ptr(), n_out)
    torch.cuda.synchronize()
    want = w.matmul_prepared(np.stack([w.prepare(r) for r in x]))
    assert close(y.cpu().numpy(), want)


@pytest.mark.parametrize("bits", [2, 4])
@pytest.mark.parametrize("shape", [(812, 768), (768, 768), (300, 3072), (8192, 768)])
@pytest.mark.parametrize("levels_kind", ["f16", "f32"])
def test_cq_tensor_core_gemm_matches_oracle(cuda, bits, shape, levels_kind):
    """The tcgen05 path (path 3) against the oracle for ragged row counts
    (partial 128-row tiles) and partial 128-output tiles. f16 codebook entries
    take the exact-level form (two MMAs per K step); plain f32 entries need the
    level remainders too (three MMAs)."""
    torch = cuda
    out, inp = shape
    if levels_kind == "f16":
        cb = cact_pack.random_codebook(np.random.default_rng(9))
    else:
        cb = (np.random.default_rng(9).normal(0.0, 0.02, 28) / np.sqrt(128)).astype(np.float32)
        assert not np.array_equal(cb, cact_pack.f16_round(cb))
    d, pp, npp, w, _, _ = make_weight(torch, out, inp, bits, 7, cb)
    levels = cact_pack.codebook_levels(cb, bits)
    rng = np.random.default_rng(11)
    for M in (9, 128, 200, 1000):
        x = rng.normal(size=(M, inp)).astype(np.float32)
        xh = np.stack([w.prepare(r) for r in x])
        y = torch.zeros(M, out, device="cuda")
        xd = dev(torch, xh)
        nb.cq_project(pp, npp, out, inp, bits, levels, xd.data_ptr(), xh.shape[1], M, y.data_ptr(), out,
                      path=3)
        torch.cuda.synchronize()
        want = w.matmul_prepared(xh)
        got = y.cpu().numpy()
        assert close(got, want), (M, float(np.abs(got - want).max()))


@pytest.mark.parametrize("shape,M", [((300, 768), 7680), ((1000, 768), 4000)])
@pytest.mark.parametrize("levels_kind", ["f16", "f32"])
def test_cq_tensor_core_persistent_tiles(cuda, shape, M, levels_kind):
    """More tiles than SMs, so every persistent CTA computes several tiles and
    the group accumulators alternate across tile boundaries: 128-row weight
    tiles at (300, 768) x 7680 (180 tiles), 192-row tiles at (1000, 768) x 4000
    (192 tiles), with f16 and plain f32 codebook entries."""
    torch = cuda
    out, inp = shape
    if levels_kind == "f16":
        cb = cact_pack.random_codebook(np.random.default_rng(9))
    else:
        cb = (np.random.default_rng(9).normal(0.0, 0.02, 28) / np.sqrt(128)).astype(np.float32)
    d, pp, npp, w, _, _ = make_weight(torch, out, inp, 2, 8, cb)
    levels = cact_pack.codebook_levels(cb, 2)
    x = np.random.default_rng(12).normal(size=(M, inp)).astype(np.float32)
    xh = np.stack([w.prepare(r) for r in x])
    y = torch.zeros(M, out, device="cuda")
    xd = dev(torch, xh)
    nb.cq_project(pp, npp, out, inp, 2, levels, xd.data_ptr(), inp, M, y.data_ptr(), out, path=3)
    torch.cuda.synchronize()
    want = w.matmul_prepared(xh)
    got = y.cpu().numpy()
    assert close(got, want), float(np.abs(got - want).max())


@pytest.mark.parametrize("bits", [2, 4])
def test_cq_tensor_core_unpacking_matches_levels(cuda, bits):
    """One-hot rotated inputs through the tensor-core path return
    norm * level[idx] per row to the precision of the hi/lo split."""
    torch = cuda
    cb = cact_pack.lloyd_codebook()
    out, inp = 300, 768
    d, pp, npp, w, idx, norms = make_weight(torch, out, inp, bits, 1, cb)
    levels = cact_pack.codebook_levels(cb, bits)
    ks = np.arange(0, inp, 7)[:16]
    xh = np.zeros((16, inp), np.float32)
    xh[np.arange(16), ks] = 1.0
    y = torch.zeros(16, out, device="cuda")
    xd = dev(torch, xh)
    nb.cq_project(pp, npp, out, inp, bits, levels, xd.data_ptr(), inp, 16, y.data_ptr(), out, path=3)
    torch.cuda.synchronize()
    yn = y.cpu().numpy()
    for m, k in enumerate(ks):
        want = (norms[:, k // 128].astype(np.float32) * levels[idx[:, k]]).astype(np.float32)
        assert np.allclose(yn[m], want, rtol=1e-6, atol=1e-9), k


def test_cq_row_ranges_and_ragged_sizes(cuda):
    torch = cuda
    cb = cact_pack.lloyd_codebook()
    d, pp, npp, w, _, _ = make_weight(torch, 80, 3072, 4, 6, cb)
    levels = cact_pack.codebook_levels(cb, 4)
    x = np.random.default_rng(1).normal(size=(67, 3072)).astype(np.float32)
    xh = np.stack([w.prepare(r) for r in x])
    for M, row0, nrows, path in ((1, 4, 4, 0), (1, 16, 16, 0), (67, 40, 24, 0), (67, 0, 80, 2), (9, 3, 61, 0),
                                 (67, 40, 24, 3), (9, 3, 61, 3)):
        y = torch.zeros(M, nrows, device="cuda")
        xd = dev(torch, xh[:M])
        nb.cq_project(pp, npp, 80, 3072, 4, levels, xd.data_ptr(), 3072, M, y.data_ptr(), nrows,
                      row0=row0, nrows=nrows, path=path)
        torch.cuda.synchronize()
        assert close(y.cpu().numpy(), w.matmul_prepared(xh[:M], row0, nrows))


def test_cq_rejects_bad_arguments(cuda):
    torch = cuda
    cb = cact_pack.lloyd_codebook()
    d, pp, npp, w, _, _ = make_weight(torch, 8, 128, 2, 0, cb)
    xh = torch.zeros(1, 128, device="cuda")
    y = torch.zeros(1, 8, device="cuda")
    with pytest.raises(nb.NeedleError):
        nb.cq_project(pp, npp, 8, 128, 2, cb[:4], xh.data_ptr(), 128, 1, y.data_ptr(), 8, row0=4, nrows=8)
    with pytest.raises(nb.NeedleError):
        nb.cq_project(pp, npp, 8, 128, 3, cb[4:12], xh.data_ptr(), 128, 1, y.data_ptr(), 8)


# ------------------------------------------------------------------ int8 KV
def test_kv_quant_is_bit_exact(cuda):
    import json
    import os
    from conftest import GOLDEN
    torch = cuda
    rng = np.random.default_rng(0)
    rows = [(rng.normal(size=48) * 10 ** rng.uniform(-4, 4)).astype(np.float32) for _ in range(3000)]
    with open(os.path.join(GOLDEN, "kv_quant_vectors.json")) as f:
        for case in json.load(f)["cases"]:
            rows += list(np.array(case["in"], np.float32).reshape(-1, case["dim"]))
    for dim in (48, 64):
        sel = [r[:dim] if len(r) >= dim else np.pad(r, (0, dim - len(r))) for r in rows]
        x = np.stack(sel).astype(np.float32)
        q = torch.zeros(x.shape, dtype=torch.int8, device="cuda")
        s = torch.zeros(len(x), device="cuda")
        xd = dev(torch, x)
        nb.kv_quant(xd.data_ptr(), len(x), dim, q.data_ptr(), s.data_ptr())
        torch.cuda.synchronize()
        want = [orc.quant_into(r) for r in x]
        assert np.array_equal(q.cpu().numpy(), np.stack([w[0] for w in want]))
        assert np.array_equal(s.cpu().numpy(), np.array([w[1] for w in want], np.float32))


@pytest.mark.parametrize("int8", [True, False])
def test_attend_step_config2(cuda, int8):
    """64 sessions, context 512, 12 query heads (qk 48),
    2 KV heads (v 64), K/V N(0,1) quantised per (position, head), q fake-quantised."""
    torch = cuda
    B, S, H, KVH, QK, VH = 64, 512, 12, 2, 48, 64
    rng = np.random.default_rng(0)
    q = rng.normal(size=(B, H, QK)).astype(np.float32)
    k = rng.normal(size=(B, S, KVH, QK)).astype(np.float32)
    v = rng.normal(size=(B, S, KVH, VH)).astype(np.float32)
    lo = np.zeros(B, np.int32)
    hi = np.full(B, S - 1, np.int32)
    if int8:
        q = np.stack([np.stack([orc.fake_quant(h) for h in s]) for s in q])
        kq = np.zeros(k.shape, np.int8)
        vq = np.zeros(v.shape, np.int8)
        ks = np.zeros((B, S, KVH), np.float32)
        vs = np.zeros((B, S, KVH), np.float32)
        for b in range(B):
            for p in range(S):
                for h in range(KVH):
                    kq[b, p, h], ks[b, p, h] = orc.quant_into(k[b, p, h])
                    vq[b, p, h], vs[b, p, h] = orc.quant_into(v[b, p, h])
        args = (dev(torch, kq), dev(torch, vq), dev(torch, ks), dev(torch, vs))
    else:
        args = (dev(torch, k), dev(torch, v), None, None)
    out = torch.zeros(B, H * VH, device="cuda")
    qd, lod, hid = dev(torch, q), dev(torch, lo), dev(torch, hi)  # keep the device copies alive
    nb.attend_step(qd.data_ptr(), args[0].data_ptr(), args[1].data_ptr(),
                   args[2].data_ptr() if int8 else None, args[3].data_ptr() if int8 else None, int8, S,
                   lod.data_ptr(), hid.data_ptr(), B, H, KVH, QK, VH, out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b in range(0, B, 7):
        if int8:
            want = orc.attend_step(q[b].ravel(), S, 0, S - 1, H, KVH, QK, VH, kq=kq[b].ravel(), ks=ks[b].ravel(),
                                   vq=vq[b].ravel(), vs=vs[b].ravel())
        else:
            want = orc.attend_step(q[b].ravel(), S, 0, S - 1, H, KVH, QK, VH, k=k[b].ravel(), v=v[b].ravel())
        assert close(got[b], want, 1e-4)


def test_attend_step_ring_wrap_and_ragged_ranges(cuda):
    torch = cuda
    B, S, H, KVH, QK, VH = 5, 17, 4, 2, 48, 64
    rng = np.random.default_rng(1)
    q = rng.normal(size=(B, H, QK)).astype(np.float32)
    k = rng.normal(size=(B, S, KVH, QK)).astype(np.float32)
    v = rng.normal(size=(B, S, KVH, VH)).astype(np.float32)
    ranges = [(0, 0), (0, 9), (3, 16), (5, 5), (20, 36)]  # the last wraps the 17-slot ring
    lo = np.array([r[0] for r in ranges], np.int32)
    hi = np.array([r[1] for r in ranges], np.int32)
    out = torch.zeros(B, H * VH, device="cuda")
    keep = [dev(torch, a) for a in (q, k, v, lo, hi)]  # keep the device copies alive until the kernel ran
    nb.attend_step(keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), None, None, 0, S,
                   keep[3].data_ptr(), keep[4].data_ptr(), B, H, KVH, QK, VH, out.data_ptr())
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for b, (l, h) in enumerate(ranges):
        want = orc.attend_step(q[b].ravel(), S, l, h, H, KVH, QK, VH, k=k[b].ravel(), v=v[b].ravel())
        assert close(got[b], want, 1e-4)


@pytest.mark.parametrize("M", [512, 40])
def test_cq_grouped_projection_is_the_separate_ones(cuda, M):
    """nd_cq_project_grouped over config 1's three matrices (768, 2304 and 3072
    rows of 768, sharing the codebook) fills y with each matrix's projection
    side by side, matching both the oracle and three nd_cq_project calls."""
    torch = cuda
    cb = cact_pack.random_codebook(np.random.default_rng(21))
    levels = cact_pack.codebook_levels(cb, 2)
    shapes = [(768, 768), (2304, 768), (3072, 768)]
    mats = [make_weight(torch, out, inp, 2, 30 + i, cb) for i, (out, inp) in enumerate(shapes)]
    inp = 768
    x = np.random.default_rng(22).normal(size=(M, inp)).astype(np.float32)
    xh = np.stack([mats[0][3].prepare(r) for r in x])
    xd = dev(torch, xh)
    total = sum(o for o, _ in shapes)
    yg = torch.zeros(M, total, device="cuda")
    nb.cq_project_grouped([(m[1], m[2], o) for m, (o, _) in zip(mats, shapes)], inp, 2, levels, xd.data_ptr(), inp,
                          M, yg.data_ptr(), total)
    ys = []
    for m, (o, _) in zip(mats, shapes):
        y = torch.zeros(M, o, device="cuda")
        nb.cq_project(m[1], m[2], o, inp, 2, levels, xd.data_ptr(), inp, M, y.data_ptr(), o)
        ys.append(y)
    torch.cuda.synchronize()
    got = yg.cpu().numpy()
    sep = np.concatenate([y.cpu().numpy() for y in ys], axis=1)
    want = np.concatenate([m[3].matmul_prepared(xh) for m in mats], axis=1)
    assert close(got, want), float(np.abs(got - want).max())
    # The same products in the same order: one launch or three agree exactly.
    assert np.array_equal(got, sep)
