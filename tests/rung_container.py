"""Test helper: write a ladder rung as a container of its own, the way
`needle build --layers N` ships one (the reference's
crates/needle-infer/tests/v3_ladder_slice.rs:1-12 compares such a file with a
load-time slice). Kept blocks' tensors are copied whole and renumbered; the
per-layer mHC scalars and the rows of the mHC lane matrices are cut to the kept
blocks; Engram sites survive with their blocks; the header's layer count,
global-layer mask and site list are rewritten. A container loaded from this at
full depth must compute exactly what the load-time slice computes."""
import struct

import numpy as np
from conftest import cact_pack

_ITEM = {cact_pack.DT_FP16: 2, cact_pack.DT_FP32: 4}


def _cq_rows(raw, rec, rows):
    """Rows of a CQ blob: packed codes [out, row_bytes] then f16 norms [out, groups]."""
    out, in_feat = rec["shape"][0], rec["shape"][1]
    group, bits = rec["group"], rec["bits"]
    in_pad = -(-in_feat // group) * group
    row_bytes, groups = in_pad * bits // 8, in_pad // group
    blob = raw[rec["offset"]:rec["offset"] + rec["nbytes"]]
    packed = np.frombuffer(blob, np.uint8, out * row_bytes).reshape(out, row_bytes)
    norms = np.frombuffer(blob, "<u2", out * groups, out * row_bytes).reshape(out, groups)
    return packed[rows].tobytes() + norms[rows].tobytes()


def write_rung(raw: bytes, kept) -> bytes:
    """`raw` (a full-depth container) cut to the blocks `kept` (ascending)."""
    words, cb, recs = cact_pack.read_directory(raw)
    words, theta = list(words[:48]), words[48]
    L, n, taps = words[10], words[15], words[19]
    gmask = words[17] | (words[18] << 32)
    sites = list(words[32:32 + words[31]])
    per = 4 + (3 if taps else 0) + 7 + 13
    blob = lambda r: raw[r["offset"]:r["offset"] + r["nbytes"]]  # noqa: E731
    w = cact_pack._Writer()

    def copy(r):
        w.recs.append((r["dtype"], tuple(r["shape"]), blob(r), r["group"], r["bits"]))

    copy(recs[0])  # embedding
    for l in kept:
        for r in recs[1 + l * per:1 + (l + 1) * per]:
            copy(r)
    at = 1 + L * per
    for width, r in zip((1, 1, 1, n, n, n * n), recs[at:at + 6]):  # a_*, b_*
        isz = _ITEM[r["dtype"]]
        rows = np.frombuffer(blob(r), np.uint8).reshape(L, width * isz)[kept]
        shape = (len(kept),) + tuple(r["shape"][1:])
        w.recs.append((r["dtype"], shape, rows.tobytes(), r["group"], r["bits"]))
    for width, r in zip((n, n, n * n), recs[at + 6:at + 9]):  # phi_pre, phi_post, phi_res
        rows = [i for l in kept for i in range(l * width, (l + 1) * width)]
        w.recs.append((r["dtype"], (len(rows), r["shape"][1]), _cq_rows(raw, r, rows), r["group"], r["bits"]))
    copy(recs[at + 9])
    copy(recs[at + 10])  # hadamard permutations
    at += 11
    new_sites = []
    for s, layer in enumerate(sites):
        if layer in kept:
            new_sites.append(kept.index(layer))
            for r in recs[at + 4 * s:at + 4 * s + 4]:
                copy(r)
    at += 4 * len(sites)
    copy(recs[at])  # final norm
    at += 1
    # Probe heads (v3.rs:745-787): cells 0 and 1 + each kept block of probes
    # (CQ rows) and gain, and the same cells on the middle axis of row_bias.
    if at < len(recs) and recs[at]["dtype"] != cact_pack.DT_RAW:
        man = recs[at]
        copy(man)
        codes = np.frombuffer(blob(man), "<f2" if man["dtype"] == cact_pack.DT_FP16 else "<f4").astype(int)
        at += 1
        cells = [0] + [k + 1 for k in kept]
        for code in codes:
            pr, ga, qu, rb, pj, bi = recs[at:at + 6]
            k = pr["shape"][0] // (L + 1)
            rows = [c * k + i for c in cells for i in range(k)]
            w.recs.append((pr["dtype"], (len(rows), pr["shape"][1]), _cq_rows(raw, pr, rows), pr["group"], pr["bits"]))
            isz = _ITEM[ga["dtype"]]
            g = np.frombuffer(blob(ga), np.uint8).reshape(L + 1, k * isz)[cells]
            w.recs.append((ga["dtype"], (len(cells), k), g.tobytes(), 0, 0))
            copy(qu)
            q = rb["shape"][0]
            b = np.frombuffer(blob(rb), np.uint8).reshape(q, L + 1, k * _ITEM[rb["dtype"]])[:, cells]
            w.recs.append((rb["dtype"], (q, len(cells), k), b.tobytes(), 0, 0))
            copy(pj)
            copy(bi)
            at += 6
            if code == 3:
                copy(recs[at])
                at += 1
    for r in recs[at:]:  # the tokenizer
        copy(r)
    new_mask = 0
    for i, l in enumerate(kept):
        if (gmask >> l) & 1:
            new_mask |= 1 << i
    words[1] = len(w.recs)
    words[10] = len(kept)
    words[17], words[18] = new_mask & 0xFFFFFFFF, new_mask >> 32
    words[31] = len(new_sites)
    words[32:48] = new_sites + [0] * (16 - len(new_sites))
    return w.build(words, theta, cb)


def header_layers(raw: bytes) -> int:
    return struct.unpack_from("<I", raw, 40)[0]
