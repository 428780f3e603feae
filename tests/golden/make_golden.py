"""Regenerate the golden fixtures in tests/golden/ (run in a container that has
the reference checkout; the committed fixtures are what the tests read).

    python tests/golden/make_golden.py /path/to/needle-rs

* kv_quant_vectors.json — the six `fake_quant` cases of the reference's
  `tests/v3_kv_quant_vectors.json` (generated upstream from
  needle.model.quantize.fake_quant; gated by
  crates/needle-core/tests/v3_kv_quant_parity.rs:18-65), copied unchanged.
* cact_v3_directory.json — header geometry and the directory of the shipped
  needle3.cact (the reference's `tests/cact_v3_vectors.json`): record dtypes,
  shapes, groups, widths and byte sizes, which pin the container canon and the
  CQ size arithmetic.
* ladder_rungs.json — the reference's `tests/v3_ladder_rungs.json` (the
  intelligence ladder of a 20-block model: block order and, per depth, the
  kept blocks, renumbered global layers and Engram sites; gated by
  crates/needle-infer/tests/v3_ladder_slice.rs:39-68), copied unchanged.
* numpy_ref_{tiny,full}.npz — logits of the reference's own numpy model
  (`tools/needle3_reference.py`, imported from the reference checkout) on
  seeded synthetic containers written by needle-rs_b200/cact_pack.py. The
  numpy model masks token id 0 as padding and needs prompts longer than the
  Engram reach, so prompts are drawn from [1, vocab) with T > 9.
"""
import hashlib
import json
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "needle-rs_b200"))
import cact_pack  # noqa: E402


def copy_ladder(ref_root):
    with open(os.path.join(ref_root, "tests", "v3_ladder_rungs.json")) as f:
        lad = json.load(f)
    with open(os.path.join(HERE, "ladder_rungs.json"), "w") as f:
        json.dump(lad, f)


def main(ref_root):
    copy_ladder(ref_root)
    with open(os.path.join(ref_root, "tests", "v3_kv_quant_vectors.json")) as f:
        kv = json.load(f)
    with open(os.path.join(HERE, "kv_quant_vectors.json"), "w") as f:
        json.dump(kv, f)
    with open(os.path.join(ref_root, "tests", "cact_v3_vectors.json")) as f:
        cv = json.load(f)
    keep = {k: cv[k] for k in ("container_bytes", "header_bytes", "record_bytes", "codebook_len", "geometry")}
    keep["records"] = [{k: r[k] for k in ("index", "dtype", "ndim", "shape", "offset", "nbytes", "group", "bits")}
                       for r in cv["records"]]
    with open(os.path.join(HERE, "cact_v3_directory.json"), "w") as f:
        json.dump(keep, f)

    sys.path.insert(0, os.path.join(ref_root, "tools"))
    import needle3_reference as ref  # the reference's own numpy model

    for name, geom, seed, T, keep_rows in (("tiny", cact_pack.tiny(), 1, 20, None),
                                           ("full", cact_pack.shipped(), 0, 16, [0, 7, 15])):
        raw = cact_pack.build_container(geom, seed=seed)
        with tempfile.TemporaryDirectory() as tmp:
            path = os.path.join(tmp, f"golden_{name}.cact")
            with open(path, "wb") as f:
                f.write(raw)
            toks = np.random.default_rng(seed).integers(1, geom.vocab_size, T).astype(np.int64)
            logits = ref.Model(path).forward(toks).astype(np.float32)
        rows = list(range(T)) if keep_rows is None else keep_rows
        np.savez_compressed(os.path.join(HERE, f"numpy_ref_{name}.npz"), tokens=toks.astype(np.uint32),
                            rows=np.array(rows), logits=logits[rows], argmax=logits.argmax(-1),
                            container_sha256=np.array(hashlib.sha256(raw).hexdigest()), seed=np.array(seed))
        print(name, logits.shape)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <path of the needle-rs checkout>")
    main(sys.argv[1])
