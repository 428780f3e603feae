import hashlib
import importlib.util
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "needle-rs_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
CACHE = os.path.join(ROOT, ".pytest_cache", "containers")


def _load_pkg():
    if "needle_b200" in sys.modules:
        return sys.modules["needle_b200"]
    spec = importlib.util.spec_from_file_location(
        "needle_b200", os.path.join(PKG_DIR, "__init__.py"), submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["needle_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


nb = _load_pkg()
from needle_b200 import cact_pack  # noqa: E402

sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as orc  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def container(geom_name: str, seed: int) -> bytes:
    """Seeded synthetic container, cached on disk between runs."""
    os.makedirs(CACHE, exist_ok=True)
    path = os.path.join(CACHE, f"{geom_name}_{seed}.cact")
    if os.path.exists(path):
        return open(path, "rb").read()
    geom = getattr(cact_pack, geom_name)()
    raw = cact_pack.build_container(geom, seed=seed)
    tmp = path + f".{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(raw)
    os.replace(tmp, path)
    return raw


@pytest.fixture(scope="session")
def tiny_raw():
    return container("tiny", 1)


@pytest.fixture(scope="session")
def full_raw():
    return container("shipped", 0)


@pytest.fixture(scope="session")
def tiny_oracle(tiny_raw):
    return orc.Model(tiny_raw)


@pytest.fixture(scope="session")
def full_oracle(full_raw):
    return orc.Model(full_raw)


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    nb.lib()
    return torch


@pytest.fixture(scope="session")
def tiny_gpu(cuda, tiny_raw):
    return nb.V3Engine.from_bytes(tiny_raw)


@pytest.fixture(scope="session")
def full_gpu(cuda, full_raw):
    return nb.V3Engine.from_bytes(full_raw)


@pytest.fixture(scope="session")
def sp_fixture():
    """A SentencePiece BPE model trained with the `sentencepiece` package, as a
    RAW tokenizer blob plus that library's ids for a set of texts
    (tests/golden/make_tokenizer_golden.py)."""
    import base64
    import json
    d = json.load(open(os.path.join(GOLDEN, "sp_bpe_tokenizer.json")))
    d["blob"] = base64.b64decode(d["blob_b64"])
    return d


@pytest.fixture(scope="session")
def text_raw(sp_fixture):
    """The shipped-geometry container of full_raw with the fixture's tokenizer
    appended as its RAW record, cached on disk like the others."""
    os.makedirs(CACHE, exist_ok=True)
    path = os.path.join(CACHE, f"shipped_tok_0_{sha256(sp_fixture['blob'])[:12]}.cact")
    if os.path.exists(path):
        return open(path, "rb").read()
    raw = cact_pack.build_container(cact_pack.shipped(), seed=0, tokenizer=sp_fixture["blob"])
    tmp = path + f".{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(raw)
    os.replace(tmp, path)
    return raw


@pytest.fixture(scope="session")
def head_text_raw(sp_fixture):
    """As text_raw, with a confidence probe head between the final norm and the
    tokenizer (the weights before it are those of full_raw)."""
    os.makedirs(CACHE, exist_ok=True)
    path = os.path.join(CACHE, f"shipped_tok_head_0_{sha256(sp_fixture['blob'])[:12]}.cact")
    if os.path.exists(path):
        return open(path, "rb").read()
    raw = cact_pack.build_container(cact_pack.shipped(), seed=0, tokenizer=sp_fixture["blob"], confidence_head=True)
    tmp = path + f".{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(raw)
    os.replace(tmp, path)
    return raw


def sha256(b: bytes) -> str:
    return hashlib.sha256(b).hexdigest()
