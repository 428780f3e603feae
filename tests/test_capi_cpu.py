"""The C ABI without a GPU: the library loads, exports every symbol the header
declares, and reports argument errors the way the reference does
(crates/needle-c/src/lib.rs:27-40: NULL/false/0 plus a thread-local message)."""
import ctypes
import os
import re

import pytest
from conftest import ROOT, nb

HEADER = os.path.join(ROOT, "include", "needle.h")


def declared():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b((?:needle|nd)_[a-z0-9_]+)\s*\(", src)))


def test_header_compiles_as_c():
    import subprocess
    r = subprocess.run(["gcc", "-std=c99", "-fsyntax-only", "-x", "c", HEADER], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_library_exports_every_declared_symbol():
    lib = nb.lib()
    names = declared()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the reference's Needle-3 surface is all there
    for n in ("needle_v3_load", "needle_v3_load_bytes", "needle_v3_load_with_depth", "needle_v3_num_layers",
              "needle_v3_run", "needle_v3_run_json", "needle_v3_reasoning", "needle_v3_generate",
              "needle_v3_run_stream", "needle_v3_has_confidence", "needle_v3_confidence_for",
              "needle_v3_kv_bytes", "needle_v3_max_seq_len", "needle_v3_free", "needle_free_str",
              "needle_last_error"):
        assert n in names


def test_null_and_bad_arguments_set_the_last_error():
    lib = nb.lib()
    assert lib.needle_v3_num_layers(None) == 0
    assert b"null" in lib.needle_last_error()
    assert lib.needle_v3_max_seq_len(None) == 0
    assert lib.needle_v3_kv_bytes(None, 10, False) == 0
    assert not lib.needle_v3_has_confidence(None)
    assert lib.needle_v3_load_bytes(None, 0) is None
    assert lib.needle_last_error() == b"data was null"
    assert lib.needle_v3_load(None) is None
    assert b"null" in lib.needle_last_error()
    lib.needle_v3_free(None)  # safe on NULL (v3.rs:378-382)
    lib.needle_free_str(None)


def test_malformed_containers_are_rejected_before_touching_the_gpu(tiny_raw):
    lib = nb.lib()
    assert lib.needle_v3_load_bytes(b"\x00" * 10, 10) is None
    assert b"too short" in lib.needle_last_error()
    bad = bytearray(tiny_raw)
    bad[0] ^= 1
    assert lib.needle_v3_load_bytes(bytes(bad), len(bad)) is None
    assert b"bad tag" in lib.needle_last_error()
    short = tiny_raw[:300]
    assert lib.needle_v3_load_bytes(short, len(short)) is None
    assert b"directory" in lib.needle_last_error()
    assert lib.needle_v3_load(b"/nonexistent/needle3.cact") is None
    assert b"cannot read" in lib.needle_last_error()


def test_error_is_thread_local():
    import threading
    lib = nb.lib()
    lib.needle_v3_num_layers(None)
    seen = []

    def other():
        seen.append(lib.needle_last_error())

    t = threading.Thread(target=other)
    t.start()
    t.join()
    assert seen == [None]
    assert lib.needle_last_error() is not None


def test_text_calls_fail_with_a_clear_message():
    lib = nb.lib()
    assert lib.needle_v3_run(None, b"q", b"[]") is None
    assert b"null" in lib.needle_last_error()
