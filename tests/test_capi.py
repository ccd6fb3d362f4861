"""The C-ABI library loads and exports every entry point the header declares
(no kernel is launched: this runs without a GPU)."""
import ctypes
import os
import re

from conftest import REPO
from hayate_b200 import _lib


def header_functions():
    src = open(os.path.join(REPO, "include", "hayate_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(hy_[a-z0-9_]+)\s*\(", src)))


def test_header_and_binding_agree():
    assert header_functions() == sorted(_lib.exported_symbols())


def test_library_exports_every_symbol():
    lib = _lib.load()
    for name in header_functions():
        assert getattr(lib, name) is not None
    assert lib.hy_version() >= 100
    assert lib.hy_get_last_error() == b""


def test_invalid_arguments_fail_without_a_gpu():
    lib = _lib.load()
    assert lib.hy_argmax(7, None, 0, 1, 1, None, None) == -1
    assert b"dtype" in lib.hy_get_last_error()
    args = [None if t is ctypes.c_void_p else 0 for t in lib.hy_pack_batch.argtypes]
    assert lib.hy_pack_batch(*args) == -1
    assert lib.hy_attention_workspace_size(0, 0, 0) == 0
