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


def test_lm_head_argmax_checks_its_arguments_on_the_host():
    """The fused LM head's argument checks run before any CUDA call: bad
    geometry and missing buffers are refused with a message, zero rows is a
    no-op, and the workspace size is fixed."""
    lib = _lib.load()
    assert lib.hy_lm_head_argmax_workspace_size() == 4096
    assert lib.hy_lm_head_argmax(None, 128, 0, None, 128, 10, 128, None, None, None, None) == 0
    buf = ctypes.create_string_buffer(8192)
    p = (ctypes.addressof(buf) + 15) // 16 * 16         # 16-byte aligned host address
    # hidden not a multiple of 64 (the kernel's 64-element chunks)
    assert lib.hy_lm_head_argmax(p, 96, 2, p, 96, 10, 96, p, p, None, None) == -3
    assert b"multiple of 64" in lib.hy_get_last_error()
    # no workspace, no output, row pitch below the row width
    assert lib.hy_lm_head_argmax(p, 128, 2, p, 128, 10, 128, p, None, None, None) == -1
    assert lib.hy_lm_head_argmax(p, 128, 2, p, 128, 10, 128, None, p, None, None) == -1
    assert lib.hy_lm_head_argmax(p, 64, 2, p, 128, 10, 128, p, p, None, None) == -1
    # TMA needs 16-byte aligned starts and pitches
    assert lib.hy_lm_head_argmax(p + 2, 128, 2, p, 128, 10, 128, p, p, None, None) == -1
    assert lib.hy_lm_head_argmax(p, 132, 2, p, 128, 10, 128, p, p, None, None) == -1
    assert b"16-byte aligned" in lib.hy_get_last_error()


def test_lm_head_argmax_wrapper_refuses_non_bf16():
    import pytest
    import torch
    from hayate_b200 import kernels as K
    x = torch.zeros(2, 64, dtype=torch.float32)
    w = torch.zeros(10, 64, dtype=torch.float32)
    out = torch.zeros(2, dtype=torch.int32)
    with pytest.raises(ValueError, match="bf16"):
        K.lm_head_argmax(x, w, out, torch.zeros(4096, dtype=torch.uint8))
