"""hy_varlen_attention_noalloc: attention for callers that cannot allocate.

Some callers cannot allocate device memory where they invoke the kernel (an
FFI or plugin host that passes only the operation's tensors, a runtime whose
pool owns all device memory, a path that must not risk cudaMalloc's implicit
synchronisation).  This entry point plans and runs the bf16 attention with the
library's built-in scratch array instead of a caller workspace.  Its output
must match the workspace entry point's, call after call.
"""
import ctypes

import pytest
import torch

from helpers import random_paged_batch
from hayate_b200 import _lib
from hayate_b200 import kernels as K

pytestmark = pytest.mark.gpu


def _with_workspace(b, kv_heads):
    out = torch.empty_like(b["q"])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.zeros(K.attention_workspace_size(b["S"], b["T"], kv_heads), dtype=torch.uint8,
                     device="cuda")
    K.attention_plan(b["cu"], b["kv"], b["S"], kv_heads, b["S"], b["T"], ws, err)
    K.varlen_attention(b["q"], out, b["cache"], b["layer"], b["bt"], b["cu"], b["kv"], b["S"],
                       b["S"], b["T"], ws, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def _no_alloc(b, kv_heads):
    lib = _lib.load()
    out = torch.full_like(b["q"], float("nan"))
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    cache = b["cache"]
    rc = lib.hy_varlen_attention_noalloc(
        b["q"].data_ptr(), out.data_ptr(), b["T"], 4 * kv_heads, kv_heads, cache.data_ptr(),
        cache.shape[0], cache.shape[1], b["layer"], b["bt"].data_ptr(), b["bt"].shape[1], None,
        b["cu"].data_ptr(), b["kv"].data_ptr(), b["S"], 1.0 / 128 ** 0.5, err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.hy_get_last_error()
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def test_no_alloc_matches_workspace_entry_point_on_consecutive_calls():
    batches = [
        random_paged_batch([1, 300, 1, 1, 40], [4000, 812, 17, 16384, 40], kv_heads=8, seed=21),
        random_paged_batch([1] * 9 + [64], [33, 1, 5000, 260, 16, 17, 999, 2048, 70, 64],
                           kv_heads=8, seed=22),
    ]
    for b in batches:                   # two calls in a row, different shapes
        want = _with_workspace(b, 8)
        got = _no_alloc(b, 8)
        assert (got.float() - want.float()).abs().max().item() <= 2e-2


def test_no_alloc_rejects_batches_beyond_its_scratch():
    lib = _lib.load()
    dummy = torch.zeros(16, dtype=torch.int32, device="cuda")
    p = dummy.data_ptr()
    rc = lib.hy_varlen_attention_noalloc(p, p, 9000, 32, 8, p, 1, 1, 0, p, 1, None, p, p, 1,
                                         0.1, None, None)
    assert rc == -1
    assert b"exceeds the built-in scratch limit" in lib.hy_get_last_error()
    rc = lib.hy_varlen_attention_noalloc(p, p, 10, 32, 8, p, 1, 1, 0, p, 1, None, p, p, 300,
                                         0.1, None, None)
    assert rc == -1
