"""hy_varlen_attention_noalloc: attention for callers that cannot allocate.

Some callers cannot allocate device memory where they invoke the kernel (an
FFI or plugin host that passes only the operation's tensors, a runtime whose
pool owns all device memory, a path that must not risk cudaMalloc's implicit
synchronisation).  This entry point plans and runs the bf16 attention with the
library's built-in scratch array instead of a caller workspace.  It runs the
same plan and kernel as the workspace entry point, so its output must equal
that entry point's bit for bit, call after call, whatever the previous call
left in the shared scratch; and it must stay within the 2e-2 attention bound of
the fp32 oracle.
"""
import pytest
import torch

from helpers import random_paged_batch, reference_attention
from hayate_b200 import _lib
from hayate_b200 import kernels as K

pytestmark = pytest.mark.gpu


def _with_workspace(b, kv_heads, bt=None, rows=None, layer=None):
    out = torch.empty_like(b["q"])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.zeros(K.attention_workspace_size(b["S"], b["T"], kv_heads), dtype=torch.uint8,
                     device="cuda")
    K.attention_plan(b["cu"], b["kv"], b["S"], kv_heads, b["S"], b["T"], ws, err)
    K.varlen_attention(b["q"], out, b["cache"], b["layer"] if layer is None else layer,
                       b["bt"] if bt is None else bt, b["cu"], b["kv"], b["S"], b["S"], b["T"], ws,
                       seq_bt_row=rows, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def _no_alloc(b, kv_heads, bt=None, rows=None, layer=None, with_err=True):
    """One call through the C ABI; returns (out, error word or None)."""
    lib = _lib.load()
    out = torch.full_like(b["q"], float("nan"))
    err = torch.zeros(1, dtype=torch.int32, device="cuda") if with_err else None
    cache = b["cache"]
    bt = b["bt"] if bt is None else bt
    rc = lib.hy_varlen_attention_noalloc(
        b["q"].data_ptr(), out.data_ptr(), b["T"], 4 * kv_heads, kv_heads, cache.data_ptr(),
        cache.shape[0], cache.shape[1], b["layer"] if layer is None else layer, bt.data_ptr(),
        bt.shape[1], None if rows is None else rows.data_ptr(), b["cu"].data_ptr(),
        b["kv"].data_ptr(), b["S"], 1.0 / 128 ** 0.5, None if err is None else err.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.hy_get_last_error()
    torch.cuda.synchronize()
    return out, None if err is None else int(err.item())


def _check(got, want_ws, b):
    assert torch.equal(got, want_ws), (got.float() - want_ws.float()).abs().max().item()
    assert (got.float() - reference_attention(b)).abs().max().item() <= 2e-2


def test_no_alloc_matches_workspace_entry_point_on_consecutive_calls():
    # 1: a 16384-token context (256 split items for one sequence) beside prefill
    b1 = random_paged_batch([1, 300, 1, 1, 40], [4000, 812, 17, 16384, 40], kv_heads=8, seed=21)
    # 2: other shapes, fewer splits per sequence, after 1 left its scratch
    b2 = random_paged_batch([1] * 9 + [64], [33, 1, 5000, 260, 16, 17, 999, 2048, 70, 64],
                            kv_heads=8, seed=22)
    for b in (b1, b2):
        got, err = _no_alloc(b, 8)
        assert err == 0
        _check(got, _with_workspace(b, 8), b)
    # 3: batch 1 again, at the other layer, with its block-table rows moved to
    # rows 6, 0, 3, 7, 2 of a larger table (seq_bt_row indirection)
    b3 = random_paged_batch([1, 300, 1, 1, 40], [4000, 812, 17, 16384, 40], kv_heads=8, seed=21,
                            layer=0)
    rows = torch.tensor([6, 0, 3, 7, 2], dtype=torch.int32, device="cuda")
    big = torch.full((8, b3["bt"].shape[1]), -1, dtype=torch.int32, device="cuda")
    big[rows.long()] = b3["bt"]
    got, err = _no_alloc(b3, 8, bt=big, rows=rows)
    assert err == 0
    _check(got, _with_workspace(b3, 8, bt=big, rows=rows), b3)
    # 4: no error word at all (nullable) on a valid batch
    got, err = _no_alloc(b2, 8, with_err=False)
    assert err is None
    _check(got, _with_workspace(b2, 8), b2)


def test_no_alloc_reports_a_bad_block_id_and_recovers():
    """A block id past the cache in a prefill sequence's table: the kernel's own
    bounds check sets HY_DEV_BOUNDS in the caller's error word (the tile reads
    zeros instead); the next call on the same scratch is exact again."""
    b = random_paged_batch([1, 40, 1], [300, 40, 100], kv_heads=8, seed=5)
    bad = b["bt"].clone()
    bad[1, 1] = b["cache"].shape[1] + 3
    _, err = _no_alloc(b, 8, bt=bad)
    assert err & K.DEV_BOUNDS
    got, err = _no_alloc(b, 8)
    assert err == 0
    _check(got, _with_workspace(b, 8), b)


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
