"""Torch-facing wrappers over the C ABI (device tensors in, launches out).

Every function launches on ``torch.cuda.current_stream()`` and returns without
synchronising.  Shapes and dtypes are checked on the host before the call;
the kernels check indices on the device and report through the int32 error
word (bits ``DEV_*``).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import check

DEV_BOUNDS, DEV_TIMEOUT, DEV_POOL, DEV_PLAN = 1, 2, 4, 8
ATTN_EARLY = 1                      # hy_varlen_attention flag HY_ATTN_EARLY
DTYPES = {torch.bfloat16: 0, torch.float32: 1}


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _i32(t: torch.Tensor, name: str):
    if t.dtype != torch.int32 or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous int32 CUDA tensor")


def _dt(t: torch.Tensor) -> int:
    try:
        return DTYPES[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}; use bf16 or fp32") from None


def describe_error(word: int) -> str:
    names = [(DEV_BOUNDS, "index out of range"), (DEV_TIMEOUT, "wait timed out"),
             (DEV_POOL, "KV block pool exhausted"), (DEV_PLAN, "attention plan overflow")]
    return ", ".join(n for b, n in names if word & b) or "none"


def block_pool_init(free_stack: torch.Tensor, free_top: torch.Tensor) -> None:
    _i32(free_stack, "free_stack")
    _i32(free_top, "free_top")
    check(_lib.load().hy_block_pool_init(_ptr(free_stack), _ptr(free_top), free_stack.numel(),
                                         _stream()), "hy_block_pool_init")


def pack_batch(sched: torch.Tensor, num_seqs: int, num_tokens: int, req_tokens: torch.Tensor,
               block_tables: torch.Tensor, req_num_blocks: torch.Tensor,
               free_stack: torch.Tensor, free_top: torch.Tensor, input_ids: torch.Tensor,
               positions: torch.Tensor, slot_mapping: torch.Tensor, cu_seqlens_q: torch.Tensor,
               seq_lens_k: torch.Tensor, sample_rows: torch.Tensor, sample_seq: torch.Tensor,
               err: torch.Tensor) -> None:
    for n, t in (("sched", sched), ("req_tokens", req_tokens), ("block_tables", block_tables),
                 ("req_num_blocks", req_num_blocks), ("free_stack", free_stack),
                 ("free_top", free_top), ("input_ids", input_ids), ("positions", positions),
                 ("slot_mapping", slot_mapping), ("cu_seqlens_q", cu_seqlens_q),
                 ("seq_lens_k", seq_lens_k), ("sample_rows", sample_rows),
                 ("sample_seq", sample_seq), ("err", err)):
        _i32(t, n)
    if sched.numel() < 4 * num_seqs or cu_seqlens_q.numel() < num_seqs + 1:
        raise ValueError("sched/cu_seqlens_q too small for num_seqs")
    if input_ids.numel() < num_tokens:
        raise ValueError("token buffers smaller than num_tokens")
    check(_lib.load().hy_pack_batch(
        _ptr(sched), num_seqs, num_tokens, _ptr(req_tokens), req_tokens.shape[1],
        req_tokens.shape[0], _ptr(block_tables), block_tables.shape[1], _ptr(req_num_blocks),
        _ptr(free_stack), _ptr(free_top), free_stack.numel(), _ptr(input_ids), _ptr(positions),
        _ptr(slot_mapping), _ptr(cu_seqlens_q), _ptr(seq_lens_k), _ptr(sample_rows),
        _ptr(sample_seq), _ptr(err), _stream()), "hy_pack_batch")


def free_blocks(slots: torch.Tensor, block_tables: torch.Tensor, req_num_blocks: torch.Tensor,
                free_stack: torch.Tensor, free_top: torch.Tensor, err: torch.Tensor,
                first_block: Optional[torch.Tensor] = None) -> None:
    """Return the listed slots' blocks to the pool (from position first_block[i]
    on, when given: the earlier blocks stay with a prefix cache)."""
    _i32(slots, "slots")
    if first_block is None:
        check(_lib.load().hy_free_blocks(
            _ptr(slots), slots.numel(), block_tables.shape[0], _ptr(block_tables),
            block_tables.shape[1], _ptr(req_num_blocks), _ptr(free_stack), _ptr(free_top),
            free_stack.numel(), _ptr(err), _stream()), "hy_free_blocks")
        return
    _i32(first_block, "first_block")
    if first_block.numel() != slots.numel():
        raise ValueError("first_block needs one entry per slot")
    check(_lib.load().hy_free_blocks_from(
        _ptr(slots), _ptr(first_block), slots.numel(), block_tables.shape[0], _ptr(block_tables),
        block_tables.shape[1], _ptr(req_num_blocks), _ptr(free_stack), _ptr(free_top),
        free_stack.numel(), _ptr(err), _stream()), "hy_free_blocks_from")


def push_blocks(block_ids: torch.Tensor, free_stack: torch.Tensor, free_top: torch.Tensor,
                err: torch.Tensor) -> None:
    """Push block ids onto the free stack (blocks a prefix cache gives up)."""
    _i32(block_ids, "block_ids")
    check(_lib.load().hy_push_blocks(_ptr(block_ids), block_ids.numel(), _ptr(free_stack),
                                     _ptr(free_top), free_stack.numel(), _ptr(err), _stream()),
          "hy_push_blocks")


def commit_tokens(next_tokens: torch.Tensor, n_sample: int, sample_seq: torch.Tensor,
                  sched: torch.Tensor, num_seqs: int, req_tokens: torch.Tensor,
                  err: torch.Tensor) -> None:
    check(_lib.load().hy_commit_tokens(
        _ptr(next_tokens), n_sample, _ptr(sample_seq), _ptr(sched), num_seqs, _ptr(req_tokens),
        req_tokens.shape[1], req_tokens.shape[0], _ptr(err), _stream()), "hy_commit_tokens")


def qk_norm_rope(qkv: torch.Tensor, q_heads: int, kv_heads: int, positions: torch.Tensor,
                 q_norm_w: torch.Tensor, k_norm_w: torch.Tensor, rope_cos: torch.Tensor,
                 rope_sin: torch.Tensor, eps: float, q_out: Optional[torch.Tensor] = None,
                 k_out: Optional[torch.Tensor] = None, kv_cache_layer: Optional[torch.Tensor] = None,
                 slot_mapping: Optional[torch.Tensor] = None, num_blocks: int = 0,
                 err: Optional[torch.Tensor] = None) -> None:
    T = qkv.shape[0]
    if qkv.stride(1) != 1:
        raise ValueError("qkv rows must be contiguous")
    for t in (q_out, k_out, kv_cache_layer):
        if t is not None and (t.dtype != qkv.dtype or not t.is_contiguous()):
            raise ValueError("outputs must be contiguous and share qkv's dtype")
    if rope_cos.dtype != torch.float32 or rope_cos.shape[1] != 64:
        raise ValueError("rope tables must be fp32 [max_pos][64]")
    check(_lib.load().hy_qk_norm_rope(
        _dt(qkv), _ptr(qkv), qkv.stride(0), T, q_heads, kv_heads, _ptr(positions),
        _ptr(q_norm_w), _ptr(k_norm_w), _ptr(rope_cos), _ptr(rope_sin), rope_cos.shape[0],
        float(eps), _ptr(q_out), _ptr(k_out), _ptr(kv_cache_layer), _ptr(slot_mapping),
        num_blocks, _ptr(err), _stream()), "hy_qk_norm_rope")


def kv_append(k: torch.Tensor, v: torch.Tensor, slot_mapping: torch.Tensor,
              kv_cache_layer: torch.Tensor, num_blocks: int,
              err: Optional[torch.Tensor] = None) -> None:
    T, kv_heads = k.shape[0], k.shape[1]
    check(_lib.load().hy_kv_append(_dt(k), _ptr(k), _ptr(v), T, kv_heads, _ptr(slot_mapping),
                                   _ptr(kv_cache_layer), num_blocks, _ptr(err), _stream()),
          "hy_kv_append")


def attention_workspace_size(max_seqs: int, max_tokens: int, kv_heads: int) -> int:
    return int(_lib.load().hy_attention_workspace_size(max_seqs, max_tokens, kv_heads))


def attention_plan(cu_seqlens_q: torch.Tensor, seq_lens_k: torch.Tensor, num_seqs: int,
                   kv_heads: int, max_seqs: int, max_tokens: int, workspace: torch.Tensor,
                   err: Optional[torch.Tensor] = None) -> None:
    check(_lib.load().hy_attention_plan(
        _ptr(cu_seqlens_q), _ptr(seq_lens_k), num_seqs, kv_heads, max_seqs, max_tokens,
        _ptr(workspace), workspace.numel() * workspace.element_size(), _ptr(err), _stream()),
        "hy_attention_plan")


def varlen_attention(q: torch.Tensor, out: torch.Tensor, kv_cache: torch.Tensor, layer: int,
                     block_tables: torch.Tensor, cu_seqlens_q: torch.Tensor,
                     seq_lens_k: torch.Tensor, num_seqs: int, max_seqs: int, max_tokens: int,
                     workspace: Optional[torch.Tensor], seq_bt_row: Optional[torch.Tensor] = None,
                     scale: Optional[float] = None, err: Optional[torch.Tensor] = None,
                     early: bool = False) -> None:
    """kv_cache: [layers][blocks][2][kv_heads][16][128]; q/out: [tokens][q_heads][128].
    ``early``: HY_ATTN_EARLY (the plan, block tables and older cache entries were
    written at least two launches back and this is not the plan's first call)."""
    T, q_heads, D = q.shape
    L, NB, two, kv_heads, bs, D2 = kv_cache.shape
    if (two, bs, D, D2) != (2, 16, 128, 128):
        raise ValueError("kv_cache must be [layers][blocks][2][kv_heads][16][128]")
    if q.dtype != kv_cache.dtype or out.dtype != q.dtype:
        raise ValueError("q, out and kv_cache must share a dtype")
    scale = (1.0 / D ** 0.5) if scale is None else scale
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    check(_lib.load().hy_varlen_attention(
        _dt(q), _ptr(q), _ptr(out), T, q_heads, kv_heads, _ptr(kv_cache), L, NB, layer,
        _ptr(block_tables), block_tables.shape[1], _ptr(seq_bt_row), _ptr(cu_seqlens_q),
        _ptr(seq_lens_k), num_seqs, float(scale), max_seqs, max_tokens, _ptr(workspace),
        ws_bytes, ATTN_EARLY if early else 0, _ptr(err), _stream()), "hy_varlen_attention")


def add_rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float,
                 delta: Optional[torch.Tensor] = None,
                 out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x += delta in place (if given), then return RMSNorm(x) * w."""
    rows, cols = x.shape
    if x.stride(1) != 1 or (delta is not None and delta.stride(1) != 1):
        raise ValueError("rows must be contiguous")
    out = torch.empty_like(x) if out is None else out
    check(_lib.load().hy_add_rms_norm(
        _dt(x), _ptr(x), x.stride(0), _ptr(delta), 0 if delta is None else delta.stride(0), rows,
        cols, _ptr(w), float(eps), _ptr(out), out.stride(0), _stream()), "hy_add_rms_norm")
    return out


def add_rms_norm_splitk(x: torch.Tensor, w: torch.Tensor, eps: float, parts: torch.Tensor,
                        out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x += round(parts.sum(0)) in place (parts: [n, rows, cols] fp32 split-K
    partials of the projection giving the residual's delta), then return
    RMSNorm(x) * w."""
    rows, cols = x.shape
    if parts.dtype != torch.float32 or parts.dim() != 3 or parts.shape[1:] != (rows, cols):
        raise ValueError("parts must be fp32 [n, rows, cols]")
    if x.stride(1) != 1 or parts.stride(2) != 1:
        raise ValueError("rows must be contiguous")
    out = torch.empty_like(x) if out is None else out
    check(_lib.load().hy_add_rms_norm_splitk(
        _dt(x), _ptr(x), x.stride(0), _ptr(parts), parts.shape[0], parts.stride(0),
        parts.stride(1), rows, cols, _ptr(w), float(eps), _ptr(out), out.stride(0), _stream()),
        "hy_add_rms_norm_splitk")
    return out


def gather_add_rms_norm(x: torch.Tensor, rows: torch.Tensor, w: torch.Tensor, eps: float,
                        delta: Optional[torch.Tensor] = None,
                        parts: Optional[torch.Tensor] = None,
                        x_out: Optional[torch.Tensor] = None,
                        out: Optional[torch.Tensor] = None,
                        err: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Output row i: r = x[rows[i]] + delta[i] (or + round(parts[:, i].sum(0)),
    fp32 split-K partials; or r = x[rows[i]] with neither), written to
    x_out[i] if given; returns RMSNorm(r) * w.  x is not modified."""
    n = rows.numel()
    cols = x.shape[1]
    _i32(rows, "rows")
    if x.stride(1) != 1 or (delta is not None and delta.stride(1) != 1):
        raise ValueError("rows must be contiguous")
    if delta is not None and parts is not None:
        raise ValueError("give delta or parts, not both")
    out = torch.empty(n, cols, dtype=x.dtype, device=x.device) if out is None else out
    if parts is not None:
        if parts.dtype != torch.float32 or parts.dim() != 3 or parts.shape[1:] != (n, cols) \
                or parts.stride(2) != 1:
            raise ValueError("parts must be fp32 [k, rows, cols] with contiguous rows")
        ldd, nparts, pstride = parts.stride(1), parts.shape[0], parts.stride(0)
    else:
        ldd = 0 if delta is None else delta.stride(0)
        nparts, pstride = 0, 0
    check(_lib.load().hy_gather_add_rms_norm(
        _dt(x), _ptr(x), x.stride(0), _ptr(rows), x.shape[0], _ptr(delta), ldd, _ptr(parts),
        nparts, pstride, n, cols, _ptr(w), float(eps), _ptr(x_out),
        0 if x_out is None else x_out.stride(0), _ptr(out), out.stride(0), _ptr(err), _stream()),
        "hy_gather_add_rms_norm")
    return out


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
    return add_rms_norm(x, w, eps, None, out)


def silu_mul(gu: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    rows, two_i = gu.shape
    inter = two_i // 2
    if gu.stride(1) != 1:
        raise ValueError("gu rows must be contiguous")
    out = torch.empty(rows, inter, dtype=gu.dtype, device=gu.device) if out is None else out
    check(_lib.load().hy_silu_mul(_dt(gu), _ptr(gu), gu.stride(0), rows, inter, _ptr(out),
                                  out.stride(0), _stream()), "hy_silu_mul")
    return out


def argmax(logits: torch.Tensor, out: torch.Tensor) -> None:
    rows, V = logits.shape
    if logits.stride(1) != 1:
        raise ValueError("logits rows must be contiguous")
    _i32(out, "out")
    check(_lib.load().hy_argmax(_dt(logits), _ptr(logits), logits.stride(0), rows, V, _ptr(out),
                                _stream()), "hy_argmax")


def lm_head_argmax_workspace_size() -> int:
    return int(_lib.load().hy_lm_head_argmax_workspace_size())


def lm_head_argmax(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor, workspace: torch.Tensor,
                   err: Optional[torch.Tensor] = None) -> None:
    """out[r] = argmax_v bf16(x[r] . w[v]): the LM head and greedy sampling in
    one kernel (bf16; ``workspace`` zeroed once, left zeroed by every call)."""
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("lm_head_argmax is bf16 only")
    rows, hidden = x.shape
    vocab, hidden_w = w.shape
    if hidden_w != hidden or x.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("x (rows, hidden) and w (vocab, hidden) need contiguous rows of one width")
    if out.numel() < rows:
        raise ValueError("out holds fewer entries than x has rows")
    _i32(out, "out")
    if workspace.numel() * workspace.element_size() < lm_head_argmax_workspace_size():
        raise ValueError("workspace smaller than hy_lm_head_argmax_workspace_size()")
    check(_lib.load().hy_lm_head_argmax(_ptr(x), x.stride(0), rows, _ptr(w), w.stride(0), vocab,
                                        hidden, _ptr(out), _ptr(workspace), _ptr(err), _stream()),
          "hy_lm_head_argmax")
