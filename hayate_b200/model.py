"""Qwen3 forward over packed ragged batches, on the paged KV cache.

One ``Runner.launch_step`` is the device half of a continuous-batching step:

  pack (on-GPU batch build + block allocation) -> attention plan ->
  embed -> RMSNorm -> 36 x [QKV GEMM, QK-norm+RoPE+KV append, varlen attention,
  O GEMM, residual add + RMSNorm, gate/up GEMM, SiLU*up, down GEMM, residual add +
  next RMSNorm] -> LM head + argmax on the sampled rows only -> commit.

It replaces ``Qwen3Model.forward`` (hayate/model/qwen.py:46-124) with its block
and attention modules (block.py:21-31, attention.py:26-66, linear.py:11-14) and
the engine's gather/scatter around it (engine.py:80-163).  The projections, the
MLP and the LM head stay on cuBLAS through torch; the residual adds fused with
the RMSNorms, and SiLU*up, are this library's row kernels with the reference's
rounding points.  The LM head runs on the last row of each sampled sequence
only, where the reference computes logits for every position (qwen.py:122-123);
in bf16 greedy steps it is this library's tcgen05 kernel with the argmax in its
epilogue (``hy_lm_head_argmax``: the logits never reach HBM), otherwise a
cuBLAS GEMM whose logits go to ``hy_argmax`` or the caller's sampler.

Nothing here synchronises: the step is a fixed sequence of launches over
static buffers, so a decode step can be captured in a CUDA graph.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from . import kernels as K
from .config import EngineConfig, ModelConfig, BLOCK_SIZE


@dataclass
class LayerWeights:
    w_qkv: torch.Tensor       # (q + 2kv, H)   rows: q_proj | k_proj | v_proj
    w_o: torch.Tensor         # (H, q)
    w_gate_up: torch.Tensor   # (2I, H)        rows: gate_proj | up_proj
    w_down: torch.Tensor      # (H, I)
    ln1: torch.Tensor         # input_layernorm
    ln2: torch.Tensor         # post_attention_layernorm
    q_norm: torch.Tensor
    k_norm: torch.Tensor


_SPLITK_ON = os.environ.get("HY_SPLITK", "1") != "0"
# HY_LM_FUSED=0: bf16 greedy steps take the cuBLAS LM head + hy_argmax instead
_LM_FUSED_ON = os.environ.get("HY_LM_FUSED", "1") != "0"


def linear_splitk(x: torch.Tensor, w: torch.Tensor, s: int) -> torch.Tensor:
    """x @ w.T as s fp32 partial products over K slices, [s, rows, out] (one
    cuBLAS batched GEMM; x [rows, K] and w [out, K] contiguous, K = s * slice)."""
    rows, k = x.shape
    n, ks = w.shape[0], k // s
    return torch.bmm(x.view(rows, s, ks).transpose(0, 1),
                     w.view(n, s, ks).transpose(0, 1).transpose(1, 2), out_dtype=torch.float32)


def rope_half_tables(cfg: ModelConfig, device):
    """fp32 cos/sin [max_pos][64]: the reference's tables (rope.py:3-13; the
    second half of each row repeats the first) computed with the same ops."""
    d = cfg.head_dim
    exps = torch.arange(0, d, 2, dtype=torch.float32)[: d // 2].float() / d
    inv_freq = 1.0 / (int(cfg.rope_theta) ** exps)
    pos = torch.arange(cfg.max_position_embeddings, dtype=torch.float32)
    ang = pos.unsqueeze(1) * inv_freq.unsqueeze(0)
    return torch.cos(ang).contiguous().to(device), torch.sin(ang).contiguous().to(device)


class Runner:
    """Device state (weights, KV cache, request rows, step buffers) + the step."""

    def __init__(self, cfg: ModelConfig, ecfg: EngineConfig, dtype: torch.dtype,
                 device: torch.device, embed: torch.Tensor, layers: List[Dict[str, torch.Tensor]],
                 norms: Optional[Dict[str, torch.Tensor]] = None):
        cfg.check_kernel_support()
        if dtype not in (torch.bfloat16, torch.float32):
            raise ValueError("dtype must be bf16 or fp32")
        if ecfg.block_size != BLOCK_SIZE:
            raise ValueError(f"block_size must be {BLOCK_SIZE}")
        self.cfg, self.ecfg, self.dtype, self.device = cfg, ecfg, dtype, device
        H, I = cfg.hidden_size, cfg.intermediate_size
        dev = device

        def dn(name, n):
            if norms is None:
                return torch.ones(n, dtype=dtype, device=dev)
            return norms[name].to(device=dev, dtype=dtype)

        self.embed = embed.to(device=dev, dtype=dtype).contiguous()
        self.layers: List[LayerWeights] = []
        for l, blk in enumerate(layers):
            g = lambda k: blk[k].to(device=dev, dtype=dtype)  # noqa: E731
            self.layers.append(LayerWeights(
                w_qkv=torch.cat([g("q_proj"), g("k_proj"), g("v_proj")], 0).contiguous(),
                w_o=g("o_proj").contiguous(),
                w_gate_up=torch.cat([g("gate_proj"), g("up_proj")], 0).contiguous(),
                w_down=g("down_proj").contiguous(),
                ln1=dn(f"layers.{l}.input_layernorm.weight", H),
                ln2=dn(f"layers.{l}.post_attention_layernorm.weight", H),
                q_norm=dn(f"layers.{l}.self_attn.q_norm.weight", cfg.head_dim),
                k_norm=dn(f"layers.{l}.self_attn.k_norm.weight", cfg.head_dim)))
            for k in list(blk):
                if blk[k].device == dev:          # drop the per-matrix device copies
                    del blk[k]
        self.final_norm = dn("norm.weight", H)
        self.rope_cos, self.rope_sin = rope_half_tables(cfg, dev)

        # ---- KV cache: [layer][block][K/V][kv_head][16][128]
        self.num_blocks = ecfg.num_kv_blocks or self._blocks_from_memory()
        self.kv_cache = torch.zeros(cfg.num_layers, self.num_blocks, 2, cfg.num_kv_heads,
                                    BLOCK_SIZE, cfg.head_dim, dtype=dtype, device=dev)
        # ---- request rows (slot max_reqs-1 is the graph padding row)
        self.max_reqs = ecfg.max_num_seqs + 1
        self.bt_pitch = -(-ecfg.max_model_len // BLOCK_SIZE)
        i32 = dict(dtype=torch.int32, device=dev)
        self.req_tokens = torch.zeros(self.max_reqs, ecfg.max_model_len + 1, **i32)
        self.block_tables = torch.zeros(self.max_reqs, self.bt_pitch, **i32)
        self.req_nblk = torch.zeros(self.max_reqs, **i32)
        self.free_stack = torch.zeros(self.num_blocks, **i32)
        self.free_top = torch.zeros(1, **i32)
        K.block_pool_init(self.free_stack, self.free_top)
        # ---- step buffers
        S, T = ecfg.max_num_seqs, ecfg.max_batched_tokens
        self.sched = torch.zeros(4 * S, **i32)
        self.input_ids = torch.zeros(T, **i32)
        self.positions = torch.zeros(T, **i32)
        self.slot_mapping = torch.zeros(T, **i32)
        self.cu_q = torch.zeros(S + 1, **i32)
        self.seq_lens_k = torch.zeros(S, **i32)
        self.sample_rows = torch.zeros(S, **i32)
        self.sample_seq = torch.zeros(S, **i32)
        self.out_buf = torch.zeros(1 + S, **i32)        # [error word | next tokens]
        self.q_buf = torch.empty(T, cfg.num_heads, cfg.head_dim, dtype=dtype, device=dev)
        self.attn_buf = torch.empty_like(self.q_buf)
        self.ws = None
        self.lm_ws = None                                # fused LM head + argmax (bf16)
        if dtype == torch.bfloat16:
            nbytes = K.attention_workspace_size(S, T, cfg.num_kv_heads)
            self.ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
            if _LM_FUSED_ON:
                self.lm_ws = torch.zeros(K.lm_head_argmax_workspace_size(), dtype=torch.uint8,
                                         device=dev)
        self.kernel_launches = 0

    # ------------------------------------------------------------------ memory
    def _blocks_from_memory(self) -> int:
        free, _ = torch.cuda.mem_get_info(self.device)
        per_block = (2 * self.cfg.num_kv_heads * BLOCK_SIZE * self.cfg.head_dim *
                     self.cfg.num_layers * torch.tensor([], dtype=self.dtype).element_size())
        act = 4 << 30                                    # activations + workspace headroom
        n = int((free - act) * self.ecfg.kv_cache_fraction) // per_block
        if n < 16:
            raise RuntimeError("not enough device memory for the KV cache")
        return n

    @property
    def error_word(self) -> torch.Tensor:
        return self.out_buf[:1]

    @property
    def next_tokens(self) -> torch.Tensor:
        return self.out_buf[1:]

    # ------------------------------------------------------------------ step
    def launch_step(self, S: int, T: int, n_sample: int, sampler=None) -> None:
        """Enqueue one step for the schedule already in ``self.sched[:4*S]``:
        pack, the model, the LM head on the sampled rows, the next tokens
        (greedy argmax kernel, or ``sampler(logits) -> (n, 1) or (n,)`` token
        ids on the device) committed to the requests' token rows.  bf16
        greedy steps run the LM head and the argmax as one kernel."""
        toks = self.next_tokens[:n_sample]
        if sampler is None and self.lm_ws is not None:
            h = self.forward_hidden(S, T, n_sample)
            if h is None:
                return
            K.lm_head_argmax(h, self.embed, toks, self.lm_ws, self.error_word)
        else:
            logits = self.forward_logits(S, T, n_sample)
            if logits is None:
                return
            if sampler is None:
                K.argmax(logits, toks)
            else:
                toks.copy_(sampler(logits).reshape(-1))
        K.commit_tokens(toks, n_sample, self.sample_seq, self.sched[:4 * S], S, self.req_tokens,
                        self.error_word)
        if sampler is not None:
            self.kernel_launches += 1
        elif self.lm_ws is not None:                # one LM-head launch per 256 rows
            self.kernel_launches += 1 + (n_sample + 255) // 256
        else:
            self.kernel_launches += 2

    def forward_logits(self, S: int, T: int, n_sample: int) -> Optional[torch.Tensor]:
        """The model half of a step: pack the schedule in ``self.sched[:4*S]``
        (allocating its KV blocks), run the layers (appending the step's K/V to
        the cache), and return the logits ``(n_sample, vocab)`` of the last
        token of each sequence that samples, in schedule order -- the reference
        model's ``logits[:, -1, :]`` (qwen.py:46-124, engine.py:143-163), or None
        when no sequence samples.  Nothing is committed: the caller appends the
        chosen tokens (``launch_step`` does, or ``commit_next_tokens``).

        The last layer needs every row only up to its attention (their K/V are
        appended there); from its o_proj on it runs on the sampled rows alone,
        gathered by ``hy_gather_add_rms_norm``, and the final norm follows on
        those rows (the reference norms and projects every position,
        qwen.py:122-123)."""
        h = self.forward_hidden(S, T, n_sample)
        return None if h is None else F.linear(h, self.embed)

    def forward_hidden(self, S: int, T: int, n_sample: int) -> Optional[torch.Tensor]:
        """``forward_logits`` up to the LM head: the final RMSNorm's output
        ``(n_sample, hidden)`` for the sampled rows (schedule order), or None
        when no sequence samples."""
        cfg, ecfg = self.cfg, self.ecfg
        err = self.error_word
        Hq, Hkv, D = cfg.num_heads, cfg.num_kv_heads, cfg.head_dim
        sched = self.sched[:4 * S]
        K.pack_batch(sched, S, T, self.req_tokens, self.block_tables, self.req_nblk,
                     self.free_stack, self.free_top, self.input_ids, self.positions,
                     self.slot_mapping, self.cu_q, self.seq_lens_k, self.sample_rows,
                     self.sample_seq, err)
        cu_q, kv_lens, slots = self.cu_q[:S + 1], self.seq_lens_k[:S], sched[:S]
        launches = 1
        if self.ws is not None:
            K.attention_plan(cu_q, kv_lens, S, Hkv, ecfg.max_num_seqs, ecfg.max_batched_tokens,
                             self.ws, err)
            launches += 1
        pos, smap = self.positions[:T], self.slot_mapping[:T]
        q, attn = self.q_buf[:T], self.attn_buf[:T]
        s_o = self.splitk_parts(T, Hq * D)
        s_d = self.splitk_parts(T, cfg.intermediate_size)
        x = F.embedding(self.input_ids[:T], self.embed)
        eps = cfg.rms_norm_eps
        h = K.add_rms_norm(x, self.layers[0].ln1, eps)
        launches += 1
        nl = len(self.layers)
        gathered = n_sample < T             # the last layer's tail runs on the sampled rows
        for l, w in enumerate(self.layers):
            last = l == nl - 1
            qkv = F.linear(h, w.w_qkv)
            K.qk_norm_rope(qkv, Hq, Hkv, pos, w.q_norm, w.k_norm, self.rope_cos, self.rope_sin,
                           eps, q_out=q, kv_cache_layer=self.kv_cache[l], slot_mapping=smap,
                           num_blocks=self.num_blocks, err=err)
            launches += 1
            if last and n_sample == 0:
                break                       # K/V appended; nothing samples this step
            # from the second layer on, the plan, the block tables and the item id
            # cache are at least two launches old: decode loads may start early
            K.varlen_attention(q, attn, self.kv_cache, l, self.block_tables, cu_q, kv_lens, S,
                               ecfg.max_num_seqs, ecfg.max_batched_tokens, self.ws,
                               seq_bt_row=slots, err=err, early=l > 0)
            launches += 1
            a2 = attn.view(T, Hq * D)
            nxt = self.final_norm if last else self.layers[l + 1].ln1
            if last and gathered:
                rows = self.sample_rows[:n_sample]
                a_s = a2.index_select(0, rows)
                xs = torch.empty(n_sample, cfg.hidden_size, dtype=self.dtype, device=self.device)
                so = self.splitk_parts(n_sample, Hq * D)
                if so > 1:
                    h = K.gather_add_rms_norm(x, rows, w.ln2, eps, parts=linear_splitk(a_s, w.w_o, so),
                                              x_out=xs, err=err)
                else:
                    h = K.gather_add_rms_norm(x, rows, w.ln2, eps, delta=F.linear(a_s, w.w_o),
                                              x_out=xs, err=err)
                act = K.silu_mul(F.linear(h, w.w_gate_up))
                sd = self.splitk_parts(n_sample, cfg.intermediate_size)
                if sd > 1:
                    h = K.add_rms_norm_splitk(xs, nxt, eps, linear_splitk(act, w.w_down, sd))
                else:
                    h = K.add_rms_norm(xs, nxt, eps, delta=F.linear(act, w.w_down))
                launches += 3
                break
            # x += o_proj(attn); h = post_attention_layernorm(x)
            if s_o > 1:
                h = K.add_rms_norm_splitk(x, w.ln2, eps, linear_splitk(a2, w.w_o, s_o))
            else:
                h = K.add_rms_norm(x, w.ln2, eps, delta=F.linear(a2, w.w_o))
            act = K.silu_mul(F.linear(h, w.w_gate_up))
            # x += mlp(h); h = next block's input_layernorm(x), or the final norm
            if s_d > 1:
                h = K.add_rms_norm_splitk(x, nxt, eps, linear_splitk(act, w.w_down, s_d))
            else:
                h = K.add_rms_norm(x, nxt, eps, delta=F.linear(act, w.w_down))
            launches += 3
        self.kernel_launches += launches
        if n_sample == 0:
            return None
        # decode steps sample every row, in order: h holds exactly those rows
        return h

    def commit_next_tokens(self, tokens: torch.Tensor, S: int, n_sample: int) -> None:
        """Append ``tokens`` (int32, one per sampled sequence, schedule order) to
        their requests' token rows: the step after ``forward_logits`` feeds them."""
        toks = self.next_tokens[:n_sample]
        toks.copy_(tokens.reshape(-1))
        K.commit_tokens(toks, n_sample, self.sample_seq, self.sched[:4 * S], S, self.req_tokens,
                        self.error_word)
        self.kernel_launches += 1

    def free_slots(self, slots: torch.Tensor, first_block: Optional[torch.Tensor] = None) -> None:
        K.free_blocks(slots, self.block_tables, self.req_nblk, self.free_stack, self.free_top,
                      self.error_word, first_block=first_block)
        self.kernel_launches += 1

    def push_blocks(self, block_ids: torch.Tensor) -> None:
        K.push_blocks(block_ids, self.free_stack, self.free_top, self.error_word)
        self.kernel_launches += 1

    def splitk_parts(self, T: int, k: int) -> int:
        """K slices for a projection of T rows and inner size k: decode-sized bf16
        steps run the o and down projections as a batched GEMM over K slices with
        fp32 partials, which the add+RMSNorm kernel sums (cuBLAS gives a GEMM of
        16 rows and K = 4096 or 9728 too few CTAs to fill the GPU: measured at
        16 rows, 8 slices take o_proj 8.6 -> 6.2 us and down_proj 15.1 -> 10.4
        us; at 64 rows 4 slices are best).  fp32 steps keep one GEMM, so their
        sums keep cuBLAS's order.  HY_SPLITK=0 turns the split off."""
        if self.dtype != torch.bfloat16 or not _SPLITK_ON:
            return 1
        for s, t_max in ((8, 32), (4, 128)):
            if T <= t_max and k % (8 * s) == 0:
                return s
        return 1

    def launches_per_step(self, n_sample: bool = True) -> int:
        """Kernels of this library one decode step (every row sampled) launches:
        pack, plan, the first RMSNorm, per layer QK-norm+RoPE, attention, two
        add+RMSNorm and SiLU*up, then the argmax (fused with the LM head in
        bf16) and commit."""
        per_layer = 5
        return 2 + (self.ws is not None) + per_layer * len(self.layers) + (2 if n_sample else 0)
