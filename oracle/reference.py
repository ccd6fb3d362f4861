"""The reference's continuous-batching path restated on the CPU (torch).

Test infrastructure only (see ``oracle/__init__.py``).  Each function cites the
reference file:line (axrshz/hayate) whose computation it restates; the same
torch operators are used in the same order, so on the CPU the results are
bit-identical to the reference's -- the fixtures in ``tests/golden`` (made by
running the reference) check exactly that.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

# engine.py:13-15
MAX_BATCH_SIZE = 20
MAX_PREFILL_BATCH = 8


# ----------------------------------------------------------------- RoPE + norms
def rope_tables(head_dim: int, theta: float, max_pos: int):
    """fp32 cos/sin tables of shape (max_pos, head_dim); rope.py:3-13.

    inv_freq = 1 / theta^(2i/d); angles = pos * inv_freq, duplicated to the full
    head dimension.
    """
    exps = torch.arange(0, head_dim, 2, dtype=torch.float32)[: head_dim // 2].float() / head_dim
    inv_freq = 1.0 / (int(theta) ** exps)
    pos = torch.arange(max_pos, dtype=torch.float32)
    ang = pos.unsqueeze(1) * inv_freq.unsqueeze(0)
    ang = torch.cat([ang, ang], dim=1)
    return torch.cos(ang), torch.sin(ang)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """nn.RMSNorm(dim, eps) forward (attention.py:23-24, block.py:18-19, qwen.py:35)."""
    return F.rms_norm(x, (x.shape[-1],), w, eps)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
         position_ids: torch.Tensor) -> torch.Tensor:
    """apply_rope_vectorized, rope.py:31-44.  x: (B, H, T, D); position_ids (B, T)."""
    half = x.shape[-1] // 2
    c = cos[position_ids].unsqueeze(1)
    s = sin[position_ids].unsqueeze(1)
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return ((x * c) + (rotated * s)).to(dtype=x.dtype)


def qk_norm_rope(q, k, wq, wk, cos, sin, positions, eps):
    """Per-token q (T, Hq, D) and k (T, Hkv, D): QK-RMSNorm then RoPE
    (attention.py:40-48).  Returns tensors of the same layout."""
    qn = rms_norm(q[None], wq, eps).transpose(1, 2)
    kn = rms_norm(k[None], wk, eps).transpose(1, 2)
    pos = positions[None].long()
    qo = rope(qn, cos, sin, pos)[0].transpose(0, 1).contiguous()
    ko = rope(kn, cos, sin, pos)[0].transpose(0, 1).contiguous()
    return qo, ko


# ----------------------------------------------------------- positions + mask
def positions_and_mask(B: int, T: int, L_prev: int, cache_lens: Optional[torch.Tensor],
                       pad_lengths: Optional[torch.Tensor], dtype: torch.dtype):
    """Position ids (B, T) and the additive mask (B, 1, T, L_prev+T); qwen.py:66-106.

    Masked: keys after the query (causal), cache columns past a request's valid
    length, and left-pad columns of the new region for real (non-pad) queries.
    """
    L_full = L_prev + T
    ar = torch.arange(T, dtype=torch.long).unsqueeze(0)
    cl = cache_lens.view(-1, 1) if cache_lens is not None else torch.zeros(B, 1, dtype=torch.long)
    if pad_lengths is not None:
        pos = (ar + cl - pad_lengths.view(-1, 1)).clamp(min=0)
    else:
        pos = ar + cl
    kp = torch.arange(L_full, dtype=torch.long).view(1, 1, -1)
    qc = (L_prev + ar).unsqueeze(-1)
    masked = kp > qc
    if L_prev > 0:
        masked = masked | ((kp < L_prev) & (kp >= cache_lens.view(-1, 1, 1)))
    if pad_lengths is not None:
        pl = pad_lengths.view(-1, 1, 1)
        real = ar.unsqueeze(-1) >= pl
        newpad = (kp >= L_prev) & ((kp - L_prev) < pl)
        masked = masked | (newpad & real)
    masked = masked.unsqueeze(1)
    return pos, torch.zeros_like(masked, dtype=dtype).masked_fill(masked, float("-inf"))


def sdpa_gqa(q, k, v, attn_mask):
    """The attention call of attention.py:58-64 (scale 1/sqrt(D), GQA broadcast)."""
    return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, dropout_p=0.0,
                                          is_causal=False, enable_gqa=True)


def varlen_attention(q: torch.Tensor, cu_q: List[int], ctx_k: List[torch.Tensor],
                     ctx_v: List[torch.Tensor]) -> torch.Tensor:
    """Attention of a packed ragged batch, one unpadded sequence at a time.

    q: (T, Hq, D) packed; ctx_k[i]/ctx_v[i]: (L_i, Hkv, D), the sequence's whole
    context with its new tokens last.  This is the reference's mask for a single
    request with a fully valid cache (qwen.py:89-91: key j visible to query row r
    iff j <= L_prev + r), computed by the same SDPA call in fp32.
    """
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    for i in range(len(ctx_k)):
        a, b = cu_q[i], cu_q[i + 1]
        T = b - a
        if T == 0:
            continue
        L = ctx_k[i].shape[0]
        L_prev = L - T
        qi = q[a:b].float().transpose(0, 1)[None]
        ki = ctx_k[i].float().transpose(0, 1)[None]
        vi = ctx_v[i].float().transpose(0, 1)[None]
        kp = torch.arange(L, device=q.device).view(1, -1)
        qc = (L_prev + torch.arange(T, device=q.device)).view(-1, 1)
        mask = torch.zeros(T, L, device=q.device).masked_fill(kp > qc, float("-inf"))
        out[a:b] = sdpa_gqa(qi, ki, vi, mask[None, None])[0].transpose(0, 1)
    return out


# -------------------------------------------------------------------- model
@dataclass
class RefWeights:
    """Module weights in the reference's layout (nn.Linear: out x in)."""
    embed: torch.Tensor
    layers: List[Dict[str, torch.Tensor]]
    cos: torch.Tensor
    sin: torch.Tensor
    eps: float
    num_heads: int
    num_kv_heads: int
    head_dim: int

    @staticmethod
    def from_host(hw, dtype=torch.float32) -> "RefWeights":
        cfg = hw.cfg
        cos, sin = rope_tables(cfg.head_dim, cfg.rope_theta, cfg.max_position_embeddings)
        layers = []
        for l, blk in enumerate(hw.layers):
            d = {k: v.to(dtype) for k, v in blk.items()}
            for n in ("input_layernorm", "post_attention_layernorm"):
                d[n] = hw.norms[f"layers.{l}.{n}.weight"].to(dtype)
            for n in ("q_norm", "k_norm"):
                d[n] = hw.norms[f"layers.{l}.self_attn.{n}.weight"].to(dtype)
            layers.append(d)
        return RefWeights(hw.embed.to(dtype), layers, cos, sin, cfg.rms_norm_eps,
                          cfg.num_heads, cfg.num_kv_heads, cfg.head_dim)

    @property
    def norm(self) -> torch.Tensor:
        return torch.ones(self.embed.shape[1], dtype=self.embed.dtype)


def forward(W: RefWeights, token_ids, prev_k=None, prev_v=None, cache_lens=None,
            pad_lengths=None):
    """Qwen3Model.forward, qwen.py:46-124 (block.py:21-31, attention.py:26-66,
    linear.py:11-14).  Returns (logits (B,T,V), new_k, new_v)."""
    B, T = token_ids.shape
    dt = W.embed.dtype
    x = F.embedding(token_ids, W.embed)
    L_prev = prev_k.shape[3] if prev_k is not None else 0
    pos, mask = positions_and_mask(B, T, L_prev, cache_lens, pad_lengths, dt)
    Hq, Hkv, D = W.num_heads, W.num_kv_heads, W.head_dim
    nks, nvs = [], []
    for l, p in enumerate(W.layers):
        sc = x
        h = rms_norm(x, p["input_layernorm"], W.eps)
        q = F.linear(h, p["q_proj"]).view(B, T, Hq, D)
        k = F.linear(h, p["k_proj"]).view(B, T, Hkv, D)
        v = F.linear(h, p["v_proj"]).view(B, T, Hkv, D)
        q = rms_norm(q, p["q_norm"], W.eps).transpose(1, 2)
        k = rms_norm(k, p["k_norm"], W.eps).transpose(1, 2)
        v = v.transpose(1, 2)
        q = rope(q, W.cos, W.sin, pos)
        k = rope(k, W.cos, W.sin, pos)
        if prev_k is not None:
            k = torch.cat([prev_k[l], k], dim=2)
            v = torch.cat([prev_v[l], v], dim=2)
        ctx = sdpa_gqa(q, k, v, mask).transpose(1, 2).reshape(B, T, Hq * D)
        x = F.linear(ctx, p["o_proj"]) + sc
        sc = x
        h = rms_norm(x, p["post_attention_layernorm"], W.eps)
        x = F.linear(F.silu(F.linear(h, p["gate_proj"])) * F.linear(h, p["up_proj"]),
                     p["down_proj"]) + sc
        nks.append(k)
        nvs.append(v)
    x = rms_norm(x, W.norm, W.eps)
    return F.linear(x, W.embed), torch.stack(nks, 0), torch.stack(nvs, 0)


# ------------------------------------------------------------------- engine
@dataclass
class RefRequest:
    """Request state of engine.py:17-32 (the cache held as two tensors)."""
    id: int
    prompt: List[int]
    max_tokens: int
    tokens: List[int] = field(default_factory=list)
    k: Optional[torch.Tensor] = None          # (layers, Hkv, L, D)
    v: Optional[torch.Tensor] = None
    cache_pos: int = 0
    is_completed: bool = False
    is_prefill: bool = True
    margins: List[float] = field(default_factory=list)


class RefEngine:
    """The reference scheduler and step loop (engine.py:63-234) over ``forward``.

    FIFO admission up to MAX_BATCH_SIZE live requests; each step runs the
    not-yet-prefilled requests in padded groups of MAX_PREFILL_BATCH, then one
    decode forward over the requests that were prefilled in earlier steps.
    """

    def __init__(self, W: RefWeights, eos_token_id: Optional[int] = None, pad_id: int = 0,
                 record_margins: bool = False):
        self.W = W
        self.eos = eos_token_id
        self.pad = pad_id
        self.pool: List[RefRequest] = []
        self.current_batch: List[RefRequest] = []
        self.request_id = 0
        self.record_margins = record_margins

    def add(self, prompt: List[int], max_tokens: int) -> RefRequest:
        r = RefRequest(self.request_id, list(prompt), max_tokens)
        self.request_id += 1
        self.pool.append(r)
        return r

    def _finalize(self, r: RefRequest, tok: int):          # engine.py:73-78
        r.tokens.append(tok)
        if tok == self.eos or len(r.tokens) >= r.max_tokens:
            r.is_completed = True

    def _gather(self, reqs):                               # engine.py:80-116
        lens = [0 if r.k is None else r.k.shape[2] for r in reqs]
        ref = next((r.k for r in reqs if r.k is not None), None)
        if ref is None:
            return None, None, None
        nl, hkv, _, d = ref.shape
        Lm = max(lens)
        pk = torch.zeros(nl, len(reqs), hkv, Lm, d, dtype=ref.dtype)
        pv = torch.zeros_like(pk)
        for i, r in enumerate(reqs):
            if lens[i] > 0:
                pk[:, i, :, :lens[i]] = r.k
                pv[:, i, :, :lens[i]] = r.v
        return pk, pv, torch.tensor(lens, dtype=torch.long)

    def _scatter(self, reqs, nk, nv, L_prev, T, pads):     # engine.py:118-141
        for i, r in enumerate(reqs):
            pl = pads[i] if pads is not None else 0
            r.k = torch.cat([nk[:, i, :, :r.cache_pos], nk[:, i, :, L_prev + pl:L_prev + T]], 2)
            r.v = torch.cat([nv[:, i, :, :r.cache_pos], nv[:, i, :, L_prev + pl:L_prev + T]], 2)

    def _forward(self, tokens, reqs, pads=None):           # engine.py:143-163
        pk, pv, cl = self._gather(reqs)
        L_prev = pk.shape[3] if pk is not None else 0
        pl = torch.tensor(pads, dtype=torch.long) if pads is not None else None
        with torch.no_grad():
            logits, nk, nv = forward(self.W, tokens, pk, pv, cl, pl)
        self._scatter(reqs, nk, nv, L_prev, tokens.shape[1], pads)
        last = logits[:, -1, :]
        if self.record_margins:
            top2 = last.float().topk(2, dim=-1).values
            for r, m in zip(reqs, (top2[:, 0] - top2[:, 1]).tolist()):
                r.margins.append(m)
        return last

    def _prefill(self, reqs):                              # engine.py:165-182
        n = max(len(r.prompt) for r in reqs)
        pads = [n - len(r.prompt) for r in reqs]
        tokens = torch.tensor([[self.pad] * p + r.prompt for p, r in zip(pads, reqs)])
        nxt = torch.argmax(self._forward(tokens, reqs, pads), dim=-1)
        for i, r in enumerate(reqs):
            self._finalize(r, int(nxt[i]))
            r.cache_pos = len(r.prompt)
            r.is_prefill = False

    def _decode(self, reqs):                               # engine.py:184-194
        tokens = torch.tensor([[r.tokens[-1]] for r in reqs])
        nxt = torch.argmax(self._forward(tokens, reqs), dim=-1)
        for i, r in enumerate(reqs):
            r.cache_pos += 1
            self._finalize(r, int(nxt[i]))

    def step(self) -> bool:                                # engine.py:196-217
        self.current_batch = [r for r in self.current_batch if not r.is_completed]
        while self.pool and len(self.current_batch) < MAX_BATCH_SIZE:
            self.current_batch.append(self.pool.pop(0))
        if not self.current_batch:
            return False
        pre = [r for r in self.current_batch if r.is_prefill]
        dec = [r for r in self.current_batch if not r.is_prefill]
        for i in range(0, len(pre), MAX_PREFILL_BATCH):
            self._prefill(pre[i:i + MAX_PREFILL_BATCH])
        if dec:
            self._decode(dec)
        return True

    def run(self, prompts: List[List[int]], max_tokens: int) -> List[RefRequest]:
        reqs = [self.add(p, max_tokens) for p in prompts]   # engine.py:219-234
        while self.step():
            pass
        return reqs
