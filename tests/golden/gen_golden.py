"""Generate the parity fixtures under tests/golden/ by running the reference.

This script is the only committed code that imports the reference
(``hayate`` from the reference checkout, default ``/root/reference``); it runs in
the development container, never on the GPU machine.  It writes:

* ``tiny_engine.json``   -- greedy tokens (+ top-2 logit margins) from the
  reference ``Engine`` (``hayate/engine/engine.py``) driving a two-layer model
  with the Qwen3-4B head geometry, fp32, for several request scenarios;
* ``tiny_forward.npz``   -- inputs and outputs of the reference
  ``Qwen3Model.forward`` (``hayate/model/qwen.py:46-124``) for the first padded
  prefill call and the first decode call of one scenario;
* ``qk_norm_rope.npz``   -- the reference QK-RMSNorm (``attention.py:23-24,40-41``)
  and RoPE (``rope.py:3-13,31-44``) on seeded inputs, bf16 and fp32;
* ``full_greedy.json``   -- greedy tokens and margins of the full-size model
  (fp32, seeded random init) for the single-request case and the first 64
  tokens of the 10-request upfront case, plus a weight fingerprint;
* ``hayate_b200/data/rng_ckpt_*.npz`` -- generator checkpoints for the exact
  block-parallel weight fill.

Usage: ``python tests/golden/gen_golden.py [--part tiny|full|all] [--ref PATH]``
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from queue import Queue

import numpy as np
import torch
import torch.nn as nn

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from hayate_b200.config import QWEN3_4B, TINY, ModelConfig  # noqa: E402
from hayate_b200 import weights as W  # noqa: E402
from hayate_b200 import workloads  # noqa: E402


# Init scale of the two-layer model: with 0.02 its greedy output repeats one token
# (the tied embedding dominates the residual stream); 0.15 gives varied tokens.
TINY_STD = 0.15


class FakeTokenizer:
    """Identity tokenizer: prompts are token-id lists."""
    eos_token_id = None
    pad_token_id = 0

    def encode(self, prompt):
        return list(prompt)

    def decode(self, tokens, skip_special_tokens=True):
        return " ".join(str(t) for t in tokens)


def build_ref_model(ref, cfg: ModelConfig, w: W.HostWeights, dtype):
    """Reference Qwen3Model with the seeded weights (constructor init skipped)."""
    Qwen3Model = ref["Qwen3Model"]
    TransformerBlock = ref["TransformerBlock"]
    m = Qwen3Model.__new__(Qwen3Model)
    nn.Module.__init__(m)
    m.num_layers, m.num_kv_groups, m.head_dim = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
    with torch.device("meta"):
        m.embed_tokens = nn.Embedding(cfg.vocab_size, cfg.hidden_size, dtype=torch.bfloat16)
        m.layers = nn.ModuleList([
            TransformerBlock(hidden_size=cfg.hidden_size, num_heads=cfg.num_heads,
                             num_kv_groups=cfg.num_kv_heads, head_dim=cfg.head_dim,
                             intermediate_size=cfg.intermediate_size,
                             rms_norm_eps=cfg.rms_norm_eps)
            for _ in range(cfg.num_layers)])
        m.norm = nn.RMSNorm(cfg.hidden_size, eps=cfg.rms_norm_eps, dtype=torch.bfloat16)
        m.out_head = nn.Linear(cfg.hidden_size, cfg.vocab_size, bias=False, dtype=torch.bfloat16)
    m.to_empty(device="cpu")
    cos, sin = ref["compute_rope_params"](head_dim=cfg.head_dim, theta_base=int(cfg.rope_theta),
                                          context_length=cfg.max_position_embeddings)
    m.register_buffer("cos", cos, persistent=False)
    m.register_buffer("sin", sin, persistent=False)
    with torch.no_grad():
        m.embed_tokens.weight.copy_(w.embed)
        for l, blk in enumerate(m.layers):
            src = w.layers[l]
            a = blk.self_attn
            for k in ("q_proj", "k_proj", "v_proj", "o_proj"):
                getattr(a, k).weight.copy_(src[k])
            for k in ("gate_proj", "up_proj", "down_proj"):
                getattr(blk.mlp, k).weight.copy_(src[k])
            for norm in (a.q_norm, a.k_norm, blk.input_layernorm, blk.post_attention_layernorm):
                norm.weight.fill_(1.0)
        m.norm.weight.fill_(1.0)
    m.out_head.weight = m.embed_tokens.weight   # utils.py:98-99
    if dtype == torch.float32:
        m.float()
    m.eval()
    return m


def build_ref_engine(ref, model):
    Engine = ref["Engine"]
    eng = Engine.__new__(Engine)
    eng.model = model
    eng.num_layers = model.num_layers
    eng.num_kv_groups = model.num_kv_groups
    eng.head_dim = model.head_dim
    eng.tokenizer = FakeTokenizer()
    eng.pool = Queue()
    eng.current_batch = []
    eng.request_id = 0
    margins = {}
    orig = eng._forward_pass

    def forward_pass(tokens, requests, pad_lengths_py=None):
        out = orig(tokens, requests, pad_lengths_py=pad_lengths_py)
        top2 = out.float().topk(2, dim=-1).values
        for r, mg in zip(requests, (top2[:, 0] - top2[:, 1]).tolist()):
            margins.setdefault(r.id, []).append(mg)
        return out

    eng._forward_pass = forward_pass
    eng._margins = margins
    return eng


def run_upfront(ref, eng, prompts, max_tokens):
    reqs = eng.generate_text([list(p) for p in prompts], max_tokens=max_tokens)
    if not isinstance(reqs, list):
        reqs = [reqs]
    return [{"prompt": list(p), "max_tokens": max_tokens, "tokens": list(r.tokens),
             "margins": eng._margins[r.id]} for p, r in zip(prompts, reqs)]


def run_staggered(ref, eng, arrivals):
    """arrivals: list of (step, prompt, max_tokens); requests join at that engine step."""
    Request = ref["Request"]
    pending = sorted(arrivals, key=lambda a: a[0])
    live = []
    step = 0
    while pending or eng.current_batch or not eng.pool.empty():
        while pending and pending[0][0] <= step:
            _, prompt, mt = pending.pop(0)
            r = Request(id=eng.request_id, prompt=list(prompt), max_tokens=mt)
            eng.request_id += 1
            eng.add_request(r)
            live.append((r, prompt, mt, step))
        eng.generate()
        step += 1
    return [{"prompt": list(p), "max_tokens": mt, "arrival_step": s, "tokens": list(r.tokens),
             "margins": eng._margins[r.id]} for r, p, mt, s in live]


def tiny_scenarios(cfg: ModelConfig):
    g = torch.Generator().manual_seed(1234)
    rnd = lambda n: torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist()  # noqa: E731
    sc = {}
    sc["single"] = {"kind": "upfront", "max_tokens": 16, "prompts": [rnd(20)]}
    sc["batch5"] = {"kind": "upfront", "max_tokens": 24,
                    "prompts": [rnd(n) for n in (3, 17, 40, 64, 33)]}
    sc["long_prompt"] = {"kind": "upfront", "max_tokens": 12, "prompts": [rnd(700), rnd(5)]}
    sc["max_tokens_one"] = {"kind": "upfront", "max_tokens": 1, "prompts": [rnd(9), rnd(1)]}
    rng = np.random.default_rng(7)
    arr = []
    for i in range(25):           # more than MAX_BATCH_SIZE=20 live at once
        arr.append((int(i // 3), rnd(int(rng.integers(1, 90))), int(rng.integers(1, 30))))
    sc["staggered25"] = {"kind": "staggered", "arrivals": arr}
    return sc


def gen_tiny(ref):
    cfg = TINY
    w = W.sequential_seeded(cfg, 0, std=TINY_STD)
    out = {"config": cfg.__dict__, "seed": 0, "std": TINY_STD, "scenarios": {}}
    for name, sc in tiny_scenarios(cfg).items():
        model = build_ref_model(ref, cfg, w, torch.float32)
        eng = build_ref_engine(ref, model)
        t0 = time.time()
        if sc["kind"] == "upfront":
            res = run_upfront(ref, eng, sc["prompts"], sc["max_tokens"])
        else:
            res = run_staggered(ref, eng, sc["arrivals"])
        out["scenarios"][name] = {"kind": sc["kind"], "requests": res}
        print(f"tiny {name}: {len(res)} requests in {time.time() - t0:.1f}s", flush=True)
    with open(os.path.join(HERE, "tiny_engine.json"), "w") as f:
        json.dump(out, f)

    # Forward-call fixture: record the first prefill and first decode call.
    model = build_ref_model(ref, cfg, w, torch.float32)
    calls = []
    orig_forward = model.forward

    def rec(token_ids, prev_k=None, prev_v=None, cache_lens=None, pad_lengths=None):
        res = orig_forward(token_ids, prev_k=prev_k, prev_v=prev_v, cache_lens=cache_lens,
                           pad_lengths=pad_lengths)
        if len(calls) < 2:
            calls.append(dict(token_ids=token_ids.clone(), prev_k=prev_k, prev_v=prev_v,
                              cache_lens=cache_lens, pad_lengths=pad_lengths,
                              logits=res[0].clone(), new_k=res[1].clone(), new_v=res[2].clone()))
        return res

    model.forward = rec
    eng = build_ref_engine(ref, model)
    prompts = [p[:n] for p, n in zip(tiny_scenarios(cfg)["batch5"]["prompts"], (3, 9, 12))]
    eng.generate_text(prompts, max_tokens=3)
    arrays = {}
    for i, c in enumerate(calls):
        for k, v in c.items():
            if v is not None:
                arrays[f"c{i}_{k}"] = v.numpy()
    arrays["prompts_flat"] = np.concatenate([np.array(p) for p in prompts])
    arrays["prompt_lens"] = np.array([len(p) for p in prompts])
    np.savez_compressed(os.path.join(HERE, "tiny_forward.npz"), **arrays)
    print("tiny forward fixture:", sorted(arrays), flush=True)


def gen_qk_norm_rope(ref):
    cfg = QWEN3_4B
    g = torch.Generator().manual_seed(99)
    T = 12
    cos, sin = ref["compute_rope_params"](head_dim=128, theta_base=int(cfg.rope_theta),
                                          context_length=cfg.max_position_embeddings)
    pos = torch.randint(0, cfg.max_position_embeddings, (T,), generator=g)
    pos[0], pos[1] = 0, cfg.max_position_embeddings - 1
    arrays = {"positions": pos.numpy(), "cos_rows": cos[pos].numpy(), "sin_rows": sin[pos].numpy()}
    for dt, tag in ((torch.bfloat16, "bf16"), (torch.float32, "fp32")):
        q = (torch.randn(T, cfg.num_heads, 128, generator=g) * 3.0).to(dt)
        k = (torch.randn(T, cfg.num_kv_heads, 128, generator=g) * 0.5).to(dt)
        wq = (1.0 + 0.1 * torch.randn(128, generator=g)).to(dt)
        wk = (1.0 + 0.1 * torch.randn(128, generator=g)).to(dt)
        qn = nn.RMSNorm(128, eps=cfg.rms_norm_eps, dtype=dt)
        kn = nn.RMSNorm(128, eps=cfg.rms_norm_eps, dtype=dt)
        with torch.no_grad():
            qn.weight.copy_(wq)
            kn.weight.copy_(wk)
            qo = ref["apply_rope_vectorized"](qn(q[None]).transpose(1, 2), cos, sin, pos[None])
            ko = ref["apply_rope_vectorized"](kn(k[None]).transpose(1, 2), cos, sin, pos[None])
        qo = qo[0].transpose(0, 1).contiguous()
        ko = ko[0].transpose(0, 1).contiguous()

        def npy(t):
            return t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
        arrays.update({f"{tag}_q": npy(q), f"{tag}_k": npy(k), f"{tag}_wq": npy(wq),
                       f"{tag}_wk": npy(wk), f"{tag}_q_out": npy(qo), f"{tag}_k_out": npy(ko)})
    np.savez_compressed(os.path.join(HERE, "qk_norm_rope.npz"), **arrays)
    print("qk_norm_rope fixture written", flush=True)


def gen_full(ref, c2_tokens: int):
    cfg = QWEN3_4B
    t0 = time.time()
    w, states = W.sequential_seeded(cfg, 0, record_states=True)
    print(f"full weights (sequential recipe) in {time.time() - t0:.0f}s", flush=True)
    W.save_checkpoints(cfg, 0, states)
    fp = W.fingerprint(w)
    model = build_ref_model(ref, cfg, w, torch.float32)
    del w
    out = {"config": cfg.__dict__, "seed": 0, "fingerprint": fp, "cases": {}}
    eng = build_ref_engine(ref, model)
    c1 = workloads.single(seed=0)
    t0 = time.time()
    out["cases"]["single"] = run_upfront(ref, eng, [r.prompt for r in c1], c1[0].max_tokens)
    print(f"single: {time.time() - t0:.1f}s", flush=True)
    eng = build_ref_engine(ref, model)
    c2 = workloads.upfront(seed=0)
    t0 = time.time()
    out["cases"]["upfront"] = run_upfront(ref, eng, [r.prompt for r in c2], c2_tokens)
    print(f"upfront ({c2_tokens} tokens): {time.time() - t0:.1f}s", flush=True)
    with open(os.path.join(HERE, "full_greedy.json"), "w") as f:
        json.dump(out, f)


def gen_tiny_ckpt():
    _, states = W.sequential_seeded(TINY, 0, record_states=True)
    W.save_checkpoints(TINY, 0, states)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--part", default="all", choices=["tiny", "full", "all"])
    ap.add_argument("--ref", default="/root/reference")
    ap.add_argument("--c2-tokens", type=int, default=64)
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.ref)
    from hayate.engine.engine import Engine, Request
    from hayate.model.qwen import Qwen3Model
    from hayate.model.block import TransformerBlock
    from hayate.model.rope import compute_rope_params, apply_rope_vectorized
    ref = dict(Engine=Engine, Request=Request, Qwen3Model=Qwen3Model,
               TransformerBlock=TransformerBlock, compute_rope_params=compute_rope_params,
               apply_rope_vectorized=apply_rope_vectorized)
    torch.set_num_threads(os.cpu_count() or 8)
    if args.part in ("tiny", "all"):
        gen_tiny(ref)
        gen_qk_norm_rope(ref)
        gen_tiny_ckpt()
    if args.part in ("full", "all"):
        gen_full(ref, args.c2_tokens)


if __name__ == "__main__":
    main()
