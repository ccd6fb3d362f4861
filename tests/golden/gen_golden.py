"""Generate the parity fixtures under tests/golden/ by running the reference.

This script is the only committed code that imports the reference
(``hayate`` from a reference checkout named by ``--ref``); it runs where that
checkout exists, never on the GPU machine.  It writes:

* ``tiny_engine.json``   -- greedy tokens (+ top-2 logit margins) from the
  reference ``Engine`` (``hayate/engine/engine.py``) driving a two-layer model
  with the Qwen3-4B head geometry, fp32, for several request scenarios;
* ``tiny_forward.npz``   -- inputs and outputs of the reference
  ``Qwen3Model.forward`` (``hayate/model/qwen.py:46-124``) for the first padded
  prefill call and the first decode call of one scenario;
* ``qk_norm_rope.npz``   -- the reference QK-RMSNorm (``attention.py:23-24,40-41``)
  and RoPE (``rope.py:3-13,31-44``) on seeded inputs, bf16 and fp32;
* ``tiny_eos.json``      -- the same two-layer model with the tokenizer's
  ``eos_token_id`` set to a token the reference emits mid-sequence, so that
  requests stop early (engine.py:76-77);
* ``tiny_paged_pin.npz`` -- what the paged spec is pinned to: the position ids
  each forward call of the reference passes to its blocks (qwen.py:66-77,
  recorded at the first block) with the call's token ids, and every request's
  compacted cache after its last step (engine.py:118-141; layer 0, the first
  4 of 128 dimensions, K and V);
* ``full_greedy.json``   -- greedy tokens and margins of the full-size model
  (fp32, seeded random init) for the single-request case and the first 64
  tokens of the 10-request upfront case, plus a weight fingerprint;
* ``full_chunked.json``  -- the same for the first 6 requests of the Poisson
  workload (prompts of 1330, 1861, 1125, 345, 280 and 256 tokens, three of
  them longer than one 512-token prefill chunk), 32 tokens each;
* ``hayate_b200/data/rng_ckpt_*.npz`` -- generator checkpoints for the exact
  block-parallel weight fill.

Usage: ``python tests/golden/gen_golden.py --ref PATH [--part tiny|eos|paged|full|chunked|all]``
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
    pad_token_id = 0

    def __init__(self, eos_token_id=None):
        self.eos_token_id = eos_token_id

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


def build_ref_engine(ref, model, eos_token_id=None):
    Engine = ref["Engine"]
    eng = Engine.__new__(Engine)
    eng.model = model
    eng.num_layers = model.num_layers
    eng.num_kv_groups = model.num_kv_groups
    eng.head_dim = model.head_dim
    eng.tokenizer = FakeTokenizer(eos_token_id)
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


# eos ids chosen from the reference's own greedy output without eos (batch5:
# 462 ends two requests at tokens 3 and 8, 254 two at tokens 10 and 18;
# staggered25: 349 recurs in several requests)
EOS_CASES = (("batch5_eos462", "batch5", 462), ("batch5_eos254", "batch5", 254),
             ("staggered25_eos349", "staggered25", 349))


def gen_eos(ref):
    cfg = TINY
    w = W.sequential_seeded(cfg, 0, std=TINY_STD)
    scen = tiny_scenarios(cfg)
    out = {"config": cfg.__dict__, "seed": 0, "std": TINY_STD, "scenarios": {}}
    for name, base, eos in EOS_CASES:
        sc = scen[base]
        eng = build_ref_engine(ref, build_ref_model(ref, cfg, w, torch.float32), eos_token_id=eos)
        if sc["kind"] == "upfront":
            res = run_upfront(ref, eng, sc["prompts"], sc["max_tokens"])
        else:
            res = run_staggered(ref, eng, sc["arrivals"])
        early = sum(1 for r in res if len(r["tokens"]) < r["max_tokens"])
        assert early > 0, f"{name}: eos {eos} stops no request early"
        out["scenarios"][name] = {"kind": sc["kind"], "eos_token_id": eos, "requests": res}
        print(f"eos {name}: {early} of {len(res)} requests stop at eos", flush=True)
    with open(os.path.join(HERE, "tiny_eos.json"), "w") as f:
        json.dump(out, f)


PIN_DIMS = 4           # leading head dimensions kept of each cached K/V row


def gen_paged_pin(ref):
    """Record the reference's position ids per forward call and its compacted
    per-request caches after the run (two-layer model, fp32), for the
    scenarios that mix padded prefill groups, decodes and a 700-token prompt."""
    cfg = TINY
    w = W.sequential_seeded(cfg, 0, std=TINY_STD)
    scen = tiny_scenarios(cfg)
    arrays = {}
    for name in ("batch5", "long_prompt", "staggered25"):
        sc = scen[name]
        model = build_ref_model(ref, cfg, w, torch.float32)
        calls = []
        blk0 = model.layers[0]
        orig_blk = blk0.forward

        def blk_forward(x, attn_mask, cos, sin, position_ids, prev_k, prev_v, _o=orig_blk):
            calls.append(position_ids.clone())
            return _o(x, attn_mask, cos, sin, position_ids, prev_k, prev_v)

        blk0.forward = blk_forward
        eng = build_ref_engine(ref, model)
        toks = []                                  # the token ids of each call, by request
        orig_fp = eng._forward_pass

        def fp(tokens, requests, pad_lengths_py=None, _o=orig_fp):
            toks.append((tokens.clone(), [r.id for r in requests],
                         list(pad_lengths_py) if pad_lengths_py is not None else None,
                         [r.cache_pos for r in requests]))
            return _o(tokens, requests, pad_lengths_py=pad_lengths_py)

        eng._forward_pass = fp
        Request = ref["Request"]
        if sc["kind"] == "upfront":
            reqs = []
            for p in sc["prompts"]:
                r = Request(id=eng.request_id, prompt=list(p), max_tokens=sc["max_tokens"])
                eng.request_id += 1
                eng.add_request(r)
                reqs.append(r)
            while eng.generate():
                pass
        else:
            reqs = []
            pending = sorted(sc["arrivals"], key=lambda a: a[0])
            step = 0
            while pending or eng.current_batch or not eng.pool.empty():
                while pending and pending[0][0] <= step:
                    _, prompt, mt = pending.pop(0)
                    r = Request(id=eng.request_id, prompt=list(prompt), max_tokens=mt)
                    eng.request_id += 1
                    eng.add_request(r)
                    reqs.append(r)
                eng.generate()
                step += 1
        assert len(calls) == len(toks)
        for i, (pos, (tk, ids, pads, cpos)) in enumerate(zip(calls, toks)):
            arrays[f"{name}_call{i}_positions"] = pos.numpy()
            arrays[f"{name}_call{i}_tokens"] = tk.numpy()
            arrays[f"{name}_call{i}_ids"] = np.array(ids)
            arrays[f"{name}_call{i}_pads"] = np.array(pads if pads is not None else [0] * len(ids))
            arrays[f"{name}_call{i}_cache_pos"] = np.array(cpos)
        arrays[f"{name}_ncalls"] = np.array(len(calls))
        for r in reqs:
            arrays[f"{name}_req{r.id}_prompt"] = np.array(r.prompt)
            arrays[f"{name}_req{r.id}_tokens"] = np.array(r.tokens)
            arrays[f"{name}_req{r.id}_k"] = r.kv_cache.k[0, :, :, :PIN_DIMS].numpy()
            arrays[f"{name}_req{r.id}_v"] = r.kv_cache.v[0, :, :, :PIN_DIMS].numpy()
        arrays[f"{name}_nreq"] = np.array(len(reqs))
        print(f"paged pin {name}: {len(calls)} forward calls, {len(reqs)} requests", flush=True)
    np.savez_compressed(os.path.join(HERE, "tiny_paged_pin.npz"), **arrays)


def gen_chunked(ref, n_req: int = 6, ntok: int = 32):
    """Full-size model, fp32: the first requests of the Poisson workload, whose
    long prompts the engine splits into 512-token chunks."""
    cfg = QWEN3_4B
    t0 = time.time()
    w = W.exact_seeded(cfg, 0)
    with open(os.path.join(HERE, "full_greedy.json")) as f:
        fp_want = json.load(f)["fingerprint"]
    assert W.fingerprint(w) == fp_want, "weights differ from the full_greedy fixture's"
    print(f"full weights in {time.time() - t0:.0f}s", flush=True)
    model = build_ref_model(ref, cfg, w, torch.float32)
    del w
    eng = build_ref_engine(ref, model)
    ws = workloads.poisson(seed=0)[:n_req]
    t0 = time.time()
    res = run_upfront(ref, eng, [r.prompt for r in ws], ntok)
    print(f"chunked slice: {time.time() - t0:.1f}s", flush=True)
    out = {"config": cfg.__dict__, "seed": 0, "fingerprint": fp_want,
           "workload": f"poisson(seed=0)[:{n_req}], {ntok} tokens each, submitted upfront",
           "requests": res}
    with open(os.path.join(HERE, "full_chunked.json"), "w") as f:
        json.dump(out, f)


PARTS = ("tiny", "eos", "paged", "full", "chunked")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--part", default="all", choices=list(PARTS) + ["all"])
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
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
    parts = PARTS if args.part == "all" else (args.part,)
    if "tiny" in parts:
        gen_tiny(ref)
        gen_qk_norm_rope(ref)
        gen_tiny_ckpt()
    if "eos" in parts:
        gen_eos(ref)
    if "paged" in parts:
        gen_paged_pin(ref)
    if "full" in parts:
        gen_full(ref, args.c2_tokens)
    if "chunked" in parts:
        gen_chunked(ref)


if __name__ == "__main__":
    main()
