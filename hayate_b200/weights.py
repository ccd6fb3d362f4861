"""Random-init weights for the Qwen3 architecture.

No checkpoint or network exists offline, so weights are drawn N(0, 0.02).  The
seeded recipe is:

1. the parameters are enumerated in the reference module's ``named_parameters``
   order (``hayate/model/qwen.py:27-37`` builds embed, 36 blocks, norm, head;
   ``block.py:10-19`` and ``attention.py:18-24`` order each block);
2. ``torch.manual_seed(seed)`` on the CPU generator, then every parameter whose
   name does not contain ``"norm"`` gets ``normal_(0, 0.02)`` in bf16, in order;
   norm weights stay 1.0 (``nn.RMSNorm`` default);
3. the output head is tied to the embedding (``hayate/utils.py:98-99``); its own
   draw comes last, so skipping it leaves every other draw unchanged.

The draw count does not depend on the standard deviation, so the generator
checkpoints below serve any ``std``; the two-layer test model uses 0.15 so that
its greedy output is not a repeated token.

Step 2 is sequential on one CPU generator (about 150 s for 4B parameters).
:func:`exact_seeded` reproduces it bit for bit in parallel: ``rng_checkpoints``
holds the generator state at the start of the embedding and of each block, taken
from one sequential run, so each block is filled by its own generator on a
worker thread.  :func:`device_seeded` is the fast path for throughput runs: the
same shapes and distribution from a CUDA generator (seed 0), not bit-identical
to the CPU recipe.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .config import ModelConfig

_DATA = os.path.join(os.path.dirname(__file__), "data")


def layer_param_specs(cfg: ModelConfig) -> List[Tuple[str, Tuple[int, ...]]]:
    """(name, shape) of one block's matrices in reference order (norms omitted)."""
    h, i = cfg.hidden_size, cfg.intermediate_size
    return [
        ("q_proj", (cfg.q_size, h)),
        ("k_proj", (cfg.kv_size, h)),
        ("v_proj", (cfg.kv_size, h)),
        ("o_proj", (h, cfg.q_size)),
        ("gate_proj", (i, h)),
        ("up_proj", (i, h)),
        ("down_proj", (h, i)),
    ]


def reference_param_order(cfg: ModelConfig) -> List[Tuple[str, Tuple[int, ...]]]:
    """Every parameter name of the reference module tree, in registration order."""
    out = [("embed_tokens.weight", (cfg.vocab_size, cfg.hidden_size))]
    d = cfg.head_dim
    for l in range(cfg.num_layers):
        p = f"layers.{l}."
        specs = dict(layer_param_specs(cfg))
        out += [(p + "self_attn.q_proj.weight", specs["q_proj"]),
                (p + "self_attn.k_proj.weight", specs["k_proj"]),
                (p + "self_attn.v_proj.weight", specs["v_proj"]),
                (p + "self_attn.o_proj.weight", specs["o_proj"]),
                (p + "self_attn.q_norm.weight", (d,)),
                (p + "self_attn.k_norm.weight", (d,)),
                (p + "mlp.gate_proj.weight", specs["gate_proj"]),
                (p + "mlp.up_proj.weight", specs["up_proj"]),
                (p + "mlp.down_proj.weight", specs["down_proj"]),
                (p + "input_layernorm.weight", (cfg.hidden_size,)),
                (p + "post_attention_layernorm.weight", (cfg.hidden_size,))]
    out += [("norm.weight", (cfg.hidden_size,)),
            ("out_head.weight", (cfg.vocab_size, cfg.hidden_size))]
    return out


@dataclass
class HostWeights:
    """Weights on the host in bf16, grouped the way the engine consumes them."""
    cfg: ModelConfig
    embed: torch.Tensor                       # (V, H)
    layers: List[Dict[str, torch.Tensor]]     # per block: name -> matrix
    norms: Dict[str, torch.Tensor]            # name -> vector (all ones here)

    def named_tensors(self):
        yield "embed_tokens.weight", self.embed
        for l, blk in enumerate(self.layers):
            for k, v in blk.items():
                yield f"layers.{l}.{k}", v


def _ones_norms(cfg: ModelConfig) -> Dict[str, torch.Tensor]:
    n = {"norm.weight": torch.ones(cfg.hidden_size, dtype=torch.bfloat16)}
    for l in range(cfg.num_layers):
        for k in ("input_layernorm", "post_attention_layernorm"):
            n[f"layers.{l}.{k}.weight"] = torch.ones(cfg.hidden_size, dtype=torch.bfloat16)
        for k in ("q_norm", "k_norm"):
            n[f"layers.{l}.self_attn.{k}.weight"] = torch.ones(cfg.head_dim, dtype=torch.bfloat16)
    return n


def _fill_block(cfg: ModelConfig, gen: torch.Generator, std: float) -> Dict[str, torch.Tensor]:
    blk = {}
    for name, shape in layer_param_specs(cfg):
        t = torch.empty(shape, dtype=torch.bfloat16)
        t.normal_(0.0, std, generator=gen)
        blk[name] = t
    return blk


def sequential_seeded(cfg: ModelConfig, seed: int = 0,
                      record_states: bool = False, std: float = 0.02):
    """The recipe run in order on the global CPU generator.

    Returns the weights and, if asked, the generator state at the start of the
    embedding and of every block (the checkpoints :func:`exact_seeded` uses).
    """
    torch.manual_seed(seed)
    states = []
    if record_states:
        states.append(torch.get_rng_state().clone())
    embed = torch.empty(cfg.vocab_size, cfg.hidden_size, dtype=torch.bfloat16)
    embed.normal_(0.0, std)
    layers = []
    for _ in range(cfg.num_layers):
        if record_states:
            states.append(torch.get_rng_state().clone())
        blk = {}
        for name, shape in layer_param_specs(cfg):
            t = torch.empty(shape, dtype=torch.bfloat16)
            t.normal_(0.0, std)
            blk[name] = t
        layers.append(blk)
    w = HostWeights(cfg, embed, layers, _ones_norms(cfg))
    return (w, states) if record_states else w


def checkpoint_path(cfg: ModelConfig, seed: int) -> str:
    return os.path.join(_DATA, f"rng_ckpt_h{cfg.hidden_size}_l{cfg.num_layers}_"
                               f"v{cfg.vocab_size}_s{seed}.npz")


def save_checkpoints(cfg: ModelConfig, seed: int, states: List[torch.Tensor]) -> str:
    os.makedirs(_DATA, exist_ok=True)
    path = checkpoint_path(cfg, seed)
    np.savez_compressed(path, states=np.stack([s.numpy() for s in states]),
                        torch_version=np.array(torch.__version__))
    return path


def exact_seeded(cfg: ModelConfig, seed: int = 0, threads: Optional[int] = None,
                 std: float = 0.02) -> HostWeights:
    """Bit-identical to :func:`sequential_seeded`, filled block-parallel.

    Falls back to the sequential recipe when no checkpoint file exists for
    this shape and seed.
    """
    path = checkpoint_path(cfg, seed)
    if not os.path.exists(path):
        return sequential_seeded(cfg, seed, std=std)
    data = np.load(path)
    states = data["states"]
    if states.shape[0] != cfg.num_layers + 1:
        raise ValueError(f"{path}: expected {cfg.num_layers + 1} states, got {states.shape[0]}")

    def gen_for(k: int) -> torch.Generator:
        g = torch.Generator()
        g.set_state(torch.from_numpy(states[k].copy()))
        return g

    def fill_embed():
        t = torch.empty(cfg.vocab_size, cfg.hidden_size, dtype=torch.bfloat16)
        t.normal_(0.0, std, generator=gen_for(0))
        return t

    threads = threads or min(32, (os.cpu_count() or 8))
    with cf.ThreadPoolExecutor(max_workers=threads) as ex:
        f_embed = ex.submit(fill_embed)
        f_layers = [ex.submit(_fill_block, cfg, gen_for(l + 1), std) for l in range(cfg.num_layers)]
        embed = f_embed.result()
        layers = [f.result() for f in f_layers]
    return HostWeights(cfg, embed, layers, _ones_norms(cfg))


def device_seeded(cfg: ModelConfig, seed: int = 0, device="cuda", dtype=torch.bfloat16,
                  std: float = 0.02) -> Tuple[torch.Tensor, List[Dict[str, torch.Tensor]]]:
    """N(0, 0.02) weights drawn on the device (fast; not the CPU recipe's values)."""
    g = torch.Generator(device=device).manual_seed(seed)
    embed = torch.empty(cfg.vocab_size, cfg.hidden_size, dtype=dtype, device=device)
    embed.normal_(0.0, std, generator=g)
    layers = []
    for _ in range(cfg.num_layers):
        blk = {}
        for name, shape in layer_param_specs(cfg):
            t = torch.empty(shape, dtype=dtype, device=device)
            t.normal_(0.0, std, generator=g)
            blk[name] = t
        layers.append(blk)
    return embed, layers


def fingerprint(w: HostWeights) -> Dict[str, float]:
    """A few float64 sums that identify a weight set (for cross-machine checks)."""
    out = {"embed": float(w.embed[:4096].double().sum())}
    for l in (0, len(w.layers) - 1):
        for k in ("q_proj", "down_proj"):
            out[f"l{l}.{k}"] = float(w.layers[l][k][:64].double().sum())
    return out
