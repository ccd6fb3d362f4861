"""Model and engine configuration.

The Qwen3-4B constants follow ``hayate/model/qwen.py:12-25`` of the reference
(vocab 151936, hidden 2560, 36 layers, 32 query heads, 8 KV heads, head_dim 128,
MLP 9728, RMSNorm eps 1e-6, RoPE theta 1e6, 40960 positions).  The engine
defaults mirror ``hayate/engine/engine.py:13-15`` (``MAX_BATCH_SIZE = 20``) and add
the knobs that paged KV and chunked prefill need.
"""
from __future__ import annotations

from dataclasses import dataclass, field, replace

# Kernel-side constants.  The CUDA kernels are specialised for these values; the
# host checks every model config against them before building an engine.
HEAD_DIM = 128
GQA_GROUP = 4          # query heads per KV head
BLOCK_SIZE = 16        # tokens per paged KV block


@dataclass(frozen=True)
class ModelConfig:
    vocab_size: int = 151_936
    hidden_size: int = 2560
    num_layers: int = 36
    num_heads: int = 32
    num_kv_heads: int = 8
    head_dim: int = HEAD_DIM
    intermediate_size: int = 9728
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    max_position_embeddings: int = 40_960
    tie_word_embeddings: bool = True

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    def check_kernel_support(self) -> None:
        if self.head_dim != HEAD_DIM:
            raise ValueError(f"kernels are built for head_dim={HEAD_DIM}, got {self.head_dim}")
        if self.num_heads != GQA_GROUP * self.num_kv_heads:
            raise ValueError(
                f"kernels are built for {GQA_GROUP} query heads per KV head, got "
                f"{self.num_heads}/{self.num_kv_heads}")

    def num_params(self) -> int:
        h, i = self.hidden_size, self.intermediate_size
        per_layer = h * self.qkv_size + self.q_size * h + 3 * h * i
        emb = self.vocab_size * h
        head = 0 if self.tie_word_embeddings else emb
        return emb + head + self.num_layers * per_layer


QWEN3_4B = ModelConfig()

# A two-layer model with the same head geometry.  The engine-level parity
# fixtures are generated with it because it runs the reference in seconds.
TINY = ModelConfig(vocab_size=512, hidden_size=256, num_layers=2, num_heads=8,
                   num_kv_heads=2, intermediate_size=512,
                   max_position_embeddings=4096)


@dataclass
class EngineConfig:
    # Admission limit; the reference admits at most MAX_BATCH_SIZE=20 requests
    # (engine.py:13).  The paged engine can hold far more; the limit only
    # bounds per-step metadata buffers.
    max_num_seqs: int = 256
    # Token budget of one step (decodes + prefill chunks).
    max_batched_tokens: int = 8192
    # Longest prefill piece that one sequence contributes to a step.
    prefill_chunk: int = 512
    block_size: int = BLOCK_SIZE
    # KV capacity in blocks; None = size from free device memory.
    num_kv_blocks: int | None = None
    kv_cache_fraction: float = 0.80
    # Longest sequence (prompt + generated) a request may reach.
    max_model_len: int = 8192
    # Capture decode-only steps in CUDA graphs.
    cuda_graphs: bool = True
    # Treat eos as an ordinary token (fixed-length generation).
    ignore_eos: bool = False
    # Share the KV of identical prompt prefixes (full 16-token blocks) between
    # requests; off by default.
    prefix_caching: bool = False
    # NVTX ranges around each step's phases (admit, schedule, launch, collect),
    # for Nsight timelines; also on when the environment sets HY_NVTX=1.
    trace: bool = False

    def with_(self, **kw) -> "EngineConfig":
        return replace(self, **kw)
