"""The engine API of the reference, driving the B200 step.

Same surface as hayate/engine/engine.py: ``Request`` (engine.py:17-32),
``Engine(model_name, compile=False)`` (:35-61), ``add_request`` (:63-67),
``sample`` (:69-71), ``generate()`` -- one continuous-batching step returning
False when there is nothing to run (:202-217) -- and ``generate_text(prompts,
max_tokens=100)`` returning one Request or a list (:219-234).  The attributes
``pool`` (a ``queue.Queue``), ``current_batch`` and ``request_id`` behave as the
benchmark expects (benchmark.py:249-264).

What changes underneath: requests live in device-side rows (token ids, block
tables) and a paged KV cache; each step is one mixed batch of decodes and
prefill chunks built on the GPU (see ``model.Runner``); decode-only steps
replay CUDA graphs; the host reads back one small array per step (the sampled
tokens and the device error word) instead of one ``.item()`` per request.

Prompts are token-id lists or strings.  Strings need a tokenizer: pass one
with ``encode``/``decode``/``eos_token_id``, or a local Hugging Face tokenizer
directory as ``model_name``; with no tokenizer, strings are encoded as UTF-8
bytes.  ``eos_token_id`` stops a request as in the reference (engine.py:76).
"""
from __future__ import annotations

import os
import time
from dataclasses import dataclass, field
from queue import Queue
from typing import Dict, List, Optional, Union

import numpy as np
import torch

from . import kernels as K
from . import weights as Wt
from .config import EngineConfig, ModelConfig, QWEN3_4B, TINY
from .model import Runner
from .prefix_cache import PrefixCache, cacheable_blocks
from .scheduler import SAMPLE, Scheduler, StepPlan, graph_bucket, graph_buckets


class _NoRange:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


_NO_RANGE = _NoRange()


class _Range:
    """An NVTX range (torch.cuda.nvtx) as a context manager."""

    def __init__(self, name: str):
        self.name = name

    def __enter__(self):
        torch.cuda.nvtx.range_push(self.name)
        return self

    def __exit__(self, *exc):
        torch.cuda.nvtx.range_pop()
        return False

MODEL_CONFIGS = {"Qwen/Qwen3-4B": QWEN3_4B, "qwen3-4b": QWEN3_4B, "tiny": TINY}


@dataclass
class Request:
    id: int = 0
    prompt: Union[str, List[int]] = ""
    max_tokens: int = 100

    prompt_tokens: List[int] = field(default_factory=list)
    tokens: List[int] = field(default_factory=list)
    kv_cache: object = None          # kept for API compatibility; KV lives in the paged pool

    cache_pos: int = 0               # tokens whose KV is in the cache
    is_completed: bool = False
    is_prefill: bool = True
    use_cache: bool = True

    response: Optional[str] = None

    # engine bookkeeping
    slot: int = -1
    _blocks: int = 0
    _pinned: Optional[torch.Tensor] = None
    _pending: int = 0             # sampled tokens launched, not yet read back
    _inflight: int = 0            # launched steps containing this request, not yet read back
    _last_launched: bool = False  # the step that samples its last token is launched
    # prefix caching: chain hashes of the prompt's cacheable blocks, how many of
    # its leading blocks the cache holds, the adopted block ids, and a pending
    # read-back of the block ids its prefill wrote
    _hashes: List[int] = field(default_factory=list)
    _shared: int = 0
    _shared_blocks: List[int] = field(default_factory=list)
    _offer: Optional[tuple] = None
    _adopt_pinned: Optional[tuple] = None   # host buffers of the adopted-block upload


class ByteTokenizer:
    """UTF-8 byte tokenizer used for string prompts when no tokenizer is given."""
    eos_token_id = None
    pad_token_id = 0

    def encode(self, text):
        return list(text.encode("utf-8")) if isinstance(text, str) else list(text)

    def decode(self, ids, skip_special_tokens=True):
        return bytes(i for i in ids if 0 <= i < 256).decode("utf-8", errors="replace")


class Engine:
    def __init__(self, model_name: str = "Qwen/Qwen3-4B", compile: bool = False, *,
                 model_config: Optional[ModelConfig] = None,
                 engine_config: Optional[EngineConfig] = None,
                 dtype: torch.dtype = torch.bfloat16, weights="device", seed: int = 0,
                 std: float = 0.02, tokenizer=None, device=None):
        """``weights``: "device" (N(0,std) drawn on the GPU, fast), "exact" (the
        CPU recipe of ``weights.py``, bit-identical to the parity fixtures), or a
        ``weights.HostWeights``.  ``compile`` turns on CUDA-graph capture of
        decode steps (the native counterpart of torch.compile's
        reduce-overhead mode, engine.py:43-57); it is also on whenever
        ``engine_config.cuda_graphs`` is set."""
        if not torch.cuda.is_available():
            raise RuntimeError("hayate_b200 needs a CUDA device (B200, sm_100a)")
        self.cfg = model_config or MODEL_CONFIGS.get(model_name, QWEN3_4B)
        self.ecfg = engine_config or EngineConfig()
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        torch.cuda.set_device(self.device)
        self.dtype = dtype
        if dtype == torch.float32:
            torch.backends.cuda.matmul.allow_tf32 = False
        self.num_layers = self.cfg.num_layers
        self.num_kv_groups = self.cfg.num_kv_heads
        self.head_dim = self.cfg.head_dim
        self.tokenizer = tokenizer if tokenizer is not None else self._load_tokenizer(model_name)
        self.eos_token_id = None if self.ecfg.ignore_eos else getattr(
            self.tokenizer, "eos_token_id", None)

        if isinstance(weights, Wt.HostWeights):
            hw = weights
            embed, layers, norms = hw.embed, hw.layers, hw.norms
        elif weights == "exact":
            hw = Wt.exact_seeded(self.cfg, seed, std=std)
            embed, layers, norms = hw.embed, hw.layers, hw.norms
        elif weights == "device":
            embed, layers = Wt.device_seeded(self.cfg, seed, self.device, dtype, std=std)
            norms = None
        else:
            raise ValueError(f"unknown weights source {weights!r}")
        self.runner = Runner(self.cfg, self.ecfg, dtype, self.device, embed, layers, norms)
        del embed, layers
        self.prefix_cache = PrefixCache() if self.ecfg.prefix_caching else None
        self.scheduler = Scheduler(self.ecfg, self.runner.num_blocks, self.runner.max_reqs,
                                   cache=self.prefix_cache)
        # A subclass that overrides ``sample`` (the reference's hook for the
        # next-token choice, engine.py:69-71) gets the step's last-token logits
        # and its choice is committed on the device; the built-in greedy choice
        # runs the argmax on the device (in bf16, inside the LM-head kernel).  Decode steps are only captured in CUDA
        # graphs for the built-in choice.
        self._sampler = None if type(self).sample is Engine.sample else self.sample
        self.use_graphs = bool(compile or self.ecfg.cuda_graphs) and self._sampler is None
        self.trace = bool(self.ecfg.trace or os.environ.get("HY_NVTX") == "1")
        self._graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self._graph_pool = None
        S = self.ecfg.max_num_seqs
        # two of each: step n+1 is prepared while step n may still be running
        self._sched_host = [torch.zeros(4 * S, dtype=torch.int32).pin_memory() for _ in range(2)]
        self._out_host = [torch.zeros(1 + S, dtype=torch.int32).pin_memory() for _ in range(2)]
        self._events = [torch.cuda.Event() for _ in range(2)]
        self._inflight = None          # (plan, buffer index) of the step not yet read back
        self._step_idx = 0
        self._pad_ready = False
        self.pool: Queue = Queue()
        self.current_batch: List[Request] = []
        self.request_id = 0
        # counters for throughput accounting
        self.h2d_bytes = 0
        self.d2h_bytes = 0
        self.steps = 0
        self.graph_steps = 0
        self.prompt_tokens_computed = 0     # prompt tokens that went through the model
        # when a list: one (num_seqs, num_tokens, num_sampled, decode_only, key
        # tokens) record per launched step, for profiling
        self.step_log: Optional[list] = None

    @staticmethod
    def _load_tokenizer(model_name):
        if os.path.isdir(model_name):
            try:
                from transformers import AutoTokenizer
                return AutoTokenizer.from_pretrained(model_name, use_fast=True)
            except Exception:                              # noqa: BLE001
                pass
        return ByteTokenizer()

    # ------------------------------------------------------------------ API
    def add_request(self, request: Request):
        """adds a request in the pool"""
        self.pool.put(request)

    def sample(self, logits: torch.Tensor) -> torch.Tensor:
        """select the next token greedily via argmax (on-GPU kernel).

        Override it to choose tokens another way: the engine then calls it once
        per step with the ``(num_sampled, vocab)`` logits of the step's last
        tokens, on the device, and commits the ``(num_sampled, 1)`` ids it
        returns."""
        logits = logits.contiguous()
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
        K.argmax(logits, out)
        return out.long().unsqueeze(-1)

    def generate(self) -> bool:
        """One continuous-batching step; False when there is nothing to run.

        The engine runs one step ahead of the host: a call launches the next
        step (its inputs -- tokens sampled by the previous step -- are committed
        on the device) and then reads back the previous step's tokens, so the
        host's bookkeeping overlaps the GPU's work.  Requests therefore report
        completion one call after their last token is sampled."""
        rng = self._range
        with rng("admit"):
            self._drain_pool()
            sch = self.scheduler
            for r in sch.admit():
                self._upload_prompt(r)
                if r._shared_blocks:
                    self._adopt_blocks(r)
            evicted = sch.take_evicted()
            if evicted:                             # cache blocks back to the device pool
                ids = torch.tensor(evicted, dtype=torch.int32).pin_memory()
                self.runner.push_blocks(ids.to(self.device, non_blocking=True))
                self.h2d_bytes += 4 * len(evicted)
        launched = False
        if sch.running:
            with rng("schedule"):
                plan = sch.schedule()
            if plan.num_seqs:
                prev = self._inflight
                with rng("launch"):
                    self._inflight = self._launch(plan)
                launched = True
                if prev is not None:
                    with rng("collect"):
                        self._collect(*prev)
        if not launched:
            if self._inflight is None:
                self.current_batch = [r for r in sch.running if not r.is_completed]
                return bool(sch.running)
            prev, self._inflight = self._inflight, None
            with rng("collect"):
                self._collect(*prev)
        self.current_batch = [r for r in sch.running if not r.is_completed]
        return True

    def generate_text(self, prompts, max_tokens: int = 100):
        """the public api for generation"""
        if isinstance(prompts, str) or (isinstance(prompts, torch.Tensor) and prompts.dim() == 1) \
                or (isinstance(prompts, list) and prompts and isinstance(prompts[0], int)):
            prompts = [prompts]
        requests = []
        for p in prompts:
            req = Request(id=self.request_id, prompt=p, max_tokens=max_tokens)
            self.request_id += 1
            self.add_request(req)
            requests.append(req)
        while self.generate():
            pass
        return requests[0] if len(requests) == 1 else requests

    # ------------------------------------------------------------------ internals
    def _range(self, name: str):
        return _Range(name) if self.trace else _NO_RANGE

    def _drain_pool(self):
        while not self.pool.empty():
            r = self.pool.get()
            if not len(r.prompt_tokens):
                if isinstance(r.prompt, torch.Tensor):
                    # device-resident prompt: stays on the GPU (copied device to device)
                    r.prompt_tokens = r.prompt.to(torch.int32).reshape(-1)
                elif isinstance(r.prompt, str):
                    r.prompt_tokens = self.tokenizer.encode(r.prompt)
                else:
                    r.prompt_tokens = list(r.prompt)
            self.scheduler.check_request(r)
            self.scheduler.waiting.append(r)

    def _upload_prompt(self, r: Request):
        if isinstance(r.prompt_tokens, torch.Tensor) and r.prompt_tokens.is_cuda:
            n = r.prompt_tokens.numel()
            self.runner.req_tokens[r.slot, :n].copy_(r.prompt_tokens, non_blocking=True)
            return
        t = torch.tensor(r.prompt_tokens, dtype=torch.int32).pin_memory()
        r._pinned = t                                  # keep alive until the copy lands
        self.runner.req_tokens[r.slot, :t.numel()].copy_(t, non_blocking=True)
        self.h2d_bytes += t.numel() * 4

    def _adopt_blocks(self, r: Request):
        """The request's leading blocks are the cache's: its block-table row starts
        with them and the pack kernel allocates only what follows."""
        k = len(r._shared_blocks)
        ids = torch.tensor(r._shared_blocks, dtype=torch.int32).pin_memory()
        cnt = torch.tensor([k], dtype=torch.int32).pin_memory()
        self.runner.block_tables[r.slot, :k].copy_(ids, non_blocking=True)
        self.runner.req_nblk[r.slot:r.slot + 1].copy_(cnt, non_blocking=True)
        r._adopt_pinned = (ids, cnt)                # alive until the copies land
        self.h2d_bytes += 4 * (k + 1)

    def _ensure_pad_slot(self, buf: int):
        """The padding row of graph batches owns one block and one token.  ``buf``
        is a host schedule buffer no launched step still reads (the one the
        caller is about to fill)."""
        if self._pad_ready:
            return
        self._pad_ready = True
        pad = self.scheduler.pad_slot
        self._write_sched([(pad, 0, 1, SAMPLE)], buf)
        self.runner.launch_step(1, 1, 1)
        torch.cuda.current_stream().synchronize()     # once, before any graph capture

    def _write_sched(self, rows, buf: int = 0):
        S = len(rows)
        host = self._sched_host[buf]
        a = host.numpy()
        for i, (slot, start, q, fl) in enumerate(rows):
            a[i], a[S + i], a[2 * S + i], a[3 * S + i] = slot, start, q, fl
        self.runner.sched[:4 * S].copy_(host[:4 * S], non_blocking=True)
        self.h2d_bytes += 16 * S

    def _launch(self, plan: StepPlan):
        """Enqueue one step and the read-back of its tokens; no synchronisation."""
        buf = self._step_idx & 1
        self._step_idx += 1
        rows = [(e.req.slot, e.start, e.q_len, e.flags) for e in plan.entries]
        S, T, ns = plan.num_seqs, plan.num_tokens, plan.num_sample
        if self.use_graphs and plan.decode_only:
            Sp = graph_bucket(S, self.ecfg.max_num_seqs)
            # the other buffer belongs to the previous step, whose schedule copy
            # may still be queued; this step's buffer is free (its last user was
            # collected)
            self._ensure_pad_slot(buf)
            pad = self.scheduler.pad_slot
            rows += [(pad, 0, 1, SAMPLE)] * (Sp - S)
            self._write_sched(rows, buf)
            g = self._graphs.get(Sp)
            if g is None:
                g = self._capture(Sp)
            g.replay()
            self.runner.kernel_launches += self.runner.launches_per_step(True)
            self.graph_steps += 1
            n_read = Sp
        else:
            self._write_sched(rows, buf)
            self.runner.launch_step(S, T, ns, sampler=self._sampler)
            n_read = ns
        self.steps += 1
        if self.step_log is not None:
            self.step_log.append((S, T, ns, plan.decode_only,
                                  sum(e.start + e.q_len for e in plan.entries)))
        self._out_host[buf][:1 + n_read].copy_(self.runner.out_buf[:1 + n_read],
                                                non_blocking=True)
        self.d2h_bytes += 4 * (1 + n_read)
        if self.prefix_cache is not None:            # prefills this step completes
            for e in plan.entries:
                if e.flags & SAMPLE and e.req.is_prefill:
                    self._read_prompt_blocks(e.req, plan)
        self._events[buf].record()
        # host state advances at launch: the next schedule builds on this step
        for e in plan.entries:
            r = e.req
            if r.is_prefill:
                self.prompt_tokens_computed += e.q_len
            r.cache_pos = e.start + e.q_len
            r._inflight += 1
            if e.flags & SAMPLE:
                r.is_prefill = False
                r._pending += 1
                if len(r.tokens) + r._pending >= self.scheduler.token_limit(r):
                    r._last_launched = True
        return plan, buf

    def _read_prompt_blocks(self, r: Request, plan: StepPlan):
        """With the step that ends a prefill: copy the ids of the prompt blocks it
        wrote (past those the cache gave) to the host, for the cache to take once
        the step is collected."""
        n = cacheable_blocks(len(r.prompt_tokens), self.ecfg.block_size)
        if n <= r._shared:
            return
        host = torch.empty(n - r._shared, dtype=torch.int32).pin_memory()
        host.copy_(self.runner.block_tables[r.slot, r._shared:n], non_blocking=True)
        r._offer = (r._shared, n, host, plan)
        self.d2h_bytes += 4 * (n - r._shared)

    def _collect(self, plan: StepPlan, buf: int):
        """Wait for a launched step, then apply its tokens and stop conditions."""
        self._events[buf].synchronize()
        toks = self._out_host[buf].numpy()
        err = int(toks[0])
        if err:
            raise K._lib.HayateError(f"device error word {err}: {K.describe_error(err)}")
        if self.prefix_cache is not None:
            for e in plan.entries:
                r = e.req
                if r._offer is not None and r._offer[3] is plan:
                    lo, hi, host, _ = r._offer
                    r._offer = None
                    taken = self.prefix_cache.offer(r._hashes[lo:hi], host.tolist())
                    self.scheduler.offered(r, taken)
        k = 0
        for e in plan.entries:
            r = e.req
            r._inflight -= 1
            if e.flags & SAMPLE:
                tok = int(toks[1 + k])
                k += 1
                r._pending -= 1
                if r.is_completed:
                    continue                    # stopped at an earlier token (eos)
                r.tokens.append(tok)
                if tok == self.eos_token_id or len(r.tokens) >= self.scheduler.token_limit(r):
                    r.is_completed = True
                    r._last_launched = True
                    r.response = self.tokenizer.decode(r.tokens, skip_special_tokens=True)
        done = [r for r in self.scheduler.running if r.is_completed and r._inflight == 0]
        if done:
            for r in done:
                self.scheduler.release(r)
                r._pinned = None
            slots = torch.tensor([r.slot for r in done], dtype=torch.int32).pin_memory()
            dslots = slots.to(self.device, non_blocking=True)
            first = None
            if self.prefix_cache is not None:        # the cache keeps the leading blocks
                f = torch.tensor([r._shared for r in done], dtype=torch.int32).pin_memory()
                first = f.to(self.device, non_blocking=True)
            self.runner.free_slots(dslots, first)
            self.h2d_bytes += 4 * len(done) * (2 if first is not None else 1)

    def _capture(self, Sp: int) -> torch.cuda.CUDAGraph:
        r = self.runner
        # warm-up on a side stream (allocator + one-time kernel setup), then capture
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        saved = r.sched[:4 * Sp].clone()
        with torch.cuda.stream(s):
            r.launch_step(Sp, Sp, Sp)
        torch.cuda.current_stream().wait_stream(s)
        # the warm-up wrote real tokens/KV for this step; replaying it rewrites
        # the same values, so capture simply re-runs from the same schedule
        r.sched[:4 * Sp].copy_(saved)
        g = torch.cuda.CUDAGraph()
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(g, pool=self._graph_pool):
            r.launch_step(Sp, Sp, Sp)
        self._graphs[Sp] = g
        return g

    def capture_graphs(self, sizes: Optional[List[int]] = None) -> int:
        """Capture the decode-step graphs of the given batch buckets (all of them by
        default) ahead of use, so that no capture happens inside a timed run.  The
        graphs record launches over the step buffers; here every row is the padding
        slot, and a replay reads the real schedule.  Call while no step is in
        flight; returns how many graphs were captured."""
        if not self.use_graphs:
            return 0
        if self._inflight is not None:
            raise RuntimeError("capture_graphs: a step is still in flight")
        self._ensure_pad_slot(self._step_idx & 1)
        pad = self.scheduler.pad_slot
        n = 0
        for Sp in (sizes or graph_buckets(self.ecfg.max_num_seqs)):
            if Sp in self._graphs:
                continue
            self._write_sched([(pad, 0, 1, SAMPLE)] * Sp, self._step_idx & 1)
            self._capture(Sp)
            torch.cuda.current_stream().synchronize()  # the host schedule buffer is reused
            n += 1
        return n

    # ------------------------------------------------------------------ info
    def check_device_errors(self) -> int:
        torch.cuda.synchronize(self.device)
        return int(self.runner.error_word.item())
