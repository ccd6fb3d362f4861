"""CUDA kernels against the oracle, through the C ABI (run on a B200)."""
import math
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from helpers import random_paged_batch, reference_attention
from hayate_b200 import kernels as K
from hayate_b200.config import QWEN3_4B
from oracle import paged as PS
from oracle import reference as R

pytestmark = pytest.mark.gpu
dev = "cuda"


def i32(a):
    return torch.as_tensor(np.asarray(a), dtype=torch.int32, device=dev).contiguous()


# ------------------------------------------------------------------ packing
class DeviceState:
    def __init__(self, st: PS.PagedState):
        self.req_tokens = i32(st.req_tokens)
        self.block_tables = i32(st.block_tables)
        self.req_nblk = i32(st.req_nblk)
        self.free_stack = torch.zeros(st.num_blocks, dtype=torch.int32, device=dev)
        self.free_top = torch.zeros(1, dtype=torch.int32, device=dev)
        K.block_pool_init(self.free_stack, self.free_top)
        self.err = torch.zeros(1, dtype=torch.int32, device=dev)


def _pack_step(ds, st, sched, T):
    S = sched.shape[1]
    outs = {n: torch.full((max(T, 1),), -7, dtype=torch.int32, device=dev)
            for n in ("input_ids", "positions", "slot_mapping")}
    cu = torch.full((S + 1,), -7, dtype=torch.int32, device=dev)
    kv = torch.full((S,), -7, dtype=torch.int32, device=dev)
    sr = torch.full((S,), -7, dtype=torch.int32, device=dev)
    ss = torch.full((S,), -7, dtype=torch.int32, device=dev)
    K.pack_batch(i32(sched.reshape(-1)), S, T, ds.req_tokens, ds.block_tables, ds.req_nblk,
                 ds.free_stack, ds.free_top, outs["input_ids"], outs["positions"],
                 outs["slot_mapping"], cu, kv, sr, ss, ds.err)
    want = PS.pack(st, sched, T)
    torch.cuda.synchronize()
    assert int(ds.err.item()) == 0, K.describe_error(int(ds.err.item()))
    for n in ("input_ids", "positions", "slot_mapping"):
        assert np.array_equal(outs[n][:T].cpu().numpy(), want[n]), n
    assert np.array_equal(cu.cpu().numpy(), want["cu_seqlens_q"])
    assert np.array_equal(kv.cpu().numpy(), want["seq_lens_k"])
    ns = len(want["sample_rows"])
    assert np.array_equal(sr[:ns].cpu().numpy(), want["sample_rows"])
    assert np.array_equal(ss[:ns].cpu().numpy(), want["sample_seq"])
    assert np.array_equal(ds.block_tables.cpu().numpy(), st.block_tables)
    assert np.array_equal(ds.req_nblk.cpu().numpy(), st.req_nblk)
    assert int(ds.free_top.item()) == st.free_top
    return want, ss[:ns]


def test_pack_commit_free_bit_exact():
    rng = np.random.default_rng(0)
    max_reqs, pitch, btp, NB = 40, 700, 48, 600
    st = PS.PagedState(max_reqs, pitch, btp, NB)
    st.req_tokens[:] = rng.integers(0, 151936, size=st.req_tokens.shape)
    ds = DeviceState(st)
    assert np.array_equal(ds.free_stack.cpu().numpy(), st.free_stack)
    lens = {s: int(rng.integers(1, 400)) for s in range(0, 36, 2)}   # prompt lengths
    done = {s: 0 for s in lens}                                       # cached tokens
    step = 0
    while any(done[s] < lens[s] + 3 for s in lens) and step < 40:
        rows = []
        for s in lens:
            total = lens[s] + 3
            if done[s] >= total:
                continue
            q = min(int(rng.integers(1, 130)), total - done[s]) if done[s] < lens[s] else 1
            q = min(q, lens[s] - done[s]) if done[s] < lens[s] else 1
            rows.append((s, done[s], q, int(done[s] + q >= lens[s])))
        order = rng.permutation(len(rows))
        rows = [rows[i] for i in order]
        sched = PS.make_sched(*zip(*rows))
        T = int(sched[2].sum())
        want, ss = _pack_step(ds, st, sched, T)
        # commit: sampled tokens land after each sequence's last token
        nxt = rng.integers(0, 151936, size=len(want["sample_seq"])).astype(np.int32)
        K.commit_tokens(i32(nxt), len(nxt), ss, i32(sched.reshape(-1)), sched.shape[1],
                        ds.req_tokens, ds.err)
        PS.commit(st, nxt, want["sample_seq"], sched)
        for s, start, q, _ in rows:
            done[s] = start + q
        # release finished requests
        fin = [s for s in lens if done[s] >= lens[s] + 3]
        if fin and step % 3 == 0:
            K.free_blocks(i32(fin), ds.block_tables, ds.req_nblk, ds.free_stack, ds.free_top,
                          ds.err)
            PS.free(st, fin)
            for s in fin:
                lens.pop(s)
                done.pop(s)
        torch.cuda.synchronize()
        assert np.array_equal(ds.req_tokens.cpu().numpy(), st.req_tokens)
        assert np.array_equal(ds.free_stack.cpu().numpy()[:st.free_top],
                              st.free_stack[:st.free_top])
        step += 1
    assert int(ds.err.item()) == 0


def test_free_from_and_push_bit_exact():
    """Prefix-cache moves of the pool: slots give back only their blocks past a
    shared prefix, and the held prefix blocks are pushed back later in a list."""
    rng = np.random.default_rng(3)
    st = PS.PagedState(12, 400, 32, 200)
    st.req_tokens[:] = rng.integers(0, 1000, size=st.req_tokens.shape)
    ds = DeviceState(st)
    lens = [37, 150, 16, 300, 5, 90]
    sched = PS.make_sched(list(range(len(lens))), [0] * len(lens), lens, [1] * len(lens))
    _pack_step(ds, st, sched, int(sum(lens)))
    slots = [4, 1, 3, 0]
    first = [0, 5, 2, 3]                             # blocks before these stay held
    held = [int(b) for s, f in zip(slots, first) for b in st.block_tables[s, :f]]
    K.free_blocks(i32(slots), ds.block_tables, ds.req_nblk, ds.free_stack, ds.free_top, ds.err,
                  first_block=i32(first))
    PS.free(st, slots, first)
    order = list(rng.permutation(len(held)))
    K.push_blocks(i32([held[i] for i in order]), ds.free_stack, ds.free_top, ds.err)
    PS.push(st, [held[i] for i in order])
    torch.cuda.synchronize()
    assert int(ds.err.item()) == 0
    assert int(ds.free_top.item()) == st.free_top
    assert np.array_equal(ds.free_stack.cpu().numpy()[:st.free_top], st.free_stack[:st.free_top])
    assert np.array_equal(ds.req_nblk.cpu().numpy(), st.req_nblk)
    # a bad id pushes nothing and is reported
    top = int(ds.free_top.item())
    K.push_blocks(i32([3, 999]), ds.free_stack, ds.free_top, ds.err)
    torch.cuda.synchronize()
    assert int(ds.free_top.item()) == top and int(ds.err.item()) & K.DEV_BOUNDS


def test_pack_reports_pool_exhaustion():
    st = PS.PagedState(4, 200, 16, 3)
    ds = DeviceState(st)
    sched = PS.make_sched([0], [0], [100], [1])    # needs 7 blocks, only 3 exist
    S, T = 1, 100
    bufs = [torch.zeros(T, dtype=torch.int32, device=dev) for _ in range(3)]
    small = [torch.zeros(2, dtype=torch.int32, device=dev) for _ in range(4)]
    K.pack_batch(i32(sched.reshape(-1)), S, T, ds.req_tokens, ds.block_tables, ds.req_nblk,
                 ds.free_stack, ds.free_top, *bufs, *small, ds.err)
    torch.cuda.synchronize()
    assert int(ds.err.item()) & K.DEV_POOL


# ------------------------------------------------------- QK-norm + RoPE + append
@pytest.mark.parametrize("tag,dt", [("bf16", torch.bfloat16), ("fp32", torch.float32)])
def test_qk_norm_rope_vs_reference_fixture(tag, dt):
    f = np.load(os.path.join(GOLDEN, "qk_norm_rope.npz"))

    def t(name):
        a = torch.from_numpy(f[f"{tag}_{name}"])
        return (a.view(torch.bfloat16) if dt == torch.bfloat16 else a).to(dev)
    q, k = t("q"), t("k")
    T, Hq, Hkv = q.shape[0], q.shape[1], k.shape[1]
    v = torch.randn(T, Hkv, 128, device=dev).to(dt)
    qkv = torch.cat([q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], 1).contiguous()
    cos, sin = R.rope_tables(128, QWEN3_4B.rope_theta, QWEN3_4B.max_position_embeddings)
    cos64, sin64 = cos[:, :64].contiguous().to(dev), sin[:, :64].contiguous().to(dev)
    pos = torch.from_numpy(f["positions"]).to(dev).int()
    q_out = torch.empty_like(q)
    k_out = torch.empty_like(k)
    NB = 8
    cache = torch.zeros(NB, 2, Hkv, 16, 128, dtype=dt, device=dev)
    slots = torch.randperm(NB * 16, device=dev)[:T].int()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    K.qk_norm_rope(qkv, Hq, Hkv, pos, t("wq"), t("wk"), cos64, sin64, QWEN3_4B.rms_norm_eps,
                   q_out=q_out, k_out=k_out, kv_cache_layer=cache, slot_mapping=slots,
                   num_blocks=NB, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    for got, want in ((q_out, t("q_out")), (k_out, t("k_out"))):
        if dt == torch.bfloat16:
            # at most one bf16 ulp: the mean-of-squares summation order differs
            gi = got.view(torch.int16).int()
            wi = want.view(torch.int16).int()
            assert (gi - wi).abs().max().item() <= 1
            assert (gi != wi).float().mean().item() < 0.02
        else:
            torch.testing.assert_close(got, want, rtol=2e-6, atol=2e-6)
    # the cache holds the rotated keys and raw values at their slots
    want_cache = np.zeros((NB, 2, Hkv, 16, 128), np.float32)
    PS.kv_append(want_cache, k_out.float().cpu().numpy(), v.float().cpu().numpy(),
                 slots.cpu().numpy())
    assert np.array_equal(cache.float().cpu().numpy(), want_cache)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_kv_append_bit_exact(dt):
    T, Hkv, NB = 57, 8, 9
    k = torch.randn(T, Hkv, 128, device=dev).to(dt)
    v = torch.randn(T, Hkv, 128, device=dev).to(dt)
    slots = torch.randperm(NB * 16, device=dev)[:T].int()
    slots[3] = -1                                    # padding rows are skipped
    cache = torch.zeros(NB, 2, Hkv, 16, 128, dtype=dt, device=dev)
    K.kv_append(k, v, slots, cache, NB)
    want = np.zeros((NB, 2, Hkv, 16, 128), np.float32)
    PS.kv_append(want, k.float().cpu().numpy(), v.float().cpu().numpy(), slots.cpu().numpy())
    torch.cuda.synchronize()
    assert np.array_equal(cache.float().cpu().numpy(), want)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_kv_append_many_tokens(dt):
    """More rows than one pass of the grid: every lane group loops."""
    T, Hkv, NB = 9000, 8, 600
    k = torch.randn(T, Hkv, 128, device=dev).to(dt)
    v = torch.randn(T, Hkv, 128, device=dev).to(dt)
    slots = torch.randperm(NB * 16, device=dev)[:T].int()
    slots[::97] = -1
    cache = torch.zeros(NB, 2, Hkv, 16, 128, dtype=dt, device=dev)
    K.kv_append(k, v, slots, cache, NB)
    want = np.zeros((NB, 2, Hkv, 16, 128), np.float32)
    PS.kv_append(want, k.float().cpu().numpy(), v.float().cpu().numpy(), slots.cpu().numpy())
    torch.cuda.synchronize()
    assert np.array_equal(cache.float().cpu().numpy(), want)


@pytest.mark.parametrize("Hq,Hkv", [(32, 8), (48, 12)])
def test_qk_norm_rope_bf16_many_tokens_vs_oracle(Hq, Hkv):
    """bf16 path over more tokens than CTAs (each CTA walks several tokens):
    for 32/8 heads a unit covers a token's 3 passes of 16 head rows; for 48/12
    (72 rows) a token is two units of up to 4 passes, the second holding one
    half-empty pass.  Against the oracle's torch ops on the CPU: at most one
    bf16 ulp."""
    T, NB = 2500, 200
    g = torch.Generator(device=dev).manual_seed(5)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * 128, device=dev, generator=g).to(torch.bfloat16)
    wq = (1 + 0.1 * torch.randn(128, device=dev, generator=g)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(128, device=dev, generator=g)).to(torch.bfloat16)
    cos, sin = R.rope_tables(128, QWEN3_4B.rope_theta, QWEN3_4B.max_position_embeddings)
    cos64, sin64 = cos[:, :64].contiguous().to(dev), sin[:, :64].contiguous().to(dev)
    pos = torch.randint(0, 40960, (T,), device=dev, generator=g).int()
    slots = torch.randperm(NB * 16, device=dev, generator=g)[:T].int()
    slots[::101] = -1                             # padding tokens
    q_out = torch.empty(T, Hq, 128, dtype=torch.bfloat16, device=dev)
    cache = torch.zeros(NB, 2, Hkv, 16, 128, dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    K.qk_norm_rope(qkv, Hq, Hkv, pos, wq, wk, cos64, sin64, QWEN3_4B.rms_norm_eps, q_out=q_out,
                   kv_cache_layer=cache, slot_mapping=slots, num_blocks=NB, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    c = qkv.cpu()
    q, k = c[:, :Hq * 128].view(T, Hq, 128), c[:, Hq * 128:(Hq + Hkv) * 128].view(T, Hkv, 128)
    vv = c[:, (Hq + Hkv) * 128:].view(T, Hkv, 128)
    wq_out, wk_out = R.qk_norm_rope(q, k, wq.cpu(), wk.cpu(), cos, sin, pos.cpu(),
                                    QWEN3_4B.rms_norm_eps)
    # One bf16 ulp of a normed element (magnitude < 8: ulp <= 2^-5) moves an
    # output by at most two such ulps with the roundings of the products and the
    # sum, also where y*cos and y'*sin cancel and the ulp distance of the tiny
    # result says little; most elements are identical.
    def close(got, want):
        d = (got.float() - want.float()).abs()
        assert d.max().item() <= 2 ** -4
        assert (got.view(torch.int16) != want.view(torch.int16)).float().mean().item() < 0.02
    close(q_out.cpu(), wq_out)
    sl = slots.cpu().long()
    keep = sl >= 0                                # padding tokens (slot -1) write no K/V
    blk, j = sl[keep] // 16, sl[keep] % 16
    cc = cache.cpu()
    got_k = cc[blk, 0, :, j]                      # (kept tokens, Hkv, 128)
    got_v = cc[blk, 1, :, j]
    close(got_k, wk_out[keep])
    assert torch.equal(got_v, vv[keep])
    written = torch.zeros(NB * 16, dtype=torch.bool)
    written[sl[keep]] = True
    flat = cc.permute(0, 3, 1, 2, 4).reshape(NB * 16, -1)   # slot-major view of the cache
    assert not flat[~written].any()               # nothing else was written


# ------------------------------------------------------------------ attention
def _run_attention(b, dt, kv_heads, bt_row=None, max_seqs=None, max_tokens=None):
    S, T = b["S"], b["T"]
    max_seqs = max_seqs or S
    max_tokens = max_tokens or T
    out = torch.full_like(b["q"], float("nan"))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = None
    if dt == torch.bfloat16:
        nbytes = K.attention_workspace_size(max_seqs, max_tokens, kv_heads)
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
        K.attention_plan(b["cu"], b["kv"], S, kv_heads, max_seqs, max_tokens, ws, err)
    bt = b["bt"] if bt_row is None else bt_row[0]
    K.varlen_attention(b["q"], out, b["cache"], b["layer"], bt, b["cu"], b["kv"], S,
                       max_seqs, max_tokens, ws, seq_bt_row=None if bt_row is None else bt_row[1],
                       err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, K.describe_error(int(err.item()))
    return out


CASES = {
    "decode_edges": ([1] * 6, [1, 15, 16, 17, 300, 1000]),
    "decode_long_split": ([1] * 3, [16384, 5000, 70]),
    "prefill_only": ([37, 64, 16, 3], [37, 164, 16, 1027]),
    "mixed": ([1, 512, 1, 5, 1, 129, 1], [1000, 4096, 33, 12, 2049, 129, 7]),
    # 376 prefill items (several per CTA), ragged 64-token tiles, prefixes
    "prefill_many": ([65, 127, 128, 200, 512, 512, 512, 512, 300, 1],
                     [65, 227, 1128, 200, 512, 1024, 2048, 600, 3000, 50]),
    # a chunk after 8192 cached tokens (129/130 key tiles per item); a 64-token
    # chunk after 16384; a ragged 36-row tile after 5000 beside a short chunk
    "prefill_long_prior": ([128, 1], [8320, 300]),
    "prefill_longer_prior": ([64, 1], [16448, 100]),
    "prefill_ragged_prior": ([100, 37, 1], [5100, 37, 2000]),
    # decode only, 18 x 8 (sequence, KV head) pairs <= 148 CTAs and contexts of at
    # most 128 blocks: one pair per CTA, partials merged in shared memory
    "decode_per_cta": ([1] * 18, [1, 16, 17, 33, 100, 128, 129, 500, 777, 1000, 1023, 1024,
                                  1025, 1500, 2000, 2047, 2048, 64]),
    # 19 x 8 pairs > 148: the split-K path with its workspace merge
    "decode_per_cta_over": ([1] * 19, [1, 16, 17, 33, 100, 128, 129, 500, 777, 1000, 1023, 1024,
                                       1025, 1500, 2000, 2047, 2048, 64, 3]),
    # a context past 128 blocks: the split-K path as well
    "decode_per_cta_long": ([1] * 3, [2049, 30, 700]),
}


@pytest.mark.parametrize("name", list(CASES))
def test_attention_bf16_vs_fp32_reference(name):
    q_lens, kv_lens = CASES[name]
    b = random_paged_batch(q_lens, kv_lens, kv_heads=8, dtype=torch.bfloat16, seed=sum(map(ord, name)))
    got = _run_attention(b, torch.bfloat16, 8)
    want = reference_attention(b)
    err = (got.float() - want).abs().max().item()
    assert err <= 2e-2, f"max abs err {err}"


EARLY_CASES = {
    # one (sequence, KV head) pair per CTA
    "per_cta": CASES["decode_per_cta"],
    # 60 short contexts: 480 items, one round of warps assigned statically
    "static": ([1] * 60, [(7 * i) % 64 + 1 for i in range(60)]),
    # the split-K path with dynamic item pulls (the flag leaves it unchanged)
    "split_k": CASES["decode_per_cta_over"],
}


@pytest.mark.parametrize("name", list(EARLY_CASES))
def test_attention_early_start_matches_plain_launch(name):
    """HY_ATTN_EARLY, as an engine step uses it from its second layer on: the
    plan's first call (layer 0) caches the item ids; the launch just before the
    flagged call appends the step's new keys and values (each sequence's last
    position, as QK-norm+RoPE does); the flagged call must give the plain
    call's output bit for bit, within 2e-2 of fp32 attention over the updated
    cache."""
    q_lens, kv_lens = EARLY_CASES[name]
    b = random_paged_batch(q_lens, kv_lens, kv_heads=8, seed=sum(map(ord, name)), layer=1)
    S, T, NB = b["S"], b["T"], b["cache"].shape[1]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(K.attention_workspace_size(S, T, 8), dtype=torch.uint8, device=dev)
    K.attention_plan(b["cu"], b["kv"], S, 8, S, T, ws, err)
    out0 = torch.empty_like(b["q"])
    K.varlen_attention(b["q"], out0, b["cache"], 0, b["bt"], b["cu"], b["kv"], S, S, T, ws,
                       err=err)
    g = torch.Generator(device=dev).manual_seed(7)
    newk = torch.randn(T, 8, 128, device=dev, generator=g).to(torch.bfloat16)
    newv = torch.randn(T, 8, 128, device=dev, generator=g).to(torch.bfloat16)
    last = [kv - 1 for kv in kv_lens]
    slots = torch.tensor([int(b["bt"][i, p // 16]) * 16 + p % 16 for i, p in enumerate(last)],
                         dtype=torch.int32, device=dev)
    outs = []
    for early in (False, True):
        out = torch.full_like(b["q"], float("nan"))
        K.kv_append(newk, newv, slots, b["cache"][1], NB, err=err)
        K.varlen_attention(b["q"], out, b["cache"], 1, b["bt"], b["cu"], b["kv"], S, S, T, ws,
                           err=err, early=early)
        outs.append(out)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, K.describe_error(int(err.item()))
    assert torch.equal(outs[0], outs[1])
    for i, p in enumerate(last):
        b["ctx_k"][i][p] = newk[i]
        b["ctx_v"][i][p] = newv[i]
    assert (outs[1].float() - reference_attention(b)).abs().max().item() <= 2e-2


@pytest.mark.parametrize("name,items", [("prefill_long_prior", 16), ("prefill_longer_prior", 8),
                                        ("prefill_ragged_prior", 24)])
def test_attention_split_prefill_pieces(name, items):
    """A step of few, long prefill items: the plan cuts each item into pieces
    over key ranges (more planned items than 64-token tiles x KV heads), the
    last piece merges the partials, and the next calls on the same plan (the
    engine's later layers) give the same output bit for bit, within 2e-2 of
    fp32 attention."""
    q_lens, kv_lens = CASES[name]
    b = random_paged_batch(q_lens, kv_lens, kv_heads=8, seed=sum(map(ord, name)) + 1)
    S, T = b["S"], b["T"]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(K.attention_workspace_size(S, T, 8), dtype=torch.uint8, device=dev)
    K.attention_plan(b["cu"], b["kv"], S, 8, S, T, ws, err)
    torch.cuda.synchronize()
    assert int(ws[:4].view(torch.int32).item()) > items
    outs = []
    for _ in range(3):
        out = torch.full_like(b["q"], float("nan"))
        K.varlen_attention(b["q"], out, b["cache"], b["layer"], b["bt"], b["cu"], b["kv"], S, S, T,
                           ws, err=err)
        outs.append(out)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, K.describe_error(int(err.item()))
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
    assert (outs[0].float() - reference_attention(b)).abs().max().item() <= 2e-2


def _plan_items(ws, S, T, kv_heads):
    """The plan's prefill items in run order, read from the workspace: header
    word 0 is their count; the sorted items follow the by-sequence ones
    (256-byte aligned int4 arrays of max_pre entries, max_pre = kv_heads x
    (T / 64 + S) + one piece slot per SM)."""
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    max_pre = kv_heads * (T // 64 + S) + sms
    a256 = lambda x: (x + 255) // 256 * 256
    off = 256 + a256(max_pre * 16)
    n = int(ws[:4].view(torch.int32).item())
    items = ws[off:off + 16 * n].view(torch.int32).view(n, 4).cpu().tolist()
    return items, sms


@pytest.mark.parametrize("name", ["prefill_long_prior", "prefill_longer_prior",
                                  "prefill_ragged_prior", "prefill_many"])
def test_attention_plan_pieces_partition_each_item(name):
    """Every 64-token query tile x KV head appears as one whole item or as
    pieces that agree on their count and partial slot, number 0..n-1 once each,
    and cover its key tiles [0, nt) exactly; at most one piece per SM; items in
    run order have non-increasing key tiles.  (prefill_many: 376 items, more
    than the SMs, so none is cut.)"""
    q_lens, kv_lens = CASES[name]
    S, T = len(q_lens), sum(q_lens)
    cu = i32(np.concatenate([[0], np.cumsum(q_lens)]).tolist())
    kv = i32(kv_lens)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(K.attention_workspace_size(S, T, 8), dtype=torch.uint8, device=dev)
    K.attention_plan(cu, kv, S, 8, S, T, ws, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    items, sms = _plan_items(ws, S, T, 8)
    groups, tiles_seen, pieces = {}, [], 0
    for seq, g, t0, w in items:
        q, k = q_lens[seq], kv_lens[seq]
        nt = (k - q + t0 + min(64, q - t0) + 63) // 64
        if w == 0:
            lo, hi, key = 0, nt, None
        else:
            ns, sp, slot = (w >> 26) & 31, (w >> 20) & 63, w & 0xFFFFF
            lo, hi = sp * nt // ns, (sp + 1) * nt // ns
            key = (ns, slot)
            pieces += 1
        groups.setdefault((seq, g, t0), []).append((lo, hi, key))
        tiles_seen.append(hi - lo)
    want = {(s, g, t0) for s, q in enumerate(q_lens) if q > 1 for g in range(8)
            for t0 in range(0, q, 64)}
    assert set(groups) == want
    for parts in groups.values():
        assert len({p[2] for p in parts}) == 1                    # one count and slot
        if parts[0][2] is not None:
            assert len(parts) == parts[0][2][0]
        cover = sorted((lo, hi) for lo, hi, _ in parts)
        assert cover[0][0] == 0 and all(a[1] == b[0] for a, b in zip(cover, cover[1:]))
        assert all(hi > lo for lo, hi in cover)
    assert pieces <= sms
    assert tiles_seen == sorted(tiles_seen, reverse=True)
    if name == "prefill_many":
        assert pieces == 0
    else:
        assert pieces > 0


def test_attention_rejects_unaligned_queries():
    """The bf16 path reads q by TMA: a q that does not start on 16 bytes is
    refused on the host (no launch), and the next aligned call is exact."""
    from hayate_b200._lib import HayateError
    b = random_paged_batch([40, 1], [300, 77], kv_heads=8, seed=9)
    S, T = b["S"], b["T"]
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(K.attention_workspace_size(S, T, 8), dtype=torch.uint8, device=dev)
    K.attention_plan(b["cu"], b["kv"], S, 8, S, T, ws, err)
    shifted = torch.empty(T * 32 * 128 + 1, dtype=torch.bfloat16, device=dev)[1:].view(T, 32, 128)
    shifted.copy_(b["q"])
    out = torch.full_like(b["q"], float("nan"))
    with pytest.raises(HayateError, match="16-byte aligned"):
        K.varlen_attention(shifted, out, b["cache"], b["layer"], b["bt"], b["cu"], b["kv"], S, S,
                           T, ws, err=err)
    K.varlen_attention(b["q"], out, b["cache"], b["layer"], b["bt"], b["cu"], b["kv"], S, S, T, ws,
                       err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert (out.float() - reference_attention(b)).abs().max().item() <= 2e-2


def test_attention_bf16_block_table_indirection_and_headroom():
    q_lens, kv_lens = [1, 40, 1, 1], [77, 300, 16, 5]
    b = random_paged_batch(q_lens, kv_lens, kv_heads=2, seed=5)
    # the rows of the real table live at rows 3, 0, 5, 1 of a larger table
    rows = [3, 0, 5, 1]
    big = torch.full((6, b["bt"].shape[1]), -1, dtype=torch.int32, device=dev)
    for i, r in enumerate(rows):
        big[r] = b["bt"][i]
    got = _run_attention(b, torch.bfloat16, 2, bt_row=(big, i32(rows)), max_seqs=64,
                         max_tokens=1024)
    want = reference_attention(b)
    assert (got.float() - want).abs().max().item() <= 2e-2


def test_attention_micro_shape_reduced():
    rng = np.random.default_rng(0)
    dec = np.round(np.exp(rng.uniform(math.log(256), math.log(16384), size=48))).astype(int)
    q_lens = [512, 512] + [1] * len(dec)
    kv_lens = [512, 512 + 1536] + dec.tolist()
    b = random_paged_batch(q_lens, kv_lens, kv_heads=8, seed=11)
    got = _run_attention(b, torch.bfloat16, 8)
    want = reference_attention(b)
    assert (got.float() - want).abs().max().item() <= 2e-2


def test_attention_operator_case_full_size():
    """The ragged attention operator case exactly as the bench times it (256
    decode sequences, contexts log-uniform in [256,16384], 4 prefill chunks of
    512 after 0/512/1536/3584 cached tokens, permuted block table, one plan as
    the bench makes it): every output row within 2e-2 of fp32 SDPA with the
    reference's causal mask."""
    from hayate_b200.microbench import attention_micro_batch
    b = attention_micro_batch()
    S, T = b["S"], b["T"]
    out = torch.full_like(b["q"], float("nan"))
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws = torch.zeros(K.attention_workspace_size(S, T, 8), dtype=torch.uint8, device=dev)
    K.attention_plan(b["cu"], b["kv"], S, 8, S, T, ws, err)
    for _ in range(2):                  # the second call runs on the cached block ids
        K.varlen_attention(b["q"], out, b["cache"], 0, b["bt"], b["cu"], b["kv"], S, S, T, ws,
                           err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0, K.describe_error(int(err.item()))
    cu = b["cu"].tolist()
    worst = 0.0
    for i in range(S):
        L, nb = b["kv_lens"][i], b["nblk"][i]
        blocks = b["cache"][0, b["bt"][i, :nb].long()]           # (nb, 2, 8, 16, 128)
        k = blocks[:, 0].permute(0, 2, 1, 3).reshape(-1, 8, 128)[:L]
        v = blocks[:, 1].permute(0, 2, 1, 3).reshape(-1, 8, 128)[:L]
        want = R.varlen_attention(b["q"][cu[i]:cu[i + 1]], [0, cu[i + 1] - cu[i]], [k], [v])
        worst = max(worst, (out[cu[i]:cu[i + 1]].float() - want).abs().max().item())
    assert worst <= 2e-2, f"max abs err {worst}"


@pytest.mark.parametrize("name", ["decode_edges", "mixed"])
def test_attention_fp32_vs_reference(name):
    q_lens, kv_lens = CASES[name]
    b = random_paged_batch(q_lens, kv_lens, kv_heads=8, dtype=torch.float32, seed=3)
    got = _run_attention(b, torch.float32, 8)
    want = reference_attention(b)
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-4)


# ------------------------------------------------------------------- argmax
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_argmax_first_index_ties(dt):
    rows, V = 7, 151936
    x = torch.randn(rows, V, device=dev).to(dt)
    x[1, 5] = x[1, 100000] = 50.0           # tie -> lowest index
    x[2, :] = 1.0                            # all equal -> 0
    x[3, V - 1] = 60.0                       # last column
    x[4, 77] = float("inf")
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    K.argmax(x, out)
    want = torch.argmax(x, dim=-1).int()
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    assert out[1].item() == 5 and out[2].item() == 0


@pytest.mark.parametrize("rows", [1, 10, 260, 1300])
def test_argmax_cluster_split_rows(rows):
    """Rows split over clusters of 8, 8, 4 and 1 CTAs: ties placed in different
    chunks resolve to the lower index; NaN wins (first NaN); a row of equal values gives 0."""
    V = 151936
    g = torch.Generator(device=dev).manual_seed(rows)
    x = torch.randn(rows, V, device=dev, generator=g).to(torch.bfloat16)
    r = rows - 1
    x[r, 3 * V // 4 + 5] = 40.0                 # tie in the last chunk ...
    x[r, V // 8 - 1] = 40.0                     # ... and in the first: lower index wins
    if rows > 1:
        x[0, 100] = float("nan")
        x[0, 90000] = float("nan")
        x[0, 5] = float("inf")
    if rows > 2:
        x[1, :] = -3.0
    if rows > 3:                                # -0 and +0 are equal: the first zero wins
        x[2, :] = -1.0
        x[2, 7] = -0.0
        x[2, 9] = 0.0
    if rows > 4:                                # all -inf: index 0
        x[3, :] = float("-inf")
    out = torch.empty(rows, dtype=torch.int32, device=dev)
    K.argmax(x, out)
    want = torch.argmax(x.float().cpu(), dim=-1).int()
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), want)
    assert out[r].item() == V // 8 - 1
    if rows > 1:
        assert out[0].item() == 100
    if rows > 2:
        assert out[1].item() == 0
    if rows > 3:
        assert out[2].item() == 7
    if rows > 4:
        assert out[3].item() == 0


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_argmax_odd_vocab_and_unaligned_rows(dt):
    rows, V = 12, 1001
    base = torch.randn(rows, V + 1, device=dev).to(dt)
    for n, x in enumerate((base[:, :V], base[:, 1:])):   # aligned rows with a tail; unaligned
        x[2, V - 1] = 99.0 + 100 * n
        out = torch.empty(rows, dtype=torch.int32, device=dev)
        K.argmax(x, out)
        want = torch.argmax(x.float().cpu(), dim=-1).int()
        torch.cuda.synchronize()
        assert torch.equal(out.cpu(), want)
        assert out[2].item() == V - 1


# --------------------------------------------------------- RMSNorm, SiLU*up
def _ulp_diff_bf16(a, b):
    return (a.view(torch.int16).int() - b.view(torch.int16).int()).abs()


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("cols", [2560, 256, 4096, 1000])
@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("rows", [37, 3000])
def test_add_rms_norm_vs_reference(dt, cols, residual, rows):
    """37 rows: one CTA per row; 3000 bf16 rows: the streamed kernel (warps
    fed by bulk copies), except for 4096 columns with a residual, whose ring
    would not fit shared memory."""
    x = (torch.randn(rows, cols, device=dev) * 3).to(dt)
    delta = (torch.randn(rows, cols, device=dev) * 3).to(dt) if residual else None
    w = (1 + 0.1 * torch.randn(cols, device=dev)).to(dt)
    want_x = x + delta if residual else x.clone()      # block.py:24,30 residual add
    want = R.rms_norm(want_x, w, 1e-6)                  # nn.RMSNorm semantics (F.rms_norm)
    got = K.add_rms_norm(x, w, 1e-6, delta=delta)
    torch.cuda.synchronize()
    assert torch.equal(x, want_x)                       # residual updated in place, exactly
    if dt == torch.bfloat16:
        d = _ulp_diff_bf16(got, want)
        assert d.max().item() <= 1 and (d > 0).float().mean().item() < 0.02
    else:
        torch.testing.assert_close(got, want, rtol=2e-6, atol=2e-6)


def test_add_rms_norm_streamed_strided_rows():
    """The streamed kernel on rows of wider tensors (row pitches 2624 and 2688
    for 2560 columns), a row count that leaves the last warps one row short."""
    rows, cols = 1187, 2560
    xb = (torch.randn(rows, cols + 64, device=dev) * 3).to(torch.bfloat16)
    db = (torch.randn(rows, cols + 128, device=dev) * 3).to(torch.bfloat16)
    x, delta = xb[:, :cols], db[:, 64:64 + cols]
    w = (1 + 0.1 * torch.randn(cols, device=dev)).to(torch.bfloat16)
    want_x = x + delta
    want = R.rms_norm(want_x, w, 1e-6)
    pad = xb[:, cols:].clone()
    got = K.add_rms_norm(x, w, 1e-6, delta=delta)
    torch.cuda.synchronize()
    assert torch.equal(x, want_x)
    assert torch.equal(xb[:, cols:], pad)               # nothing written past the rows
    d = _ulp_diff_bf16(got, want)
    assert d.max().item() <= 1 and (d > 0).float().mean().item() < 0.02


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("nparts,rows,cols", [(8, 16, 2560), (4, 64, 2560), (1, 5, 256),
                                              (3, 37, 1000)])
def test_add_rms_norm_splitk_vs_reference(dt, nparts, rows, cols):
    """The residual's delta given as fp32 split-K partials: x gains round(sum of
    the partials in order) exactly, as the unsplit projection's rounded output
    would give it, and y is the reference RMSNorm of the new x."""
    x = (torch.randn(rows, cols, device=dev) * 3).to(dt)
    # partials in a strided [n, rows, cols] view, as a batched GEMM writes them
    big = torch.randn(nparts, rows + 3, cols + 8, device=dev)
    parts = big[:, 1:rows + 1, 4:cols + 4]
    w = (1 + 0.1 * torch.randn(cols, device=dev)).to(dt)
    acc = parts[0].clone()
    for p in range(1, nparts):                          # fp32 sum in the kernel's order
        acc = acc + parts[p]
    want_x = x + acc.to(dt)                              # block.py:24,30 on the rounded output
    want = R.rms_norm(want_x, w, 1e-6)
    got = K.add_rms_norm_splitk(x, w, 1e-6, parts)
    torch.cuda.synchronize()
    assert torch.equal(x, want_x)
    if dt == torch.bfloat16:
        d = _ulp_diff_bf16(got, want)
        assert d.max().item() <= 1 and (d > 0).float().mean().item() < 0.02
    else:
        torch.testing.assert_close(got, want, rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("mode", ["delta", "parts", "none"])
def test_gather_add_rms_norm_vs_reference(dt, mode):
    """Rows gathered by index (repeats allowed), the residual's delta added (a
    tensor, fp32 split-K partials, or none), the updated rows written to x_out
    and normed; the source rows are left untouched.  An index out of range sets
    the bounds bit and leaves its output row unwritten."""
    g = torch.Generator(device=dev).manual_seed(17)
    cols = 2560
    src = (torch.randn(50, cols, device=dev, generator=g) * 3).to(dt)
    keep = src.clone()
    idx = [49, 3, 3, 17, 0, 21]
    rows = i32(idx)
    n = len(idx)
    w = (1 + 0.1 * torch.randn(cols, device=dev, generator=g)).to(dt)
    delta = parts = None
    base = src[torch.tensor(idx, device=dev).long()]
    if mode == "delta":
        delta = (torch.randn(n, cols, device=dev, generator=g) * 3).to(dt)
        want_x = base + delta
    elif mode == "parts":
        big = torch.randn(4, n + 2, cols + 8, device=dev, generator=g)
        parts = big[:, 1:n + 1, 4:cols + 4]
        acc = parts[0].clone()
        for p in range(1, 4):
            acc = acc + parts[p]
        want_x = base + acc.to(dt)
    else:
        want_x = base
    want = R.rms_norm(want_x, w, 1e-6)
    x_out = torch.full((n, cols), 7.0, dtype=dt, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    got = K.gather_add_rms_norm(src, rows, w, 1e-6, delta=delta, parts=parts, x_out=x_out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert torch.equal(src, keep)
    assert torch.equal(x_out, want_x)
    if dt == torch.bfloat16:
        d = _ulp_diff_bf16(got, want)
        assert d.max().item() <= 1 and (d > 0).float().mean().item() < 0.02
    else:
        torch.testing.assert_close(got, want, rtol=2e-6, atol=2e-6)
    bad = i32([2, 50, -1])
    out = torch.zeros(3, cols, dtype=dt, device=dev)
    K.gather_add_rms_norm(src, bad, w, 1e-6, out=out, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) & K.DEV_BOUNDS
    assert torch.equal(out[1:], torch.zeros_like(out[1:]))
    torch.testing.assert_close(out[0].float(), R.rms_norm(src[2:3], w, 1e-6)[0].float())


def test_splitk_projection_matches_one_gemm():
    """o_proj / down_proj as a batched GEMM over K slices + the partial sums in
    add+RMSNorm give the residual and normed rows of one GEMM + add+RMSNorm, up
    to the bf16 rounding of a differently ordered fp32 sum (decode step shapes)."""
    import torch.nn.functional as F
    from hayate_b200.model import linear_splitk
    g = torch.Generator(device=dev).manual_seed(3)
    for k, s in ((4096, 8), (9728, 8), (9728, 4)):
        a = torch.randn(16, k, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(2560, k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn(16, 2560, device=dev, generator=g).to(torch.bfloat16)
        ln = (1 + 0.1 * torch.randn(2560, device=dev, generator=g)).to(torch.bfloat16)
        parts = linear_splitk(a, w, s)
        assert parts.shape == (s, 16, 2560) and parts.dtype == torch.float32
        x1, x2 = x.clone(), x.clone()
        y1 = K.add_rms_norm(x1, ln, 1e-6, delta=F.linear(a, w))
        y2 = K.add_rms_norm_splitk(x2, ln, 1e-6, parts)
        torch.cuda.synchronize()
        # the two fp32 sums may round delta to neighbouring bf16 values (one
        # ulp of delta, |delta| ~ 1.3-2): a few elements move by that much
        for got, want in ((x2, x1), (y2, y1)):
            torch.testing.assert_close(got.float(), want.float(), rtol=1e-2, atol=3e-2)
            assert (got != want).float().mean().item() < 0.05


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_silu_mul_vs_reference(dt):
    gu = (torch.randn(19, 2 * 9728, device=dev) * 2).to(dt)
    got = K.silu_mul(gu)
    I = 9728
    want = torch.nn.functional.silu(gu[:, :I]) * gu[:, I:]   # linear.py:13
    torch.cuda.synchronize()
    if dt == torch.bfloat16:
        d = _ulp_diff_bf16(got, want)
        assert d.max().item() <= 1 and (d > 0).float().mean().item() < 0.01
    else:
        torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)


# ------------------------------------------------------- bounded device waits
def test_bounded_wait_gives_up_and_reports():
    """A wait nothing completes ends after its limit with HY_DEV_TIMEOUT set; the
    context stays usable (a kernel runs correctly right after)."""
    from hayate_b200 import _lib
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = _lib.load().hy_selftest_wait_timeout(err.data_ptr(), 50, done.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(done.item()) == 1
    assert int(err.item()) & K.DEV_TIMEOUT
    x = torch.randn(3, 1000, device=dev)
    out = torch.empty(3, dtype=torch.int32, device=dev)
    K.argmax(x, out)
    assert torch.equal(out, torch.argmax(x, -1).int())


def test_exp2_poly_accuracy_against_cuda_exp2():
    """The prefill softmax's polynomial 2^x (range reduction + a degree-3
    minimax polynomial on the FMA pipe) against CUDA's exp2f (torch.exp2 on the
    device): relative error below 1e-4 on (-126, 8] (weights are rounded to
    bf16, 2^-9 relative, before the P V product) and 2e-4 at -126 (a subnormal
    result); exactly 0 below -126 and at -inf."""
    from hayate_b200 import _lib
    x = torch.cat([torch.linspace(-125.99, 8.0, 200001, device=dev),
                   torch.tensor([0.0, -0.5, 0.5, 1.0, -1.0, 7.5, -125.5], device=dev)])
    y = torch.empty_like(x)
    assert _lib.load().hy_selftest_exp2_poly(x.data_ptr(), y.data_ptr(), x.numel(),
                                             torch.cuda.current_stream().cuda_stream) == 0
    want = torch.exp2(x)
    rel = ((y - want).abs() / want).max().item()
    assert rel < 1e-4, rel
    edge = torch.tensor([-126.0], device=dev)
    ye = torch.empty_like(edge)
    _lib.load().hy_selftest_exp2_poly(edge.data_ptr(), ye.data_ptr(), 1,
                                      torch.cuda.current_stream().cuda_stream)
    assert ((ye - torch.exp2(edge)).abs() / torch.exp2(edge)).item() < 2e-4
    lo = torch.tensor([-126.5, -127.0, -200.0, float("-inf")], device=dev)
    out = torch.full_like(lo, 5.0)
    _lib.load().hy_selftest_exp2_poly(lo.data_ptr(), out.data_ptr(), lo.numel(),
                                      torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert torch.equal(out, torch.zeros_like(lo))
