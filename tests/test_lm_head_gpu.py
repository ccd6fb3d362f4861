"""hy_lm_head_argmax: the LM head and the greedy choice in one tcgen05 kernel.

The reference computes bf16 logits (hayate/model/qwen.py:122-123) and takes
torch.argmax of the last position's row (hayate/engine/engine.py:69-71).  The
oracle here is the same: fp32 products summed in fp32 (torch, TF32 off),
rounded to bf16, argmax with torch's rules.  The kernel sums in another order,
so a logit whose fp32 sum lies within rounding distance of a bf16 boundary may
round to the neighbouring bf16 value; its choice must therefore be the
oracle's argmax, or a column whose bf16 logit is within one bf16 step of the
row maximum (a near tie), and must equal the oracle's on nearly every row.
Ties, NaN, signed zeros and the ragged last vocabulary tile are checked
exactly on planted inputs.
"""
import pytest
import torch
import torch.nn.functional as F

from hayate_b200 import kernels as K

pytestmark = pytest.mark.gpu

VOCAB, HIDDEN = 151936, 2560


def oracle_logits(x, w):
    """bf16-rounded logits of fp32 products summed in fp32, as floats."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return (x.float() @ w.float().t()).bfloat16().float()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def bf16_step(v: torch.Tensor) -> torch.Tensor:
    """Spacing of bf16 values at |v| (8 significant bits)."""
    e = torch.floor(torch.log2(v.abs().clamp_min(2.0 ** -126)))
    return torch.exp2(e - 7)


def check_choice(tokens, logits, min_exact):
    want = logits.argmax(dim=1)
    mx = logits.max(dim=1).values
    got = logits.gather(1, tokens.long().view(-1, 1)).view(-1)
    assert bool((tokens >= 0).all()) and bool((tokens < logits.shape[1]).all())
    assert bool((got >= mx - bf16_step(mx)).all()), "a choice is not within one bf16 step of the max"
    exact = (tokens.long() == want).float().mean().item()
    assert exact >= min_exact, exact
    return exact


def run(x, w, ws=None, err=None):
    out = torch.full((x.shape[0],), -7, dtype=torch.int32, device="cuda")
    if ws is None:
        ws = torch.zeros(K.lm_head_argmax_workspace_size(), dtype=torch.uint8, device="cuda")
    K.lm_head_argmax(x, w, out, ws, err)
    torch.cuda.synchronize()
    return out


@pytest.fixture(scope="module")
def qwen_head():
    g = torch.Generator(device="cuda").manual_seed(0)
    w = (torch.randn(VOCAB, HIDDEN, device="cuda", generator=g) * 0.02).bfloat16()
    return w, g


@pytest.mark.parametrize("rows", [1, 10, 128, 129, 256, 300])
def test_lm_head_argmax_matches_the_oracle_at_qwen3_sizes(qwen_head, rows):
    w, g = qwen_head
    x = torch.randn(rows, HIDDEN, device="cuda", generator=g).bfloat16()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    ws = torch.zeros(K.lm_head_argmax_workspace_size(), dtype=torch.uint8, device="cuda")
    tok = run(x, w, ws, err)
    assert int(err.item()) == 0
    assert int(ws.count_nonzero().item()) == 0          # the call left its workspace zeroed
    check_choice(tok, oracle_logits(x, w), 0.95 if rows >= 20 else 0.0)
    # the path it replaces: cuBLAS bf16 logits, then hy_argmax
    unfused = torch.empty(rows, dtype=torch.int32, device="cuda")
    K.argmax(F.linear(x, w), unfused)
    torch.cuda.synchronize()
    same = (unfused == tok).float().mean().item()
    assert same >= (0.95 if rows >= 20 else 0.0)


def test_lm_head_argmax_consecutive_calls_share_one_workspace(qwen_head):
    w, g = qwen_head
    ws = torch.zeros(K.lm_head_argmax_workspace_size(), dtype=torch.uint8, device="cuda")
    outs, xs = [], []
    for rows in (200, 7, 200):
        x = torch.randn(rows, HIDDEN, device="cuda", generator=g).bfloat16()
        outs.append(run(x, w, ws))
        xs.append(x)
    for x, tok in zip(xs, outs):
        assert torch.equal(tok, run(x, w))                # a fresh workspace gives the same
        check_choice(tok, oracle_logits(x, w), 0.9)


def test_lm_head_argmax_ties_nan_zeros_and_the_ragged_last_tile():
    g = torch.Generator(device="cuda").manual_seed(3)
    vocab, hidden, rows = 1000, 128, 8                 # 1000 = 4 x 208 + 168: a ragged last tile
    x = torch.randn(rows, hidden, device="cuda", generator=g).bfloat16()
    w = (torch.randn(vocab, hidden, device="cuda", generator=g) * 0.02).bfloat16()
    # equal rows of W give bit-equal logits: the lower index wins
    w[3] = (x[0].float() * 0.5).bfloat16()
    w[900] = w[3]
    # the maximum of row 1 in the last, partial tile
    w[999] = (x[1].float() * 0.5).bfloat16()
    tok = run(x, w)
    assert int(tok[0]) == 3 and int(tok[1]) == 999
    check_choice(tok, oracle_logits(x, w), 0.0)
    # all logits negative: the zero-filled columns past the vocabulary must not win
    xp = x.abs()
    wn = -w.abs()
    tok = run(xp, wn)
    lg = oracle_logits(xp, wn)
    assert bool((lg < 0).all())
    check_choice(tok, lg, 0.0)
    # NaN counts above every number, the first NaN column winning
    wnan = w.clone()
    wnan[777, 5] = float("nan")
    wnan[950, 0] = float("nan")
    assert torch.equal(run(x, wnan), torch.full((rows,), 777, dtype=torch.int32, device="cuda"))
    # all logits zero (either sign): index 0
    z = torch.zeros(rows, hidden, device="cuda", dtype=torch.bfloat16)
    assert torch.equal(run(z, w), torch.zeros(rows, dtype=torch.int32, device="cuda"))


def test_lm_head_argmax_rejects_bad_arguments():
    from hayate_b200 import _lib
    lib = _lib.load()
    buf = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    p = buf.data_ptr()
    # hidden not a multiple of 64
    assert lib.hy_lm_head_argmax(p, 100, 2, p, 100, 10, 100, p, p, None, None) == -3
    # no workspace
    assert lib.hy_lm_head_argmax(p, 128, 2, p, 128, 10, 128, p, None, None, None) == -1
    # misaligned x
    assert lib.hy_lm_head_argmax(p + 2, 128, 2, p, 128, 10, 128, p, p, None, None) == -1
    # zero rows: nothing to do
    assert lib.hy_lm_head_argmax(None, 128, 0, None, 128, 10, 128, None, None, None, None) == 0
