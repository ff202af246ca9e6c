"""loom_lm_head_argmax (greedy selection fused into the LM-head GEMM) against a plain PyTorch fp32
reference of the same product.

The fused kernel accumulates exact bf16 products in f32 on the tensor cores, in an order no other GEMM
shares, so its logits agree with torch's fp32 matmul to rounding (TOL below), not bit for bit. The checks:
  * the chosen id's reference logit is within TOL of the reference row maximum (it is an argmax);
  * where the reference top-2 gap exceeds 2 * TOL, the id is exactly the reference argmax;
  * the returned logit and log-sum-exp match the reference within TOL (absolute, logits of order 1-10);
  * the selection rule of Generator::argmax (src/core/generation.cpp:64-74) on exactly equal logits
    (duplicated weight rows: the lowest id wins) and a NaN at id 0 (it wins).
"""
import pytest
import torch

import loom_select as ls

pytestmark = pytest.mark.gpu

TOL = 2e-3


def _case(rows, hdim, vocab, seed, plant=True):
    g = torch.Generator(device="cuda").manual_seed(seed)
    hidden = torch.randn(rows, hdim, generator=g, device="cuda").to(torch.bfloat16)
    weight = (torch.randn(vocab, hdim, generator=g, device="cuda") * (1.0 / hdim ** 0.5)).to(torch.bfloat16)
    if plant:
        # every third row gets a clear winner: a weight row aligned with the hidden state
        win = torch.randint(0, vocab, (rows,), generator=g, device="cuda")
        for r in range(0, rows, 3):
            weight[win[r]] = (hidden[r].float() * (3.0 / hdim ** 0.5)).to(torch.bfloat16)
    return hidden, weight


def _reference(hidden, weight):
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return hidden.float() @ weight.float().t()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = old


def _check(hidden, weight):
    ids, logit, lse = ls.lm_head_argmax(hidden, weight)
    torch.cuda.synchronize()
    ref = _reference(hidden, weight)
    top2 = ref.topk(2, dim=1)
    ref_max = top2.values[:, 0]
    ids_l = ids.long()
    assert ids_l.min() >= 0 and ids_l.max() < weight.shape[0]
    chosen = ref.gather(1, ids_l[:, None])[:, 0]
    assert torch.all(chosen >= ref_max - TOL), "a chosen id is not an argmax of the reference logits"
    clear = (top2.values[:, 0] - top2.values[:, 1]) > 2 * TOL
    assert torch.equal(ids_l[clear], top2.indices[clear, 0])
    assert torch.allclose(logit, ref_max, atol=TOL, rtol=0)
    assert torch.allclose(lse, torch.logsumexp(ref, dim=1), atol=TOL, rtol=0)
    return ids


@pytest.mark.parametrize("rows,hdim,vocab", [
    (1, 2048, 151936),     # one decode row, Qwen-size vocabulary
    (5, 1024, 1000),       # vocabulary not a multiple of the 256-id tile
    (200, 512, 4099),      # two row tiles, the second ragged; a 3-id last vocabulary tile
    (128, 64, 256),        # one K slice, exactly one tile
    (16, 1024, 151936),    # the largest call that loads a 16-row hidden tile
    (17, 512, 30011),      # the smallest that loads the full 128-row tile
    (1024, 2048, 151936),  # the 1024-row batch
])
def test_lm_head_matches_fp32_reference(rows, hdim, vocab):
    hidden, weight = _case(rows, hdim, vocab, seed=rows * 7 + hdim + vocab)
    _check(hidden, weight)


def test_lm_head_without_optional_outputs():
    hidden, weight = _case(33, 256, 5000, seed=3)
    ids_full, _, _ = ls.lm_head_argmax(hidden, weight)
    ids_only, logit, lse = ls.lm_head_argmax(hidden, weight, want_logit=False, want_lse=False)
    assert logit is None and lse is None
    assert torch.equal(ids_full, ids_only)


def test_lm_head_equal_logits_lowest_id_wins():
    rows, hdim, vocab = 6, 256, 70001
    hidden, weight = _case(rows, hdim, vocab, seed=11, plant=False)
    # rows 0-2: the winner duplicated in another tile (100 and 70000); rows 3-5: in the same tile (300, 301)
    for r, (a, b) in enumerate([(100, 70000)] * 3 + [(300, 301)] * 3):
        w = (hidden[r].float() * (4.0 / hdim ** 0.5)).to(torch.bfloat16)
        weight[a] = w
        weight[b] = w
    ids, logit, _ = ls.lm_head_argmax(hidden, weight)
    torch.cuda.synchronize()
    ref = _reference(hidden, weight)
    expect = [100, 100, 100, 300, 300, 300]
    for r in range(rows):
        # the two duplicated columns hold the same sum; only a row whose maximum they are is checked
        if ref[r].argmax().item() in (expect[r], 70000 if expect[r] == 100 else 301):
            assert ids[r].item() == expect[r], (r, ids[r].item())


def test_lm_head_nan_at_id_zero_wins():
    hidden, weight = _case(4, 128, 3000, seed=5)
    weight[0] = float("nan")
    weight[1] = float("nan")
    ids, logit, lse = ls.lm_head_argmax(hidden, weight)
    torch.cuda.synchronize()
    assert ids.tolist() == [0, 0, 0, 0]
    assert torch.isnan(logit).all()


def test_lm_head_nan_elsewhere_never_wins():
    hidden, weight = _case(4, 128, 3000, seed=6)
    weight[1234] = float("nan")
    ids = _check_nan_free(hidden, weight, skip=1234)
    assert (ids != 1234).all()


def _check_nan_free(hidden, weight, skip):
    ids, _, _ = ls.lm_head_argmax(hidden, weight, want_lse=False)
    torch.cuda.synchronize()
    ref = _reference(hidden, weight)
    ref[:, skip] = -float("inf")
    ref_max = ref.max(dim=1).values
    chosen = ref.gather(1, ids.long()[:, None])[:, 0]
    assert torch.all(chosen >= ref_max - TOL)
    return ids


def test_lm_head_two_calls_share_a_workspace():
    ws = ls.Workspace(torch.device("cuda", torch.cuda.current_device()))
    h1, w1 = _case(300, 256, 20000, seed=21)
    h2, w2 = _case(7, 512, 9000, seed=22)
    a1, _, _ = ls.lm_head_argmax(h1, w1, workspace=ws)
    a2, _, _ = ls.lm_head_argmax(h2, w2, workspace=ws)
    b1, _, _ = ls.lm_head_argmax(h1, w1)
    torch.cuda.synchronize()
    assert torch.equal(a1, b1)
    assert ws.read_status() == ls.OK
    _check(h2, w2)
