"""Vocabulary-sharded sampling (K2 partial + K4 merge) on one GPU.

The 8 shards run one after another on cuda:0 and their records are concatenated in rank order --
exactly what ncclAllGather produces on 8 GPUs -- then merged. The result must equal the unsharded
chain: ids and top-k sets bit-exact, probabilities within 1e-5 relative, log-probs within 1e-5 on
the probability scale.
"""
import os

import numpy as np
import pytest
import torch

import synth
from test_gpu_sample import assert_parity, host_of

pytestmark = pytest.mark.gpu
NT = os.cpu_count() or 4


def sharded(sel, x, u, T, r, k, p, G, hist=None):
    rows, V = x.shape
    rb = sel.shard_record_bytes(k)
    recs = torch.empty(G, rows * rb, dtype=torch.uint8, device=x.device)
    for g in range(G):
        lo, hi = g * V // G, (g + 1) * V // G
        sel.shard_partial_into(x[:, lo:hi], recs[g], lo, V, T, r, k, p, history=hist)
    ids = torch.empty(rows, dtype=torch.int32, device=x.device)
    prob = torch.empty(rows, dtype=torch.float32, device=x.device)
    logp = torch.empty(rows, dtype=torch.float32, device=x.device)
    topk = torch.empty(rows, k, dtype=torch.int32, device=x.device)
    sel.shard_merge_into(recs, G, rows, u, ids, prob, T, k, p, logp, topk)
    torch.cuda.synchronize()
    return dict(ids=ids.cpu().numpy(), prob=prob.cpu().numpy(), logp=logp.cpu().numpy(), topk=topk.cpu().numpy())


def test_gemma_vocab_8_shards(sel, dev, oracle):
    # [256, 262144] bf16, N(0, 2.5^2) + Zipf(1.1) log-bias, T 1, top-k 64, top-p 0.95, 8 shards of 32768
    x, u = synth.gemma_vocab(256, device="cuda")
    got = sharded(sel, x, u, 1.0, 1.0, 64, 0.95, 8)
    want = oracle.sample_rows(host_of(x), u.cpu().numpy(), 1.0, 1.0, 64, 0.95, None, nthreads=NT)
    assert_parity(got, want)


def test_shards_with_penalty_and_ties(sel, dev, oracle):
    rng = np.random.default_rng(12)
    V, rows, G = 40000, 10, 8
    x = rng.normal(0, 2, (rows, V)).astype(np.float32)
    x[3, 4000:26000] = 5.0                         # a tie spanning several shards
    x[4, :] = np.nan
    x[4, 39990] = 1.0                              # fewer non-NaN values than k, in the last shard
    xt = torch.from_numpy(x).to(dev)
    hist = torch.from_numpy(rng.integers(0, V, (rows, 100)).astype(np.int32)).to(dev)
    u = torch.from_numpy(rng.random(rows).astype(np.float32)).to(dev)
    got = sharded(sel, xt, u, 0.9, 1.3, 64, 0.9, G, hist)
    want = oracle.sample_rows(x, u.cpu().numpy(), 0.9, 1.3, 64, 0.9, hist.cpu().numpy(), nthreads=NT)
    assert_parity(got, want)


def test_shard_records_match_oracle_records(sel, dev, oracle):
    rng = np.random.default_rng(2)
    V, rows, G, k = 16384, 6, 4, 64
    x = rng.normal(0, 2.5, (rows, V)).astype(np.float32)
    xt = torch.from_numpy(x).to(dev)
    rb = sel.shard_record_bytes(k)
    for g in range(G):
        lo, hi = g * V // G, (g + 1) * V // G
        rec = torch.zeros(rows * rb, dtype=torch.uint8, device=dev)
        sel.shard_partial_into(xt[:, lo:hi], rec, lo, V, 1.0, 1.0, k)
        got = rec.cpu().numpy().reshape(rows, rb)
        st, want = oracle.shard_partial(np.ascontiguousarray(x[:, lo:hi]), lo, V, 1.0, 1.0, k)
        assert st == 0
        want = want.reshape(rows, rb)
        # count and the (value, id) pairs are exact; (m, s) are partial sums within tolerance
        np.testing.assert_array_equal(got[:, 0:4], want[:, 0:4])
        np.testing.assert_array_equal(got[:, 16:], want[:, 16:])
        gm, wm = got[:, 4:12].copy().view(np.float32), want[:, 4:12].copy().view(np.float32)
        np.testing.assert_allclose(gm, wm, rtol=1e-5)
