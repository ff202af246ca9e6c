"""The fused sampling chain on the GPU (K2) against the oracle.

loom.cpp has no sampler, so parity is with the oracle (pinned by the chain's written semantics and
an independent numpy restatement in test_oracle_semantics.py), on the same input bytes. Ids and
top-k sets must be bit-exact; probabilities within 1e-5 relative (the bar stated for this stage; the
kernels are built to match bit for bit, which test_probabilities_bit_exact checks); log-probs within
1e-5 on the probability scale (|d logp| <= 1e-5 * max(1, |logp|)).
"""
import os

import numpy as np
import pytest
import torch

import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NT = os.cpu_count() or 4
PROB_RTOL = 1e-5
LOGP_TOL = 1e-5


def run_gpu(sel, x, hist, u, T, r, k, p, logp=True, workspace=None):
    ids, prob, lp, topk = sel.sample_rows(x, u, T, r, k, p, history=hist, want_logp=True, want_topk=True,
                                          workspace=workspace)
    torch.cuda.synchronize()
    return dict(ids=ids.cpu().numpy(), prob=prob.cpu().numpy(), logp=lp.cpu().numpy(), topk=topk.cpu().numpy())


def host_of(x):
    return synth.bf16_bits(x) if x.dtype == torch.bfloat16 else x.cpu().numpy()


def assert_parity(got, want, check_logp=True):
    np.testing.assert_array_equal(got["topk"], want["topk"])
    np.testing.assert_array_equal(got["ids"], want["ids"])
    gp, wp = got["prob"].astype(np.float64), want["prob"].astype(np.float64)
    both_nan = np.isnan(gp) & np.isnan(wp)
    assert np.all(both_nan | (np.abs(gp - wp) <= PROB_RTOL * np.abs(wp))), (gp, wp)
    if check_logp:
        gl, wl = got["logp"].astype(np.float64), want["logp"].astype(np.float64)
        fin = np.isfinite(wl)
        assert np.all(np.isnan(gl[np.isnan(wl)]))
        assert np.all(np.abs(gl[fin] - wl[fin]) <= LOGP_TOL * np.maximum(1.0, np.abs(wl[fin]))), (gl, wl)


def vs_oracle(sel, oracle, x, hist, u, T, r, k, p, workspace=None):
    got = run_gpu(sel, x, hist, u, T, r, k, p, workspace=workspace)
    want = oracle.sample_rows(host_of(x), u.cpu().numpy(), T, r, k, p,
                              None if hist is None else hist.cpu().numpy(), nthreads=NT)
    assert want["status"] == 0
    assert_parity(got, want)
    return got, want


def test_fixture_cases(sel, dev):
    g = np.load(os.path.join(GOLDEN, "sample_oracle.npz"))
    x = torch.from_numpy(g["x"]).to(dev)
    hist = torch.from_numpy(g["hist"]).to(dev)
    u = torch.from_numpy(g["u"]).to(dev)
    for name in ("chain", "boost", "greedy", "k1", "kbig"):
        T, r, k, p = g[f"{name}_params"]
        got = run_gpu(sel, x, hist, u, float(T), float(r), int(k), float(p))
        want = dict(ids=g[f"{name}_ids"], prob=g[f"{name}_prob"], logp=g[f"{name}_logp"], topk=g[f"{name}_topk"])
        assert_parity(got, want)


def test_chain_64_rows(sel, dev, oracle):
    # [64, 151936] f32 N(0, 3^2), 256-id history, penalty 1.1, T 0.7, top-k 40, top-p 0.9
    x, hist, u = synth.sample_chain(64, device="cuda")
    vs_oracle(sel, oracle, x, hist, u, 0.7, 1.1, 40, 0.9)


def test_probabilities_bit_exact(sel, dev, oracle):
    x, hist, u = synth.sample_chain(64, seed=9, device="cuda")
    got, want = vs_oracle(sel, oracle, x, hist, u, 0.7, 1.1, 40, 0.9)
    np.testing.assert_array_equal(got["prob"].view(np.uint32), want["prob"].view(np.uint32))


@pytest.mark.parametrize("rows", [1, 2, 16, 128, 149])
def test_split_rows(sel, dev, oracle, rows):
    # few rows: each row is cut across several CTAs, merged by the last one
    x, hist, u = synth.sample_chain(rows, seed=rows, device="cuda")
    vs_oracle(sel, oracle, x, hist, u, 0.7, 1.1, 40, 0.9)


@pytest.mark.parametrize("rows,k", [(300, 40), (597, 40), (297, 300)])
def test_whole_row_ranges(sel, dev, oracle, rows, k):
    # at least as many rows as CTAs: each CTA takes whole rows, the same number each (300 rows on a
    # B200: 150 CTAs of 2; 597: 199 of 3), for both kernels (k <= 128 and k > 128)
    x, hist, u = synth.sample_chain(rows, seed=rows + 7, device="cuda")
    vs_oracle(sel, oracle, x, hist, u, 0.7, 1.1, k, 0.9)


@pytest.mark.parametrize("T,r,k,p", [(1.0, 1.0, 1, 1.0), (0.3, 1.5, 1024, 0.95), (2.0, 0.7, 64, 0.5),
                                     (0.0, 1.1, 40, 0.9), (1e-3, 1.0, 7, 0.999), (25.0, 1.05, 200, 1.0)])
def test_parameters(sel, dev, oracle, T, r, k, p):
    x, hist, u = synth.sample_chain(20, seed=int(k * 10 + T * 7), device="cuda")
    vs_oracle(sel, oracle, x, hist, u, T, r, k, p)


def _adversarial_rows(rng, rows, V):
    x = rng.normal(0, 3, (rows, V)).astype(np.float32)
    x[0, :] = 1.5                                        # all equal: the lowest k ids
    x[1, :] = np.round(x[1, :])                          # many ties
    x[2, rng.integers(0, V, 500)] = np.nan
    x[3, 0] = np.nan
    x[4, rng.integers(0, V, 3)] = np.inf
    x[5, :] = np.nan
    x[5, rng.integers(0, V, 4)] = 0.5                    # fewer non-NaN values than k
    x[6, :] = -np.inf
    x[7, :] = np.arange(V, dtype=np.float32) * 1e-3      # ascending: every element passes
    x[8, :] = -np.arange(V, dtype=np.float32) * 1e-3     # descending
    x[9, ::2] = -0.0
    x[9, 1::2] = 0.0
    x[10, :] = np.float32(3.0) * np.float32(1.0000001) ** np.arange(V).astype(np.float32)
    x[11, V // 2:V // 2 + 3000] = 8.0                    # a wide tie in the middle of the row
    return x


@pytest.mark.parametrize("V,rows", [(1000, 12), (8191, 12), (70001, 12), (151936, 12)])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_adversarial_rows(sel, dev, oracle, V, rows, dtype):
    rng = np.random.default_rng(V)
    x = torch.from_numpy(_adversarial_rows(rng, rows, V)).to(dev)
    if dtype == "bf16":
        x = x.to(torch.bfloat16)
    hist = torch.from_numpy(rng.integers(0, V, (rows, 64)).astype(np.int32)).to(dev)
    hist[0, :] = 0                                       # one id, repeated
    u = torch.from_numpy(rng.random(rows).astype(np.float32)).to(dev)
    vs_oracle(sel, oracle, x, hist, u, 0.8, 1.2, 40, 0.9)
    vs_oracle(sel, oracle, x, hist, u, 0.0, 1.2, 16, 1.0)


def test_strided_rows(sel, dev, oracle):
    rng = np.random.default_rng(4)
    V, pad, rows = 151936, 3, 7
    full = torch.from_numpy(rng.normal(0, 3, (rows, V + pad)).astype(np.float32)).to(dev)
    x = full[:, :V]
    hist = torch.from_numpy(rng.integers(0, V, (rows, 256)).astype(np.int32)).to(dev)
    u = torch.rand(rows, device=dev)
    got = run_gpu(sel, x, hist, u, 0.7, 1.1, 40, 0.9)
    want = oracle.sample_rows(np.ascontiguousarray(x.cpu().numpy()), u.cpu().numpy(), 0.7, 1.1, 40, 0.9,
                              hist.cpu().numpy(), nthreads=NT)
    assert_parity(got, want)


def test_no_history(sel, dev, oracle):
    x, _, u = synth.sample_chain(8, seed=77, device="cuda")
    vs_oracle(sel, oracle, x, None, u, 0.7, 1.0, 40, 0.9)


def test_history_out_of_range(sel, dev):
    x, hist, u = synth.sample_chain(4, seed=5, device="cuda")
    hist[2, 7] = x.shape[1]
    ws = sel.Workspace(dev)
    got = run_gpu(sel, x, hist, u, 0.7, 1.1, 40, 0.9, workspace=ws)
    assert ws.read_status() == sel.EHISTORY
    assert got["ids"][2] == -1 and np.all(got["topk"][2] == -1)
    assert np.all(got["ids"][[0, 1, 3]] >= 0)
    assert ws.read_status() == sel.OK                    # read_status clears it


@pytest.mark.parametrize("rows", [1024])
def test_full_batch(sel, dev, oracle, rows):
    # the headline shape: [1024, 151936] f32
    x, hist, u = synth.sample_chain(rows, device="cuda")
    vs_oracle(sel, oracle, x, hist, u, 0.7, 1.1, 40, 0.9)


def test_repeat_calls_same_result(sel, dev):
    x, hist, u = synth.sample_chain(33, seed=3, device="cuda")
    ws = sel.Workspace(dev)
    first = run_gpu(sel, x, hist, u, 0.7, 1.1, 40, 0.9, workspace=ws)
    for _ in range(10):
        again = run_gpu(sel, x, hist, u, 0.7, 1.1, 40, 0.9, workspace=ws)
        for key in ("ids", "topk", "prob"):
            np.testing.assert_array_equal(first[key], again[key])
    assert ws.read_status() == sel.OK


def test_one_workspace_for_calls_of_every_size(sel, dev, oracle):
    # One workspace serves calls of any size and kind: growing and shrinking row counts, another k,
    # argmax and CTC calls in between (the tickets must stay where every call expects them).
    ws = sel.Workspace(dev)
    for rows, k in [(16, 40), (128, 40), (1, 64), (149, 1024), (2, 40), (128, 40), (5, 3)]:
        x, hist, u = synth.sample_chain(rows, seed=rows + k, device="cuda")
        vs_oracle(sel, oracle, x, hist, u, 0.7, 1.1, k, 0.9, workspace=ws)
        out = torch.empty(rows, dtype=torch.int32, device=dev)
        sel.argmax_rows_into(x, out, workspace=ws)
        np.testing.assert_array_equal(out.cpu().numpy(), oracle.argmax_rows(x.cpu().numpy(), nthreads=NT))
        f = synth.ctc_frames(3, 500 + rows, seed=rows, device="cuda")
        ids, frames, lens = sel.ctc_greedy(f, synth.CTC_BLANK, workspace=ws)
        seqs, _, _ = oracle.ctc_greedy(f.cpu().numpy(), synth.CTC_BLANK, nthreads=NT)
        for utt, (wi, wf) in enumerate(seqs):
            n = int(lens[utt].item())
            np.testing.assert_array_equal(ids[utt, :n].cpu().numpy(), wi)
    assert ws.read_status() == sel.OK
