"""loom_sample_rows_noalloc (the sampling chain on the library's own fixed scratch) against loom_sample_rows.

Collected last on purpose: it must give the same results whether it runs alone in a fresh process
(its first call looks the scratch up on the device) or after every other test. Calls in a row
share the scratch, so each one after the first also checks that the one before left it fit for reuse. Ids and top-k
sets must be equal; probabilities within 1e-5 relative, log-probs within 1e-5 on the probability
scale (the tolerance of the sampling tests; both entry points run the same kernel).
"""
import ctypes

import numpy as np
import pytest
import torch

import synth

pytestmark = pytest.mark.gpu
PROB_RTOL = 1e-5
LOGP_TOL = 1e-5


def with_workspace(sel, x, hist, u, T, r, k, p):
    ids, prob, lp, topk = sel.sample_rows(x, u, T, r, k, p, history=hist, want_logp=True, want_topk=True)
    return ids, prob, lp, topk


def without_workspace(sel, x, hist, u, T, r, k, p):
    rows, dev = x.shape[0], x.device
    ids = torch.empty(rows, dtype=torch.int32, device=dev)
    prob = torch.empty(rows, dtype=torch.float32, device=dev)
    lp = torch.empty(rows, dtype=torch.float32, device=dev)
    topk = torch.empty(rows, k, dtype=torch.int32, device=dev)
    status = torch.full((1,), -7, dtype=torch.int32, device=dev)
    sel.sample_rows_noalloc_into(x, u, ids, prob, T, r, k, p, history=hist, out_logp=lp, out_topk=topk,
                                 out_status=status)
    return ids, prob, lp, topk, status


def assert_same(got, want):
    g_ids, g_prob, g_lp, g_topk = (t.cpu().numpy() for t in got[:4])
    w_ids, w_prob, w_lp, w_topk = (t.cpu().numpy() for t in want)
    np.testing.assert_array_equal(g_topk, w_topk)
    np.testing.assert_array_equal(g_ids, w_ids)
    gp, wp = g_prob.astype(np.float64), w_prob.astype(np.float64)
    assert np.all((np.isnan(gp) & np.isnan(wp)) | (np.abs(gp - wp) <= PROB_RTOL * np.abs(wp)))
    gl, wl = g_lp.astype(np.float64), w_lp.astype(np.float64)
    fin = np.isfinite(wl)
    assert np.all(np.isnan(gl[np.isnan(wl)]))
    assert np.all(np.abs(gl[fin] - wl[fin]) <= LOGP_TOL * np.maximum(1.0, np.abs(wl[fin])))


def test_calls_in_a_row_match_loom_sample_rows(sel, dev):
    # call 1: [512, 151936] f32 with a 256-id history (at least as many rows as CTAs: whole rows per
    # CTA, no tickets); call 2: [96, 262144] bf16 without history at the largest top-k this entry point
    # takes (fewer rows than CTAs: rows cut across CTAs, merged through the tickets and records of the
    # scratch); call 3: [40, 151936] f32 with history, again cut across CTAs, on the tickets call 2
    # just used. All are enqueued before any is read back, so each runs on the scratch the one before
    # it left behind.
    x1, h1, u1 = synth.sample_chain(512, seed=41, device="cuda")
    x2, u2 = synth.gemma_vocab(96, seed=43, device="cuda")
    x3, h3, u3 = synth.sample_chain(40, seed=47, device="cuda")
    calls = [(x1, h1, u1, 0.7, 1.1, 40, 0.9), (x2, None, u2, 1.3, 1.0, 64, 0.95), (x3, h3, u3, 0.8, 1.2, 50, 0.8)]
    got = [without_workspace(sel, *c) for c in calls]
    torch.cuda.synchronize()
    want = [with_workspace(sel, *c) for c in calls]
    torch.cuda.synchronize()
    for g, w in zip(got, want):
        assert g[4].item() == sel.OK
        assert_same(g, w)


def test_device_status_and_size_limit(sel, dev):
    x, hist, u = synth.sample_chain(4, seed=5, device="cuda")
    hist[2, 7] = x.shape[1]                              # an id outside the vocabulary
    ids, _, _, topk, status = without_workspace(sel, x, hist, u, 0.7, 1.1, 40, 0.9)
    torch.cuda.synchronize()
    assert status.item() == sel.EHISTORY
    assert ids[2].item() == -1 and bool(torch.all(topk[2] == -1))
    # the next call clears the status word itself
    hist[2, 7] = 0
    _, _, _, _, status = without_workspace(sel, x, hist, u, 0.7, 1.1, 40, 0.9)
    torch.cuda.synchronize()
    assert status.item() == sel.OK
    # top_k beyond the scratch's limit is refused before anything is enqueued
    limit = 64
    out = torch.empty(4, dtype=torch.int32, device=dev)
    prob = torch.empty(4, dtype=torch.float32, device=dev)
    p = sel.SampleParams(0.7, 1.0, limit + 1, 0.9)
    rc = sel.lib().loom_sample_rows_noalloc(x.data_ptr(), 0, 4, x.shape[1], x.shape[1], None, 0, u.data_ptr(),
                                            ctypes.byref(p), out.data_ptr(), prob.data_ptr(), None, None, None,
                                            None)
    assert rc == sel.ESHAPE
