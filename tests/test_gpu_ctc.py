"""Greedy CTC decode on the GPU (K3) against loom.cpp's own ctc_greedy_decode and the oracle.

Token sequences, frame offsets and per-frame ids are bit-exact; per-frame log-probs within 1e-5 on
the probability scale. Citations are paths in the loom.cpp tree.
"""
import os

import numpy as np
import pytest
import torch

import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NT = os.cpu_count() or 4


def test_known_answers(sel, dev):
    # tests/ci/test_ctc_decode.cpp:12-38
    g = np.load(os.path.join(GOLDEN, "ctc_reference.npz"))
    for case in ("ka1", "ka2", "ka3"):
        x = torch.from_numpy(g[case]).to(dev)
        assert sel.ctc_greedy_decode(x, 3) == g[f"{case}_expected"].tolist(), case


def test_reference_fixture(sel, dev):
    # seeded utterances with many ties, an all-blank utterance, NaNs; expected ids from loom.cpp's code
    g = np.load(os.path.join(GOLDEN, "ctc_reference.npz"))
    x = torch.from_numpy(g["utt"]).to(dev)
    ids, frames, lens = sel.ctc_greedy(x, int(g["blank"]))
    lens = lens.cpu().numpy()
    np.testing.assert_array_equal(lens, g["ref_lens"])
    ids = ids.cpu().numpy()
    for u in range(x.shape[0]):
        np.testing.assert_array_equal(ids[u, :lens[u]], g["ref_ids"][u, :lens[u]])


def _check(sel, oracle, x, blank, logp=True):
    ids, frames, lens, fid, flp = sel.ctc_greedy(x, blank, want_frame_ids=True, want_frame_logp=True)
    torch.cuda.synchronize()
    host = synth.bf16_bits(x) if x.dtype == torch.bfloat16 else x.cpu().numpy()
    seqs, want_fid, want_flp = oracle.ctc_greedy(host, blank, want_logp=True, nthreads=NT)
    lens = lens.cpu().numpy()
    ids, frames = ids.cpu().numpy(), frames.cpu().numpy()
    np.testing.assert_array_equal(fid.cpu().numpy(), want_fid)
    for u, (wi, wf) in enumerate(seqs):
        assert lens[u] == len(wi), u
        np.testing.assert_array_equal(ids[u, :lens[u]], wi)
        np.testing.assert_array_equal(frames[u, :lens[u]], wf)
    if logp:
        g, w = flp.cpu().numpy().astype(np.float64), want_flp.astype(np.float64)
        fin = np.isfinite(w)
        assert np.all(np.abs(g[fin] - w[fin]) <= 1e-5 * np.maximum(1.0, np.abs(w[fin])))


def test_asr_batch(sel, dev, oracle):
    # [32, 1500, 1025] f32, blank 1024: 70% blank frames, the rest a random non-blank id
    x = synth.ctc_frames(32, 1500, device="cuda")
    _check(sel, oracle, x, synth.CTC_BLANK)


def test_asr_batch_bf16(sel, dev, oracle):
    x = synth.ctc_frames(8, 777, seed=5, device="cuda").to(torch.bfloat16)
    _check(sel, oracle, x, synth.CTC_BLANK)


@pytest.mark.parametrize("U,F,C,blank", [(1, 1, 5, 4), (3, 17, 3, 0), (5, 2001, 129, 64), (2, 999, 4097, 4096),
                                         (40, 50, 1025, 1024), (7, 300, 33, 99)])
def test_shapes(sel, dev, oracle, U, F, C, blank):
    rng = np.random.default_rng(U * F + C)
    x = np.round(rng.normal(0, 1, (U, F, C)) * 2).astype(np.float32)  # integer logits: ties
    x[0, F // 2, 0] = np.nan
    _check(sel, oracle, torch.from_numpy(x).to(dev), blank)


def test_frame_argmax_is_argmax_rows(sel, dev, oracle):
    # loom.argmax_rows over a [48000, 1025] frame matrix (lua_bridge.cpp:343-365) -- the short-row path
    x = synth.ctc_frames(32, 1500, seed=8, device="cuda").reshape(-1, 1025)
    out = torch.empty(x.shape[0], dtype=torch.int32, device=dev)
    sel.argmax_rows_into(x, out)
    np.testing.assert_array_equal(out.cpu().numpy(), oracle.argmax_rows(x.cpu().numpy(), nthreads=NT))


def test_repeat_calls(sel, dev):
    x = synth.ctc_frames(4, 321, seed=2, device="cuda")
    ws = sel.Workspace(dev)
    a = sel.ctc_greedy(x, synth.CTC_BLANK, workspace=ws)
    lens = a[2].cpu().numpy()
    for _ in range(5):
        b = sel.ctc_greedy(x, synth.CTC_BLANK, workspace=ws)
        np.testing.assert_array_equal(lens, b[2].cpu().numpy())
        for u, n in enumerate(lens):
            np.testing.assert_array_equal(a[0][u, :n].cpu().numpy(), b[0][u, :n].cpu().numpy())
            np.testing.assert_array_equal(a[1][u, :n].cpu().numpy(), b[1][u, :n].cpu().numpy())
    assert ws.read_status() == sel.OK
