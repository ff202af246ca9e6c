"""Several argmax windows of the same rows in one launch (loom_argmax_windows), against the oracle.

What it replaces: one argmax_tensor_row call per window (src/core/lua_bridge.cpp:302-330), which
Whisper's driver makes through loom.argmax_row_range (lua_bridge.cpp:779-797) for the language block
and the timestamp block of a decoder row. The shapes are Whisper's multilingual vocabulary: 51865 ids,
the 99 language ids 50259..50357, the timestamp ids 50364..51864, the text ids below 50257. Ids are
bit-exact; the chunked kernel behind it also serves loom_argmax_rows for small batches.
"""
import ctypes

import numpy as np
import pytest
import torch

import synth

pytestmark = pytest.mark.gpu
NT = 8
WHISPER_V = 51865
WHISPER_WINDOWS = [(50259, 50358), (50364, 51865), (0, 50257), (0, -1)]


def _adversarial(rng, rows, V):
    x = rng.normal(0, 3, (rows, V)).astype(np.float32)
    for r in range(rows):
        kind = r % 6
        if kind == 1:
            x[r, 50259:50358] = np.round(x[r, 50259:50358])   # ties inside the language block
        elif kind == 2:
            x[r, 50259] = np.nan                              # NaN at a window's first id wins there
        elif kind == 3:
            x[r, rng.integers(0, V, 300)] = np.nan            # NaNs that never win
        elif kind == 4:
            x[r, 50364:] = -np.inf
            x[r, V - 1] = -2.0                                # only the last timestamp is finite
        elif kind == 5:
            x[r, :] = -0.0
            x[r, rng.integers(0, V, 3)] = 0.0                 # +0 == -0: each window's first id
    return x


def _want(oracle, host, windows):
    V = host.shape[1]
    cols = []
    for lo, hi in windows:
        hi_ = V if hi < 0 else hi
        cols.append(oracle.argmax_rows(np.ascontiguousarray(host[:, lo:hi_]), nthreads=NT) + lo)
    return np.stack(cols, axis=1)


@pytest.mark.parametrize("rows", [1, 5, 64, 600])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_whisper_windows_vs_oracle(sel, dev, oracle, rows, dtype):
    rng = np.random.default_rng(rows * 31 + (1 if dtype == "bf16" else 0))
    x = _adversarial(rng, rows, WHISPER_V)
    xt = torch.from_numpy(x).to(dev)
    host = x
    if dtype == "bf16":
        xt = xt.to(torch.bfloat16)
        host = synth.bf16_bits(xt)
    got = sel.argmax_windows(xt, WHISPER_WINDOWS).cpu().numpy()
    np.testing.assert_array_equal(got, _want(oracle, host, WHISPER_WINDOWS))


def test_language_window_excludes_words(sel, dev):
    # the reason the binding exists (BACKLOG.md, the Whisper prompt): a word outscores every language id,
    # and the windowed argmax still answers with the best language id
    x = torch.full((1, WHISPER_V), -5.0, device=dev)
    x[0, 1234] = 30.0                 # a word
    x[0, 50300] = 1.0                 # the best language
    x[0, 51000] = 2.0                 # the best timestamp
    got = sel.argmax_windows(x, WHISPER_WINDOWS).cpu().numpy()
    assert got.tolist() == [[50300, 51000, 1234, 1234]]


def test_strided_rows_and_small_windows(sel, dev, oracle):
    rng = np.random.default_rng(3)
    V, pad, rows = 70001, 3, 7
    full = rng.normal(0, 1, (rows, V + pad)).astype(np.float32)
    xt = torch.from_numpy(full).to(dev)[:, :V]      # rows off 16-byte boundaries
    windows = [(0, 1), (1, 2), (5, 22), (69990, 70001), (1, 70000), (4097, 12289)]
    got = sel.argmax_windows(xt, windows).cpu().numpy()
    np.testing.assert_array_equal(got, _want(oracle, full[:, :V], windows))


def test_errors_before_launch(sel, dev):
    x = torch.zeros(2, 100, device=dev)
    out = torch.empty(2, 8, dtype=torch.int32, device=dev)
    for windows, code in [([(5, 5)], sel.EWINDOW), ([(0, 101)], sel.EWINDOW), ([(-1, 4)], sel.EWINDOW),
                          ([], sel.EINVAL), ([(0, 10)] * 9, sel.EINVAL)]:
        with pytest.raises(sel.SelectError) as e:
            sel.argmax_windows_into(x, windows, out)
        assert e.value.status == code


def test_shared_workspace_with_other_kernels(sel, dev, oracle):
    # the pair records live in a region no other kernel writes, and return to zero after each call
    ws = sel.Workspace(dev)
    x, hist, u = synth.sample_chain(40, seed=9, device="cuda")          # split rows: records + tickets
    y = torch.from_numpy(_adversarial(np.random.default_rng(5), 3, WHISPER_V)).to(dev)
    want = _want(oracle, y.cpu().numpy(), WHISPER_WINDOWS)
    for _ in range(3):
        sel.sample_rows(x, u, 0.7, 1.1, 40, 0.9, history=hist, workspace=ws)
        out = torch.empty(3, len(WHISPER_WINDOWS), dtype=torch.int32, device=dev)
        sel.argmax_windows_into(y, WHISPER_WINDOWS, out, workspace=ws)
        np.testing.assert_array_equal(out.cpu().numpy(), want)
        ids = torch.empty(40, dtype=torch.int32, device=dev)
        sel.argmax_rows_into(x, ids, workspace=ws)                     # small batch: the chunked path
        np.testing.assert_array_equal(ids.cpu().numpy(), oracle.argmax_rows(x.cpu().numpy(), nthreads=NT))
    assert ws.read_status() == sel.OK
    # the raw entry point with NULL window arrays is refused
    lib = sel.lib()
    rc = lib.loom_argmax_windows(y.data_ptr(), 0, 3, WHISPER_V, WHISPER_V, None, None, 1, out.data_ptr(),
                                 ws.buf.data_ptr(), ws.buf.numel(), None)
    assert rc == sel.EINVAL
