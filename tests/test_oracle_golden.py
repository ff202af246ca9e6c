"""The oracle pinned against loom.cpp: its known-answer tests, and fixtures made by its own code.

Citations are paths in the loom.cpp tree. These run without a GPU.
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


# ---- tests/ci/test_ctc_decode.cpp:12-38 ----

def test_ctc_known_answers(oracle):
    g = _load("ctc_reference.npz")
    for case in ("ka1", "ka2", "ka3"):
        seqs, _, _ = oracle.ctc_greedy(g[case], 3)
        np.testing.assert_array_equal(seqs[0][0], g[f"{case}_expected"])
        np.testing.assert_array_equal(g[f"{case}_ref"], g[f"{case}_expected"])


def test_ctc_known_answer_frames(oracle):
    # frame-wise argmax 1,1,3,2,2,0,0,3 (test_ctc_decode.cpp:12-23); emitted at frames 0, 3, 5
    g = _load("ctc_reference.npz")
    seqs, fid, _ = oracle.ctc_greedy(g["ka1"], 3)
    np.testing.assert_array_equal(fid[0], [1, 1, 3, 2, 2, 0, 0, 3])
    np.testing.assert_array_equal(seqs[0][1], [0, 3, 5])


def test_ctc_matches_reference_fixture(oracle):
    g = _load("ctc_reference.npz")
    utt, blank = g["utt"], int(g["blank"])
    seqs, _, _ = oracle.ctc_greedy(utt, blank)
    for u, (ids, _) in enumerate(seqs):
        n = int(g["ref_lens"][u])
        np.testing.assert_array_equal(ids, g["ref_ids"][u, :n])
    assert int(g["ref_lens"][2]) == 0  # the all-blank utterance collapses to nothing


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(GOLDEN), "..", "oracle", "_ref",
                                                    "libref_ctc.so")),
                    reason="loom.cpp's compiled ctc_decode.cpp (oracle/_ref) is built only where its tree is")
def test_ctc_oracle_vs_reference_random(oracle):
    rng = np.random.default_rng(7)
    for trial in range(30):
        F, C = int(rng.integers(1, 300)), int(rng.integers(2, 70))
        x = np.round(rng.normal(0, 1, (F, C)) * 2).astype(np.float32)
        if trial % 5 == 0:
            x[rng.integers(0, F), 0] = np.nan
        blank = int(rng.integers(0, C))
        seqs, _, _ = oracle.ctc_greedy(x, blank)
        np.testing.assert_array_equal(seqs[0][0], oracle.ref_ctc_greedy_decode(x, blank))


# ---- the argmax scans: generation.cpp:64-74, lua_bridge.cpp:320-329, :358-362, :744-758 ----

def test_argmax_matches_reference_fixture(oracle):
    g = _load("argmax_reference.npz")
    rows, ref = g["rows"], g["ref_argmax"]
    for r in range(rows.shape[0]):
        assert oracle.argmax(rows[r]) == ref[r], r
    st, ids = oracle.argmax_tensor_rows(rows)
    assert st == 0
    np.testing.assert_array_equal(ids, ref)
    np.testing.assert_array_equal(oracle.argmax_rows(rows), ref)


def test_argmax_row_array_form(oracle):
    # tests/ci/test_lua_bridge.cpp:139-145: flat=[1,5,2, 9,0,3], n_vocab=3, row_index=1 -> 0
    st, i = oracle.argmax_row_array([1, 5, 2, 9, 0, 3], 3, 1)
    assert st == 0 and i == 0
    st, _ = oracle.argmax_row_array([1, 5, 2], 3, 1)  # row past the array (lua_bridge.cpp:748-750)
    assert st != 0


def test_argmax_window_excludes_winner(oracle):
    # tests/ci/test_lua_bridge_retained_outputs.cpp:152-174: a window that excludes the unrestricted
    # winner must return the window's own best, as an ABSOLUTE id
    x = np.array([[0.5, 4.0, 1.0, 2.0, 3.5, 0.0]], dtype=np.float32)
    st, full = oracle.argmax_tensor_row(x, -1)
    assert st == 0 and full == 1
    st, got = oracle.argmax_tensor_row(x, -1, 3, 6)
    assert st == 0 and got == 4
    assert got != full and 3 <= got < 6


def test_argmax_window_errors(oracle):
    # lua_bridge.cpp:310-319 / test_lua_bridge_retained_outputs.cpp:229-241 (cases 6 and 7)
    x = np.zeros((3, 6), dtype=np.float32)
    assert oracle.argmax_tensor_row(x, -1, 2, 99)[0] != 0   # hi past the row
    assert oracle.argmax_tensor_row(x, -1, 3, 3)[0] != 0    # empty window
    assert oracle.argmax_tensor_row(x, 3)[0] != 0           # row out of range
    assert oracle.argmax_tensor_row(x, -1, -1, 2)[0] != 0   # negative lo
    assert oracle.argmax_tensor_row(x, -1, 0, -1) == (0, 0)  # hi < 0 means the whole row


def test_argmax_bf16_is_widened_exactly(oracle):
    rng = np.random.default_rng(3)
    x = rng.normal(0, 2, (5, 513)).astype(np.float32)
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)           # truncate to bf16 bit patterns
    widened = (bits.astype(np.uint32) << 16).view(np.float32)
    np.testing.assert_array_equal(oracle.argmax_rows(bits), oracle.argmax_rows(widened))


# ---- sampling chain: the oracle against its own committed fixture ----

def test_sample_oracle_fixture(oracle):
    g = _load("sample_oracle.npz")
    for name in ("chain", "boost", "greedy", "k1", "kbig"):
        T, r, k, p = g[f"{name}_params"]
        res = oracle.sample_rows(g["x"], g["u"], float(T), float(r), int(k), float(p), g["hist"])
        assert res["status"] == 0
        np.testing.assert_array_equal(res["ids"], g[f"{name}_ids"], err_msg=name)
        np.testing.assert_array_equal(res["topk"], g[f"{name}_topk"], err_msg=name)
        np.testing.assert_array_equal(res["prob"].view(np.uint32), g[f"{name}_prob"].view(np.uint32), err_msg=name)
