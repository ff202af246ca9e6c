"""Generates the golden fixtures of tests/golden/ (run in a checkout that has the loom.cpp tree).

    python tests/golden/make_golden.py [--reference /path/to/loom.cpp]

Pinned by loom.cpp's OWN code: oracle/_ref/libref_ctc.so is loom.cpp's src/core/ctc_decode.cpp
compiled from its tree (oracle/Makefile, target `ref`).
  ctc_reference.npz     the three known answers of tests/ci/test_ctc_decode.cpp:12-38, and seeded
                        utterances (with frequent ties) decoded by loom.cpp's ctc_greedy_decode.
  argmax_reference.npz  adversarial rows (ties, NaN at 0 and elsewhere, +-0, +-inf, all-equal,
                        all-NaN) with the argmax that loom.cpp's own scan returns. The scan of
                        ctc_greedy_decode (ctc_decode.cpp:9-20) is the same strict '>' scan as
                        Generator::argmax (generation.cpp:64-74); it is read out by decoding each
                        row between separator frames whose argmax is the blank id, so that every
                        row's argmax is emitted once and never collapsed.
Pinned by the oracle only (loom.cpp has no sampler):
  sample_oracle.npz     small sampling-chain cases and the oracle's outputs, so that a change to
                        the oracle shows up as a fixture mismatch.
"""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle_binding as ob  # noqa: E402


def argmax_via_reference(rows):
    """Per-row argmax computed by loom.cpp's compiled ctc_greedy_decode."""
    rows = np.asarray(rows, dtype=np.float32)
    n_rows, n = rows.shape
    C = n + 1
    sep = np.full(C, -np.inf, dtype=np.float32)
    sep[n] = 0.0
    frames = [sep]
    for r in rows:
        frames.append(np.concatenate([r, np.array([-np.inf], dtype=np.float32)]))
        frames.append(sep)
    frames = np.stack(frames)
    out = ob.ref_ctc_greedy_decode(frames, n)
    assert out.shape[0] == n_rows, (out.shape, n_rows)
    return out


def adversarial_rows(rng, n=37):
    nan, inf = np.float32(np.nan), np.float32(np.inf)
    rows = []
    base = rng.normal(0, 1, n).astype(np.float32)
    rows.append(base.copy())
    r = base.copy(); r[5] = r[20] = r[30] = 9.0; rows.append(r)          # ties: lowest index
    r = base.copy(); r[0] = nan; rows.append(r)                            # NaN at 0 wins
    r = base.copy(); r[3] = nan; r[10] = 5.0; rows.append(r)               # NaN elsewhere never
    r = np.zeros(n, np.float32); r[2] = -0.0; r[7] = 0.0; r[:2] = -1; rows.append(r)  # -0 == +0
    r = np.full(n, -0.0, np.float32); r[6] = 0.0; rows.append(r)
    r = base.copy(); r[11] = inf; r[12] = inf; rows.append(r)              # +inf tie
    r = np.full(n, -inf, np.float32); rows.append(r)                       # all -inf -> 0
    r = np.full(n, -inf, np.float32); r[0] = nan; r[4] = 1.0; rows.append(r)
    r = np.full(n, nan, np.float32); rows.append(r)                        # all NaN -> 0
    r = np.full(n, nan, np.float32); r[9] = -inf; rows.append(r)           # NaN at 0 -> 0
    r = np.full(n, 3.0, np.float32); rows.append(r)                        # all equal -> 0
    r = np.arange(n, dtype=np.float32); rows.append(r)                     # ascending -> n-1
    r = np.arange(n, dtype=np.float32)[::-1].copy(); rows.append(r)        # descending -> 0
    r = np.round(rng.normal(0, 1, n)).astype(np.float32); rows.append(r)   # many ties
    for _ in range(16):
        rows.append(np.round(rng.normal(0, 2, n) * 2).astype(np.float32))
    return np.stack(rows)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("LOOM_REFERENCE") or os.path.join(os.path.dirname(ROOT), "reference"))
    a = ap.parse_args()
    os.environ["REF"] = a.reference
    import subprocess

    subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), f"REF={a.reference}", "liboracle.so", "ref"],
                   check=True)
    rng = np.random.default_rng(20261201)

    # ---- CTC: known answers of tests/ci/test_ctc_decode.cpp:12-38, plus seeded utterances ----
    ka1 = np.array([0, 5, 0, 0, 0, 4, 1, 0, 0, 0, 0, 9, 0, 0, 7, 1, 1, 0, 6, 0, 8, 0, 0, 1, 7, 0, 0, 2, 0, 0, 0, 9],
                   dtype=np.float32).reshape(8, 4)
    ka2 = np.array([0, 0, 0, 9, 0, 5, 0, 0], dtype=np.float32).reshape(2, 4)
    ka3 = np.array([0, 0, 0, 9, 0, 0, 0, 9, 0, 0, 0, 9], dtype=np.float32).reshape(3, 4)
    U, F, C, blank = 4, 200, 29, 28
    utt = np.round(rng.normal(0, 1.0, (U, F, C)) * 2).astype(np.float32)   # integer values: many ties
    is_blank = rng.random((U, F)) < 0.6
    for u in range(U):
        for f in range(F):
            utt[u, f, blank if is_blank[u, f] else rng.integers(0, C - 1)] += 3.0
    utt[1, 50:80, :] = 0.0      # all-equal frames: argmax 0
    utt[2, :, blank] = 100.0    # an all-blank utterance
    utt[3, 10, 0] = np.nan      # NaN at column 0 wins its frame
    utt[3, 11, 5] = np.nan      # NaN elsewhere never wins
    ref_seqs = [ob.ref_ctc_greedy_decode(utt[u], blank) for u in range(U)]
    lens = np.array([len(s) for s in ref_seqs], dtype=np.int32)
    ref_ids = np.zeros((U, F), dtype=np.int32)
    for u, s in enumerate(ref_seqs):
        ref_ids[u, :len(s)] = s
    np.savez_compressed(
        os.path.join(HERE, "ctc_reference.npz"),
        ka1=ka1, ka1_expected=np.array([1, 2, 0], np.int32),
        ka2=ka2, ka2_expected=np.array([1], np.int32),
        ka3=ka3, ka3_expected=np.zeros(0, np.int32),
        ka1_ref=ob.ref_ctc_greedy_decode(ka1, 3), ka2_ref=ob.ref_ctc_greedy_decode(ka2, 3),
        ka3_ref=ob.ref_ctc_greedy_decode(ka3, 3),
        utt=utt, blank=np.int32(blank), ref_ids=ref_ids, ref_lens=lens,
    )

    # ---- argmax rows through loom.cpp's own scan ----
    rows = adversarial_rows(rng)
    np.savez_compressed(os.path.join(HERE, "argmax_reference.npz"), rows=rows,
                        ref_argmax=argmax_via_reference(rows).astype(np.int32))

    # ---- sampling chain: oracle outputs (no loom.cpp counterpart) ----
    cases = {}
    V = 777
    x = rng.normal(0, 3, (12, V)).astype(np.float32)
    x[1, 100:140] = 7.5                           # a 40-way tie at the top
    x[2, :] = np.round(x[2, :])                   # many ties
    x[3, 5] = np.nan
    x[4, 7] = np.inf
    x[5, :] = -np.inf; x[5, 3] = 1.0              # one finite value
    x[6, :] = np.nan; x[6, 9] = 2.0               # fewer than k non-NaN values
    x[7, :] = 0.0; x[7, ::2] = -0.0               # +-0 everywhere
    hist = rng.integers(0, V, (12, 24)).astype(np.int32)
    hist[8, :] = 11                               # one id repeated: applied once
    u = rng.random(12).astype(np.float32)
    u[9] = 0.0
    u[10] = np.float32(0.99999994)
    for name, (T, r, k, p) in {
        "chain": (0.7, 1.1, 40, 0.9),
        "boost": (1.3, 0.8, 17, 0.5),
        "greedy": (0.0, 1.1, 5, 1.0),
        "k1": (1.0, 1.0, 1, 1.0),
        "kbig": (0.5, 1.2, 300, 0.95),
    }.items():
        res = ob.sample_rows(x, u, T, r, k, p, hist)
        assert res["status"] == 0
        cases[f"{name}_params"] = np.array([T, r, k, p], dtype=np.float64)
        cases[f"{name}_ids"] = res["ids"]
        cases[f"{name}_prob"] = res["prob"]
        cases[f"{name}_logp"] = res["logp"]
        cases[f"{name}_topk"] = res["topk"]
    np.savez_compressed(os.path.join(HERE, "sample_oracle.npz"), x=x, hist=hist, u=u, **cases)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
