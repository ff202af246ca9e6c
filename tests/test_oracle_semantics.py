"""The sampling-chain oracle against an independent numpy restatement of the same semantics.

loom.cpp has no sampler, so the chain's parity is pinned by its written semantics (penalty over the
distinct history ids, fp32 temperature divide, key = value desc / id asc with NaN lowest and
-0 == +0, top-k, double-precision survivor softmax, top-p, inverse-CDF draw). This file restates them
a second time with numpy sorting and Python floats, and checks the C oracle against it.
"""
import math
import os

import numpy as np
import pytest


def chain_numpy(x_row, hist_row, u, T, r, k, p):
    x = np.array(x_row, dtype=np.float32, copy=True)
    r32 = np.float32(r)
    for v in sorted(set(int(h) for h in hist_row)):
        x[v] = np.float32(x[v] / r32) if x[v] > 0 else np.float32(x[v] * r32)
    y = x if T == 0 else (x / np.float32(T)).astype(np.float32)
    V = y.size
    isnan = np.isnan(y)
    order = np.lexsort((np.arange(V), -np.where(isnan, 0, y), isnan))
    top = order[:k]
    ys = y[top]
    m = ys[0]

    def weight(yi):
        if math.isnan(yi) or math.isnan(m):
            return 0.0
        if yi == m:
            return 1.0
        return math.exp(float(yi) - float(m))

    e = [weight(float(v)) for v in ys]
    S = []
    acc = 0.0
    for w in e:
        acc = w if not S else acc + w
        S.append(acc)
    if T == 0:
        sel_id = 0 if math.isnan(x[0]) else int(top[0])
        return sel_id, 1.0, top
    target = float(np.float32(p)) * S[-1]
    n = next((j + 1 for j in range(k) if S[j] >= target), k)
    draw = float(np.float32(u)) * S[n - 1]
    sel = next((i for i in range(n) if draw < S[i]), n - 1)
    prob = e[sel] / S[n - 1] if S[n - 1] != 0.0 else float("nan")  # IEEE 0/0
    return int(top[sel]), prob, top


def _check(oracle, x, hist, u, T, r, k, p):
    res = oracle.sample_rows(x, u, T, r, k, p, hist)
    assert res["status"] == 0
    for row in range(x.shape[0]):
        sid, prob, top = chain_numpy(x[row], hist[row], u[row], T, r, k, p)
        np.testing.assert_array_equal(res["topk"][row], top, err_msg=f"row {row}")
        assert res["ids"][row] == sid, f"row {row}"
        if math.isnan(prob):
            assert math.isnan(res["prob"][row])
        else:
            assert abs(float(res["prob"][row]) - prob) <= 1e-6 * max(prob, 1e-30), row


@pytest.mark.parametrize("T,r,k,p", [(0.7, 1.1, 40, 0.9), (1.0, 1.0, 1, 1.0), (1.7, 0.6, 64, 0.3),
                                     (0.0, 1.3, 8, 1.0), (0.2, 2.0, 333, 0.99)])
def test_chain_matches_numpy(oracle, T, r, k, p):
    rng = np.random.default_rng(int(T * 100 + k))
    V = 1501
    x = rng.normal(0, 3, (8, V)).astype(np.float32)
    x[1, 200:260] = 9.0
    x[2] = np.round(x[2])
    x[3, 0] = np.nan
    x[4, 10:20] = np.inf
    x[5, 1::2] = -0.0
    x[5, ::2] = 0.0
    hist = rng.integers(0, V, (8, 50)).astype(np.int32)
    hist[6] = 3
    u = rng.random(8).astype(np.float32)
    _check(oracle, x, hist, u, T, r, k, p)


def test_fewer_values_than_k(oracle):
    V = 300
    x = np.full((3, V), np.nan, dtype=np.float32)
    x[0, 17] = 1.0
    x[1, 5] = -np.inf
    hist = np.zeros((3, 1), dtype=np.int32)
    u = np.array([0.3, 0.9, 0.5], dtype=np.float32)
    _check(oracle, x, hist, u, 0.9, 1.0, 10, 0.8)


def test_history_out_of_range_is_an_error(oracle):
    x = np.zeros((2, 100), dtype=np.float32)
    hist = np.array([[3, 100], [1, 2]], dtype=np.int32)
    res = oracle.sample_rows(x, np.zeros(2, np.float32), 1.0, 1.1, 5, 1.0, hist)
    assert res["status"] == 7  # LOOM_SELECT_EHISTORY
    assert res["ids"][0] == -1 and res["ids"][1] == 0


def test_parameter_checks(oracle):
    x = np.zeros((1, 10), dtype=np.float32)
    u = np.zeros(1, np.float32)
    for T, r, k, p in [(-1.0, 1.0, 1, 1.0), (1.0, 0.0, 1, 1.0), (1.0, 1.0, 0, 1.0), (1.0, 1.0, 11, 1.0),
                       (1.0, 1.0, 1, 0.0), (1.0, 1.0, 1, 1.5), (float("inf"), 1.0, 1, 1.0)]:
        assert oracle.sample_rows(x, u, T, r, k, p)["status"] == 8


def test_logp_is_the_full_row_log_softmax(oracle):
    rng = np.random.default_rng(11)
    x = rng.normal(0, 3, (4, 2000)).astype(np.float32)
    hist = rng.integers(0, 2000, (4, 30)).astype(np.int32)
    u = rng.random(4).astype(np.float32)
    T, r = 0.7, 1.1
    res = oracle.sample_rows(x, u, T, r, 40, 0.9, hist)
    for row in range(4):
        xx = x[row].copy()
        for v in set(hist[row].tolist()):
            xx[v] = np.float32(xx[v] / np.float32(r)) if xx[v] > 0 else np.float32(xx[v] * np.float32(r))
        y = (xx / np.float32(T)).astype(np.float64)
        lse = y.max() + math.log(np.exp(y - y.max()).sum())
        assert abs(res["logp"][row] - (y[res["ids"][row]] - lse)) < 1e-5


def test_shard_merge_equals_full_row(oracle):
    rng = np.random.default_rng(5)
    V, G, rows, k = 4096, 8, 6, 64
    x = rng.normal(0, 2.5, (rows, V)).astype(np.float32)
    x[2, 1000:1100] = 6.0                      # a tie that crosses shard boundaries
    hist = rng.integers(0, V, (rows, 20)).astype(np.int32)
    u = rng.random(rows).astype(np.float32)
    T, r, p = 0.8, 1.15, 0.95
    full = oracle.sample_rows(x, u, T, r, k, p, hist)
    parts = []
    for g in range(G):
        st, rec = oracle.shard_partial(x[:, g * V // G:(g + 1) * V // G], g * V // G, V, T, r, k, hist)
        assert st == 0
        parts.append(rec)
    merged = oracle.shard_merge(np.concatenate(parts), G, rows, u, T, k, p)
    np.testing.assert_array_equal(merged["ids"], full["ids"])
    np.testing.assert_array_equal(merged["topk"], full["topk"])
    np.testing.assert_array_equal(merged["prob"].view(np.uint32), full["prob"].view(np.uint32))
    np.testing.assert_allclose(merged["logp"], full["logp"], rtol=1e-5, atol=1e-6)


def test_exp_d_accuracy(oracle):
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-745, 0, 20000), rng.uniform(-8, 0, 20000), rng.uniform(-1e-3, 0, 2000),
                         [0.0, -0.0, -1e-300, -708.3, -744.4, -745.1]])
    worst = 0.0
    for x in xs:
        a, b = oracle.exp_d(x), math.exp(x)
        if b == 0.0:
            assert a == 0.0
            continue
        if b < 2.2250738585072014e-308:  # subnormal results: absolute error in units of the smallest subnormal
            assert abs(a - b) <= 5e-324
            continue
        worst = max(worst, abs(a - b) / math.ulp(b))
    assert worst <= 1.0
    assert oracle.exp_d(0.0) == 1.0
    assert oracle.exp_d(-800.0) == 0.0
    assert math.isnan(oracle.exp_d(float("nan")))


def test_kernel_division_by_temperature_equals_ieee_divide(oracle):
    """The sampling kernels divide by T (and by the penalty r) with Markstein's method -- a product with
    the correctly rounded reciprocal and one FMA correction -- instead of a divide instruction. That
    must give the IEEE quotient bit for bit: checked for every float mantissa of x against 64
    divisors (the headline's T 0.7 and r 1.1, extremes, and seeded random ones)."""
    import ctypes

    import numpy as np

    f = oracle.lib().oracle_div_check
    f.restype = ctypes.c_int64
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
    rng = np.random.default_rng(20261202)
    fixed = [0.7, 0.001, 1.3, 2.5, 0.9, 1.0, 0.5, 0.25, 3.0, 1e-4, 1e4, 0.1, 0.3333333, 1.9999999, 1.0000001,
             0.99999994, 1.1, 1.2, 1.05, 0.8, 1.5, 2.0]
    Ts = np.concatenate([np.array(fixed, np.float32), (2.0 ** rng.uniform(-12, 12, 42)).astype(np.float32)])
    bx, bT = ctypes.c_float(), ctypes.c_float()
    bad = f(Ts.ctypes.data, len(Ts), os.cpu_count() or 1, ctypes.byref(bx), ctypes.byref(bT))
    assert bad == 0, f"{bad} mismatches, first at x={bx.value!r}, T={bT.value!r}"
