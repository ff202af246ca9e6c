"""Greedy argmax on the GPU (K1 long rows, warp-per-row short rows) against loom.cpp and the oracle.

Bit-exact ids everywhere. Citations are paths in the loom.cpp tree.
"""
import os

import numpy as np
import pytest
import torch

import synth

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
NT = os.cpu_count() or 4


def _ids(sel, x, lo=0, hi=-1):
    out = torch.empty(x.shape[0], dtype=torch.int32, device=x.device)
    sel.argmax_rows_into(x, out, lo, hi)
    return out.cpu().numpy()


def test_known_answers(sel, dev):
    # tests/ci/test_lua_bridge.cpp:139-145: rows [1,5,2] and [9,0,3]; row 1 -> 0
    x = torch.tensor([[1, 5, 2], [9, 0, 3]], dtype=torch.float32, device=dev)
    assert sel.argmax_row(x, 1) == 0.0
    assert sel.argmax_row(x) == 0.0                      # row -1 is the last row
    assert sel.argmax_rows(x) == [1.0, 0.0]


def test_window_excludes_winner_and_errors(sel, dev):
    # tests/ci/test_lua_bridge_retained_outputs.cpp:152-174 and :229-241 (cases 6, 7)
    x = torch.tensor([[0.5, 4.0, 1.0, 2.0, 3.5, 0.0]], dtype=torch.float32, device=dev)
    full = sel.argmax_row(x, -1)
    got = sel.argmax_row_range(x, -1, 3, 6)
    assert full == 1.0 and got == 4.0
    for lo, hi in [(2, 99), (3, 3), (-1, 4)]:
        with pytest.raises(sel.SelectError) as e:
            sel.argmax_row_range(x, -1, lo, hi)
        assert e.value.status == sel.EWINDOW
    with pytest.raises(sel.SelectError):
        sel.argmax_row(x, 1)                             # row out of range


def test_reference_fixture_rows(sel, dev):
    g = np.load(os.path.join(GOLDEN, "argmax_reference.npz"))
    rows, ref = g["rows"], g["ref_argmax"]
    x = torch.from_numpy(rows).to(dev)
    np.testing.assert_array_equal(_ids(sel, x), ref)
    # the same rows at the head of long rows (K1): filler -inf never wins, so the answer is unchanged
    W = 40000
    wide = np.full((rows.shape[0], W), -np.inf, dtype=np.float32)
    wide[:, :rows.shape[1]] = rows
    np.testing.assert_array_equal(_ids(sel, torch.from_numpy(wide).to(dev)), ref)


def _adversarial(rng, rows, V):
    x = rng.normal(0, 3, (rows, V)).astype(np.float32)
    for r in range(rows):
        kind = r % 8
        if kind == 1:
            pos = rng.integers(0, V, 5)
            x[r, pos] = x[r].max() + 1.0          # a tie at the top, far apart
        elif kind == 2:
            x[r, rng.integers(1, V, 50)] = np.nan  # NaNs that never win
        elif kind == 3:
            x[r, 0] = np.nan                       # NaN in column 0 wins
        elif kind == 4:
            x[r] = np.round(x[r])                  # many ties
        elif kind == 5:
            x[r] = 2.0                             # all equal -> lowest
        elif kind == 6:
            x[r] = -np.inf
            x[r, V - 1] = -1.0                     # only the last is finite
        elif kind == 7:
            x[r, :] = -0.0
            x[r, rng.integers(0, V)] = 0.0         # +0 == -0 -> column 0
    return x


@pytest.mark.parametrize("V", [8192, 8193, 100003, 151936, 262144])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_rows_vs_oracle(sel, dev, oracle, V, dtype):
    rng = np.random.default_rng(V + (7 if dtype == "bf16" else 0))
    rows = 24
    x = _adversarial(rng, rows, V)
    xt = torch.from_numpy(x).to(dev)
    if dtype == "bf16":
        xt = xt.to(torch.bfloat16)
        host = synth.bf16_bits(xt)
    else:
        host = x
    np.testing.assert_array_equal(_ids(sel, xt), oracle.argmax_rows(host, nthreads=NT))


@pytest.mark.parametrize("V,pad,lo,hi", [(151936, 3, 0, -1), (151936, 5, 7, 151929), (50001, 1, 3, 50000),
                                          (3000, 2, 1, 2999), (262144, 8, 131071, 262143)])
def test_strided_and_windowed_vs_oracle(sel, dev, oracle, V, pad, lo, hi):
    # row stride V + pad leaves most rows off 16-byte boundaries; windows start off them too
    rng = np.random.default_rng(V + pad + lo)
    rows = 9
    x = _adversarial(rng, rows, V + pad)
    xt = torch.from_numpy(x).to(dev)[:, :V]
    got = _ids(sel, xt, lo, hi)
    hi_ = V if hi < 0 else hi
    want = oracle.argmax_rows(np.ascontiguousarray(x[:, lo:hi_]), nthreads=NT) + lo
    np.testing.assert_array_equal(got, want)


def test_greedy_decode_512_steps(sel, dev, oracle):
    # [1, 151936] f32 per decode step, 512 steps, each seeded from (seed, step); one call per step
    out = torch.empty(512, dtype=torch.int32, device=dev)
    host = []
    for s in range(512):
        x = synth.greedy_decode_step(s).to(dev)
        sel.argmax_rows_into(x, out[s:s + 1])
        host.append(x.cpu().numpy())
    want = oracle.argmax_rows(np.concatenate(host), nthreads=NT)
    np.testing.assert_array_equal(out.cpu().numpy(), want)


@pytest.mark.parametrize("rows", [1, 3, 148, 149, 300, 1024])
def test_batch_vs_oracle(sel, dev, oracle, rows):
    x, _, _ = synth.sample_chain(rows, device="cuda")
    np.testing.assert_array_equal(_ids(sel, x), oracle.argmax_rows(x.cpu().numpy(), nthreads=NT))


def test_repeat_calls_leave_workspace_clean(sel, dev, oracle):
    # split rows use tickets in the workspace; they must be back at zero after every call
    x, _, _ = synth.sample_chain(5, device="cuda")
    want = oracle.argmax_rows(x.cpu().numpy(), nthreads=NT)
    ws = sel.Workspace(dev)
    for _ in range(20):
        out = torch.empty(5, dtype=torch.int32, device=dev)
        sel.argmax_rows_into(x, out, workspace=ws)
        np.testing.assert_array_equal(out.cpu().numpy(), want)
    assert ws.read_status() == sel.OK
