"""The C-ABI library without a GPU: it loads, exports every declared symbol, and rejects bad
arguments on the host before touching CUDA (loom.cpp's argument errors, lua_bridge.cpp:302-319)."""
import ctypes
import os
import re

import pytest

import loom_select as ls

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FAKE = ctypes.c_void_p(1 << 20)  # never dereferenced: every call below fails its host-side checks


def declared_symbols():
    text = open(os.path.join(ROOT, "include", "loom_select.h")).read()
    return set(re.findall(r"LOOM_SELECT_API\s+[\w\s\*]+?\b(loom_\w+)\s*\(", text))


def test_library_loads_and_exports_every_declared_symbol():
    lib = ls.lib()
    declared = declared_symbols()
    assert declared == set(ls.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.loom_select_abi_version() == 100


def test_strerror_covers_every_status():
    lib = ls.lib()
    for code in range(10):
        assert lib.loom_select_strerror(code).decode() != "unknown status"
    assert lib.loom_select_strerror(99).decode() == "unknown status"


def test_workspace_sizes_are_device_independent_and_aligned():
    lib = ls.lib()
    a = lib.loom_argmax_workspace_size(1024, 151936)
    s = lib.loom_sample_workspace_size(1024, 151936, 40)
    c = lib.loom_ctc_workspace_size(32, 1500)
    for v in (a, s, c):
        assert v > 0 and v % 256 == 0
    assert lib.loom_sample_workspace_size(1024, 151936, 1024) > s
    assert c >= 32 * 1500 * 4
    assert lib.loom_shard_record_bytes(64) == 16 + 8 * 64


def _argmax(lib, dtype=0, rows=2, n=10, stride=10, lo=0, hi=-1, out=FAKE, ws=FAKE, ws_bytes=1 << 30, logits=FAKE):
    return lib.loom_argmax_rows(logits, dtype, rows, n, stride, lo, hi, out, ws, ws_bytes, None)


def test_argmax_argument_checks():
    lib = ls.lib()
    assert _argmax(lib, dtype=7) == ls.EDTYPE
    assert _argmax(lib, logits=None) == ls.EINVAL
    assert _argmax(lib, out=None) == ls.EINVAL
    assert _argmax(lib, rows=0) == ls.EINVAL
    assert _argmax(lib, stride=9) == ls.EINVAL
    assert _argmax(lib, lo=3, hi=3) == ls.EWINDOW     # empty window
    assert _argmax(lib, lo=2, hi=99) == ls.EWINDOW    # past the row
    assert _argmax(lib, lo=-1, hi=5) == ls.EWINDOW
    assert _argmax(lib, ws=None) == ls.EWORKSPACE
    assert _argmax(lib, ws_bytes=16) == ls.EWORKSPACE
    assert _argmax(lib, ws=ctypes.c_void_p((1 << 20) + 8)) == ls.EWORKSPACE  # not 256-byte aligned


def _sample(lib, T=0.7, r=1.1, k=40, p=0.9, hl=0, hist=None, n=1000, ws_bytes=1 << 30, u=FAKE):
    prm = ls.SampleParams(T, r, k, p)
    return lib.loom_sample_rows(FAKE, 0, 4, n, n, hist, hl, u, ctypes.byref(prm), FAKE, FAKE, None, None, FAKE,
                                ws_bytes, None)


def test_sample_argument_checks():
    lib = ls.lib()
    assert _sample(lib, T=-1.0) == ls.EPARAM
    assert _sample(lib, T=float("inf")) == ls.EPARAM
    assert _sample(lib, T=float("nan")) == ls.EPARAM
    assert _sample(lib, r=0.0) == ls.EPARAM
    assert _sample(lib, k=0) == ls.EPARAM
    assert _sample(lib, k=1025) == ls.EPARAM
    assert _sample(lib, k=1001) == ls.EPARAM          # k > vocabulary
    assert _sample(lib, p=0.0) == ls.EPARAM
    assert _sample(lib, p=1.01) == ls.EPARAM
    assert _sample(lib, hl=3, hist=None) == ls.EINVAL
    assert _sample(lib, hl=4096, hist=FAKE) == ls.ESHAPE
    assert _sample(lib, u=None) == ls.EINVAL
    assert _sample(lib, ws_bytes=100) == ls.EWORKSPACE


def test_shard_argument_checks():
    lib = ls.lib()
    prm = ls.SampleParams(1.0, 1.0, 64, 0.95)
    # shard past the vocabulary
    assert lib.loom_sample_shard_partial(FAKE, 1, 4, 100, 100, 950, 1000, None, 0, ctypes.byref(prm), FAKE, FAKE,
                                         1 << 30, None) == ls.EINVAL
    greedy = ls.SampleParams(0.0, 1.0, 64, 0.95)
    assert lib.loom_sample_shard_partial(FAKE, 1, 4, 100, 100, 0, 1000, None, 0, ctypes.byref(greedy), FAKE, FAKE,
                                         1 << 30, None) == ls.EPARAM
    assert lib.loom_sample_shard_merge(FAKE, 0, 4, FAKE, ctypes.byref(prm), FAKE, FAKE, None, None, None) == ls.EINVAL


def test_ctc_argument_checks():
    lib = ls.lib()
    assert lib.loom_ctc_greedy(FAKE, 5, 1, 10, 4, 3, FAKE, FAKE, FAKE, None, None, FAKE, 1 << 30, None) == ls.EDTYPE
    assert lib.loom_ctc_greedy(FAKE, 0, 0, 10, 4, 3, FAKE, FAKE, FAKE, None, None, FAKE, 1 << 30, None) == ls.EINVAL
    assert lib.loom_ctc_greedy(FAKE, 0, 1, 10, 4, 3, FAKE, FAKE, FAKE, None, None, FAKE, 64, None) == ls.EWORKSPACE


def test_lm_head_argument_checks():
    lib = ls.lib()
    # hidden_dim not a multiple of 64, then null pointers, then a workspace that is too small
    assert lib.loom_lm_head_argmax(FAKE, FAKE, 4, 100, 1000, FAKE, None, None, FAKE, 1 << 30, None) == ls.ESHAPE
    assert lib.loom_lm_head_argmax(None, FAKE, 4, 128, 1000, FAKE, None, None, FAKE, 1 << 30, None) == ls.EINVAL
    assert lib.loom_lm_head_argmax(FAKE, FAKE, 0, 128, 1000, FAKE, None, None, FAKE, 1 << 30, None) == ls.EINVAL
    assert lib.loom_lm_head_argmax(FAKE, FAKE, 4, 128, 1000, FAKE, None, None, FAKE, 64, None) == ls.EWORKSPACE
    need = lib.loom_lm_head_workspace_size(4, 1000)
    assert need % 256 == 0 and need >= 256 + 4 * 4 * 16


def test_python_mirror_raises_select_error():
    with pytest.raises(ls.SelectError) as e:
        ls.check(ls.EWINDOW, "loom.argmax_row_range")
    assert "not a non-empty sub-range" in str(e.value)
