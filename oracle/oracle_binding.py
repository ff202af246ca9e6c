"""ctypes binding of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

The oracle (select_oracle.c, built into liboracle.so by the Makefile beside this file) is the checker
the CUDA kernels are compared against. Only the tests, the smoke check and the bench's CPU-baseline
and reference legs may use this module. `ref_ctc_greedy_decode` calls loom.cpp's own
src/core/ctc_decode.cpp, compiled into _ref/libref_ctc.so when the loom.cpp tree is present.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libref_ctc.so")
REFPATH_PATH = os.path.join(HERE, "librefpath.so")

F32 = 0
BF16 = 1

_LIB = None
_REF = None
_REFPATH = None


def build(ref=False):
    """make the oracle (and, with ref=True and the loom.cpp tree present, _ref/)."""
    subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    if ref:
        subprocess.run(["make", "-s", "-C", HERE, "ref"], check=True)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def lib():
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            build()
        l = ctypes.CDLL(LIB_PATH)
        vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_float
        l.oracle_argmax.restype = i32
        l.oracle_argmax.argtypes = [vp, i64]
        l.oracle_argmax_tensor_row.restype = ctypes.c_int
        l.oracle_argmax_tensor_row.argtypes = [vp, i64, i64, i64, i64, i64, i64, ctypes.POINTER(i64)]
        l.oracle_argmax_tensor_rows.restype = ctypes.c_int
        l.oracle_argmax_tensor_rows.argtypes = [vp, i64, i64, i64, vp]
        l.oracle_argmax_row_array.restype = ctypes.c_int
        l.oracle_argmax_row_array.argtypes = [vp, i64, i64, i64, ctypes.POINTER(i64)]
        l.oracle_argmax_rows.restype = ctypes.c_int
        l.oracle_argmax_rows.argtypes = [vp, ctypes.c_int, i64, i64, i64, i64, i64, vp, ctypes.c_int]
        l.oracle_ctc_greedy.restype = ctypes.c_int
        l.oracle_ctc_greedy.argtypes = [vp, ctypes.c_int, i64, i64, i64, i32, vp, vp, vp, vp, vp, ctypes.c_int]
        l.oracle_sample_rows.restype = ctypes.c_int
        l.oracle_sample_rows.argtypes = [vp, ctypes.c_int, i64, i64, i64, vp, i32, vp, f32, f32, i32, f32, vp, vp, vp,
                                         vp, ctypes.c_int]
        l.oracle_shard_record_bytes.restype = ctypes.c_size_t
        l.oracle_shard_record_bytes.argtypes = [i32]
        l.oracle_shard_partial.restype = ctypes.c_int
        l.oracle_shard_partial.argtypes = [vp, ctypes.c_int, i64, i64, i64, i64, i64, vp, i32, f32, f32, i32, vp,
                                           ctypes.c_int]
        l.oracle_shard_merge.restype = ctypes.c_int
        l.oracle_shard_merge.argtypes = [vp, i32, i64, vp, f32, i32, f32, vp, vp, vp, vp]
        l.oracle_exp_d.restype = ctypes.c_double
        l.oracle_exp_d.argtypes = [ctypes.c_double]
        _LIB = l
    return _LIB


def ref_available():
    return os.path.exists(REF_PATH)


def ref_lib():
    global _REF
    if _REF is None:
        l = ctypes.CDLL(REF_PATH)
        l.ref_ctc_greedy_decode.restype = ctypes.c_int64
        l.ref_ctc_greedy_decode.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int32,
                                            ctypes.c_void_p, ctypes.c_int64]
        _REF = l
    return _REF


def refpath_lib():
    """librefpath.so: loom.cpp's host path (device-to-host copy per row, then the scan), timed in C."""
    global _REFPATH
    if _REFPATH is None:
        if not os.path.exists(REFPATH_PATH):
            subprocess.run(["make", "-s", "-C", HERE, "librefpath.so"], check=True)
        l = ctypes.CDLL(REFPATH_PATH)
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        l.refpath_greedy_decode.restype = ctypes.c_double
        l.refpath_greedy_decode.argtypes = [vp, i64, i64, i64, vp]
        l.refpath_argmax_tensor_rows.restype = ctypes.c_double
        l.refpath_argmax_tensor_rows.argtypes = [vp, i64, i64, i64, vp]
        l.refpath_ctc_driver.restype = ctypes.c_double
        l.refpath_ctc_driver.argtypes = [vp, i64, i64, i64, i32, vp, vp]
        _REFPATH = l
    return _REFPATH


def _dtype_of(a):
    if a.dtype == np.float32:
        return F32
    if a.dtype == np.uint16:  # bf16 bit patterns
        return BF16
    raise TypeError(f"oracle logits must be float32 or uint16 (bf16 bits), got {a.dtype}")


# ---------------------------------------------------------------------------------------------

def argmax(row):
    row = np.ascontiguousarray(row, dtype=np.float32)
    return int(lib().oracle_argmax(_ptr(row), row.size))


def argmax_tensor_row(data, requested_row, lo=0, hi=-1):
    """Returns (status, id)."""
    data = np.ascontiguousarray(data, dtype=np.float32)
    rows, n = data.shape
    out = ctypes.c_int64(-1)
    st = lib().oracle_argmax_tensor_row(_ptr(data), n, rows, n, requested_row, lo, hi, ctypes.byref(out))
    return st, out.value


def argmax_tensor_rows(data):
    data = np.ascontiguousarray(data, dtype=np.float32)
    rows, n = data.shape
    out = np.zeros(rows, dtype=np.int32)
    st = lib().oracle_argmax_tensor_rows(_ptr(data), n, rows, n, _ptr(out))
    return st, out


def argmax_row_array(flat, n_vocab, row_index):
    flat = np.ascontiguousarray(flat, dtype=np.float64)
    out = ctypes.c_int64(-1)
    st = lib().oracle_argmax_row_array(_ptr(flat), flat.size, n_vocab, row_index, ctypes.byref(out))
    return st, out.value


def argmax_rows(logits, lo=0, hi=-1, nthreads=1):
    logits = np.ascontiguousarray(logits)
    rows, n = logits.shape
    out = np.zeros(rows, dtype=np.int32)
    st = lib().oracle_argmax_rows(_ptr(logits), _dtype_of(logits), rows, n, n, lo, hi, _ptr(out), nthreads)
    if st:
        raise RuntimeError(f"oracle_argmax_rows status {st}")
    return out


def ctc_greedy(logits, blank, want_logp=False, nthreads=1):
    """logits [n_utt, n_frames, n_classes] -> list of (ids, frames) per utterance, frame ids, frame logp."""
    logits = np.ascontiguousarray(logits)
    if logits.ndim == 2:
        logits = logits[None]
    U, F, C = logits.shape
    ids = np.zeros((U, F), dtype=np.int32)
    frames = np.zeros((U, F), dtype=np.int32)
    lens = np.zeros(U, dtype=np.int32)
    fid = np.zeros((U, F), dtype=np.int32)
    flp = np.zeros((U, F), dtype=np.float32) if want_logp else None
    st = lib().oracle_ctc_greedy(_ptr(logits), _dtype_of(logits), U, F, C, blank, _ptr(ids), _ptr(frames), _ptr(lens),
                                 _ptr(fid), _ptr(flp), nthreads)
    if st:
        raise RuntimeError(f"oracle_ctc_greedy status {st}")
    seqs = [(ids[u, :lens[u]].copy(), frames[u, :lens[u]].copy()) for u in range(U)]
    return seqs, fid, flp


def ref_ctc_greedy_decode(logits2d, blank):
    """loom.cpp's own ctc_greedy_decode (needs oracle/_ref/)."""
    logits2d = np.ascontiguousarray(logits2d, dtype=np.float32)
    F, C = logits2d.shape
    out = np.zeros(F, dtype=np.int32)
    n = ref_lib().ref_ctc_greedy_decode(_ptr(logits2d), F, C, blank, _ptr(out), F)
    return out[:n].copy()


def sample_rows(logits, u, temperature, repetition_penalty=1.0, top_k=40, top_p=1.0, history=None, want_logp=True,
                nthreads=1):
    """Returns dict(status, ids, prob, logp, topk)."""
    logits = np.ascontiguousarray(logits)
    rows, n = logits.shape
    u = np.ascontiguousarray(u, dtype=np.float32)
    hist = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
    hl = 0 if hist is None else hist.shape[1]
    ids = np.zeros(rows, dtype=np.int32)
    prob = np.zeros(rows, dtype=np.float32)
    logp = np.zeros(rows, dtype=np.float32) if want_logp else None
    topk = np.zeros((rows, top_k), dtype=np.int32)
    st = lib().oracle_sample_rows(_ptr(logits), _dtype_of(logits), rows, n, n, _ptr(hist), hl, _ptr(u), temperature,
                                  repetition_penalty, top_k, top_p, _ptr(ids), _ptr(prob), _ptr(logp), _ptr(topk),
                                  nthreads)
    return dict(status=st, ids=ids, prob=prob, logp=logp, topk=topk)


def shard_record_bytes(top_k):
    return int(lib().oracle_shard_record_bytes(top_k))


def shard_partial(logits, vocab_offset, vocab_total, temperature, repetition_penalty=1.0, top_k=64, history=None,
                  nthreads=1):
    logits = np.ascontiguousarray(logits)
    rows, n = logits.shape
    hist = None if history is None else np.ascontiguousarray(history, dtype=np.int32)
    hl = 0 if hist is None else hist.shape[1]
    rec = np.zeros(rows * shard_record_bytes(top_k), dtype=np.uint8)
    st = lib().oracle_shard_partial(_ptr(logits), _dtype_of(logits), rows, n, n, vocab_offset, vocab_total, _ptr(hist),
                                    hl, temperature, repetition_penalty, top_k, _ptr(rec), nthreads)
    return st, rec


def shard_merge(records, n_shards, rows, u, temperature, top_k=64, top_p=1.0):
    records = np.ascontiguousarray(records, dtype=np.uint8)
    u = np.ascontiguousarray(u, dtype=np.float32)
    ids = np.zeros(rows, dtype=np.int32)
    prob = np.zeros(rows, dtype=np.float32)
    logp = np.zeros(rows, dtype=np.float32)
    topk = np.zeros((rows, top_k), dtype=np.int32)
    st = lib().oracle_shard_merge(_ptr(records), n_shards, rows, _ptr(u), temperature, top_k, top_p, _ptr(ids),
                                  _ptr(prob), _ptr(logp), _ptr(topk))
    return dict(status=st, ids=ids, prob=prob, logp=logp, topk=topk)


def exp_d(x):
    return float(lib().oracle_exp_d(float(x)))
