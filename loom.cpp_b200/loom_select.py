"""Python mirror of loom.cpp's logits->token selection, running on the B200 kernels.

This module binds the C-ABI of include/loom_select.h (libloom_select.so, built in place by
build.py next to this file) with ctypes, and offers the selection calls of loom.cpp under their
loom.cpp names on CUDA tensors:

    argmax_row(logits, row=-1)               loom.argmax_row(module, row)     src/core/lua_bridge.cpp:729-743
    argmax_row_range(logits, row, lo, hi)    loom.argmax_row_range(...)       src/core/lua_bridge.cpp:779-797
    argmax_rows(logits)                      loom.argmax_rows(module)         src/core/lua_bridge.cpp:808-822
    ctc_greedy_decode(logits, blank_id)      loom::ctc_greedy_decode          src/core/ctc_decode.cpp:7-31
    sample_rows(logits, ...)                 the sampling chain (no loom.cpp counterpart)
    shard_partial / shard_merge              the vocabulary-sharded chain (no loom.cpp counterpart)

Errors raise SelectError, as loom.cpp raises loom::Error (include/loom/loom_errors.h:10) and its
Lua bindings turn that into a Lua error (lua_bridge.cpp:26-32). The library must be present: there
is no fallback of any kind, and importing this module on a machine without it fails.

torch is used for device memory, streams and host<->device copies only.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libloom_select.so")

F32 = 0
BF16 = 1
MAX_TOP_K = 1024
MAX_WINDOWS = 8

OK = 0
EINVAL = 1
EDTYPE = 2
EWINDOW = 3
EWORKSPACE = 4
ECUDA = 5
ETIMEOUT = 6
EHISTORY = 7
EPARAM = 8
ESHAPE = 9

# Every entry point include/loom_select.h declares.
EXPORTS = (
    "loom_select_strerror",
    "loom_select_abi_version",
    "loom_argmax_workspace_size",
    "loom_sample_workspace_size",
    "loom_ctc_workspace_size",
    "loom_select_workspace_init",
    "loom_select_read_status",
    "loom_select_test_wait_fault",
    "loom_argmax_rows",
    "loom_argmax_windows_workspace_size",
    "loom_argmax_windows",
    "loom_sample_rows",
    "loom_sample_rows_noalloc",
    "loom_shard_record_bytes",
    "loom_sample_shard_partial",
    "loom_sample_shard_merge",
    "loom_ctc_greedy",
    "loom_lm_head_workspace_size",
    "loom_lm_head_argmax",
)


class SampleParams(ctypes.Structure):
    _fields_ = [
        ("temperature", ctypes.c_float),
        ("repetition_penalty", ctypes.c_float),
        ("top_k", ctypes.c_int32),
        ("top_p", ctypes.c_float),
    ]


class SelectError(RuntimeError):
    def __init__(self, status, what=""):
        self.status = status
        msg = _lib().loom_select_strerror(status).decode()
        super().__init__(f"{what}: {msg} (status {status})" if what else f"{msg} (status {status})")


_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python {os.path.join(_HERE, 'build.py')}`")
        lib = ctypes.CDLL(LIB_PATH)
        vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
        sig = {
            "loom_select_strerror": (ctypes.c_char_p, [ctypes.c_int]),
            "loom_select_abi_version": (ctypes.c_int, []),
            "loom_argmax_workspace_size": (sz, [i64, i64]),
            "loom_sample_workspace_size": (sz, [i64, i64, i32]),
            "loom_ctc_workspace_size": (sz, [i64, i64]),
            "loom_select_workspace_init": (ctypes.c_int, [vp, sz, vp]),
            "loom_select_read_status": (ctypes.c_int, [vp, vp]),
            "loom_select_test_wait_fault": (ctypes.c_int, [vp, i64, i32, vp]),
            "loom_argmax_rows": (ctypes.c_int, [vp, ctypes.c_int, i64, i64, i64, i64, i64, vp, vp, sz, vp]),
            "loom_argmax_windows_workspace_size": (sz, [i64, i32]),
            "loom_argmax_windows": (ctypes.c_int, [vp, ctypes.c_int, i64, i64, i64, vp, vp, i32, vp, vp, sz, vp]),
            "loom_sample_rows": (ctypes.c_int, [vp, ctypes.c_int, i64, i64, i64, vp, i32, vp,
                                                ctypes.POINTER(SampleParams), vp, vp, vp, vp, vp, sz, vp]),
            "loom_sample_rows_noalloc": (ctypes.c_int, [vp, ctypes.c_int, i64, i64, i64, vp, i32, vp,
                                                        ctypes.POINTER(SampleParams), vp, vp, vp, vp, vp, vp]),
            "loom_shard_record_bytes": (sz, [i32]),
            "loom_sample_shard_partial": (ctypes.c_int, [vp, ctypes.c_int, i64, i64, i64, i64, i64, vp, i32,
                                                         ctypes.POINTER(SampleParams), vp, vp, sz, vp]),
            "loom_sample_shard_merge": (ctypes.c_int, [vp, i32, i64, vp, ctypes.POINTER(SampleParams),
                                                       vp, vp, vp, vp, vp]),
            "loom_ctc_greedy": (ctypes.c_int, [vp, ctypes.c_int, i64, i64, i64, i32, vp, vp, vp, vp, vp, vp, sz, vp]),
            "loom_lm_head_workspace_size": (sz, [i64, i64]),
            "loom_lm_head_argmax": (ctypes.c_int, [vp, vp, i64, i64, i64, vp, vp, vp, vp, sz, vp]),
        }
        for name, (res, args) in sig.items():
            f = getattr(lib, name)
            f.restype = res
            f.argtypes = args
        _LIB = lib
    return _LIB


def lib():
    """The loaded libloom_select.so (ctypes.CDLL)."""
    return _lib()


def check(status, what=""):
    if status != OK:
        raise SelectError(status, what)


# ----------------------------------------------------------------------------------------------
# torch plumbing

def _torch():
    import torch
    return torch


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream_handle(stream=None):
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _dtype_code(t):
    torch = _torch()
    if t.dtype == torch.float32:
        return F32
    if t.dtype == torch.bfloat16:
        return BF16
    raise SelectError(EDTYPE, f"logits dtype {t.dtype}")


def _rows_view(logits):
    """(rows, n_vocab, row_stride) of a 1-D or 2-D CUDA tensor with unit column stride."""
    if logits.dim() == 1:
        return 1, logits.shape[0], logits.shape[0]
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise SelectError(EINVAL, "logits must be [rows, n_vocab] with contiguous rows")
    return logits.shape[0], logits.shape[1], logits.stride(0)


class Workspace:
    """A caller-owned workspace (a CUDA uint8 tensor), zeroed once, grown on demand."""

    def __init__(self, device=None):
        self.device = device
        self.buf = None

    def get(self, nbytes, stream=None):
        torch = _torch()
        nbytes = max(int(nbytes), 256)
        if self.buf is None or self.buf.numel() < nbytes:
            dev = self.device if self.device is not None else torch.device("cuda", torch.cuda.current_device())
            self.buf = torch.empty(nbytes + 256, dtype=torch.uint8, device=dev)
            check(_lib().loom_select_workspace_init(_ptr(self.buf), self.buf.numel(), _stream_handle(stream)),
                  "loom_select_workspace_init")
        return self.buf

    def read_status(self, stream=None):
        if self.buf is None:
            return OK
        return _lib().loom_select_read_status(_ptr(self.buf), _stream_handle(stream))


_DEFAULT_WS = {}


def default_workspace():
    torch = _torch()
    dev = torch.cuda.current_device()
    if dev not in _DEFAULT_WS:
        _DEFAULT_WS[dev] = Workspace(torch.device("cuda", dev))
    return _DEFAULT_WS[dev]


# ----------------------------------------------------------------------------------------------
# greedy argmax

def argmax_rows_into(logits, out, lo=0, hi=-1, workspace=None, stream=None):
    """One absolute id per row over [lo, hi) into the int32 CUDA tensor `out` (asynchronous)."""
    rows, n_vocab, stride = _rows_view(logits)
    ws = workspace or default_workspace()
    need = _lib().loom_argmax_workspace_size(rows, n_vocab)
    buf = ws.get(need, stream)
    check(_lib().loom_argmax_rows(_ptr(logits), _dtype_code(logits), rows, n_vocab, stride, lo, hi, _ptr(out),
                                  _ptr(buf), buf.numel(), _stream_handle(stream)), "loom_argmax_rows")
    return out


def argmax_rows(logits, lo=0, hi=-1, workspace=None, stream=None):
    """loom.argmax_rows: one id per row, as a list of floats like the Lua binding returns."""
    torch = _torch()
    rows, _, _ = _rows_view(logits)
    out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    argmax_rows_into(logits, out, lo, hi, workspace, stream)
    return [float(v) for v in out.cpu().tolist()]


def argmax_row_range(logits, row, lo, hi, workspace=None, stream=None):
    """loom.argmax_row_range / argmax_tensor_row (lua_bridge.cpp:302-330): row < 0 means the last row,
    hi < 0 means n_vocab, the id is absolute; an empty or out-of-range window or row raises."""
    torch = _torch()
    rows, n_vocab, _ = _rows_view(logits)
    r = rows - 1 if row < 0 else row
    if n_vocab <= 0 or r < 0 or r >= rows:
        raise SelectError(EWINDOW, f"row {row} out of range for an output with {rows} row(s) of width {n_vocab}")
    view = logits if logits.dim() == 1 else logits[r:r + 1]
    out = torch.empty(1, dtype=torch.int32, device=logits.device)
    argmax_rows_into(view, out, lo, hi, workspace, stream)
    return float(out.item())


def argmax_windows_into(logits, windows, out, workspace=None, stream=None):
    """Every row's absolute argmax over each [lo, hi) of `windows` (a list of (lo, hi), hi < 0 meaning
    n_vocab) into the int32 CUDA tensor `out` of shape [rows, len(windows)], in one launch."""
    rows, n_vocab, stride = _rows_view(logits)
    n = len(windows)
    lo = (ctypes.c_int64 * max(n, 1))(*[int(w[0]) for w in windows])
    hi = (ctypes.c_int64 * max(n, 1))(*[int(w[1]) for w in windows])
    ws = workspace or default_workspace()
    buf = ws.get(_lib().loom_argmax_windows_workspace_size(rows, max(n, 1)), stream)
    check(_lib().loom_argmax_windows(_ptr(logits), _dtype_code(logits), rows, n_vocab, stride, lo, hi, n, _ptr(out),
                                     _ptr(buf), buf.numel(), _stream_handle(stream)), "loom_argmax_windows")
    return out


def argmax_windows(logits, windows, workspace=None, stream=None):
    """loom.argmax_row_range over several windows of every row at once: an int32 CUDA tensor
    [rows, len(windows)] of absolute ids (lua_bridge.cpp:779-797, batched)."""
    torch = _torch()
    rows, _, _ = _rows_view(logits)
    out = torch.empty(rows, len(windows), dtype=torch.int32, device=logits.device)
    return argmax_windows_into(logits, windows, out, workspace, stream)


def argmax_row(logits, row=-1, workspace=None, stream=None):
    """loom.argmax_row (module form) / Generator::argmax on one row."""
    return argmax_row_range(logits, row, 0, -1, workspace, stream)


# ----------------------------------------------------------------------------------------------
# sampling chain

def sample_rows_into(logits, u, out_ids, out_prob, temperature, repetition_penalty=1.0, top_k=40, top_p=1.0,
                     history=None, out_logp=None, out_topk=None, workspace=None, stream=None):
    """The fused sampling chain on device tensors (asynchronous). history: int32 [rows, H] or None."""
    rows, n_vocab, stride = _rows_view(logits)
    hl = 0 if history is None else int(history.shape[-1])
    p = SampleParams(temperature, repetition_penalty, top_k, top_p)
    ws = workspace or default_workspace()
    buf = ws.get(_lib().loom_sample_workspace_size(rows, n_vocab, top_k), stream)
    check(_lib().loom_sample_rows(_ptr(logits), _dtype_code(logits), rows, n_vocab, stride, _ptr(history), hl,
                                  _ptr(u), ctypes.byref(p), _ptr(out_ids), _ptr(out_prob), _ptr(out_logp),
                                  _ptr(out_topk), _ptr(buf), buf.numel(), _stream_handle(stream)),
          "loom_sample_rows")


def sample_rows_noalloc_into(logits, u, out_ids, out_prob, temperature, repetition_penalty=1.0, top_k=40,
                             top_p=1.0, history=None, out_logp=None, out_topk=None, out_status=None, stream=None):
    """sample_rows_into without a workspace: the library's own fixed scratch (top_k <= 64; calls must
    not overlap on the GPU). out_status: an int32 device tensor of one element, or None."""
    rows, n_vocab, stride = _rows_view(logits)
    hl = 0 if history is None else int(history.shape[-1])
    p = SampleParams(temperature, repetition_penalty, top_k, top_p)
    check(_lib().loom_sample_rows_noalloc(_ptr(logits), _dtype_code(logits), rows, n_vocab, stride, _ptr(history),
                                          hl, _ptr(u), ctypes.byref(p), _ptr(out_ids), _ptr(out_prob),
                                          _ptr(out_logp), _ptr(out_topk), _ptr(out_status),
                                          _stream_handle(stream)),
          "loom_sample_rows_noalloc")


def sample_rows(logits, u, temperature, repetition_penalty=1.0, top_k=40, top_p=1.0, history=None,
                want_logp=False, want_topk=False, workspace=None, stream=None):
    """Returns (ids int32, probs f32[, logp f32][, topk int32 [rows, k]]) as CUDA tensors."""
    torch = _torch()
    rows, _, _ = _rows_view(logits)
    dev = logits.device
    ids = torch.empty(rows, dtype=torch.int32, device=dev)
    prob = torch.empty(rows, dtype=torch.float32, device=dev)
    logp = torch.empty(rows, dtype=torch.float32, device=dev) if want_logp else None
    topk = torch.empty(rows, top_k, dtype=torch.int32, device=dev) if want_topk else None
    sample_rows_into(logits, u, ids, prob, temperature, repetition_penalty, top_k, top_p, history, logp, topk,
                     workspace, stream)
    out = [ids, prob]
    if want_logp:
        out.append(logp)
    if want_topk:
        out.append(topk)
    return tuple(out)


def shard_record_bytes(top_k):
    return int(_lib().loom_shard_record_bytes(top_k))


def shard_partial_into(logits, out_records, vocab_offset, vocab_total, temperature, repetition_penalty=1.0,
                       top_k=64, top_p=1.0, history=None, workspace=None, stream=None):
    """This GPU's shard [rows, shard_vocab] -> rows records of shard_record_bytes(top_k) (uint8 tensor)."""
    rows, n_vocab, stride = _rows_view(logits)
    hl = 0 if history is None else int(history.shape[-1])
    p = SampleParams(temperature, repetition_penalty, top_k, top_p)
    ws = workspace or default_workspace()
    buf = ws.get(_lib().loom_sample_workspace_size(rows, n_vocab, top_k), stream)
    check(_lib().loom_sample_shard_partial(_ptr(logits), _dtype_code(logits), rows, n_vocab, stride, vocab_offset,
                                           vocab_total, _ptr(history), hl, ctypes.byref(p), _ptr(out_records),
                                           _ptr(buf), buf.numel(), _stream_handle(stream)),
          "loom_sample_shard_partial")


def shard_merge_into(records, n_shards, rows, u, out_ids, out_prob, temperature, top_k=64, top_p=1.0,
                     out_logp=None, out_topk=None, stream=None):
    """Gathered records [n_shards][rows] -> the same outputs as sample_rows over the whole vocabulary."""
    p = SampleParams(temperature, 1.0, top_k, top_p)
    check(_lib().loom_sample_shard_merge(_ptr(records), n_shards, rows, _ptr(u), ctypes.byref(p), _ptr(out_ids),
                                         _ptr(out_prob), _ptr(out_logp), _ptr(out_topk), _stream_handle(stream)),
          "loom_sample_shard_merge")


# ----------------------------------------------------------------------------------------------
# CTC

def ctc_greedy_into(logits, blank, out_ids, out_frames, out_len, out_frame_ids=None, out_frame_logp=None,
                    workspace=None, stream=None):
    """logits: [n_utt, n_frames, n_classes] (or [n_frames, n_classes]) contiguous CUDA tensor."""
    if logits.dim() == 2:
        n_utt, (n_frames, n_classes) = 1, logits.shape
    else:
        n_utt, n_frames, n_classes = logits.shape
    if not logits.is_contiguous():
        raise SelectError(EINVAL, "CTC logits must be contiguous")
    ws = workspace or default_workspace()
    buf = ws.get(_lib().loom_ctc_workspace_size(n_utt, n_frames), stream)
    check(_lib().loom_ctc_greedy(_ptr(logits), _dtype_code(logits), n_utt, n_frames, n_classes, blank, _ptr(out_ids),
                                 _ptr(out_frames), _ptr(out_len), _ptr(out_frame_ids), _ptr(out_frame_logp),
                                 _ptr(buf), buf.numel(), _stream_handle(stream)), "loom_ctc_greedy")


def ctc_greedy(logits, blank, want_frame_ids=False, want_frame_logp=False, workspace=None, stream=None):
    """Returns (ids [n_utt, n_frames], frames [n_utt, n_frames], lens [n_utt][, frame_ids][, frame_logp])."""
    torch = _torch()
    n_utt, n_frames = (1, logits.shape[0]) if logits.dim() == 2 else (logits.shape[0], logits.shape[1])
    dev = logits.device
    ids = torch.empty(n_utt, n_frames, dtype=torch.int32, device=dev)
    frames = torch.empty(n_utt, n_frames, dtype=torch.int32, device=dev)
    lens = torch.empty(n_utt, dtype=torch.int32, device=dev)
    fid = torch.empty(n_utt, n_frames, dtype=torch.int32, device=dev) if want_frame_ids else None
    flp = torch.empty(n_utt, n_frames, dtype=torch.float32, device=dev) if want_frame_logp else None
    ctc_greedy_into(logits, blank, ids, frames, lens, fid, flp, workspace, stream)
    out = [ids, frames, lens]
    if want_frame_ids:
        out.append(fid)
    if want_frame_logp:
        out.append(flp)
    return tuple(out)


def ctc_greedy_decode(logits, blank_id, workspace=None, stream=None):
    """loom::ctc_greedy_decode(logits, n_frames, n_classes, blank_id) on a [n_frames, n_classes] CUDA
    tensor: the collapsed token ids as a list."""
    ids, _, lens = ctc_greedy(logits, blank_id, workspace=workspace, stream=stream)
    n = int(lens[0].item())
    return ids[0, :n].cpu().tolist()


# ----------------------------------------------------------------------------------------------
# greedy selection fused into the LM-head GEMM

def lm_head_argmax_into(hidden, weight, out_ids, out_logit=None, out_lse=None, workspace=None, stream=None):
    """Greedy ids of logits = hidden @ weight.T without materialising the logits (asynchronous).

    hidden [rows, hidden_dim] and weight [n_vocab, hidden_dim] are contiguous bf16 CUDA tensors (the
    weight in ggml's lm_head layout); out_ids int32 [rows]; out_logit / out_lse f32 [rows] or None."""
    torch = _torch()
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise SelectError(EDTYPE, "lm_head_argmax takes bf16 hidden states and weight")
    if hidden.dim() == 1:
        hidden = hidden.view(1, -1)
    if hidden.dim() != 2 or weight.dim() != 2 or not hidden.is_contiguous() or not weight.is_contiguous():
        raise SelectError(EINVAL, "hidden [rows, hidden_dim] and weight [n_vocab, hidden_dim] must be contiguous")
    if hidden.shape[1] != weight.shape[1]:
        raise SelectError(EINVAL, "hidden and weight disagree on hidden_dim")
    rows, hdim = hidden.shape
    n_vocab = weight.shape[0]
    ws = workspace or default_workspace()
    need = _lib().loom_lm_head_workspace_size(rows, n_vocab)
    buf = ws.get(need, stream)
    check(_lib().loom_lm_head_argmax(_ptr(hidden), _ptr(weight), rows, hdim, n_vocab, _ptr(out_ids),
                                     _ptr(out_logit), _ptr(out_lse), _ptr(buf), buf.numel(), _stream_handle(stream)),
          "loom_lm_head_argmax")
    return out_ids


def lm_head_argmax(hidden, weight, want_logit=True, want_lse=True, workspace=None, stream=None):
    """(ids, logit or None, log-sum-exp or None) per row of hidden @ weight.T."""
    torch = _torch()
    rows = 1 if hidden.dim() == 1 else hidden.shape[0]
    dev = hidden.device
    ids = torch.empty(rows, dtype=torch.int32, device=dev)
    logit = torch.empty(rows, dtype=torch.float32, device=dev) if want_logit else None
    lse = torch.empty(rows, dtype=torch.float32, device=dev) if want_lse else None
    lm_head_argmax_into(hidden, weight, ids, logit, lse, workspace, stream)
    return ids, logit, lse
