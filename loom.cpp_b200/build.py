"""Builds libloom_select.so -- the logits->token kernels for sm_100a -- in place, with nvcc.

Usage: python loom.cpp_b200/build.py [--force]

Objects go to _build/loom_select/ at the repository root; the shared library is written next to this
file so it travels with the source tree. A source is recompiled when it or any header is newer than
its object.
"""
import argparse
import concurrent.futures
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
OPS = os.path.join(PKG, "src", "ops")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "libloom_select.so")
OBJDIR = os.path.join(ROOT, "_build", "loom_select")

# (source, object name, extra flags), compiled in parallel
SOURCES = [("select_capi.cu", "select_capi.o", []),
           ("select_argmax.cu", "select_argmax.o", []),
           ("select_ctc.cu", "select_ctc.o", []),
           ("select_sample.cu", "select_sample.o", []),
           ("select_noalloc.cu", "select_noalloc.o", []),
           ("select_windows.cu", "select_windows.o", []),
           ("select_lmhead.cu", "select_lmhead.o", [])]

# sm_100a only. --fmad=false: no multiply-add contraction anywhere, so every float expression
# rounds as written (the decision arithmetic also spells its operations as explicit intrinsics).
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17", "--fmad=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", INCLUDE, "-I", OPS,
]


def _nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if cand and (os.path.isabs(cand) and os.path.exists(cand) or not os.path.isabs(cand)):
            return cand
    return "nvcc"


def _headers():
    hs = []
    for d in (OPS, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                hs.append(os.path.join(d, f))
    return hs


def _stale(obj, src, newest_header):
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return os.path.getmtime(src) > t or newest_header > t


def build(force=False, jobs=None, verbose=False):
    """Compiles every kernel source for sm_100a and links libloom_select.so. Returns its path."""
    os.makedirs(OBJDIR, exist_ok=True)
    nvcc = _nvcc()
    newest_header = max(os.path.getmtime(h) for h in _headers())
    todo = []
    objs = []
    for s, oname, extra in SOURCES:
        src = os.path.join(OPS, s)
        obj = os.path.join(OBJDIR, oname)
        objs.append(obj)
        if force or _stale(obj, src, newest_header):
            todo.append((src, obj, extra))

    def compile_one(job):
        src, obj, extra = job
        cmd = [nvcc] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        return obj

    jobs = jobs or os.cpu_count() or 4
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        list(ex.map(compile_one, todo))

    if todo or force or not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", LIB] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
