"""Benchmark of the logits->token stage on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {b200,reference}] [--workload NAME]

Headline (the JSON line's value): the full sampling chain -- repetition penalty 1.1 over a 256-id
history, temperature 0.7, top-k 40, top-p 0.9, inverse-CDF draw -- on f32 logits [1024, 151936]
(Qwen3-0.6B vocabulary) per GPU, synthetic N(0, 3^2). A step is one call of loom_sample_rows over the
whole batch. Every rank samples its own 1024 rows with no collective ("weak" scaling); `value` is all
ranks' rows / the slowest rank's time. A timed region is exactly K steps between a barrier and a
synchronize; regions repeat until they hold at least a second of device time, and the line reports
the median region (max over ranks).

The same line carries, under their own keys, the other workloads of the stage, each timed on the
device with CUDA events (max over ranks) and each checked against the oracle once:
  sweep   the chain on a GLOBAL batch B in {1, 16, 128, 1024, 4096} whose rows are split across the
          N ranks (strong scaling; B = 1024 is the strong split of the headline batch)
  shard   the Gemma-3-vocabulary chain, [256, 262144] bf16, T 1, top-k 64, top-p 0.95: each rank owns
          262144 / N ids, runs loom_sample_shard_partial on its slice, the records are all-gathered
          (NCCL over NVLink when N > 1) and loom_sample_shard_merge recombines them
  decode  greedy decode, [1, 151936] f32 x 512 steps (one row per step): device time per step, the
          host-synchronised step of a decode loop, and one CUDA graph of the 512 steps
  greedy  argmax of the headline batch
  ctc     greedy CTC of [32, 1500, 1025] f32, blank 1024
On rank 0 at N = 1 it also times the CPU paths: the oracle's sampling chain (loom.cpp has no sampler)
and loom.cpp's own host path where one exists -- a device-to-host copy per row or frame, then the
strict '>' scan on one thread (oracle/refpath.c), and loom.cpp's own compiled ctc_greedy_decode.

--workload NAME runs one workload alone (for profiling); --impl reference times the CPU arm on the
headline configuration (the oracle's chain: the only CPU implementation of it) with all host threads.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "loom.cpp_b200"))

VOCAB = 151936
ROWS = 1024
HIST = 256
T, R, K, P = 0.7, 1.1, 40, 0.9
METRIC = "rows/sec logits->token at V=151936,B=1024 (1/2/4/8 GPU); HBM GB/s vs peak"
L2_BYTES = 126 * 2**20
POOL_BYTES = 400 * 10**6  # inputs rotate through at least this much memory: > 3x the L2
SWEEP_B = (1, 16, 128, 1024, 4096)
GEMMA_VOCAB, SHARD_ROWS, SHARD_K, SHARD_P = 262144, 256, 64, 0.95
DECODE_STEPS = 512
CTC_SHAPE, CTC_BLANK = (32, 1500, 1025), 1024


def headline_config():
    return {"workload": "sampling chain: penalty 1.1 (256-id history), T 0.7, top-k 40, top-p 0.9, draw",
            "rows_per_gpu": ROWS, "vocab": VOCAB, "logits": "f32", "global_batch": None,
            "l2": "inputs larger than L2 (two alternating 622 MB batches per GPU)"}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(name):
    """DRAM bytes per launch from a committed ncu summary (profiles/<name>.txt), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", f"{name}.txt")) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed regions run."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
                power.append(float(f[3]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "sm_mhz_min": min(sm), "reasons": sorted(reasons),
                "samples": len(sm), "power_w_max": max(power) if power else None}


# ------------------------------------------------------------------------------------------------
# process group and timing

def dist_setup(n_gpus):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    import torch.distributed as dist

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def reduce_max(values, world):
    """Element-wise max over ranks of a list of floats (every rank gets the result)."""
    import torch
    import torch.distributed as dist

    if world == 1:
        return list(values)
    t = torch.tensor(list(values), dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.cpu().tolist()


def all_true(flag, world):
    return reduce_max([0.0 if flag else 1.0], world)[0] == 0.0


def timed_regions(step, steps, world, min_device_s, max_regions=400, clocks=None):
    """Regions of exactly `steps` calls of step(i), each between a barrier and a synchronize, timed with
    CUDA events on the current stream (the region, and every call in it). The first region decides how
    many follow (the same count on every rank) so that they hold min_device_s of device time.
    Returns (region times in ms, max over ranks per region; mean call time in ms, max over ranks)."""
    import torch

    stream = torch.cuda.current_stream()
    regions, calls = [], []
    i = 0

    def one_region():
        nonlocal i
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        barrier(world)
        s0.record(stream)
        for j in range(steps):
            ev[j][0].record(stream)
            step(i)
            ev[j][1].record(stream)
            i += 1
        s1.record(stream)
        barrier(world)
        regions.append(s0.elapsed_time(s1))
        calls.extend(a.elapsed_time(b) for a, b in ev)

    one_region()
    first = reduce_max([regions[0]], world)[0]
    n = max(1, min(max_regions, int(math.ceil(min_device_s * 1e3 / max(first, 1e-3)))))
    for _ in range(n - 1):
        one_region()
    regions = reduce_max(regions, world)
    call_ms = reduce_max([sum(calls) / len(calls)], world)[0]
    return regions, call_ms


# ------------------------------------------------------------------------------------------------
# inputs

def sample_pool(synth, torch, rows_per_step, seed, min_rows=2):
    """A pool of distinct sampling-chain rows (logits, history, u) on the device, at least POOL_BYTES of
    logits and at least two steps' worth, so consecutive steps never find their inputs in L2."""
    n = max(min_rows * rows_per_step, int(math.ceil(POOL_BYTES / (VOCAB * 4))))
    n = (n // rows_per_step) * rows_per_step if rows_per_step else n
    x, hist, u = synth.sample_chain(n, seed=seed, vocab=VOCAB, hist_len=HIST, device="cuda")
    return x, hist, u, n // max(rows_per_step, 1)


def oracle_mod():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_binding

    return oracle_binding


def check_sample(ob, x, hist, u, ids, prob, nthreads, T_=T, R_=R, K_=K, P_=P):
    want = ob.sample_rows(x.cpu().numpy(), u.cpu().numpy(), T_, R_, K_, P_,
                          None if hist is None else hist.cpu().numpy(), want_logp=False, nthreads=nthreads)
    import numpy as np

    ok_ids = bool(np.array_equal(ids.cpu().numpy(), want["ids"]))
    gp, wp = prob.cpu().numpy().astype(np.float64), want["prob"].astype(np.float64)
    ok_prob = bool(np.all(np.abs(gp - wp) <= 1e-5 * np.abs(wp)))
    return ok_ids and ok_prob


# ------------------------------------------------------------------------------------------------
# workloads (all ranks run each one; each returns a dict for the line)

def run_headline(args, sel, synth, torch, dev, rank, world, clocks_index):
    bufs = []
    for b in range(2):  # two batches, alternated: 1.24 GB, ten times the L2
        bufs.append(synth.sample_chain(ROWS, seed=2 + 1000 * rank + b, vocab=VOCAB, hist_len=HIST, device="cuda"))
    ids = torch.empty(ROWS, dtype=torch.int32, device=dev)
    prob = torch.empty(ROWS, dtype=torch.float32, device=dev)
    ws = sel.Workspace(dev)

    def step(i):
        x, hist, u = bufs[i & 1]
        sel.sample_rows_into(x, u, ids, prob, T, R, K, P, history=hist, workspace=ws)

    for i in range(args.warmup):
        step(i)
    barrier(world)
    with ClockSampler(clocks_index) as clocks:
        time.sleep(0.3)  # let the sampler start
        regions, call_ms = timed_regions(step, args.steps, world, args.min_seconds, clocks=clocks)
    med = statistics.median(regions)
    out = {"regions": regions, "median_ms": med, "call_ms": call_ms, "clocks": clocks.summary()}

    # parity of one batch's result (rank 0; the oracle on all host threads)
    if rank == 0:
        x, hist, u = bufs[0]
        sel.sample_rows_into(x, u, ids, prob, T, R, K, P, history=hist, workspace=ws)
        torch.cuda.synchronize()
        out["parity"] = check_sample(oracle_mod(), x, hist, u, ids, prob, os.cpu_count() or 1)
    barrier(world)

    # end to end through the public API: host (pinned) logits/history/uniforms in, ids/probs out
    if not args.no_e2e:
        hx = bufs[0][0].cpu().pin_memory()
        hh = bufs[0][1].cpu().pin_memory()
        hu = bufs[0][2].cpu().pin_memory()
        dx, dh, du = torch.empty_like(bufs[0][0]), torch.empty_like(bufs[0][1]), torch.empty_like(bufs[0][2])
        hid = torch.empty(ROWS, dtype=torch.int32).pin_memory()
        hpr = torch.empty(ROWS, dtype=torch.float32).pin_memory()

        def e2e(i):
            dx.copy_(hx, non_blocking=True)
            dh.copy_(hh, non_blocking=True)
            du.copy_(hu, non_blocking=True)
            sel.sample_rows_into(dx, du, ids, prob, T, R, K, P, history=dh, workspace=ws)
            hid.copy_(ids, non_blocking=True)
            hpr.copy_(prob, non_blocking=True)

        for i in range(2):
            e2e(i)
        n_e2e = max(3, min(args.steps, 20))
        e_regions, _ = timed_regions(e2e, n_e2e, world, 0.0, max_regions=1)
        out["e2e"] = {"value": ROWS * world * n_e2e / (e_regions[0] / 1e3), "unit": "rows/s",
                      "h2d_bytes_per_step": hx.numel() * 4 + hh.numel() * 4 + hu.numel() * 4,
                      "d2h_bytes_per_step": ROWS * 8, "steps": n_e2e,
                      "path": "pinned host logits/history/uniforms -> H2D -> loom_sample_rows -> D2H ids/probs"}
    del bufs
    return out


def run_sweep(args, sel, synth, torch, dev, rank, world, peak):
    import select_dist

    res = []
    nthreads = os.cpu_count() or 1
    for B in SWEEP_B:
        lo, hi = select_dist.split(B, world, rank)
        n = hi - lo
        ws = sel.Workspace(dev)
        if n > 0:
            x, hist, u, n_slices = sample_pool(synth, torch, n, seed=5000 + B * 16 + rank)
            ids = torch.empty(n, dtype=torch.int32, device=dev)
            prob = torch.empty(n, dtype=torch.float32, device=dev)

            def step(i):
                s = (i % n_slices) * n
                sel.sample_rows_into(x[s:s + n], u[s:s + n], ids, prob, T, R, K, P, history=hist[s:s + n],
                                     workspace=ws)
        else:
            def step(i):
                pass
        for i in range(3):
            step(i)
        steps = max(args.steps, 20)
        regions, call_ms = timed_regions(step, steps, world, args.extra_seconds)
        med = statistics.median(regions) / steps
        ok = True
        if n > 0:
            step(0)
            torch.cuda.synchronize()
            ok = check_sample(oracle_mod(), x[:n], hist[:n], u[:n], ids, prob, nthreads)
        ok = all_true(ok, world)
        gbs = B * VOCAB * 4 / (med / 1e3) / 1e9
        res.append({"global_batch": B, "rows_per_gpu_max": -(-B // world), "ms_per_step": med,
                    "rows_per_s": B / (med / 1e3), "hbm_gbs": gbs, "hbm_frac": gbs / (peak * world),
                    "parity_ok": ok})
        if n > 0:
            del x, hist, u
        torch.cuda.empty_cache()
    return res


def run_shard(args, sel, synth, torch, dev, rank, world):
    """The vocabulary-sharded chain: partial on this rank's slice, all-gather of the records, merge."""
    import numpy as np
    import torch.distributed as dist

    import select_dist

    V, rows, k = GEMMA_VOCAB, SHARD_ROWS, SHARD_K
    v0, v1 = select_dist.split(V, world, rank)
    sv = v1 - v0
    slice_bytes = rows * sv * 2
    n_bufs = max(2, int(math.ceil(POOL_BYTES / slice_bytes)))
    xs, us = [], []
    full0 = None
    for b in range(n_bufs):
        x, u = synth.gemma_vocab(rows, seed=3 + 100 * b, device="cuda")  # identical on every rank
        xs.append(x[:, v0:v1].contiguous())
        us.append(u)
        if b == 0:
            full0 = x
        else:
            del x
    rb = sel.shard_record_bytes(k)
    local = torch.empty(rows * rb, dtype=torch.uint8, device=dev)
    gathered = torch.empty(world, rows * rb, dtype=torch.uint8, device=dev)
    ids = torch.empty(rows, dtype=torch.int32, device=dev)
    prob = torch.empty(rows, dtype=torch.float32, device=dev)
    logp = torch.empty(rows, dtype=torch.float32, device=dev)
    ws = sel.Workspace(dev)
    stream = torch.cuda.current_stream()
    phases = []  # per step: (after partial, after gather) events

    def step(i, record=True):
        b = i % n_bufs
        sel.shard_partial_into(xs[b], local, v0, V, 1.0, 1.0, k, SHARD_P, workspace=ws)
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record(stream)
        if world > 1:
            dist.all_gather_into_tensor(gathered.view(-1), local)
        else:
            gathered[0].copy_(local)
        e2 = torch.cuda.Event(enable_timing=True)
        e2.record(stream)
        sel.shard_merge_into(gathered, world, rows, us[b], ids, prob, 1.0, k, SHARD_P, out_logp=logp)
        if record:
            phases.append((e1, e2))

    for i in range(3):
        step(i, record=False)
    steps = max(args.steps, 20)
    phases.clear()
    # the step's own start and end events, paired with its phase events
    starts, ends = [], []

    def timed_step(i):
        s = torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step(i)
        e = torch.cuda.Event(enable_timing=True)
        e.record(stream)
        starts.append(s)
        ends.append(e)

    regions, _ = timed_regions(timed_step, steps, world, args.extra_seconds)
    part = [s.elapsed_time(p[0]) for s, p in zip(starts, phases)]
    gath = [p[0].elapsed_time(p[1]) for p in phases]
    merg = [p[1].elapsed_time(e) for p, e in zip(phases, ends)]
    part_ms, gath_ms, merg_ms = reduce_max([statistics.median(part), statistics.median(gath),
                                            statistics.median(merg)], world)
    med = statistics.median(regions) / steps
    # parity: every rank's merged result of batch 0 against the oracle's unsharded chain (rank 0 checks)
    step(0, record=False)
    torch.cuda.synchronize()
    ok = True
    if rank == 0:
        ob = oracle_mod()
        bits = synth.bf16_bits(full0)
        want = ob.sample_rows(bits, us[0].cpu().numpy(), 1.0, 1.0, k, SHARD_P, None, want_logp=True,
                              nthreads=os.cpu_count() or 1)
        ok = bool(np.array_equal(ids.cpu().numpy(), want["ids"]))
        gp, wp = prob.cpu().numpy().astype(np.float64), want["prob"].astype(np.float64)
        ok = ok and bool(np.all(np.abs(gp - wp) <= 1e-5 * np.abs(wp)))
        gl, wl = logp.cpu().numpy().astype(np.float64), want["logp"].astype(np.float64)
        ok = ok and bool(np.all(np.abs(gl - wl) <= 1e-5 * np.maximum(1.0, np.abs(wl))))
    ok = all_true(ok, world)
    gbs = rows * V * 2 / (med / 1e3) / 1e9
    return {"config": "[256, 262144] bf16 (Gemma-3 vocabulary, N(0, 2.5^2) + Zipf(1.1) log-bias), T 1, top-k 64, "
                      "top-p 0.95, log-prob out", "shards": world, "shard_vocab": sv,
            "exchange": "NCCL all_gather_into_tensor" if world > 1 else "none (one shard)",
            "record_bytes_per_gpu": rows * rb, "ms_per_step": med, "rows_per_s": rows / (med / 1e3),
            "partial_us": 1e3 * part_ms, "allgather_us": 1e3 * gath_ms, "merge_us": 1e3 * merg_ms,
            "logit_gbs_per_gpu": rows * sv * 2 / (part_ms / 1e3) / 1e9,
            "l2": f"{n_bufs} alternating slices of {slice_bytes / 1e6:.1f} MB per GPU (> 3x L2)",
            "parity_ok": ok, "aggregate_logit_gbs": gbs}


def run_decode(args, sel, synth, torch, dev, rank, world, cpu):
    """Config 1: greedy decode, one [1, 151936] row per step, 512 steps."""
    import numpy as np

    rows = torch.cat([synth.greedy_decode_step(s, seed=1, device="cuda") for s in range(DECODE_STEPS)])
    out = torch.empty(DECODE_STEPS, dtype=torch.int32, device=dev)
    ws = sel.Workspace(dev)
    stream = torch.cuda.current_stream()
    for s in range(8):
        sel.argmax_rows_into(rows[s], out[s:s + 1], workspace=ws)
    torch.cuda.synchronize()
    # (a) device time per step, launches back to back
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(DECODE_STEPS)]
    barrier(world)
    for s in range(DECODE_STEPS):
        ev[s][0].record(stream)
        sel.argmax_rows_into(rows[s], out[s:s + 1], workspace=ws)
        ev[s][1].record(stream)
    torch.cuda.synchronize()
    dev_us = statistics.median(a.elapsed_time(b) for a, b in ev) * 1e3
    ids_a = out.cpu().numpy().copy()
    # (b) a decode loop's step: launch, read the id back (pinned), synchronise
    hid = torch.empty(1, dtype=torch.int32).pin_memory()
    lat = []
    for s in range(DECODE_STEPS):
        t0 = time.perf_counter()
        sel.argmax_rows_into(rows[s], out[s:s + 1], workspace=ws)
        hid.copy_(out[s:s + 1], non_blocking=True)
        stream.synchronize()
        lat.append(time.perf_counter() - t0)
    loop_us = statistics.median(lat) * 1e6
    # (c) one CUDA graph of the 512 steps
    graph_us = None
    try:
        g = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream()
        cap.wait_stream(stream)
        with torch.cuda.stream(cap):
            sel.argmax_rows_into(rows[0], out[0:1], workspace=ws)  # warm on the capture stream
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=cap):
            for s in range(DECODE_STEPS):
                sel.argmax_rows_into(rows[s], out[s:s + 1], workspace=ws)
        out.fill_(-1)
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(5):
            g.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        graph_us = e0.elapsed_time(e1) * 1e3 / (5 * DECODE_STEPS)
        ids_g = out.cpu().numpy().copy()
        del g
    except Exception as e:  # noqa: BLE001 -- reported, not hidden
        ids_g = None
        graph_us = f"capture failed: {e}"
    dev_us, loop_us = reduce_max([dev_us, loop_us], world)
    if isinstance(graph_us, float):
        graph_us = reduce_max([graph_us], world)[0]
    ob = oracle_mod()
    want = ob.argmax_rows(rows.cpu().numpy(), nthreads=os.cpu_count() or 1)
    ok = bool(np.array_equal(ids_a, want)) and (ids_g is None or bool(np.array_equal(ids_g, want)))
    res = {"config": "greedy argmax, [1, 151936] f32 N(0, 3^2) + 8 spikes of +10, 512 steps (one row each)",
           "device_us_per_step": graph_us if isinstance(graph_us, float) else None,
           "device_time": "the 512 steps as one CUDA graph, replayed (no host launch gaps)",
           "launch_us_per_step": dev_us,
           "launch_time": "events around each launch from Python: bound by the host's launch rate",
           "decode_loop_us_per_step": loop_us, "graph_us_per_step": graph_us, "steps": DECODE_STEPS,
           "parity_ok": all_true(ok, world)}
    if cpu:
        got = np.zeros(DECODE_STEPS, dtype=np.int32)
        secs = ob.refpath_lib().refpath_greedy_decode(rows.data_ptr(), DECODE_STEPS, VOCAB, VOCAB,
                                                      got.ctypes.data)
        res["cpu_reference_equivalent"] = {
            "us_per_step": secs * 1e6 / DECODE_STEPS, "cores": 1, "kind": "reference-equivalent",
            "sample": "512 steps: cudaMemcpy of the row to pageable host memory, then the strict '>' scan on "
                      "one thread (generation.cpp:56-74, oracle/refpath.c)",
            "parity_ok": bool(np.array_equal(got, want))}
    del rows
    return res


def run_greedy(args, sel, synth, torch, dev, rank, world, peak, cpu):
    import numpy as np

    bufs = [synth.sample_chain(ROWS, seed=2 + 1000 * rank + b, device="cuda")[0] for b in range(2)]
    ids = torch.empty(ROWS, dtype=torch.int32, device=dev)
    ws = sel.Workspace(dev)

    def step(i):
        sel.argmax_rows_into(bufs[i & 1], ids, workspace=ws)

    for i in range(3):
        step(i)
    steps = max(args.steps, 20)
    regions, call_ms = timed_regions(step, steps, world, args.extra_seconds)
    med = statistics.median(regions) / steps
    step(0)
    torch.cuda.synchronize()
    ob = oracle_mod()
    host = bufs[0].cpu().numpy()
    want = ob.argmax_rows(host, nthreads=os.cpu_count() or 1)
    ok = all_true(bool(np.array_equal(ids.cpu().numpy(), want)), world)
    gbs = ROWS * VOCAB * 4 / (call_ms / 1e3) / 1e9
    res = {"config": "argmax of [1024, 151936] f32 per GPU", "ms_per_step": med,
           "rows_per_s": ROWS * world / (med / 1e3), "hbm_gbs": gbs, "hbm_frac": gbs / peak,
           "traffic": profiled_traffic("argmax_stream_kernel_greedy"), "parity_ok": ok}
    if cpu:
        got = np.zeros(ROWS, dtype=np.int32)
        secs = ob.refpath_lib().refpath_argmax_tensor_rows(bufs[0].data_ptr(), ROWS, VOCAB, VOCAB, got.ctypes.data)
        nt = os.cpu_count() or 1
        t0 = time.perf_counter()
        ob.argmax_rows(host, nthreads=nt)
        par = time.perf_counter() - t0
        res["cpu_reference_equivalent"] = {
            "rows_per_s": ROWS / secs, "cores": 1, "kind": "reference-equivalent",
            "sample": "1024 rows: one cudaMemcpy per row to pageable host memory, then the strict '>' scan "
                      "(argmax_tensor_rows, lua_bridge.cpp:343-365; oracle/refpath.c)",
            "parity_ok": bool(np.array_equal(got, want))}
        res["cpu_host_parallel"] = {"rows_per_s": ROWS / par, "cores": nt, "kind": "port",
                                    "sample": "the same scan, rows over all host threads, logits in host memory"}
    del bufs
    return res


def run_ctc(args, sel, synth, torch, dev, rank, world, peak, cpu):
    import concurrent.futures

    import numpy as np

    U, F, C = CTC_SHAPE
    bufs = [synth.ctc_frames(U, F, seed=4 + 1000 * rank + b, device="cuda") for b in range(2)]
    ids = torch.empty(U, F, dtype=torch.int32, device=dev)
    fr = torch.empty(U, F, dtype=torch.int32, device=dev)
    ln = torch.empty(U, dtype=torch.int32, device=dev)
    ws = sel.Workspace(dev)

    def step(i):
        sel.ctc_greedy_into(bufs[i & 1], CTC_BLANK, ids, fr, ln, workspace=ws)

    for i in range(3):
        step(i)
    steps = max(args.steps, 20)
    regions, call_ms = timed_regions(step, steps, world, args.extra_seconds)
    med = statistics.median(regions) / steps
    step(0)
    torch.cuda.synchronize()
    ob = oracle_mod()
    host = bufs[0].cpu().numpy()
    nt = os.cpu_count() or 1
    use_ref = ob.ref_available()
    ok = True
    for u in range(U):
        n = int(ln[u].item())
        want = ob.ref_ctc_greedy_decode(host[u], CTC_BLANK) if use_ref else ob.ctc_greedy(host[u], CTC_BLANK)[0][0][0]
        ok = ok and bool(np.array_equal(ids[u, :n].cpu().numpy(), want))
    ok = all_true(ok, world)
    gbs = U * F * C * 4 / (call_ms / 1e3) / 1e9
    res = {"config": "greedy CTC, [32, 1500, 1025] f32 N(0, 1) (+4 on the blank 1024 for 70% of frames, else on a "
                     "random id)", "ms_per_step": med, "frames_per_s": U * F * world / (med / 1e3),
           "hbm_gbs": gbs, "hbm_frac": gbs / peak, "traffic": profiled_traffic("ctc_ring_kernel_ctc"),
           "parity_ok": ok, "parity_against": "loom.cpp's own ctc_greedy_decode" if use_ref else "the oracle"}
    if cpu:
        got = np.zeros((U, F), dtype=np.int32)
        glen = np.zeros(U, dtype=np.int32)
        secs = ob.refpath_lib().refpath_ctc_driver(bufs[0].data_ptr(), U, F, C, CTC_BLANK, got.ctypes.data,
                                                   glen.ctypes.data)
        okr = all(np.array_equal(got[u, :glen[u]], ids[u, :glen[u]].cpu().numpy()) for u in range(U))
        res["cpu_reference_equivalent"] = {
            "frames_per_s": U * F / secs, "cores": 1, "kind": "reference-equivalent",
            "sample": "32 x 1500 frames: one cudaMemcpy per frame (argmax_tensor_rows, lua_bridge.cpp:343-365), "
                      "the scan, then the collapse of ctc_decode.cpp:22-29 (oracle/refpath.c)", "parity_ok": bool(okr)}
        if use_ref:
            t0 = time.perf_counter()
            hb = bufs[0].cpu().numpy()
            t1 = time.perf_counter()
            for u in range(U):
                ob.ref_ctc_greedy_decode(hb[u], CTC_BLANK)
            t2 = time.perf_counter()
            with concurrent.futures.ThreadPoolExecutor(nt) as ex:
                t3 = time.perf_counter()
                list(ex.map(lambda u: ob.ref_ctc_greedy_decode(hb[u], CTC_BLANK), range(U)))
                t4 = time.perf_counter()
            res["cpu_reference"] = {
                "frames_per_s": U * F / (t2 - t0), "cores": 1, "kind": "reference",
                "sample": "one device-to-host copy of the batch, then loom.cpp's own compiled ctc_greedy_decode "
                          "(src/core/ctc_decode.cpp, oracle/_ref) per utterance on one thread",
                "copy_s": t1 - t0}
            res["cpu_reference_parallel"] = {
                "frames_per_s": U * F / (t4 - t3), "cores": nt, "kind": "reference",
                "sample": "loom.cpp's own ctc_greedy_decode, utterances over all host threads, logits in host memory"}
    del bufs
    return res


def run_lm_head(args, sel, torch, dev, rank, world, peak):
    """Greedy selection fused into the LM-head GEMM (loom_lm_head_argmax) against the unfused path the
    engine runs today: a library GEMM writing bf16 logits, then loom_argmax_rows reading them back.
    [rows, 2048] bf16 hidden states x a [151936, 2048] bf16 weight (a Qwen-size LM head, 622 MB; two
    copies alternate, so the weight is never L2-resident). Tensor-bound at 1024 rows, HBM-bound at 1."""
    hdim, tol = 2048, 2e-3
    g = torch.Generator(device=dev).manual_seed(17 + rank)
    weights = [(torch.randn(VOCAB, hdim, generator=g, device=dev) * (1.0 / hdim ** 0.5)).to(torch.bfloat16)
               for _ in range(2)]
    ws = sel.Workspace(dev)
    out = {"config": f"hidden [rows, {hdim}] bf16 x lm_head [{VOCAB}, {hdim}] bf16 (two alternating copies), "
                     "greedy id + logit + log-sum-exp per row",
           "tensor_peak_tflops": 1590.0, "tensor_peak_source": "fallback (no measured bf16 figure here)"}
    for rows in (1, 16, 128, ROWS):
        hidden = torch.randn(rows, hdim, generator=g, device=dev).to(torch.bfloat16)
        ids = torch.empty(rows, dtype=torch.int32, device=dev)
        logit = torch.empty(rows, dtype=torch.float32, device=dev)
        lse = torch.empty(rows, dtype=torch.float32, device=dev)
        ids_u = torch.empty(rows, dtype=torch.int32, device=dev)

        def fused(i):
            sel.lm_head_argmax_into(hidden, weights[i & 1], ids, logit, lse, workspace=ws)

        def unfused(i):
            sel.argmax_rows_into(hidden @ weights[i & 1].t(), ids_u, workspace=ws)

        res = {}
        for name, fn in (("fused", fused), ("unfused_gemm_then_argmax", unfused)):
            for i in range(3):
                fn(i)
            steps = max(args.steps, 20)
            regions, call_ms = timed_regions(fn, steps, world, args.extra_seconds / 4)
            res[name + "_us"] = 1e3 * statistics.median(regions) / steps
        fused(0)
        torch.cuda.synchronize()
        ref = hidden.float() @ weights[0].float().t()
        chosen = ref.gather(1, ids.long()[:, None])[:, 0]
        ok = bool((chosen >= ref.max(dim=1).values - tol).all()) and \
            bool(torch.allclose(lse, torch.logsumexp(ref, dim=1), atol=tol, rtol=0)) and \
            ws.read_status() == sel.OK
        del ref
        us = res["fused_us"]
        flops = 2.0 * rows * hdim * VOCAB
        res.update({"rows_per_s": rows * world / (us / 1e6), "tflops": flops / (us / 1e6) / 1e12,
                    "weight_gbs": VOCAB * hdim * 2 / (us / 1e6) / 1e9,
                    "speedup_vs_unfused": res["unfused_gemm_then_argmax_us"] / us,
                    "parity_ok": all_true(ok, world)})
        res["tensor_frac"] = res["tflops"] / out["tensor_peak_tflops"]
        res["hbm_frac"] = res["weight_gbs"] / peak
        out[f"rows_{rows}"] = res
    del weights
    return out


def cpu_baseline_sample(synth, rows=1024, min_seconds=10.0):
    """The oracle's sampling chain on the [rows, V] host batch with all host threads, repeated until at
    least `min_seconds` have passed (a bounded sample). Returns (rows/s, seconds, passes, threads)."""
    ob = oracle_mod()
    nthreads = os.cpu_count() or 1
    x, hist, u = synth.sample_chain(rows, seed=2, device="cpu")
    xn, hn, un = x.numpy(), hist.numpy(), u.numpy()
    ob.sample_rows(xn[:8], un[:8], T, R, K, P, hn[:8], want_logp=False, nthreads=nthreads)  # warm
    passes = 0
    t0 = time.perf_counter()
    while True:
        ob.sample_rows(xn, un, T, R, K, P, hn, want_logp=False, nthreads=nthreads)
        passes += 1
        dt = time.perf_counter() - t0
        if dt >= min_seconds:
            break
    t1 = time.perf_counter()
    ob.sample_rows(xn[:64], un[:64], T, R, K, P, hn[:64], want_logp=False, nthreads=1)
    single = 64 / (time.perf_counter() - t1)
    return rows * passes / dt, dt, passes, nthreads, single


# ------------------------------------------------------------------------------------------------

def run_reference(args):
    """The CPU arm: the oracle's sampling chain (the only CPU implementation of it; loom.cpp has none)
    on the headline configuration -- every row of the [1024, 151936] batch each step, all host threads."""
    import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    ob = oracle_mod()
    nthreads = os.cpu_count() or 1
    x, hist, u = synth.sample_chain(ROWS, seed=2, device="cpu")
    xn, hn, un = x.numpy(), hist.numpy(), u.numpy()
    for _ in range(args.warmup):
        ob.sample_rows(xn, un, T, R, K, P, hn, want_logp=False, nthreads=nthreads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ob.sample_rows(xn, un, T, R, K, P, hn, want_logp=False, nthreads=nthreads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = ROWS * args.steps / total
    sample = f"all {ROWS} rows of the batch per step, logits in host memory, {nthreads} threads"
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": headline_config(),
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": nthreads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "loom.cpp has no sampler; the CPU implementation of this chain is the oracle port "
                    "(oracle/select_oracle.c), run on every row with all host threads"}
    print(json.dumps(line))
    return 0


def run_b200(args):
    import torch

    import loom_select as sel
    import synth

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    peak, peak_kind = measured_peak()
    cpu = rank == 0 and world == 1 and not args.no_cpu_baseline
    only = args.workload

    line = {"metric": METRIC, "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": headline_config()}
    if only in (None, "sample"):
        h = run_headline(args, sel, synth, torch, dev, rank, world, local)
        med = h["median_ms"]
        achieved = ROWS * VOCAB * 4 / (h["call_ms"] / 1e3) / 1e9
        line.update({
            "value": ROWS * world * args.steps / (med / 1e3), "ms_per_step": med / args.steps,
            "timed_regions": {"count": len(h["regions"]), "steps_each": args.steps, "median_ms": med,
                              "min_ms": min(h["regions"]), "max_ms": max(h["regions"]),
                              "device_s": sum(h["regions"]) / 1e3, "statistic": "median region, max over ranks"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "traffic": profiled_traffic("sample_stream_kernel_sample"), "peak_source": peak_kind,
                         "kernel": "sample_stream_kernel", "algorithmic_bytes_per_launch": ROWS * VOCAB * 4,
                         "avg_launch_ms": h["call_ms"]},
            "gpu_launches": args.steps * len(h["regions"]),
            "gpu_launches_note": "sample_stream_kernel launches in all timed regions (one per step)",
            "clocks": h["clocks"]})
        if "parity" in h:
            line["parity_ok"] = h["parity"]
        if "e2e" in h:
            line["e2e"] = h["e2e"]
    extras = {}
    if only in (None, "sweep"):
        extras["sweep"] = run_sweep(args, sel, synth, torch, dev, rank, world, peak)
    if only in (None, "shard"):
        extras["shard"] = run_shard(args, sel, synth, torch, dev, rank, world)
    if only in (None, "decode"):
        extras["decode"] = run_decode(args, sel, synth, torch, dev, rank, world, cpu)
    if only in (None, "greedy"):
        extras["greedy"] = run_greedy(args, sel, synth, torch, dev, rank, world, peak, cpu)
    if only in (None, "ctc"):
        extras["ctc"] = run_ctc(args, sel, synth, torch, dev, rank, world, peak, cpu)
    if only in (None, "lm_head"):
        extras["lm_head"] = run_lm_head(args, sel, torch, dev, rank, world, peak)
    line.update(extras)
    if "sweep" in extras:
        strong = [s for s in extras["sweep"] if s["global_batch"] == ROWS][0]
        line["strong_split"] = {"global_batch": ROWS, "rows_per_gpu": ROWS // world, "ms_per_step":
                                strong["ms_per_step"], "rows_per_s": strong["rows_per_s"]}
    if cpu and only in (None, "sample"):
        v, dt, passes, nthreads, single = cpu_baseline_sample(synth)
        line["cpu_baseline"] = {"value": v, "unit": "rows/s", "cores": nthreads, "kind": "port",
                                "sample": f"the [1024, {VOCAB}] f32 batch of the same workload, {passes} passes "
                                          f"({dt:.1f} s), host memory",
                                "single_thread_rows_per_s": single}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    global ROWS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default=None, choices=["sample", "sweep", "shard", "decode", "greedy", "ctc", "lm_head"],
                    help="run one workload alone (profiling)")
    ap.add_argument("--min-seconds", type=float, default=1.0, help="device time of the headline's timed regions")
    ap.add_argument("--extra-seconds", type=float, default=0.25, help="device time of each other workload")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffers) measurement")
    ap.add_argument("--rows", type=int, default=ROWS, help="rows per GPU of the headline (profiling a smaller case)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    ROWS = args.rows
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
