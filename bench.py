"""Benchmark of the logits->token stage on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl {b200,reference}] [--workload NAME]

Default workload (the headline): the full sampling chain -- repetition penalty 1.1 over a 256-id
history, temperature 0.7, top-k 40, top-p 0.9, inverse-CDF draw -- on f32 logits [1024, 151936]
(Qwen3-0.6B vocabulary) per GPU, synthetic N(0, 3^2). A step is one call of loom_sample_rows over
the whole batch. Rows are partitioned across GPUs with no collective: every rank samples its own
1024 rows ("weak" scaling), and `value` is all ranks' rows / the slowest rank's time.

Other workloads (--workload): greedy (argmax of the same batch), ctc ([32, 1500, 1025] f32, blank
1024), shard (one GPU's shard of the Gemma-3-vocabulary chain: [256, 32768] bf16, T 1, top-k 64,
top-p 0.95, plus the merge of 8 shards' records).

--impl reference times the reference's CPU path on this host's cores: loom.cpp has no sampler, so
for the sampling chain that is the CPU oracle (a C restatement of the chain, all host threads).
"""
import argparse
import json
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


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profiled_traffic(name):
    """dram bytes per launch from a committed ncu summary (profiles/<name>.txt), or None."""
    path = os.path.join(ROOT, "profiles", f"{name}.txt")
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return int(float(line.split(":", 1)[1].strip()))
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle samples while the timed region runs."""

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
                                          "--format=csv,noheader,nounits", "-lms", "100"],
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
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


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

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    import torch
    import torch.distributed as dist

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def max_over_ranks(v, world):
    import torch
    import torch.distributed as dist

    if world == 1:
        return v
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ------------------------------------------------------------------------------------------------
# workloads: each returns (step_fn(i), rows_per_step, algorithmic_bytes_per_step, launches_per_step,
#                          e2e_fn or None, config dict, kernel name)

def workload_sample(sel, synth, torch, dev, rank):
    bufs = []
    for b in range(2):  # two batches, alternated: 1.24 GB, ten times the L2
        x, hist, u = synth.sample_chain(ROWS, seed=2 + 1000 * rank + b, vocab=VOCAB, hist_len=HIST, device="cuda")
        bufs.append((x, hist, u))
    ids = torch.empty(ROWS, dtype=torch.int32, device=dev)
    prob = torch.empty(ROWS, dtype=torch.float32, device=dev)
    ws = sel.Workspace(dev)

    def step(i):
        x, hist, u = bufs[i & 1]
        sel.sample_rows_into(x, u, ids, prob, T, R, K, P, history=hist, workspace=ws)

    # end to end through the public API: host (pinned) logits/history/uniforms in, ids/probs out
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

    h2d = hx.numel() * 4 + hh.numel() * 4 + hu.numel() * 4
    d2h = ROWS * 8
    cfg = {"workload": "sampling chain: penalty 1.1 (256-id history), T 0.7, top-k 40, top-p 0.9, draw",
           "rows_per_gpu": ROWS, "vocab": VOCAB, "logits": "f32", "global_batch": None,
           "l2": "inputs larger than L2 (two alternating 622 MB batches per GPU)"}
    return step, ROWS, ROWS * VOCAB * 4, 1, (e2e, h2d, d2h), cfg, "sample_stream_kernel", bufs


def workload_greedy(sel, synth, torch, dev, rank):
    bufs = [synth.sample_chain(ROWS, seed=2 + 1000 * rank + b, device="cuda")[0] for b in range(2)]
    ids = torch.empty(ROWS, dtype=torch.int32, device=dev)
    ws = sel.Workspace(dev)

    def step(i):
        sel.argmax_rows_into(bufs[i & 1], ids, workspace=ws)

    cfg = {"workload": "greedy argmax", "rows_per_gpu": ROWS, "vocab": VOCAB, "logits": "f32",
           "l2": "inputs larger than L2 (two alternating 622 MB batches per GPU)"}
    return step, ROWS, ROWS * VOCAB * 4, 1, None, cfg, "argmax_stream_kernel", bufs


def workload_ctc(sel, synth, torch, dev, rank):
    bufs = [synth.ctc_frames(32, 1500, seed=4 + 1000 * rank + b, device="cuda") for b in range(2)]
    ids = torch.empty(32, 1500, dtype=torch.int32, device=dev)
    fr = torch.empty(32, 1500, dtype=torch.int32, device=dev)
    ln = torch.empty(32, dtype=torch.int32, device=dev)
    ws = sel.Workspace(dev)

    def step(i):
        sel.ctc_greedy_into(bufs[i & 1], synth.CTC_BLANK, ids, fr, ln, workspace=ws)

    cfg = {"workload": "CTC greedy decode", "utterances": 32, "frames": 1500, "classes": 1025, "blank": 1024,
           "logits": "f32", "l2": "inputs larger than L2 (two alternating 197 MB batches per GPU)"}
    return step, 32 * 1500, 32 * 1500 * 1025 * 4, 1, None, cfg, "ctc_kernel", bufs


def workload_shard(sel, synth, torch, dev, rank):
    rows, G, k = 256, 8, 64
    x, u = synth.gemma_vocab(rows, seed=3 + rank, device="cuda")
    shard = [x[:, 0:32768].contiguous() for _ in range(2)]
    rb = sel.shard_record_bytes(k)
    recs = torch.zeros(G, rows * rb, dtype=torch.uint8, device=dev)
    ids = torch.empty(rows, dtype=torch.int32, device=dev)
    prob = torch.empty(rows, dtype=torch.float32, device=dev)
    ws = sel.Workspace(dev)
    for g in range(G):
        sel.shard_partial_into(x[:, g * 32768:(g + 1) * 32768], recs[g], g * 32768, 262144, 1.0, 1.0, k, 0.95,
                               workspace=ws)

    def step(i):
        sel.shard_partial_into(shard[i & 1], recs[0], 0, 262144, 1.0, 1.0, k, 0.95, workspace=ws)
        sel.shard_merge_into(recs, G, rows, u, ids, prob, 1.0, k, 0.95)

    cfg = {"workload": "vocab shard of the Gemma-3 chain (1 of 8) + merge of 8 shard records", "rows": rows,
           "shard_vocab": 32768, "vocab": 262144, "logits": "bf16",
           "l2": "inputs smaller than L2 (16.8 MB shard): L2-resident, reported as such"}
    return step, rows, rows * 32768 * 2, 2, None, cfg, "sample_stream_kernel", [x, shard]


WORKLOADS = {"sample": workload_sample, "greedy": workload_greedy, "ctc": workload_ctc, "shard": workload_shard}


def cpu_baseline_sample(synth, torch, nthreads, rows=1024, min_seconds=10.0):
    """The oracle's sampling chain on the [rows, V] host batch with all host threads, repeated until
    at least `min_seconds` of CPU time have passed (a bounded sample). Returns (rows/s, seconds, passes)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_binding as ob

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
    return rows * passes / dt, dt, passes


def run_reference(args):
    import torch

    import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if args.workload != "sample":
        print(json.dumps({"impl": "reference", "unavailable": "reference arm is defined for the sampling chain"}))
        return 0
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_binding as ob

    nthreads = os.cpu_count() or 1
    rows = 256  # a bounded sample of the 1024-row batch per step
    x, hist, u = synth.sample_chain(rows, seed=2, device="cpu")
    xn, hn, un = x.numpy(), hist.numpy(), u.numpy()
    for _ in range(args.warmup):
        ob.sample_rows(xn, un, T, R, K, P, hn, want_logp=False, nthreads=nthreads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        ob.sample_rows(xn, un, T, R, K, P, hn, want_logp=False, nthreads=nthreads)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = rows * args.steps / total
    sample = f"{rows} of the 1024 rows per step, logits in host memory, {nthreads} threads"
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * total / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "sampling chain: penalty 1.1 (256-id history), T 0.7, top-k 40, top-p 0.9, draw",
                       "rows_per_gpu": ROWS, "vocab": VOCAB, "logits": "f32"},
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": nthreads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "loom.cpp has no sampler; its CPU path for this chain is the oracle port (C, all host threads)"}
    print(json.dumps(line))
    return 0


def run_b200(args):
    import torch

    import loom_select as sel
    import synth

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    step, rows, bytes_per_step, launches, e2e, cfg, kname, _keep = WORKLOADS[args.workload](sel, synth, torch, dev,
                                                                                              rank)
    stream = torch.cuda.current_stream()
    for i in range(args.warmup):
        step(i)
    barrier(world)

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        time.sleep(0.3)  # let the sampler start
        barrier(world)
        for i in range(args.steps):
            starts[i].record(stream)
            step(i)
            ends[i].record(stream)
        barrier(world)
    total_ms = starts[0].elapsed_time(ends[-1])
    per_launch_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    total_ms = max_over_ranks(total_ms, world)
    avg_ms = max_over_ranks(sum(per_launch_ms) / len(per_launch_ms), world)

    e2e_obj = None
    if e2e is not None and not args.no_e2e:
        fn, h2d, d2h = e2e
        for i in range(2):
            fn(i)
        barrier(world)
        e_s, e_e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = max(3, min(args.steps, 20))
        e_s.record(stream)
        for i in range(n_e2e):
            fn(i)
        e_e.record(stream)
        barrier(world)
        e_ms = max_over_ranks(e_s.elapsed_time(e_e), world)
        e2e_obj = {"value": rows * world * n_e2e / (e_ms / 1e3), "unit": "rows/s", "h2d_bytes_per_step": h2d,
                   "d2h_bytes_per_step": d2h, "steps": n_e2e,
                   "path": "pinned host logits/history/uniforms -> H2D -> loom_sample_rows -> D2H ids/probs"}

    peak, peak_kind = measured_peak()
    # one step is one launch of the dominant kernel (plus the merge for the shard workload)
    achieved = bytes_per_step / (avg_ms / 1e3) / 1e9
    value = rows * world * args.steps / (total_ms / 1e3)
    line = {
        "metric": METRIC if args.workload == "sample" else f"rows/sec ({args.workload})",
        "value": value, "unit": "rows/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32" if args.workload != "shard" else "bf16", "data": "synthetic", "config": cfg,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": profiled_traffic(f"{kname}_{args.workload}"), "peak_source": peak_kind,
                     "kernel": kname, "algorithmic_bytes_per_launch": bytes_per_step,
                     "avg_launch_ms": avg_ms},
        "gpu_launches": launches * args.steps,
        "clocks": clocks.summary(),
    }
    if e2e_obj is not None:
        line["e2e"] = e2e_obj
    if rank == 0 and world == 1 and args.workload == "sample" and not args.no_cpu_baseline:
        nthreads = os.cpu_count() or 1
        v, dt, passes = cpu_baseline_sample(synth, torch, nthreads)
        line["cpu_baseline"] = {"value": v, "unit": "rows/s", "cores": nthreads, "kind": "port",
                                "sample": f"the [1024, {VOCAB}] f32 batch of the same workload, {passes} passes "
                                          f"({dt:.1f} s), host memory"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


def set_rows(n):
    global ROWS
    ROWS = n


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--workload", default="sample", choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end (host buffers) measurement")
    ap.add_argument("--rows", type=int, default=ROWS, help="rows per GPU (profiling a smaller case)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    set_rows(args.rows)
    if args.impl == "reference":
        return run_reference(args)
    return run_b200(args)


if __name__ == "__main__":
    sys.exit(main())
